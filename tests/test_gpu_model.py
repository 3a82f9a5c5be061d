"""LlamaModel forward / greedy decode on the GPU against the oracle.

Logits within 1e-4 relative L2 of the oracle's f32 result; greedy token ids
identical for the first 32 tokens (the north-star parity bar).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


from gguf_cuda import synth
from tiny_models import forward_runs_hp, forward_runs_tensors, min_llama_hp, min_llama_tensors

REL_L2 = 1e-4


def rel_l2(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def top2_margin(logits):
    s = np.sort(np.asarray(logits, np.float64))
    return (s[-1] - s[-2]) / max(abs(s[-1]), 1e-30)


# ---- the reference's own tiny models ---------------------------------------
def test_forward_runs_tiny(ggc, orc, ctx):   # llama.rs:788-899
    m = ggc.LlamaModel(forward_runs_hp(), forward_runs_tensors(), max_ctx=16, ctx=ctx)
    o = orc.Model(forward_runs_hp(), forward_runs_tensors())
    got = m.forward([1, 0], [0, 1])
    want = o.forward([1, 0], [0, 1])
    assert got.size == 8 and np.all(np.isfinite(got))
    assert np.allclose(got, want, atol=1e-6)
    assert m.cache_len() == 2


def test_min_llama_greedy(ggc, ctx):   # tests/inference.rs:275-308
    m = ggc.LlamaModel(min_llama_hp(), min_llama_tensors(), max_ctx=32, ctx=ctx)
    # all logits tie at 0.0: the last maximum wins (sampler.rs:117-122)
    assert m.generate_greedy([0, 0, 1], 5, eos=255) == [7, 7, 7, 7, 7]
    assert m.cache_len() == 3 + 5
    m.reset_cache()
    assert m.generate_greedy([0, 0, 1], 4, eos=7) == []
    assert m.cache_len() == 3
    m2 = ggc.LlamaModel(min_llama_hp(), min_llama_tensors(), max_ctx=32, ctx=ctx)
    assert m2.generate_greedy([0], 8, eos=255) == ggc.LlamaModel(min_llama_hp(), min_llama_tensors(), max_ctx=32,
                                                                 ctx=ctx).generate_greedy([0], 8, eos=255)


# ---- synthetic models of the workload shapes --------------------------------
MINI = dict(vocab_size=1000, embed_dim=512, n_heads=8, n_kv_heads=2, ffn_dim=1024, n_layers=2, rope_freq_base=1e4,
            qkv_bias=True, weights="q4_k_m")


def model_pair(ggc, orc, ctx, cfg, n_layers=None, vocab=None, max_ctx=256, seed=0, kv_f16=False):
    hp, ts = synth.make_model(cfg, n_layers=n_layers, seed=seed, vocab_size=vocab)
    m = ggc.LlamaModel(hp, ts, max_ctx=max_ctx, kv_f16=kv_f16, ctx=ctx)
    o = orc.Model(hp, ts)
    return hp, m, o


CASES = [
    ("mini-q4_k_m", MINI, None, None),
    ("mini-q8_0", dict(MINI, weights="q8_0_normal"), None, None),
    ("mini-q4_0", dict(MINI, weights=2, qkv_bias=False), None, None),
    ("qwen2-0.5b-q8_0-2layers", "qwen2-0.5b-q8_0", 2, None),
    ("llama2-7b-q4_k_m-2layers", "llama2-7b-q4_k_m", 2, None),
    ("llama3-8b-q4_0-1layer", "llama3-8b-q4_0", 1, 32000),
    # every other block format on the span GEMV, whole model
    ("mini-q5_k", dict(MINI, weights=13), None, None),
    ("mini-q3_k_m", dict(MINI, weights=112), None, None),
    ("mini-q3_k_s", dict(MINI, weights=11, qkv_bias=False), None, None),
    ("mini-q2_k", dict(MINI, weights=10), None, None),
    ("mini-q4_1", dict(MINI, weights=3), None, None),
    ("mini-q5_0", dict(MINI, weights=6, qkv_bias=False), None, None),
    ("mini-q5_1", dict(MINI, weights=7), None, None),
    ("mini-q8_k", dict(MINI, weights=15), None, None),
]


@pytest.mark.parametrize("name,cfg,n_layers,vocab", CASES, ids=[c[0] for c in CASES])
def test_prompt_logits_match_oracle(ggc, orc, ctx, name, cfg, n_layers, vocab):
    hp, m, o = model_pair(ggc, orc, ctx, cfg, n_layers, vocab)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, hp["vocab_size"], size=8).astype(np.uint32)
    pos = np.arange(8, dtype=np.int64)
    got = m.forward(prompt, pos)
    want = o.forward(prompt, pos)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, want) <= REL_L2, rel_l2(got, want)
    assert m.cache_len() == o.cache_len() == 8
    # K/V rows in the cache match the oracle's (RoPE + bias applied)
    k, v = m.cache_read(0)
    ko, vo = o.cache_read(0)
    assert rel_l2(k, ko) <= REL_L2 and rel_l2(v, vo) <= REL_L2
    # one more decode step on the cache
    got = m.forward([int(prompt[0])], [8])
    want = o.forward([int(prompt[0])], [8])
    assert rel_l2(got, want) <= REL_L2
    assert m.last_argmax == orc.greedy(got)


@pytest.mark.parametrize("name,cfg,n_layers,vocab", CASES[:4], ids=[c[0] for c in CASES[:4]])
def test_greedy_ids_match_oracle_32(ggc, orc, ctx, name, cfg, n_layers, vocab):
    """Greedy ids identical for the first 32 generated tokens."""
    hp, m, o = model_pair(ggc, orc, ctx, cfg, n_layers, vocab)
    prompt = np.random.default_rng(9).integers(0, hp["vocab_size"], size=6).astype(np.uint32)
    got = m.generate_greedy(prompt, 32)
    want = o.generate_greedy(prompt, 32)
    assert len(got) == 32
    assert got == want
    assert m.cache_len() == o.cache_len() == 6 + 32


def test_generate_equals_step_by_step_forward(ggc, ctx):
    """The device-side loop equals forward() + host argmax, step by step."""
    hp, ts = synth.make_model(MINI, seed=3)
    a = ggc.LlamaModel(hp, ts, max_ctx=128, ctx=ctx)
    b = ggc.LlamaModel(hp, ts, max_ctx=128, ctx=ctx)
    prompt = [1, 2, 3, 4]
    ids = a.generate_greedy(prompt, 16)
    logits = b.forward(prompt, list(range(4)))
    pos, host_ids = 4, []
    for _ in range(16):
        nxt = int(np.flatnonzero(logits == logits.max())[-1])
        host_ids.append(nxt)
        logits = b.forward([nxt], [pos])
        pos += 1
    assert ids == host_ids


def test_generate_continues_cache(ggc, orc, ctx):   # engine.rs:89: generate never resets the cache
    hp, m, o = model_pair(ggc, orc, ctx, MINI, seed=4)
    assert m.generate_greedy([5, 6], 4) == o.generate_greedy([5, 6], 4)
    assert m.generate_greedy([7], 4, start_pos=6) == o.generate_greedy([7], 4, start_pos=6)
    assert m.cache_len() == o.cache_len() == 11


def test_cache_append_read_truncate(ggc, orc, ctx):   # cache.rs:46-93
    hp, m, o = model_pair(ggc, orc, ctx, MINI, seed=6, max_ctx=64)
    kvd = m.kv_dim
    rng = np.random.default_rng(1)
    k = rng.normal(size=(5, kvd)).astype(np.float32)
    v = rng.normal(size=(5, kvd)).astype(np.float32)
    for l in range(hp["n_layers"]):
        m.cache_append(l, k, v)
        o.cache_append(l, k, v)
    assert m.cache_len() == 5
    kk, vv = m.cache_read(1)
    assert np.array_equal(kk, k.reshape(-1)) and np.array_equal(vv, v.reshape(-1))
    # attention over the planted cache
    got = m.forward([3], [5])
    want = o.forward([3], [5])
    assert rel_l2(got, want) <= REL_L2
    m.truncate(2); o.truncate(2)
    assert m.cache_len() == 2
    m.truncate(10)
    assert m.cache_len() == 2
    assert rel_l2(m.forward([4], [2]), o.forward([4], [2])) <= REL_L2
    m.reset_cache()
    assert m.cache_len() == 0


# ---- long cached context: every attention split spans several K/V tiles ------
# (the fused decode attention streams 16 KB tiles through a 3-stage ring; the
# general pair covers the shapes the fused kernel does not take)
HD256 = dict(vocab_size=512, embed_dim=1024, n_heads=4, n_kv_heads=1, ffn_dim=512, n_layers=1, rope_freq_base=1e4,
             qkv_bias=False, weights="q8_0_normal")
LONG_CASES = [
    ("llama2-7b-1layer-ctx1000", "llama2-7b-q4_k_m", 1, 4000, 1000, False),   # hd 128, group 1, 4 tiles / split
    ("mini-ctx3000", MINI, None, None, 3000, False),                            # hd 64, group 4
    ("mini-ctx3000-kv-f16", MINI, None, None, 3000, True),                      # hd 64, f16 cache
    ("llama3-8b-1layer-ctx1500-kv-f16", "llama3-8b-q4_0", 1, 4000, 1500, True),  # hd 128, group 4, f16 cache
    ("hd256-g4-ctx2500", HD256, None, None, 2500, False),                       # hd 256, group 4
    ("hd256-g8-ctx600", dict(HD256, embed_dim=2048, n_heads=8), None, None, 600, False),   # general pair
    ("hd64-g8-ctx2000", dict(MINI, n_kv_heads=1), None, None, 2000, False),     # group 8
    ("hd32-g2-ctx700", dict(MINI, n_heads=16, n_kv_heads=8), None, None, 700, False),      # hd 32: general pair
]


@pytest.mark.parametrize("name,cfg,n_layers,vocab,ctx_len,kv_f16", LONG_CASES, ids=[c[0] for c in LONG_CASES])
def test_long_cached_context(ggc, orc, ctx, name, cfg, n_layers, vocab, ctx_len, kv_f16):
    hp, m, o = model_pair(ggc, orc, ctx, cfg, n_layers=n_layers, vocab=vocab, max_ctx=ctx_len + 8, seed=21,
                          kv_f16=kv_f16)
    kvd = m.kv_dim
    rng = np.random.default_rng(2)
    for l in range(hp["n_layers"]):
        k = rng.normal(size=(ctx_len, kvd)).astype(np.float32)
        v = rng.normal(size=(ctx_len, kvd)).astype(np.float32)
        m.cache_append(l, k, v)
        o.cache_append(l, k, v)
    kk, vv = m.cache_read(hp["n_layers"] - 1)
    if kv_f16:
        assert np.array_equal(kk, k.astype(np.float16).astype(np.float32).reshape(-1))
    else:
        assert np.array_equal(kk, k.reshape(-1)) and np.array_equal(vv, v.reshape(-1))
    got = m.forward([7], [ctx_len])
    want = o.forward([7], [ctx_len])
    assert np.all(np.isfinite(got))
    assert rel_l2(got, want) <= (1e-2 if kv_f16 else REL_L2), rel_l2(got, want)
    if not kv_f16:   # the device loop past the planted context
        assert m.generate_greedy([11], 4, start_pos=ctx_len + 1) == o.generate_greedy([11], 4, start_pos=ctx_len + 1)
        assert m.cache_len() == o.cache_len() == ctx_len + 6


def test_positions_mask_by_absolute_position(ggc, orc, ctx):   # llama.rs:523-529
    """Re-running positions 0.. on a filled cache masks later cache rows (s > pos)."""
    hp, m, o = model_pair(ggc, orc, ctx, MINI, seed=8)
    m.forward([1, 2, 3], [0, 1, 2]); o.forward([1, 2, 3], [0, 1, 2])
    got = m.forward([4, 5], [0, 1])
    want = o.forward([4, 5], [0, 1])
    assert rel_l2(got, want) <= REL_L2
    assert m.cache_len() == o.cache_len() == 5


def test_errors(ggc, ctx):
    hp, ts = synth.make_model(MINI, seed=2)
    m = ggc.LlamaModel(hp, ts, max_ctx=8, ctx=ctx)
    with pytest.raises(ggc.InferenceError):          # llama.rs:277-280 empty input
        m.forward([], [])
    with pytest.raises(ggc.InferenceError):          # llama.rs:374-379 embed out of bounds
        m.forward([hp["vocab_size"] + 5], [0])
    m.reset_cache()
    with pytest.raises(ggc.KvCacheOverflow):          # capacity of the HBM cache
        m.forward(list(range(9)), list(range(9)))
    # the model stays usable after an error
    m.reset_cache()
    assert np.all(np.isfinite(m.forward([1, 2], [0, 1])))


def test_nan_guard(ggc, ctx):   # llama.rs:300-307: NaN after attention -> InferenceError
    hp, ts = synth.make_model(dict(MINI, weights=0, qkv_bias=False), seed=2)
    wo = ts[3 + 7]
    bad = wo["raw"].view(np.float32).copy()
    bad[:] = np.nan
    ts[3 + 7] = dict(wo, raw=bad.view(np.uint8))
    m = ggc.LlamaModel(hp, ts, max_ctx=8, ctx=ctx)
    with pytest.raises(ggc.InferenceError, match="NaN after layer 0 attention"):
        m.forward([1], [0])


def test_missing_tensor(ggc, ctx):   # llama.rs:621-632 MissingTensor
    hp, ts = synth.make_model(MINI, seed=2)
    ts[3 + 1] = None
    with pytest.raises(ggc.MissingTensor):
        ggc.LlamaModel(hp, ts, max_ctx=8, ctx=ctx)


def test_kv_f16_close(ggc, orc, ctx):
    """f16 KV cache (the Llama-3 workload's option): close to the f32 reference."""
    hp, m, o = model_pair(ggc, orc, ctx, MINI, seed=12, kv_f16=True)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    got = m.forward(prompt, list(range(8)))
    want = o.forward(prompt, list(range(8)))
    assert rel_l2(got, want) <= 1e-2


def test_determinism(ggc, ctx):
    hp, ts = synth.make_model(MINI, seed=13)
    a = ggc.LlamaModel(hp, ts, max_ctx=64, ctx=ctx)
    b = ggc.LlamaModel(hp, ts, max_ctx=64, ctx=ctx)
    la = a.forward([1, 2, 3], [0, 1, 2])
    lb = b.forward([1, 2, 3], [0, 1, 2])
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))


# ---- decode GEMV chains (GGC_DECODE_CHAIN=1: one persistent launch per run of GEMVs) ----
CHAIN_CASES = [
    ("mini-q4_k_m", MINI, None, None),
    ("qwen2-0.5b-q8_0-2layers", "qwen2-0.5b-q8_0", 2, None),
    ("llama2-7b-q4_k_m-2layers", "llama2-7b-q4_k_m", 2, None),   # Q4_K and Q6_K ops in one chain
    ("llama3-8b-q4_0-1layer", "llama3-8b-q4_0", 1, 32000),
]


@pytest.mark.parametrize("name,cfg,n_layers,vocab", CHAIN_CASES, ids=[c[0] for c in CHAIN_CASES])
def test_chain_decode_matches_oracle(ggc, orc, ctx, monkeypatch, name, cfg, n_layers, vocab):
    monkeypatch.setenv("GGC_DECODE_CHAIN", "1")
    hp, m, o = model_pair(ggc, orc, ctx, cfg, n_layers, vocab)
    prompt = np.random.default_rng(9).integers(0, hp["vocab_size"], size=6).astype(np.uint32)
    got = m.forward(prompt, np.arange(6, dtype=np.int64))
    want = o.forward(prompt, np.arange(6, dtype=np.int64))
    assert rel_l2(got, want) <= REL_L2, rel_l2(got, want)
    ids = m.decode(32)
    want_ids, lg, pos = [], want, 6
    for _ in range(32):
        want_ids.append(orc.greedy(lg))
        lg = o.forward([want_ids[-1]], [pos])
        pos += 1
    assert ids == want_ids
    m.close()


# ---- models built back to back on one context ----
# A model's buffers are zero-filled and its norm weights and biases uploaded on the
# context stream, which does not synchronise with the legacy default stream: a fill
# issued there could land after an upload and zero the weights of whichever model
# reused the memory of the one before (seen as a layer's RMSNorm weight reading 0,
# the layer's q/k/v then equal to their biases).  Several models of one shape, each
# closed before the next is built, must all match the oracle on a multi-position
# prompt (one position would not notice: its attention weight is 1).
BACK_TO_BACK = [dict(MINI, ffn_dim=2048), dict(MINI, embed_dim=1024, n_heads=16, n_kv_heads=4)]


@pytest.mark.parametrize("cfg", BACK_TO_BACK, ids=["ffn2048", "dim1024"])
def test_models_built_back_to_back_keep_their_weights(ggc, orc, ctx, cfg):
    hp, ts = synth.make_model(cfg, seed=0)
    prompt = np.random.default_rng(9).integers(0, hp["vocab_size"], size=6).astype(np.uint32)
    pos = np.arange(6, dtype=np.int64)
    want = orc.Model(hp, ts).forward(prompt, pos)
    for rep in range(6):
        m = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
        got = m.forward(prompt, pos)
        m.close()
        assert rel_l2(got, want) <= REL_L2, (rep, rel_l2(got, want))


def test_device_repack_model_matches_host_repack(ggc, ctx, monkeypatch):
    """A model whose weights were split on the GPU at load (the default) and one split
    on the host (GGC_REPACK=host) give bit-identical logits: the q/k RoPE row order and
    the fused up/gate rows go through the device repack too."""
    hp, ts = synth.make_model(MINI, seed=5)
    toks, pos = [3, 17, 250, 9, 41], [0, 1, 2, 3, 4]
    monkeypatch.delenv("GGC_REPACK", raising=False)
    dev = ggc.LlamaModel(hp, ts, max_ctx=64, ctx=ctx).forward(toks, pos)
    monkeypatch.setenv("GGC_REPACK", "host")
    host = ggc.LlamaModel(hp, ts, max_ctx=64, ctx=ctx).forward(toks, pos)
    assert np.array_equal(np.asarray(dev).view(np.uint32), np.asarray(host).view(np.uint32))

"""The batched prompt path (prefill: tcgen05 products + batched attention) against
the oracle, and against the token-by-token decode path.

A prompt longer than 64 tokens runs its prefix through the batched kernels and
its last token through the decode step: logits within 1e-4 relative L2 of the
oracle, K/V cache rows within 1e-4, greedy ids identical, and the same NaN /
embedding / position errors as the reference.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import synth

REL_L2 = 1e-4
MINI = dict(vocab_size=1000, embed_dim=512, n_heads=8, n_kv_heads=2, ffn_dim=1024, n_layers=2, rope_freq_base=1e4,
            qkv_bias=True, weights="q4_k_m")


def rel_l2(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


CASES = [
    ("mini-q4_k_m", MINI, None, None),
    ("qwen2-0.5b-q8_0-2layers", "qwen2-0.5b-q8_0", 2, None),
    ("llama2-7b-q4_k_m-2layers", "llama2-7b-q4_k_m", 2, None),
    ("llama3-8b-q4_0-1layer", "llama3-8b-q4_0", 1, 32000),
]


@pytest.mark.parametrize("name,cfg,n_layers,vocab", CASES, ids=[c[0] for c in CASES])
def test_prefill_matches_oracle(ggc, orc, ctx, name, cfg, n_layers, vocab):
    hp, ts = synth.make_model(cfg, n_layers=n_layers, seed=0, vocab_size=vocab)
    m = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
    o = orc.Model(hp, ts)
    prompt = np.random.default_rng(7).integers(0, hp["vocab_size"], size=100).astype(np.uint32)
    pos = np.arange(100, dtype=np.int64)
    got = m.forward(prompt, pos)
    want = o.forward(prompt, pos)
    assert rel_l2(got, want) <= REL_L2, rel_l2(got, want)
    assert m.cache_len() == 100
    for layer in (0, hp["n_layers"] - 1):
        k, v = m.cache_read(layer)
        ko, vo = o.cache_read(layer)
        assert rel_l2(k, ko) <= REL_L2 and rel_l2(v, vo) <= REL_L2, layer
    # decode continues on the batched cache
    got = m.forward([int(prompt[3])], [100])
    want = o.forward([int(prompt[3])], [100])
    assert rel_l2(got, want) <= REL_L2


@pytest.mark.parametrize("name,cfg,n_layers,vocab", CASES[:3], ids=[c[0] for c in CASES[:3]])
def test_prefill_greedy_ids_match_oracle(ggc, orc, ctx, name, cfg, n_layers, vocab):
    hp, ts = synth.make_model(cfg, n_layers=n_layers, seed=1, vocab_size=vocab)
    m = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
    o = orc.Model(hp, ts)
    prompt = np.random.default_rng(8).integers(0, hp["vocab_size"], size=90).astype(np.uint32)
    got = m.generate_greedy(prompt, 32)
    want = o.generate_greedy(prompt, 32)
    assert got == want
    assert m.cache_len() == o.cache_len() == 90 + 32


def test_prefill_two_passes_and_cache_base(ggc, orc, ctx):
    """600 tokens (two passes of 512) after 10 tokens already cached, positions offset."""
    hp, ts = synth.make_model(MINI, seed=2)
    m = ggc.LlamaModel(hp, ts, max_ctx=1024, ctx=ctx)
    o = orc.Model(hp, ts)
    rng = np.random.default_rng(9)
    head = rng.integers(0, hp["vocab_size"], size=10).astype(np.uint32)
    body = rng.integers(0, hp["vocab_size"], size=600).astype(np.uint32)
    for model in (m, o):
        model.forward(head, np.arange(10, dtype=np.int64))
    got = m.forward(body, np.arange(10, 610, dtype=np.int64))
    want = o.forward(body, np.arange(10, 610, dtype=np.int64))
    assert rel_l2(got, want) <= REL_L2, rel_l2(got, want)
    k, v = m.cache_read(1)
    ko, vo = o.cache_read(1)
    assert rel_l2(k, ko) <= REL_L2 and rel_l2(v, vo) <= REL_L2


def test_prefill_equals_token_by_token(ggc, ctx, monkeypatch):
    hp, ts = synth.make_model(MINI, seed=3)
    a = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
    monkeypatch.setenv("GGC_PREFILL", "0")
    b = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
    prompt = np.random.default_rng(10).integers(0, hp["vocab_size"], size=80).astype(np.uint32)
    pos = np.arange(80, dtype=np.int64)
    la, lb = a.forward(prompt, pos), b.forward(prompt, pos)
    assert rel_l2(la, lb) <= REL_L2
    assert a.generate_greedy([5], 16, start_pos=80) == b.generate_greedy([5], 16, start_pos=80)


def test_prefill_f16_cache_equals_token_by_token(ggc, ctx, monkeypatch):
    """The batched attention reading an f16 cache (a prompt on top of cached rows)
    against the token-by-token path over its own f16 cache.  The two paths round
    K/V to f16 from slightly different f32 products (tensor-core vs integer GEMV),
    so a few cache entries differ by one f16 ulp (~1e-3 relative): 5e-3 bound."""
    hp, ts = synth.make_model(MINI, seed=4)
    a = ggc.LlamaModel(hp, ts, max_ctx=256, kv_f16=True, ctx=ctx)
    monkeypatch.setenv("GGC_PREFILL", "0")
    b = ggc.LlamaModel(hp, ts, max_ctx=256, kv_f16=True, ctx=ctx)
    rng = np.random.default_rng(11)
    head = rng.integers(0, hp["vocab_size"], size=5).astype(np.uint32)
    body = rng.integers(0, hp["vocab_size"], size=90).astype(np.uint32)
    for model in (a, b):
        model.forward(head, np.arange(5, dtype=np.int64))
    la = a.forward(body, np.arange(5, 95, dtype=np.int64))
    lb = b.forward(body, np.arange(5, 95, dtype=np.int64))
    assert rel_l2(la, lb) <= 5e-3, rel_l2(la, lb)
    assert a.cache_len() == b.cache_len() == 95


def test_prefill_errors(ggc, ctx):
    hp, ts = synth.make_model(dict(MINI, weights=0, qkv_bias=False), seed=4)
    m = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
    prompt = np.arange(70, dtype=np.uint32)
    bad = prompt.copy()
    bad[30] = hp["vocab_size"] + 5                      # embed out of bounds inside the batched prefix
    with pytest.raises(ggc.InferenceError, match="embed"):
        m.forward(bad, np.arange(70, dtype=np.int64))
    m.reset_cache()
    with pytest.raises(ggc.InferenceError, match="position"):
        m.forward(prompt, np.arange(70, dtype=np.int64) - 1)
    m.reset_cache()
    assert np.all(np.isfinite(m.forward(prompt, np.arange(70, dtype=np.int64))))   # usable after errors
    wo = ts[3 + 7]
    w = wo["raw"].view(np.float32).copy()
    w[:] = np.nan
    ts[3 + 7] = dict(wo, raw=w.view(np.uint8))
    m2 = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
    with pytest.raises(ggc.InferenceError, match="NaN after layer 0 attention"):
        m2.forward(prompt, np.arange(70, dtype=np.int64))

"""Tensor-parallel decode on 2 GPUs (one process per GPU, NCCL) against the oracle.

Every rank makes the same calls; the model shards q/k/v/up/gate rows and
attn_output/ffn_down columns (ggc_tp_plan) and all-reduces the hidden state
after each of the two.  Logits within 1e-4 relative L2 of the oracle, identical
on every rank, and greedy ids identical for 32 tokens.  Skipped with fewer
than two GPUs.  Both all-reduce paths run: the fused one over peer memory
(default) and NCCL (GGC_TP_ALLREDUCE=nccl).  GGC_TEST_TP_WORLD sets the rank
count (default 2); cases whose heads it does not divide are skipped.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import synth

REL_L2 = 1e-4
WORLD = int(os.environ.get("GGC_TEST_TP_WORLD", "2"))

MINI = dict(vocab_size=1000, embed_dim=512, n_heads=8, n_kv_heads=2, ffn_dim=1024, n_layers=2, rope_freq_base=1e4,
            qkv_bias=True, weights="q4_k_m")
CASES = [
    ("mini-q4_k_m", MINI, None, None),
    ("mini-f32-bias", dict(MINI, weights=0), None, None),
    ("llama2-7b-q4_k_m-2layers", "llama2-7b-q4_k_m", 2, None),     # ffn 43 super-blocks: 22 + 21
    ("llama3-8b-q4_0-1layer", "llama3-8b-q4_0", 1, 32000),
]


def rel_l2(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def _need_gpus():
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")


def _worker(rank, world, nid, jobs, q):
    """One rank: one context, then every job (same calls on every rank), each
    with its all-reduce path (GGC_TP_ALLREDUCE is read when a model is made).
    A collective that never completes ends at the library's host deadline."""
    import time
    os.environ.setdefault("GGC_NCCL_TIMEOUT_MS", "120000")
    out = {}
    try:
        import torch  # noqa: F401  -- loads the NCCL the parent's unique id came from
        import gguf_cuda as ggc
        ctx = ggc.Context(device=rank, rank=rank, world=world, nccl_id=nid)
        log = os.environ.get("GGC_TEST_TP_LOG")
        for key, job, allreduce in jobs:
            if log:   # progress per rank, so a stall names its job
                with open(f"{log}.rank{rank}", "a") as f:
                    f.write(f"{time.time():.1f} start {key}\n")
            if allreduce == "nccl":
                os.environ["GGC_TP_ALLREDUCE"] = "nccl"
            else:
                os.environ.pop("GGC_TP_ALLREDUCE", None)
            try:
                out[key] = job(ggc, ctx)
            except Exception as e:   # reported to the parent (as text: the library's errors do not pickle)
                out[key] = RuntimeError(f"rank {rank}: {type(e).__name__}: {e}")
            if log:
                with open(f"{log}.rank{rank}", "a") as f:
                    f.write(f"{time.time():.1f} done {key}\n")
    except Exception as e:
        out = RuntimeError(f"rank {rank}: {type(e).__name__}: {e}")
    q.put((rank, out))


def run_ranks(jobs, timeout=1200):
    """Spawns WORLD ranks once and runs `jobs` [(key, job, allreduce)] in each;
    returns {key: [result of rank 0, rank 1, ...]}."""
    import multiprocessing as mp
    import torch  # noqa: F401  -- the library binds the NCCL already loaded (PyTorch's)
    import gguf_cuda as ggc
    nid = ggc.Context.nccl_unique_id()
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    procs = [mctx.Process(target=_worker, args=(r, WORLD, nid, jobs, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=timeout) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(WORLD):
        if isinstance(res[r], Exception):
            raise res[r]
    return {key: [res[r][key] for r in range(WORLD)] for key, _, _ in jobs}


class PromptJob:
    def __init__(self, cfg, n_layers, vocab, seed=0):
        self.cfg, self.n_layers, self.vocab, self.seed = cfg, n_layers, vocab, seed

    def __call__(self, ggc, ctx):
        hp, ts = synth.make_model(self.cfg, n_layers=self.n_layers, seed=self.seed, vocab_size=self.vocab)
        m = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
        prompt = np.random.default_rng(5).integers(0, hp["vocab_size"], size=8).astype(np.uint32)
        logits = m.forward(prompt, np.arange(8, dtype=np.int64))
        k, v = m.cache_read(0)
        step = m.forward([int(prompt[0])], [8])
        m.reset_cache()
        ids = m.generate_greedy(np.random.default_rng(9).integers(0, hp["vocab_size"], size=6), 32)
        return dict(logits=logits, k=k, v=v, step=step, ids=ids, cache_len=m.cache_len(), allreduce=m.allreduce)


@pytest.fixture(scope="module")
def tp_results():
    """Every job of this module in one spawn of WORLD ranks."""
    _need_gpus()
    jobs = []
    for allreduce in ("peer", "nccl"):
        for name, cfg, n_layers, vocab in CASES:
            hp = synth.hparams(cfg if isinstance(cfg, dict) else synth.CONFIGS[cfg], n_layers)
            if hp["n_kv_heads"] % WORLD == 0:
                jobs.append((("prompt", name, allreduce), PromptJob(cfg, n_layers, vocab), allreduce))
        if 2 % WORLD == 0:
            jobs.append((("nan", allreduce), NanJob(), allreduce))
    jobs.append((("long",), LongPromptJob(), "peer"))
    return run_ranks(jobs)


@pytest.mark.parametrize("allreduce", ["peer", "nccl"])
@pytest.mark.parametrize("name,cfg,n_layers,vocab", CASES, ids=[c[0] for c in CASES])
def test_tp_matches_oracle(ggc, orc, tp_results, name, cfg, n_layers, vocab, allreduce):
    hp, ts = synth.make_model(cfg, n_layers=n_layers, seed=0, vocab_size=vocab)
    if hp["n_kv_heads"] % WORLD:
        pytest.skip(f"{WORLD} ranks do not divide {hp['n_kv_heads']} kv heads")
    res = tp_results[("prompt", name, allreduce)]
    for r in res:
        if isinstance(r, Exception):
            raise r
    o = orc.Model(hp, ts)
    prompt = np.random.default_rng(5).integers(0, hp["vocab_size"], size=8).astype(np.uint32)
    want = o.forward(prompt, np.arange(8, dtype=np.int64))
    ko, vo = o.cache_read(0)
    want_step = o.forward([int(prompt[0])], [8])
    o.reset_cache()
    want_ids = o.generate_greedy(np.random.default_rng(9).integers(0, hp["vocab_size"], size=6).astype(np.uint32), 32)
    hd = hp["embed_dim"] // hp["n_heads"]
    kvw = hp["n_kv_heads"] * hd
    for rank, r in enumerate(res):
        assert r["allreduce"] == allreduce
        assert rel_l2(r["logits"], want) <= REL_L2, (rank, rel_l2(r["logits"], want))
        assert rel_l2(r["step"], want_step) <= REL_L2
        assert r["ids"] == want_ids
        assert r["cache_len"] == 6 + 32
        # the rank's cache holds its own kv heads
        p = ggc.tp_plan(hp, ts[3 + 7]["dtype"], ts[3 + 11]["dtype"], rank, WORLD)
        h0, nh = p["kv_heads"]
        sl = slice(h0 * hd, (h0 + nh) * hd)
        assert rel_l2(r["k"], ko.reshape(-1, kvw)[:, sl].ravel()) <= REL_L2
        assert rel_l2(r["v"], vo.reshape(-1, kvw)[:, sl].ravel()) <= REL_L2
    # replicated lm_head over the same reduced hidden state: identical on every rank
    for r in res[1:]:
        assert np.array_equal(res[0]["logits"], r["logits"])


class LongPromptJob:
    """An 80-token prompt: its prefix runs through the batched prefill (NCCL
    all-reduce of the partial products), the last token and the decode through
    the step graph."""

    def __call__(self, ggc, ctx):
        hp, ts = synth.make_model("llama2-7b-q4_k_m", n_layers=2, seed=3)
        m = ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx)
        prompt = np.random.default_rng(11).integers(0, hp["vocab_size"], size=80).astype(np.uint32)
        logits = m.forward(prompt, np.arange(80, dtype=np.int64))
        ids = m.decode(16)
        return dict(logits=logits, ids=ids)


def test_tp_long_prompt_prefill_matches_oracle(ggc, orc, tp_results):
    res = tp_results[("long",)]
    for r in res:
        if isinstance(r, Exception):
            raise r
    hp, ts = synth.make_model("llama2-7b-q4_k_m", n_layers=2, seed=3)
    o = orc.Model(hp, ts)
    prompt = np.random.default_rng(11).integers(0, hp["vocab_size"], size=80).astype(np.uint32)
    want = o.forward(prompt, np.arange(80, dtype=np.int64))
    for r in res:
        assert rel_l2(r["logits"], want) <= REL_L2, rel_l2(r["logits"], want)
    assert all(np.array_equal(res[0]["logits"], r["logits"]) for r in res[1:])
    assert all(r["ids"] == res[0]["ids"] for r in res[1:]) and len(res[0]["ids"]) == 16
    assert res[0]["ids"][0] == orc.greedy(want)


class NanJob:
    """NaN planted in the attn_output columns that only the last rank holds."""

    def __call__(self, ggc, ctx):
        hp, ts = synth.make_model(dict(MINI, weights=0, qkv_bias=False), seed=2)
        wo = ts[3 + 7]
        w = wo["raw"].view(np.float32).copy().reshape(hp["embed_dim"], hp["embed_dim"])
        w[:, hp["embed_dim"] - hp["embed_dim"] // WORLD:] = np.nan
        ts[3 + 7] = dict(wo, raw=w.ravel().view(np.uint8))
        m = ggc.LlamaModel(hp, ts, max_ctx=8, ctx=ctx)
        try:
            m.forward([1], [0])
        except ggc.InferenceError as e:
            return str(e)
        return None


@pytest.mark.parametrize("allreduce", ["peer", "nccl"])
def test_tp_nan_guard_same_on_every_rank(ggc, tp_results, allreduce):
    if 2 % WORLD:
        pytest.skip("the planted model has 2 kv heads")
    res = tp_results[("nan", allreduce)]
    for r in res:
        assert isinstance(r, str) and "NaN after layer 0 attention" in r, r


# ---- the fused all-reduce's bounded wait, on one GPU ------------------------------
def test_allreduce_probe_sums_in_rank_order(ggc, ctx):
    rng = np.random.default_rng(3)
    p0 = rng.normal(size=1000).astype(np.float32)
    p1 = rng.normal(size=1000).astype(np.float32)
    got = ggc.allreduce_probe(p0, p1, peer_writes=True, ctx=ctx)
    assert np.array_equal(got, (p0 + p1).astype(np.float32))


def test_allreduce_probe_lost_peer_times_out_and_context_stays_usable(ggc, ctx):
    """The peer's words never arrive: the poll gives up (a bounded wait, no GPU
    fault or hang), the call returns DeviceTimeout, and the context still works."""
    import time
    p = np.ones(64, np.float32)
    t0 = time.perf_counter()
    with pytest.raises(ggc.DeviceTimeout, match="bounded poll"):
        ggc.allreduce_probe(p, p, peer_writes=False, ctx=ctx)
    assert time.perf_counter() - t0 < 30
    assert np.array_equal(ggc.allreduce_probe(p, 2 * p, peer_writes=True, ctx=ctx), 3 * p)

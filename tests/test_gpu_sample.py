"""Device sampling (ggc_sample / ggc_model_sample) against the oracle's
restatement of Sampler::sample (sampler.rs:86-186), both given the same uniform
draw u.

The device sums the softmax denominator in parallel, so its probabilities can
differ from the reference's serial sum by a few ulp; a pick is compared only
when the oracle gives the same token for u - 1e-5, u and u + 1e-5 (u is not on
a cumulative boundary), and at least 95 % of the draws must be comparable.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import synth

MINI = dict(vocab_size=1000, embed_dim=512, n_heads=8, n_kv_heads=2, ffn_dim=1024, n_layers=2, rope_freq_base=1e4,
            qkv_bias=True, weights="q4_k_m")

CFGS = [
    dict(),                                                          # reference defaults: T 1, top_k 40, top_p 0.95
    dict(temperature=0.7, top_k=1),
    dict(temperature=1.3, top_k=1024, top_p=0.5, min_p=0.05, repeat_penalty=1.3),
    dict(temperature=0.0, repeat_penalty=1.5),                        # greedy on the penalised logits
    dict(temperature=1.0, top_k=200, top_p=1.0, min_p=0.0, repeat_penalty=1.0),
    dict(temperature=2.0, top_k=7, top_p=0.8, min_p=0.3),
]


def compare(draw, orc, logits, cfg, seen, n_draws=150, seed=0):
    us = np.random.default_rng(seed).random(n_draws).astype(np.float32)
    checked, distinct = 0, set()
    for u in us:
        u = float(u)
        want = orc.sample(logits, cfg, seen, u)
        lo, hi = max(u - 1e-5, 0.0), min(u + 1e-5, 0.99999994)
        if orc.sample(logits, cfg, seen, lo) != want or orc.sample(logits, cfg, seen, hi) != want:
            continue   # u on a boundary: a few-ulp difference in the sum may move the pick
        assert draw(cfg, seen, u) == want, (cfg, u)
        checked += 1
        distinct.add(want)
    assert checked >= 0.95 * n_draws
    return distinct


@pytest.mark.parametrize("vocab", [32000, 151936])
@pytest.mark.parametrize("cfg", CFGS, ids=[f"cfg{i}" for i in range(len(CFGS))])
def test_sample_matches_oracle(ggc, orc, ctx, cfg, vocab):
    rng = np.random.default_rng(vocab)
    logits = rng.normal(0.0, 2.5, vocab).astype(np.float32)
    logits[rng.integers(0, vocab, 64)] = 9.0        # exact ties among the top: index order breaks them
    seen = [int(i) for i in np.argsort(logits)[-6:]] + [17, 17, vocab - 1, vocab + 5]   # + a duplicate, + out of range
    got = compare(lambda c, s, u: ggc.sample(logits, c, s, u, ctx=ctx), orc, logits, cfg, seen)
    if cfg.get("temperature", 1.0) > 0 and cfg.get("top_k", 40) > 1:
        assert len(got) > 1                          # the draws really spread over candidates


def test_sample_device_logits_and_whole_small_vocab(ggc, orc, ctx):
    """Device logits; vocab <= 1024 without top-k: the candidates stay in index
    order (no sort) when top_p is 1 and are sorted when top_p < 1."""
    import torch
    logits = np.random.default_rng(3).normal(0.0, 1.5, 1000).astype(np.float32)
    dl = torch.from_numpy(logits).cuda()
    torch.cuda.synchronize()
    for cfg in (dict(top_k=0, top_p=1.0), dict(top_k=0, top_p=0.9, min_p=0.01), dict(top_k=1000, top_p=1.0)):
        compare(lambda c, s, u: ggc.sample(dl, c, s, u, ctx=ctx), orc, logits, cfg, [3, 4], seed=1)


def test_model_sample_uses_the_last_logits(ggc, orc, ctx):
    hp, ts = synth.make_model(MINI, seed=7)
    m = ggc.LlamaModel(hp, ts, max_ctx=64, ctx=ctx)
    logits = m.forward([1, 2], [0, 1])
    assert m.sample(dict(temperature=0.0, repeat_penalty=1.0)) == m.last_argmax
    hot = dict(temperature=40.0, top_k=50, top_p=0.9)   # flatten the random-init logits
    compare(lambda c, s, u: m.sample(c, s, u), orc, logits, hot, [m.last_argmax], n_draws=60)
    ids = m.decode(3)                                   # decoding continues: sampling only reads the logits
    assert len(ids) == 3


def test_sample_rejects(ggc, ctx):
    logits = np.zeros(32000, np.float32)
    with pytest.raises(ggc.InvalidArgument):
        ggc.sample(logits, dict(), u=1.0, ctx=ctx)                    # u outside [0, 1)
    with pytest.raises(ggc.InvalidArgument, match="top_k"):
        ggc.sample(logits, dict(top_k=0), ctx=ctx)                    # 32000 candidates: beyond the device limit
    with pytest.raises(ggc.InvalidArgument, match="top_k"):
        ggc.sample(logits, dict(top_k=2000), ctx=ctx)
    logits[5] = np.nan
    with pytest.raises(ggc.InferenceError, match="NaN"):
        ggc.sample(logits, dict(), ctx=ctx)
    assert ggc.sample(np.arange(10, dtype=np.float32), dict(temperature=0.0), ctx=ctx) == 9   # still usable

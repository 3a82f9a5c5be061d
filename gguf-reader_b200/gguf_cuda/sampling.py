"""Sampler::sample on the host, for the configurations the device kernel does not
take (more than 1024 candidates after top-k: top_k = 0, or top_k > 1024, over a
vocabulary of more than 1024 entries).

Restates src/infer/sampler.rs:86-186 step by step in f32: repeat penalty on the
seen ids, temperature (<= 1e-6: greedy, last maximum), softmax with a serial f32
sum, top-k by a stable descending sort, top-p (stable sort, serial cumulative
sum, cut at the first index reaching total * top_p), min-p, then the pick with
the caller's uniform draw `u` (the reference's `rng.gen_range(0.0..1.0)`).  With
top_k = 0 and top_p >= 1 the candidates stay in index order, as there.
Host logic, like the reference's: it reads one logits vector per sampled token.
"""
from __future__ import annotations

import numpy as np

DEVICE_MAX_CANDIDATES = 1024


def device_can_sample(cfg: dict, vocab: int) -> bool:
    """Whether ggc_sample takes this configuration (at most 1024 candidates after top-k)."""
    if cfg.get("temperature", 1.0) <= 1e-6:
        return True
    k = int(cfg.get("top_k", 40))
    return vocab <= DEVICE_MAX_CANDIDATES or 0 < k <= DEVICE_MAX_CANDIDATES


def _serial_sum(v: np.ndarray) -> np.float32:
    return np.add.accumulate(v, dtype=np.float32)[-1] if v.size else np.float32(0)


def _last_argmax(v: np.ndarray) -> int:
    """max_by over partial_cmp: the last of equal maxima (sampler.rs:117-122)."""
    return int(v.size - 1 - np.argmax(v[::-1]))


def sample_host(logits, cfg: dict, seen=(), u: float = 0.5) -> int:
    lg = np.asarray(logits, dtype=np.float32)
    vocab = lg.size
    if vocab == 0:
        raise ValueError("empty logits")
    if np.isnan(lg).any():
        raise ValueError("NaN logits")   # the reference panics in partial_cmp().unwrap()
    f32 = np.float32
    pen = f32(cfg.get("repeat_penalty", 1.1))
    v = lg.copy()
    if pen != f32(1.0):
        for i in set(int(t) for t in seen):
            if 0 <= i < vocab:
                v[i] = v[i] / pen if v[i] > 0 else v[i] * pen
    temp = f32(cfg.get("temperature", 1.0))
    if not temp > f32(1e-6):
        return _last_argmax(v)
    scaled = (v / temp).astype(np.float32)
    mx = scaled.max()
    exps = np.exp((scaled - mx).astype(np.float32)).astype(np.float32)
    probs = (exps / _serial_sum(exps)).astype(np.float32)
    idx = np.arange(vocab)
    top_k = int(cfg.get("top_k", 40))
    if 0 < top_k < vocab:
        order = np.argsort(-probs, kind="stable")[:top_k]
        idx = order
    cp = probs[idx]
    top_p = f32(cfg.get("top_p", 0.95))
    if top_p < f32(1.0):
        o = np.argsort(-cp, kind="stable")
        idx, cp = idx[o], cp[o]
        thr = _serial_sum(cp) * top_p
        cum = np.add.accumulate(cp, dtype=np.float32)
        hit = np.nonzero(cum >= thr)[0]
        cut = int(hit[0]) + 1 if hit.size else cp.size
        idx, cp = idx[:cut], cp[:cut]
    min_p = f32(cfg.get("min_p", 0.0))
    if min_p > f32(0.0):
        thr = (cp.max() if cp.size else f32(0)) * min_p
        keep = cp >= thr
        idx, cp = idx[keep], cp[keep]
    if idx.size == 0:
        return _last_argmax(scaled)
    r = f32(u) * _serial_sum(cp)
    for i, p in zip(idx, cp):
        r = f32(r - p)
        if r <= f32(0.0):
            return int(i)
    return int(idx[-1])

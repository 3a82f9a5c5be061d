"""Seeded synthetic GGUF tensors and model shapes for tests and benchmarks.

No real checkpoints are available offline; every weight is generated from a seed
with the value distributions of the workloads:
  * legacy 32-element blocks: fp16 d (and m) ~ U[1e-3, 1e-2], quant bits uniform;
  * K-quant super-blocks: fp16 d/dmin ~ U[1e-4, 1e-3], scale bytes and bits uniform;
    Q8_K: d drawn as f32 ~ U[1e-4, 1e-3];
  * F16/BF16/F32: N(0, 0.02);
  * Q8_0 "quantised" weights: N(0, 0.02) floats quantised with the standard Q8_0
    rule (d = amax/127 stored as fp16, q = round-half-away(x/d)).
The reference has no quantiser, so this generator defines those bytes.
Each tensor draws from its own seed (base seed, role, layer), so a model with
fewer layers holds exactly the first layers of the full model.
"""
from __future__ import annotations

import numpy as np

from ._lib import (BF16, BLOCK, F16, F32, Q2_K, Q3_K_L, Q3_K_M, Q3_K_S, Q4_0, Q4_1, Q4_K, Q5_0, Q5_1, Q5_K, Q6_K,
                   Q8_0, Q8_K)

# per-format byte offsets of the fp16 scale fields: (offset, kind) kind "d" or "m"
_SCALE_FIELDS = {
    Q4_0: [0], Q4_1: [0, 2], Q5_0: [0], Q5_1: [0, 2], Q8_0: [0],
    Q2_K: [80, 82], Q3_K_S: [108], Q3_K_L: [108], Q3_K_M: [112],
    Q4_K: [0, 2], Q5_K: [0, 2], Q6_K: [208],
}
_LEGACY = {Q4_0, Q4_1, Q5_0, Q5_1, Q8_0}

TENSOR_ROLES = ["token_embd", "output_norm", "output"]
LAYER_ROLES = ["attn_norm", "attn_q", "attn_q.bias", "attn_k", "attn_k.bias", "attn_v", "attn_v.bias",
               "attn_output", "ffn_norm", "ffn_up", "ffn_gate", "ffn_down"]


def rng_for(seed: int, *key: int) -> np.random.Generator:
    return np.random.default_rng([int(seed)] + [int(k) for k in key])


def random_blocks(dtype: int, n_elements: int, rng: np.random.Generator) -> np.ndarray:
    """Raw GGUF bytes of `n_elements` elements of `dtype` (seeded)."""
    bs, bb = BLOCK[dtype]
    assert n_elements % bs == 0, (n_elements, bs)
    nb = n_elements // bs
    if dtype in (F32, F16, BF16):
        v = rng.normal(0.0, 0.02, size=n_elements).astype(np.float32)
        if dtype == F32:
            return v.view(np.uint8).copy()
        if dtype == F16:
            return v.astype(np.float16).view(np.uint8).copy()
        b = v.view(np.uint32).astype(np.uint64)
        b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)   # round to nearest even
        return b.view(np.uint8).copy()
    raw = np.frombuffer(rng.bytes(nb * bb), dtype=np.uint8).copy().reshape(nb, bb)
    if dtype == Q8_K:
        d = rng.uniform(1e-4, 1e-3, size=nb).astype(np.float32)
        raw[:, 0:4] = d.view(np.uint8).reshape(nb, 4)
    else:
        lo, hi = (1e-3, 1e-2) if dtype in _LEGACY else (1e-4, 1e-3)
        for off in _SCALE_FIELDS[dtype]:
            d = rng.uniform(lo, hi, size=nb).astype(np.float16)
            raw[:, off:off + 2] = d.view(np.uint8).reshape(nb, 2)
    return raw.reshape(-1)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Standard Q8_0 quantisation of f32 values (blocks of 32)."""
    x = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / 127.0).astype(np.float32)
    inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1.0), 0.0).astype(np.float32)
    v = x * inv[:, None]
    q = np.clip(np.trunc(v + np.copysign(0.5, v)), -128, 127).astype(np.int8)
    out = np.empty((x.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def tensor(raw: np.ndarray, dtype: int, n: int, name: str = "") -> dict:
    return {"raw": raw, "dtype": dtype, "n_elements": n, "name": name}


# ---- model shapes ---------------------------------------------------------------
CONFIGS = {
    # Qwen2-0.5B shape, Q8_0 weights quantised from N(0, 0.02), QKV bias
    "qwen2-0.5b-q8_0": dict(vocab_size=151936, embed_dim=896, n_heads=14, n_kv_heads=2, ffn_dim=4864, n_layers=24,
                            rope_freq_base=1e6, qkv_bias=True, weights="q8_0_normal"),
    # Llama-2-7B shape, Q4_K_M mix (Q6_K for output and for attn_v / ffn_down of even layers)
    "llama2-7b-q4_k_m": dict(vocab_size=32000, embed_dim=4096, n_heads=32, n_kv_heads=32, ffn_dim=11008, n_layers=32,
                             rope_freq_base=1e4, qkv_bias=False, weights="q4_k_m"),
    # Llama-3-8B shape (GQA 32/8), Q4_0 or Q8_0 blocks
    "llama3-8b-q4_0": dict(vocab_size=128256, embed_dim=4096, n_heads=32, n_kv_heads=8, ffn_dim=14336, n_layers=32,
                           rope_freq_base=5e5, qkv_bias=False, weights=Q4_0),
    "llama3-8b-q8_0": dict(vocab_size=128256, embed_dim=4096, n_heads=32, n_kv_heads=8, ffn_dim=14336, n_layers=32,
                           rope_freq_base=5e5, qkv_bias=False, weights=Q8_0),
}


def hparams(cfg: dict, n_layers: int | None = None) -> dict:
    hp = {k: cfg[k] for k in ("vocab_size", "embed_dim", "n_heads", "n_kv_heads", "ffn_dim", "n_layers",
                              "rope_freq_base")}
    if n_layers is not None:
        hp["n_layers"] = n_layers
    return hp


def _weight_dtype(cfg: dict, role: str, layer: int) -> int:
    w = cfg["weights"]
    if w == "q4_k_m":
        if role == "output":
            return Q6_K
        if role in ("attn_v", "ffn_down") and layer % 2 == 0:
            return Q6_K
        return Q4_K
    if w == "q8_0_normal":
        return Q8_0
    return int(w)


def make_model(cfg: dict | str, n_layers: int | None = None, seed: int = 0, vocab_size: int | None = None) -> tuple:
    """(hparams, tensors in role order) of a seeded synthetic model."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    cfg = dict(cfg)
    if vocab_size is not None:
        cfg["vocab_size"] = vocab_size
    hp = hparams(cfg, n_layers)
    d, f, V = hp["embed_dim"], hp["ffn_dim"], hp["vocab_size"]
    hd = d // hp["n_heads"]
    qd, kvd = hp["n_heads"] * hd, hp["n_kv_heads"] * hd

    def weight(role: str, layer: int, rows: int, cols: int, role_id: int) -> dict:
        dt = _weight_dtype(cfg, role, layer)
        rng = rng_for(seed, role_id, layer)
        if cfg["weights"] == "q8_0_normal":
            raw = quantize_q8_0(rng.normal(0.0, 0.02, size=rows * cols).astype(np.float32))
        else:
            raw = random_blocks(dt, rows * cols, rng)
        return tensor(raw, dt, rows * cols, role)

    def ones(n: int, role: str) -> dict:
        return tensor(np.ones(n, dtype=np.float32).view(np.uint8), F32, n, role)

    def bias(n: int, role_id: int, layer: int, role: str):
        if not cfg.get("qkv_bias"):
            return None
        v = rng_for(seed, role_id, layer).normal(0.0, 0.02, size=n).astype(np.float32)
        return tensor(v.view(np.uint8), F32, n, role)

    ts = [weight("token_embd", 0, V, d, 100), ones(d, "output_norm"), weight("output", 0, V, d, 101)]
    for l in range(hp["n_layers"]):
        ts += [ones(d, "attn_norm"),
               weight("attn_q", l, qd, d, 1), bias(qd, 2, l, "attn_q.bias"),
               weight("attn_k", l, kvd, d, 3), bias(kvd, 4, l, "attn_k.bias"),
               weight("attn_v", l, kvd, d, 5), bias(kvd, 6, l, "attn_v.bias"),
               weight("attn_output", l, d, qd, 7),
               ones(d, "ffn_norm"),
               weight("ffn_up", l, f, d, 9), weight("ffn_gate", l, f, d, 10), weight("ffn_down", l, d, f, 11)]
    return hp, ts


def weight_bytes_per_token(tensors: list) -> int:
    """HBM bytes of the weights one decode step streams (all but token_embd)."""
    return sum(t["raw"].nbytes for t in tensors[1:] if t is not None)


def kv_bytes_per_token(hp: dict, ctx_len: int, kv_elem_bytes: int = 4) -> int:
    """K and V bytes attention reads at context length ctx_len."""
    hd = hp["embed_dim"] // hp["n_heads"]
    return 2 * hp["n_layers"] * ctx_len * hp["n_kv_heads"] * hd * kv_elem_bytes

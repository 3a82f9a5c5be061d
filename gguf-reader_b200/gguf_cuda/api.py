"""Host-side mirror of gguf-reader's infer API over libgguf_cuda.

Names, argument meanings and errors follow the Rust crate:
  quant::dequantize / quant::quant_matvec       (src/infer/quant.rs:403, :526)
  LlamaModel::{forward, forward_cached, cache_len, reset_cache}  (model/llama.rs:214-239)
  Engine greedy generate loop                   (src/infer/engine.rs:74-148)
Arrays are numpy (host) or torch CUDA tensors (device); results come back in the
same kind of memory the caller passed.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from ._lib import check, lib


def _ptr(a):
    """(address, nbytes) of a numpy array or a torch tensor."""
    if a is None:
        return None, 0
    if isinstance(a, np.ndarray):
        return a.ctypes.data, a.nbytes
    if hasattr(a, "data_ptr"):
        return a.data_ptr(), a.numel() * a.element_size()
    raise TypeError(f"unsupported buffer type {type(a)}")


def _as_bytes(data) -> np.ndarray:
    if isinstance(data, (bytes, bytearray, memoryview)):
        return np.frombuffer(data, dtype=np.uint8)
    if isinstance(data, np.ndarray):
        return np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    return data   # torch tensor (device bytes)


class Context:
    """One CUDA stream on one GPU (ggc_ctx)."""

    def __init__(self, device: int = 0, rank: int = 0, world: int = 1, nccl_id: bytes | None = None):
        h = C.c_void_p()
        if world > 1:
            buf = C.create_string_buffer(bytes(nccl_id), 128)
            check(lib().ggc_ctx_create_tp(device, rank, world, C.cast(buf, C.c_void_p), C.byref(h)))
        else:
            check(lib().ggc_ctx_create(device, C.byref(h)))
        self.h = h
        self.device = device
        self.rank = rank
        self.world = world

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib().ggc_nccl_unique_id(C.cast(buf, C.c_void_p)))
        return buf.raw

    @property
    def stream(self) -> int:
        return lib().ggc_ctx_stream(self.h) or 0

    def synchronize(self):
        check(lib().ggc_ctx_synchronize(self.h))

    def kernel_launches(self) -> int:
        return int(lib().ggc_ctx_kernel_launches(self.h))

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            lib().ggc_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default_ctx: Context | None = None


def default_context() -> Context:
    global _default_ctx
    if _default_ctx is None:
        _default_ctx = Context(0)
    return _default_ctx


# ---- quant.rs ----------------------------------------------------------------
def block_size(dtype: int):
    v = lib().ggc_block_size(dtype)
    return None if v < 0 else v


def block_bytes(dtype: int):
    v = lib().ggc_block_bytes(dtype)
    return None if v < 0 else v


def dequantize(data, dtype: int, n: int, out=None, ctx: Context | None = None):
    """quant::dequantize: n elements of `dtype` -> f32 (bit-exact with the reference)."""
    ctx = ctx or default_context()
    raw = _as_bytes(data)
    rp, rn = _ptr(raw)
    if out is None:
        out = np.empty(n, dtype=np.float32)
    op, _ = _ptr(out)
    check(lib().ggc_dequantize(ctx.h, dtype, rp if rn else None, rn, n, op))
    return out


def quant_matvec(w, dtype: int, rows: int, cols: int, x, y=None, ctx: Context | None = None):
    """quant::quant_matvec: y[r] = sum_c W[r, c] x[c] over raw GGUF rows."""
    ctx = ctx or default_context()
    wb = _as_bytes(w)
    if isinstance(x, np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
    if y is None:
        y = np.zeros(rows, dtype=np.float32)
    wp, wn = _ptr(wb)
    xp, xn = _ptr(x)
    yp, yn = _ptr(y)
    check(lib().ggc_quant_matvec(ctx.h, dtype, wp, wn, rows, cols, xp, xn // 4, yp, yn // 4))
    return y


def infer_k_quant_dtype(span: int, n: int, marked: int):
    v = lib().ggc_infer_k_quant_dtype(span, n, marked)
    return None if v < 0 else v


class Tensor:
    """A GGUF tensor resident in HBM (plane layout when repack=True)."""

    def __init__(self, raw, dtype: int, ne, repack: bool = True, ctx: Context | None = None):
        self.ctx = ctx or default_context()
        raw = _as_bytes(raw)
        ne_arr = (C.c_uint64 * len(ne))(*ne)
        h = C.c_void_p()
        rp, rn = _ptr(raw)
        check(lib().ggc_tensor_upload(self.ctx.h, rp, rn, dtype, ne_arr, len(ne), 1 if repack else 0, C.byref(h)))
        self.h, self.dtype, self.ne = h, dtype, tuple(ne)
        self.rows = int(np.prod(ne[1:])) if len(ne) > 1 else 1
        self.cols = ne[0]

    def matvec(self, x, y=None):
        if isinstance(x, np.ndarray):
            x = np.ascontiguousarray(x, dtype=np.float32)
        if y is None:
            y = np.zeros(self.rows, dtype=np.float32)
        check(lib().ggc_tensor_matvec(self.ctx.h, self.h, _ptr(x)[0], _ptr(y)[0]))
        return y

    @staticmethod
    def matvec_batch(tensors, x, y):
        """y = W_i x for each tensor in turn, queued on the context stream (device x, y)."""
        if not tensors:
            return y
        ctx = tensors[0].ctx
        arr = (C.c_void_p * len(tensors))(*[t.h.value for t in tensors])
        check(lib().ggc_tensor_matvec_batch(ctx.h, arr, len(tensors), _ptr(x)[0], _ptr(y)[0]))
        return y

    def matmul(self, x, m: int | None = None, y=None):
        """ops::matmul with this tensor transposed: y[m][rows] = x[m][cols] . W^T on the
        tensor cores (upload with repack=False)."""
        if isinstance(x, np.ndarray):
            x = np.ascontiguousarray(x, dtype=np.float32)
            m = x.size // self.cols if m is None else m
        elif m is None:
            m = x.numel() // self.cols
        if y is None:
            y = np.zeros((m, self.rows), dtype=np.float32)
        check(lib().ggc_tensor_matmul(self.ctx.h, self.h, _ptr(x)[0], m, _ptr(y)[0]))
        return y

    def dequantize(self, out=None):
        if out is None:
            out = np.empty(self.rows * self.cols, dtype=np.float32)
        check(lib().ggc_tensor_dequantize(self.ctx.h, self.h, _ptr(out)[0]))
        return out

    def free(self):
        if getattr(self, "h", None) is not None and self.h.value:
            lib().ggc_tensor_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _hparams(hp: dict, max_ctx: int = 0, kv_f16: bool = False):
    return L.HParams(hp["vocab_size"], hp["embed_dim"], hp["n_heads"], hp["n_kv_heads"], hp["ffn_dim"],
                     hp["n_layers"], float(hp["rope_freq_base"]), max_ctx, 1 if kv_f16 else 0)


def allreduce_probe(part0, part1, peer_writes: bool = True, ctx: Context | None = None):
    """One fused all-reduce step of a world-2 group on this GPU alone
    (ggc_allreduce_probe): part0 + part1 when the peer's words are written; with
    peer_writes=False they never arrive and DeviceTimeout is raised once the
    bounded poll gives up."""
    ctx = ctx or default_context()
    p0 = np.ascontiguousarray(part0, dtype=np.float32)
    p1 = np.ascontiguousarray(part1, dtype=np.float32)
    out = np.zeros_like(p0)
    check(lib().ggc_allreduce_probe(ctx.h, p0.size, 1 if peer_writes else 0, p0.ctypes.data, p1.ctypes.data,
                                    out.ctypes.data))
    return out


def tp_plan(hp: dict, attn_output_dtype: int, ffn_down_dtype: int, rank: int, world: int) -> dict:
    """The tensor-parallel shard of one layer kept by `rank` of `world` (ggc_tp_plan):
    q heads, kv heads and ffn rows as (first, count) pairs."""
    out = L.TpShard()
    check(lib().ggc_tp_plan(C.byref(_hparams(hp)), attn_output_dtype, ffn_down_dtype, rank, world, C.byref(out)))
    return {"heads": (out.head0, out.heads), "kv_heads": (out.kv_head0, out.kv_heads),
            "ffn": (out.ffn0, out.ffn_len)}


# ---- sampler.rs ----------------------------------------------------------------
def _sampler_args(cfg, seen):
    cfg = cfg or {}
    c = L.SamplerConfig(cfg.get("temperature", 1.0), cfg.get("top_k", 40), cfg.get("top_p", 0.95),
                        cfg.get("min_p", 0.0), cfg.get("repeat_penalty", 1.1))
    return c, np.ascontiguousarray(list(seen), dtype=np.uint32)


def sample(logits, cfg: dict | None = None, seen=(), u: float = 0.5, ctx: Context | None = None) -> int:
    """Sampler::sample (sampler.rs:86-186) on the device (ggc_sample): `u` is the
    caller's uniform draw in [0, 1) (the reference's rng.gen_range(0.0..1.0));
    cfg keys as SamplerConfig, reference defaults temperature 1.0, top_k 40,
    top_p 0.95, min_p 0.0, repeat_penalty 1.1; seen: ids with a repeat count."""
    ctx = ctx or default_context()
    if isinstance(logits, np.ndarray):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
    n = logits.size if isinstance(logits, np.ndarray) else logits.numel()
    c, ids = _sampler_args(cfg, seen)
    out = C.c_uint32(0)
    check(lib().ggc_sample(ctx.h, _ptr(logits)[0], n, C.byref(c), ids.ctypes.data if ids.size else None, ids.size,
                           float(u), C.byref(out)))
    return int(out.value)


# ---- model/llama.rs ------------------------------------------------------------
class LlamaModel:
    """LlamaModel over tensors given in role order (see synth.TENSOR_ROLES)."""

    def __init__(self, hp: dict, tensors: list, max_ctx: int = 2048, kv_f16: bool = False,
                 ctx: Context | None = None):
        self.ctx = ctx or default_context()
        descs = (L.TensorDesc * len(tensors))()
        keep = []
        for i, t in enumerate(tensors):
            if t is None:
                descs[i] = L.TensorDesc(None, 0, 0, 0)
                continue
            raw = _as_bytes(t["raw"])
            keep.append(raw)
            descs[i] = L.TensorDesc(raw.ctypes.data, raw.nbytes, t["dtype"], t["n_elements"])
        self.hp = _hparams(hp, max_ctx, kv_f16)
        h = C.c_void_p()
        check(lib().ggc_model_create(self.ctx.h, C.byref(self.hp), descs, len(tensors), C.byref(h)))
        self.h = h
        self.vocab = hp["vocab_size"]
        # cache rows hold this rank's kv heads under tensor parallelism
        self.kv_dim = hp["n_kv_heads"] // self.ctx.world * (hp["embed_dim"] // hp["n_heads"])

    @classmethod
    def from_gguf(cls, path, max_ctx: int = 2048, kv_f16: bool = False, ctx: Context | None = None):
        """LlamaModel::new over a .gguf file (gguf_cuda.loader: header, HParams,
        tensor names, the physical-span dtype re-inference)."""
        from . import loader
        f = loader.GgufFile.open(path)
        hp, tensors = loader.model_tensors(f)
        m = cls(hp, tensors, max_ctx=max_ctx, kv_f16=kv_f16, ctx=ctx)
        m.gguf = f
        return m

    def forward(self, tokens, positions, logits=None, want_logits=True):
        """LlamaModel::forward: logits (vocab f32) of the last token; appends K/V."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32) if not hasattr(tokens, "data_ptr") else tokens
        p = np.ascontiguousarray(positions, dtype=np.int64) if not hasattr(positions, "data_ptr") else positions
        n = t.size if isinstance(t, np.ndarray) else t.numel()
        if want_logits and logits is None:
            logits = np.zeros(self.vocab, dtype=np.float32)
        am = np.zeros(1, dtype=np.uint32)
        check(lib().ggc_model_forward(self.h, _ptr(t)[0], _ptr(p)[0], n, _ptr(logits)[0] if want_logits else None,
                                      am.ctypes.data))
        self.last_argmax = int(am[0])
        return logits if want_logits else self.last_argmax

    forward_cached = forward

    def cache_len(self) -> int:
        return int(lib().ggc_model_cache_len(self.h))

    def reset_cache(self):
        check(lib().ggc_model_reset_cache(self.h))

    def sample(self, cfg: dict | None = None, seen=(), u: float = 0.5) -> int:
        """Sampler::sample on the device over the last forward's logits (ggc_model_sample)."""
        c, ids = _sampler_args(cfg, seen)
        out = C.c_uint32(0)
        check(lib().ggc_model_sample(self.h, C.byref(c), ids.ctypes.data if ids.size else None, ids.size, float(u),
                                     C.byref(out)))
        return int(out.value)

    @property
    def allreduce(self) -> str:
        """How the tensor-parallel partials are summed: "none", "nccl" or "peer"."""
        return ("none", "nccl", "peer")[lib().ggc_model_allreduce_kind(self.h)]

    def truncate(self, new_len: int):
        check(lib().ggc_model_truncate(self.h, new_len))

    def cache_append(self, layer: int, k, v):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        check(lib().ggc_model_cache_append(self.h, layer, k.ctypes.data, v.ctypes.data, k.size // self.kv_dim))

    def cache_read(self, layer: int):
        n = self.cache_len() * self.kv_dim
        k = np.zeros(n, dtype=np.float32)
        v = np.zeros(n, dtype=np.float32)
        check(lib().ggc_model_cache_read(self.h, layer, k.ctypes.data, v.ctypes.data))
        return k, v

    def generate_greedy(self, prompt, max_tokens: int, eos: int = -1, start_pos: int = 0) -> list:
        """Engine::generate's loop with the greedy sampler, run on the device."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(max_tokens, 1), dtype=np.uint32)
        n = C.c_uint64(0)
        check(lib().ggc_model_generate_greedy(self.h, p.ctypes.data, p.size, start_pos, max_tokens, eos,
                                              out.ctypes.data, C.byref(n)))
        return out[: n.value].tolist()

    def decode(self, steps: int, eos: int = -1, sync: bool = True):
        """Continues greedy decoding from the last forward's logits (sample -> forward, on the device)."""
        out = np.zeros(max(steps, 1), dtype=np.uint32)
        n = C.c_uint64(0)
        check(lib().ggc_model_decode(self.h, steps, eos, 1 if sync else 0, out.ctypes.data if sync else None,
                                     C.byref(n)))
        return out[: n.value].tolist() if sync else None

    def wait(self, max_ids: int = 0) -> list:
        out = np.zeros(max(max_ids, 1), dtype=np.uint32)
        n = C.c_uint64(0)
        check(lib().ggc_model_wait(self.h, out.ctypes.data if max_ids else None, C.byref(n)))
        return out[: min(n.value, max_ids)].tolist()

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            lib().ggc_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

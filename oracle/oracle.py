"""ctypes view of the CPU oracle (oracle/_build/liborc.so).

TEST INFRASTRUCTURE ONLY: the parity checker and the CPU-baseline timer.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this
module.  The oracle restates chaos-asimo/gguf-reader's Rust CPU path
(src/infer/quant.rs, ops.rs, cache.rs, model/llama.rs, engine.rs) in C++.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liborc.so"

# GGUF on-disk dtype ids (src/types.rs:122-160) + API-only Q3_K_L / Q3_K_M
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
Q2_K, Q3_K_S, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 10, 11, 12, 13, 14, 15, 30
Q3_K_L, Q3_K_M = 111, 112

OK, ERR_DEQUANT, ERR_INVALID_TENSOR_SHAPE, ERR_MISSING_TENSOR = 0, 1, 2, 3
ERR_UNSUPPORTED_ARCH, ERR_INFERENCE, ERR_KV_CACHE_OVERFLOW, ERR_INVALID_ARG = 4, 5, 6, 7


class OracleError(RuntimeError):
    def __init__(self, status, expected=0, actual=0, elements=0, block=0, message=""):
        super().__init__(f"status={status} expected={expected} actual={actual} "
                         f"elements={elements} block={block} {message}")
        self.status, self.expected, self.actual = status, expected, actual
        self.elements, self.block, self.message = elements, block, message


class _Err(C.Structure):
    _fields_ = [("status", C.c_int), ("expected", C.c_uint64), ("actual", C.c_uint64),
                ("elements", C.c_uint64), ("block", C.c_uint64), ("message", C.c_char * 256)]


class TensorDesc(C.Structure):
    _fields_ = [("data", C.c_void_p), ("nbytes", C.c_uint64), ("dtype", C.c_int),
                ("n_elements", C.c_uint64)]


class HParams(C.Structure):
    _fields_ = [("vocab_size", C.c_uint32), ("embed_dim", C.c_uint32), ("n_heads", C.c_uint32),
                ("n_kv_heads", C.c_uint32), ("ffn_dim", C.c_uint32), ("n_layers", C.c_uint32),
                ("rope_freq_base", C.c_double)]


_lib = None


def build():
    """Compile the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        u64, i64, vp, fp = C.c_uint64, C.c_int64, C.c_void_p, C.POINTER(C.c_float)
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_bf16_to_f32.restype = C.c_float
        L.orc_bf16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_block_size.restype = i64
        L.orc_block_bytes.restype = i64
        L.orc_dequantize_block.argtypes = [vp, u64, C.c_int, vp]
        L.orc_dequantize.argtypes = [vp, u64, C.c_int, u64, vp]
        L.orc_quant_matvec.argtypes = [vp, u64, C.c_int, u64, u64, vp, u64, vp, u64]
        L.orc_matvec.argtypes = [vp, u64, u64, u64, vp, u64, vp, u64, vp]
        L.orc_matmul.argtypes = [vp, u64, u64, u64, vp, u64, u64, vp, u64]
        L.orc_matvec_colmajor_trans.argtypes = [vp, u64, u64, u64, vp, u64, vp, u64, vp]
        L.orc_matvec_colmajor.argtypes = [vp, u64, u64, u64, vp, u64, vp, u64, vp]
        L.orc_silu.argtypes = [vp, u64]
        L.orc_gelu.argtypes = [vp, u64]
        L.orc_rmsnorm.argtypes = [vp, u64, vp, u64, C.c_float]
        L.orc_layernorm.argtypes = [vp, u64, vp, u64, vp, u64, C.c_float]
        L.orc_softmax.argtypes = [vp, u64]
        L.orc_rope.argtypes = [vp, u64, vp, u64, vp, u64]
        L.orc_build_inv_freq.argtypes = [u64, C.c_double, vp]
        L.orc_rope_freqs.argtypes = [u64, C.c_float, u64, vp]
        L.orc_infer_k_quant_dtype.argtypes = [u64, u64, C.c_int]
        L.orc_model_create.argtypes = [C.POINTER(HParams), C.POINTER(TensorDesc), u64, C.POINTER(vp)]
        L.orc_model_destroy.argtypes = [vp]
        L.orc_model_forward.argtypes = [vp, vp, vp, u64, vp]
        L.orc_model_cache_len.restype = u64
        L.orc_model_cache_len.argtypes = [vp]
        L.orc_model_reset_cache.argtypes = [vp]
        L.orc_model_truncate.argtypes = [vp, u64]
        L.orc_model_cache_append.argtypes = [vp, C.c_uint32, vp, vp, u64]
        L.orc_model_cache_read.argtypes = [vp, C.c_uint32, vp, vp]
        L.orc_generate_greedy.argtypes = [vp, vp, u64, i64, u64, i64, vp, C.POINTER(u64)]
        L.orc_greedy.restype = C.c_uint32
        L.orc_greedy.argtypes = [vp, u64]
        L.orc_sample.argtypes = [vp, u64, C.POINTER(SamplerCfg), vp, u64, C.c_float, C.POINTER(C.c_uint32)]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_last_error.argtypes = [C.POINTER(_Err)]
        _lib = L
    return _lib


def set_threads(n: int):
    lib().orc_set_threads(int(n))


def get_threads() -> int:
    return lib().orc_get_threads()


def _check(status):
    if status != OK:
        e = _Err()
        lib().orc_last_error(C.byref(e))
        raise OracleError(status, e.expected, e.actual, e.elements, e.block,
                          e.message.decode(errors="replace"))


def _ptr(a):
    return None if a is None else a.ctypes.data


def f16_to_f32(bits: int) -> float:
    return lib().orc_f16_to_f32(bits)


def f32_to_f16(v: float) -> int:
    return lib().orc_f32_to_f16(v)


def block_size(dtype):
    v = lib().orc_block_size(dtype)
    return None if v < 0 else v


def block_bytes(dtype):
    v = lib().orc_block_bytes(dtype)
    return None if v < 0 else v


def dequantize_block(data: bytes, dtype: int, out_len: int = 256) -> np.ndarray:
    buf = np.frombuffer(bytes(data), dtype=np.uint8)
    out = np.zeros(max(out_len, 256), dtype=np.float32)
    _check(lib().orc_dequantize_block(_ptr(buf) if buf.size else None, buf.size, dtype, _ptr(out)))
    return out[:out_len]


def dequantize(data, dtype: int, n: int) -> np.ndarray:
    buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray)) else data).view(np.uint8)
    out = np.empty(n, dtype=np.float32)
    _check(lib().orc_dequantize(_ptr(buf) if buf.size else None, buf.size, dtype, n, _ptr(out)))
    return out


def quant_matvec(w, dtype: int, rows: int, cols: int, x: np.ndarray, y_len: int | None = None) -> np.ndarray:
    wb = np.ascontiguousarray(np.frombuffer(w, dtype=np.uint8) if isinstance(w, (bytes, bytearray)) else w).view(np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows if y_len is None else y_len, dtype=np.float32)
    _check(lib().orc_quant_matvec(_ptr(wb), wb.size, dtype, rows, cols, _ptr(x), x.size, _ptr(y), y.size))
    return y


def matvec_colmajor_trans(a, dim0, dim1, x, b=None):
    a = np.ascontiguousarray(a, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(dim1, dtype=np.float32)
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
    _check(lib().orc_matvec_colmajor_trans(_ptr(a), a.size, dim0, dim1, _ptr(x), x.size, _ptr(y), y.size, _ptr(bb)))
    return y


def matvec_colmajor(a, rows, cols, x, b=None):
    a = np.ascontiguousarray(a, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
    _check(lib().orc_matvec_colmajor(_ptr(a), a.size, rows, cols, _ptr(x), x.size, _ptr(y), y.size,
                                     None if bb is None else _ptr(bb)))
    return y


def matvec(a, rows, cols, x, b=None):
    a = np.ascontiguousarray(a, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
    _check(lib().orc_matvec(_ptr(a), a.size, rows, cols, _ptr(x), x.size, _ptr(y), y.size, _ptr(bb)))
    return y


def matmul(a, ra, ca, b, cb):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    c = np.zeros(ra * cb, dtype=np.float32)
    _check(lib().orc_matmul(_ptr(a), a.size, ra, ca, _ptr(b), b.size, cb, _ptr(c), c.size))
    return c


def silu(x):
    x = np.array(x, dtype=np.float32)
    lib().orc_silu(_ptr(x), x.size)
    return x


def gelu(x):
    x = np.array(x, dtype=np.float32)
    lib().orc_gelu(_ptr(x), x.size)
    return x


def rmsnorm(x, w, eps=1e-6):
    x = np.array(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    lib().orc_rmsnorm(_ptr(x), x.size, _ptr(w), w.size, eps)
    return x


def layernorm(x, w, b, eps=1e-6):
    x = np.array(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    lib().orc_layernorm(_ptr(x), x.size, _ptr(w), w.size, _ptr(b), b.size, eps)
    return x


def softmax(x):
    x = np.array(x, dtype=np.float32)
    lib().orc_softmax(_ptr(x) if x.size else None, x.size)
    return x


def rope(x, positions, freqs):
    x = np.array(x, dtype=np.float32)
    p = np.ascontiguousarray(positions, dtype=np.int64)
    f = np.ascontiguousarray(freqs, dtype=np.float32)
    lib().orc_rope(_ptr(x), x.size, _ptr(p), p.size, _ptr(f), f.size)
    return x


def build_inv_freq(head_dim, base):
    out = np.zeros(head_dim // 2, dtype=np.float32)
    lib().orc_build_inv_freq(head_dim, float(base), _ptr(out))
    return out


def rope_freqs(dim, base, max_seq_len):
    out = np.zeros(max_seq_len * (dim // 2), dtype=np.float32)
    lib().orc_rope_freqs(dim, base, max_seq_len, _ptr(out))
    return out.reshape(max_seq_len, dim // 2)


def infer_k_quant_dtype(span, n, marked):
    v = lib().orc_infer_k_quant_dtype(span, n, marked)
    return None if v < 0 else v


class SamplerCfg(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float), ("min_p", C.c_float),
                ("repeat_penalty", C.c_float)]


def sample(logits, cfg: dict, seen=(), u: float = 0.5) -> int:
    """Sampler::sample (sampler.rs:86-186) with `u` as its uniform draw."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    sd = np.ascontiguousarray(sorted(set(int(s) for s in seen)), dtype=np.uint32)
    c = SamplerCfg(cfg.get("temperature", 1.0), cfg.get("top_k", 40), cfg.get("top_p", 0.95), cfg.get("min_p", 0.0),
                   cfg.get("repeat_penalty", 1.1))
    out = C.c_uint32(0)
    _check(lib().orc_sample(_ptr(lg), lg.size, C.byref(c), _ptr(sd) if sd.size else None, sd.size, float(u),
                            C.byref(out)))
    return int(out.value)


def greedy(logits) -> int:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_greedy(_ptr(lg), lg.size))


class Model:
    """Oracle LlamaModel over the tensors of a synthetic model (see tensor_order)."""

    def __init__(self, hp: dict, tensors: list):
        self._keep = []
        descs = (TensorDesc * len(tensors))()
        for i, t in enumerate(tensors):
            if t is None:
                descs[i] = TensorDesc(None, 0, 0, 0)
                continue
            raw = np.ascontiguousarray(t["raw"]).view(np.uint8)
            self._keep.append(raw)
            descs[i] = TensorDesc(raw.ctypes.data, raw.size, t["dtype"], t["n_elements"])
        self.hp = HParams(hp["vocab_size"], hp["embed_dim"], hp["n_heads"], hp["n_kv_heads"],
                          hp["ffn_dim"], hp["n_layers"], float(hp["rope_freq_base"]))
        h = C.c_void_p()
        _check(lib().orc_model_create(C.byref(self.hp), descs, len(tensors), C.byref(h)))
        self._keep = []   # the oracle holds its own dequantised f32 copies
        self.h = h

    def __del__(self):
        h = getattr(self, "h", None)
        if h is not None and h.value:
            lib().orc_model_destroy(h)
            self.h = None

    def forward(self, tokens, positions) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.int64)
        logits = np.zeros(self.hp.vocab_size, dtype=np.float32)
        _check(lib().orc_model_forward(self.h, _ptr(t), _ptr(p), t.size, _ptr(logits)))
        return logits

    def cache_len(self) -> int:
        return int(lib().orc_model_cache_len(self.h))

    def reset_cache(self):
        lib().orc_model_reset_cache(self.h)

    def truncate(self, n):
        lib().orc_model_truncate(self.h, n)

    def cache_append(self, layer, k, v):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        kvdim = self.hp.n_kv_heads * (self.hp.embed_dim // self.hp.n_heads)
        _check(lib().orc_model_cache_append(self.h, layer, _ptr(k), _ptr(v), k.size // kvdim))

    def cache_read(self, layer):
        kvdim = self.hp.n_kv_heads * (self.hp.embed_dim // self.hp.n_heads)
        n = self.cache_len() * kvdim
        k = np.zeros(n, dtype=np.float32)
        v = np.zeros(n, dtype=np.float32)
        _check(lib().orc_model_cache_read(self.h, layer, _ptr(k), _ptr(v)))
        return k, v

    def generate_greedy(self, prompt, max_tokens, eos=-1, start_pos=0):
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(max_tokens, 1), dtype=np.uint32)
        n = C.c_uint64(0)
        _check(lib().orc_generate_greedy(self.h, _ptr(p), p.size, start_pos, max_tokens, eos,
                                         _ptr(out), C.byref(n)))
        return out[: n.value].tolist()

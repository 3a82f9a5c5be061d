"""ctypes binding of libgguf_cuda.so (the C ABI in include/gguf_cuda.h).

The library is built in-tree (gguf-reader_b200/lib/libgguf_cuda.so).  There is no
CPU fallback: if the library is missing the import fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent          # gguf-reader_b200/
LIB_PATH = Path(os.environ.get("GGC_LIB", PKG_ROOT / "lib" / "libgguf_cuda.so"))

# dtype ids (GGUF on-disk ids, src/types.rs:122-160) + API-only Q3_K_L / Q3_K_M
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
Q2_K, Q3_K_S, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 10, 11, 12, 13, 14, 15, 30
Q3_K_L, Q3_K_M = 111, 112
ALL_DTYPES = [F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K_S, Q3_K_M, Q3_K_L, Q4_K, Q5_K, Q6_K, Q8_K]
DTYPE_NAMES = {F32: "F32", F16: "F16", BF16: "BF16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1",
               Q8_0: "Q8_0", Q2_K: "Q2_K", Q3_K_S: "Q3_K_S", Q3_K_M: "Q3_K_M", Q3_K_L: "Q3_K_L", Q4_K: "Q4_K",
               Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_K: "Q8_K"}
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24),
         Q8_0: (32, 34), Q2_K: (256, 84), Q3_K_S: (256, 110), Q3_K_L: (256, 110), Q3_K_M: (256, 114),
         Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), Q8_K: (256, 292)}

OK, ERR_DEQUANT, ERR_INVALID_TENSOR_SHAPE, ERR_MISSING_TENSOR, ERR_UNSUPPORTED_ARCH = 0, 1, 2, 3, 4
ERR_INFERENCE, ERR_KV_CACHE_OVERFLOW, ERR_INVALID_ARG, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT = 5, 6, 7, 8, 9, 10


class ErrorInfo(C.Structure):
    _fields_ = [("status", C.c_int), ("dtype", C.c_char * 16), ("expected", C.c_uint64), ("actual", C.c_uint64),
                ("elements", C.c_uint64), ("block", C.c_uint64), ("message", C.c_char * 256)]


class HParams(C.Structure):
    _fields_ = [("vocab_size", C.c_uint32), ("embed_dim", C.c_uint32), ("n_heads", C.c_uint32),
                ("n_kv_heads", C.c_uint32), ("ffn_dim", C.c_uint32), ("n_layers", C.c_uint32),
                ("rope_freq_base", C.c_double), ("max_ctx", C.c_uint32), ("kv_f16", C.c_uint32)]


class TpShard(C.Structure):
    _fields_ = [("head0", C.c_uint32), ("heads", C.c_uint32), ("kv_head0", C.c_uint32), ("kv_heads", C.c_uint32),
                ("ffn0", C.c_uint64), ("ffn_len", C.c_uint64)]


class SamplerConfig(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float), ("min_p", C.c_float),
                ("repeat_penalty", C.c_float)]


class TensorDesc(C.Structure):
    _fields_ = [("data", C.c_void_p), ("nbytes", C.c_uint64), ("dtype", C.c_int), ("n_elements", C.c_uint64)]


# ---- GgufError variants (src/error.rs:5-58) --------------------------------
class GgufError(RuntimeError):
    status = -1

    def __init__(self, info: ErrorInfo):
        self.info = info
        self.message = info.message.decode(errors="replace")
        super().__init__(self.message)


class DequantError(GgufError):
    status = ERR_DEQUANT

    @property
    def dtype(self): return self.info.dtype.decode()

    @property
    def expected(self): return self.info.expected

    @property
    def actual(self): return self.info.actual


class InvalidTensorShape(GgufError):
    status = ERR_INVALID_TENSOR_SHAPE

    @property
    def elements(self): return self.info.elements

    @property
    def block(self): return self.info.block


class MissingTensor(GgufError):
    status = ERR_MISSING_TENSOR


class UnsupportedArchitecture(GgufError):
    status = ERR_UNSUPPORTED_ARCH


class InferenceError(GgufError):
    status = ERR_INFERENCE


class KvCacheOverflow(GgufError):
    status = ERR_KV_CACHE_OVERFLOW


class InvalidArgument(GgufError):
    status = ERR_INVALID_ARG


class CudaError(GgufError):
    status = ERR_CUDA


class NcclError(GgufError):
    status = ERR_NCCL


class DeviceTimeout(GgufError):
    status = ERR_TIMEOUT


_ERRORS = {c.status: c for c in (DequantError, InvalidTensorShape, MissingTensor, UnsupportedArchitecture,
                                 InferenceError, KvCacheOverflow, InvalidArgument, CudaError, NcclError, DeviceTimeout)}

# exported symbols: name -> (restype, argtypes)
_u64, _i64, _vp, _i32, _u32 = C.c_uint64, C.c_int64, C.c_void_p, C.c_int, C.c_uint32
SIGNATURES = {
    "ggc_last_error": (_i32, [C.POINTER(ErrorInfo)]),
    "ggc_block_size": (_i64, [_i32]),
    "ggc_block_bytes": (_i64, [_i32]),
    "ggc_ctx_create": (_i32, [_i32, C.POINTER(_vp)]),
    "ggc_ctx_create_tp": (_i32, [_i32, _i32, _i32, _vp, C.POINTER(_vp)]),
    "ggc_nccl_unique_id": (_i32, [_vp]),
    "ggc_ctx_destroy": (_i32, [_vp]),
    "ggc_ctx_stream": (_vp, [_vp]),
    "ggc_ctx_synchronize": (_i32, [_vp]),
    "ggc_ctx_kernel_launches": (_u64, [_vp]),
    "ggc_dequantize": (_i32, [_vp, _i32, _vp, _u64, _u64, _vp]),
    "ggc_quant_matvec": (_i32, [_vp, _i32, _vp, _u64, _u64, _u64, _vp, _u64, _vp, _u64]),
    "ggc_quant_matvec_static": (_i32, [_i32, _vp, _u64, _u64, _u64, _vp, _u64, _vp, _u64, _vp]),
    "ggc_tensor_upload": (_i32, [_vp, _vp, _u64, _i32, C.POINTER(_u64), _i32, _i32, C.POINTER(_vp)]),
    "ggc_tensor_free": (_i32, [_vp]),
    "ggc_tensor_matvec": (_i32, [_vp, _vp, _vp, _vp]),
    "ggc_tensor_matvec_batch": (_i32, [_vp, C.POINTER(_vp), _u64, _vp, _vp]),
    "ggc_tensor_dequantize": (_i32, [_vp, _vp, _vp]),
    "ggc_tensor_matmul": (_i32, [_vp, _vp, _vp, _u64, _vp]),
    "ggc_infer_k_quant_dtype": (_i32, [_u64, _u64, _i32]),
    "ggc_tp_plan": (_i32, [C.POINTER(HParams), _i32, _i32, _i32, _i32, C.POINTER(TpShard)]),
    "ggc_model_create": (_i32, [_vp, C.POINTER(HParams), C.POINTER(TensorDesc), _u64, C.POINTER(_vp)]),
    "ggc_model_destroy": (_i32, [_vp]),
    "ggc_model_forward": (_i32, [_vp, _vp, _vp, _u64, _vp, _vp]),
    "ggc_model_cache_len": (_u64, [_vp]),
    "ggc_model_allreduce_kind": (_i32, [_vp]),
    "ggc_allreduce_probe": (_i32, [_vp, _u32, _i32, _vp, _vp, _vp]),
    "ggc_model_sample": (_i32, [_vp, C.POINTER(SamplerConfig), _vp, _u64, C.c_float, C.POINTER(_u32)]),
    "ggc_ops_matvec": (_i32, [_vp, _vp, _u64, _u64, _u64, _vp, _u64, _vp, _u64, _vp]),
    "ggc_ops_matvec_colmajor": (_i32, [_vp, _vp, _u64, _u64, _u64, _vp, _u64, _vp, _u64, _vp]),
    "ggc_ops_matvec_colmajor_trans": (_i32, [_vp, _vp, _u64, _u64, _u64, _vp, _u64, _vp, _u64, _vp]),
    "ggc_ops_matmul": (_i32, [_vp, _vp, _u64, _u64, _u64, _vp, _u64, _u64, _vp, _u64]),
    "ggc_ops_silu": (_i32, [_vp, _vp, _u64]),
    "ggc_ops_gelu": (_i32, [_vp, _vp, _u64]),
    "ggc_ops_rmsnorm": (_i32, [_vp, _vp, _u64, _vp, _u64, C.c_float]),
    "ggc_ops_layernorm": (_i32, [_vp, _vp, _u64, _vp, _u64, _vp, _u64, C.c_float]),
    "ggc_ops_softmax": (_i32, [_vp, _vp, _u64]),
    "ggc_ops_rope": (_i32, [_vp, _vp, _u64, _vp, _u64, _vp, _u64]),
    "ggc_sample": (_i32, [_vp, _vp, _u64, C.POINTER(SamplerConfig), _vp, _u64, C.c_float, C.POINTER(_u32)]),
    "ggc_model_reset_cache": (_i32, [_vp]),
    "ggc_model_truncate": (_i32, [_vp, _u64]),
    "ggc_model_cache_append": (_i32, [_vp, _u32, _vp, _vp, _u64]),
    "ggc_model_cache_read": (_i32, [_vp, _u32, _vp, _vp]),
    "ggc_model_generate_greedy": (_i32, [_vp, _vp, _u64, _i64, _u64, _i64, _vp, C.POINTER(_u64)]),
    "ggc_model_decode": (_i32, [_vp, _u64, _i64, _i32, _vp, C.POINTER(_u64)]),
    "ggc_model_wait": (_i32, [_vp, _vp, C.POINTER(_u64)]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads libgguf_cuda.so; raises if it has not been built (no CPU fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} not found: build it with `make -C gguf-reader_b200/csrc` "
                              "(or __graft_entry__.build()); there is no CPU fallback")
        L = C.CDLL(str(LIB_PATH), mode=C.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def host_error(cls, message: str, **fields) -> GgufError:
    """An error of the reference's kind raised by host code (the loader), with
    the same payload fields as one raised through the C ABI."""
    info = ErrorInfo()
    info.status = cls.status
    info.message = message.encode()[:255]
    for k, v in fields.items():
        setattr(info, k, v.encode()[:15] if isinstance(v, str) else v)
    return cls(info)


def check(status: int):
    if status != OK:
        info = ErrorInfo()
        lib().ggc_last_error(C.byref(info))
        raise _ERRORS.get(status, GgufError)(info)

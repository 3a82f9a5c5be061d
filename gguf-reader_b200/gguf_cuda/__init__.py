"""gguf_cuda -- B200 (sm_100a) implementation of gguf-reader's quantized inference
hot path, driven through the C ABI of libgguf_cuda.so (include/gguf_cuda.h)."""
from ._lib import (ALL_DTYPES, BF16, BLOCK, DTYPE_NAMES, F16, F32, Q2_K, Q3_K_L, Q3_K_M, Q3_K_S, Q4_0, Q4_1, Q4_K,
                   Q5_0, Q5_1, Q5_K, Q6_K, Q8_0, Q8_K, CudaError, DequantError, DeviceTimeout, GgufError,
                   InferenceError, InvalidArgument, InvalidTensorShape, KvCacheOverflow, MissingTensor, NcclError,
                   UnsupportedArchitecture, lib)
from .api import (Context, LlamaModel, Tensor, allreduce_probe, block_bytes, block_size, default_context, dequantize,
                  infer_k_quant_dtype, quant_matvec, sample, tp_plan)
from . import engine, loader, ops

__all__ = [n for n in dir() if not n.startswith("_")]

"""The C-ABI library loads without a GPU, exports every symbol include/gguf_cuda.h
declares, and reports the reference's errors for bad arguments before touching
the device (quant.rs:358-369, :404-425, :534-555)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "gguf_cuda.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ggc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(ggc):
    lib = ggc.lib()
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_header(ggc):
    from gguf_cuda._lib import SIGNATURES
    assert set(declared_symbols()) <= set(SIGNATURES)


def test_rust_ffi_declares_every_header_symbol():
    """The gguf-cuda crate's raw bindings name each C entry point once (no Rust
    toolchain here, so the declarations are checked as text)."""
    ffi = (ROOT / "gguf-reader_b200" / "rust" / "gguf-cuda" / "src" / "ffi.rs").read_text()
    rust = re.findall(r"pub fn (ggc_[a-z0-9_]+)\s*\(", ffi)
    assert len(rust) == len(set(rust))
    assert sorted(set(rust)) == declared_symbols()


def test_block_geometry(ggc):
    from gguf_cuda._lib import BLOCK
    for dt, (bs, bb) in BLOCK.items():
        assert ggc.block_size(dt) == bs and ggc.block_bytes(dt) == bb
    assert ggc.block_size(4) is None and ggc.block_bytes(4) is None   # Q4_2: None


def test_dequantize_errors_without_device(ggc):
    lib = ggc.lib()
    out = np.zeros(64, np.float32)
    # unsupported dtype -> DequantError { expected: 0, actual: 0 }
    with pytest.raises(ggc.DequantError):
        ggc._lib.check(lib.ggc_dequantize(None, 4, None, 0, 32, out.ctypes.data))
    # n not a multiple of the block -> InvalidTensorShape
    with pytest.raises(ggc.InvalidTensorShape) as e:
        ggc._lib.check(lib.ggc_dequantize(None, ggc.Q4_0, None, 0, 33, out.ctypes.data))
    assert e.value.elements == 33 and e.value.block == 32
    # short data -> DequantError { expected: 18, actual: 8 }
    raw = np.zeros(8, np.uint8)
    with pytest.raises(ggc.DequantError) as e:
        ggc._lib.check(lib.ggc_dequantize(None, ggc.Q4_0, raw.ctypes.data, 8, 32, out.ctypes.data))
    assert (e.value.expected, e.value.actual, e.value.dtype) == (18, 8, "Q4_0")


def test_quant_matvec_errors_without_device(ggc):
    lib = ggc.lib()
    x = np.ones(16, np.float32)
    y = np.zeros(1, np.float32)
    w = np.zeros(16, np.uint8)
    # quant.rs:1013-1022: x.len() != cols
    with pytest.raises(ggc.DequantError) as e:
        ggc._lib.check(lib.ggc_quant_matvec(None, ggc.Q4_0, w.ctypes.data, 16, 1, 32, x.ctypes.data, 16, y.ctypes.data, 1))
    assert (e.value.expected, e.value.actual) == (32, 16)
    # cols not a multiple of the block -> InvalidTensorShape
    with pytest.raises(ggc.InvalidTensorShape):
        ggc._lib.check(lib.ggc_quant_matvec(None, ggc.Q4_K, w.ctypes.data, 16, 1, 100, x.ctypes.data, 100, y.ctypes.data, 1))
    # y.len() != rows
    x32 = np.ones(32, np.float32)
    with pytest.raises(ggc.DequantError) as e:
        ggc._lib.check(lib.ggc_quant_matvec(None, ggc.Q4_0, w.ctypes.data, 16, 2, 32, x32.ctypes.data, 32, y.ctypes.data, 1))
    assert (e.value.expected, e.value.actual) == (2, 1)
    # rows * row_bytes > w.len()
    with pytest.raises(ggc.DequantError) as e:
        ggc._lib.check(lib.ggc_quant_matvec(None, ggc.Q4_0, w.ctypes.data, 16, 1, 32, x32.ctypes.data, 32, y.ctypes.data, 1))
    assert (e.value.expected, e.value.actual) == (18, 16)


def test_infer_k_quant_dtype_matches_oracle(ggc, orc):
    n = 4096 * 4096
    cases = [(n // 32 * 18, n, ggc.Q4_0), (n // 256 * 176, n, ggc.Q4_K), (n // 256 * 114, n, ggc.Q3_K_S),
             (210, 256, ggc.Q5_1), (n // 256 * 210, n, ggc.Q5_1), (100, n, ggc.F32), (0, 0, ggc.Q4_K)]
    for span, nn, marked in cases:
        assert ggc.infer_k_quant_dtype(span, nn, marked) == orc.infer_k_quant_dtype(span, nn, marked)

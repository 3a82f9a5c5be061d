"""ggc_quant_matvec_static -- the allocation-free entry point (scratch in a
file-scope device array) -- against the oracle's quant_matvec (the reference's
quant.rs:526-570) and against the existing ggc_quant_matvec entry, both called
through the C ABI on the same device buffers.

Kept in its own file, collected last, so it runs both alone and after every
other GPU test in the same process (the static scratch then has seen earlier
launches of the library's other kernels).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import synth
from gguf_cuda._lib import BLOCK, DTYPE_NAMES, ERR_INVALID_ARG, ErrorInfo

REL_L2 = 1e-4        # same bar as ggc_quant_matvec against the oracle
MAX_ROWS = 65536     # the entry's static-scratch row limit

CASES = [
    (8, 4096, 4096),     # Q8_0 square
    (2, 4096, 4096),     # Q4_0 square
    (12, 64, 65536),     # Q4_K, few long rows: 32 column splits
    (14, 11008, 4096),   # Q6_K FFN shape
    (112, 37, 1024),     # Q3_K_M ragged row count
    (1, 130, 2048),      # F16
    (13, MAX_ROWS, 256), # Q5_K at the row limit
    (0, 3, 40),          # F32, a single short split
]


def rel_l2(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def last_error(lib):
    info = ErrorInfo()
    lib.ggc_last_error(C.byref(info))
    return info


def device_case(dt, rows, cols, seed):
    import torch
    rng = synth.rng_for(seed, dt, rows, cols)
    w = synth.random_blocks(dt, rows * cols, rng)
    x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
    return torch.from_numpy(w.copy()).cuda(), torch.from_numpy(x).cuda()


def call_static(lib, dt, dw, rows, cols, dx, dy, stream):
    return lib.ggc_quant_matvec_static(dt, dw.data_ptr(), dw.numel(), rows, cols, dx.data_ptr(), dx.numel(),
                                       dy.data_ptr(), dy.numel(), stream)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{DTYPE_NAMES[c[0]]}-{c[1]}x{c[2]}")
def test_static_matches_oracle_and_existing_entry_twice(ggc, orc, ctx, case):
    import torch
    dt, rows, cols = case
    lib = ggc.lib()
    dw, dx = device_case(dt, rows, cols, 91)
    want_orc = orc.quant_matvec(dw.cpu().numpy(), dt, rows, cols, dx.cpu().numpy())
    y_ref = torch.zeros(rows, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ggc._lib.check(lib.ggc_quant_matvec(ctx.h, dt, dw.data_ptr(), dw.numel(), rows, cols, dx.data_ptr(),
                                        dx.numel(), y_ref.data_ptr(), rows))
    ctx.synchronize()
    want = y_ref.cpu().numpy()

    stream = torch.cuda.current_stream().cuda_stream
    got = []
    for _ in range(2):    # two calls in a row: the tickets must come back to zero
        y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        ggc._lib.check(call_static(lib, dt, dw, rows, cols, dx, y, stream))
        torch.cuda.synchronize()
        got.append(y.cpu().numpy())
    for g in got:
        assert np.all(np.isfinite(g))
        assert rel_l2(g, want_orc) <= REL_L2, (rel_l2(g, want_orc), DTYPE_NAMES[dt])
        assert rel_l2(g, want) <= REL_L2, (rel_l2(g, want), DTYPE_NAMES[dt])
    assert np.array_equal(got[0], got[1])    # fixed split order: deterministic


def test_static_allocates_nothing(ggc):
    """After the one-time set-up, repeated calls leave the device's free memory unchanged."""
    import torch
    lib = ggc.lib()
    dt, rows, cols = 12, 512, 8192
    dw, dx = device_case(dt, rows, cols, 92)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ggc._lib.check(call_static(lib, dt, dw, rows, cols, dx, y, stream))   # set-up happens here at the latest
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(8):
        ggc._lib.check(call_static(lib, dt, dw, rows, cols, dx, y, stream))
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] >= free0


def test_static_rejects_rows_beyond_scratch_and_host_buffers(ggc, ctx):
    import torch
    lib = ggc.lib()
    dt, cols = 8, 32
    rows = MAX_ROWS + 1
    dw, dx = device_case(dt, rows, cols, 93)
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert call_static(lib, dt, dw, rows, cols, dx, y, stream) == ERR_INVALID_ARG
    msg = last_error(lib).message.decode()
    assert "65536" in msg and "scratch" in msg
    # host buffers are refused (the entry never stages)
    wh = np.zeros(BLOCK[dt][1], np.uint8)
    xh = np.zeros(cols, np.float32)
    yh = np.zeros(1, np.float32)
    assert lib.ggc_quant_matvec_static(dt, wh.ctypes.data, wh.size, 1, cols, xh.ctypes.data, cols,
                                       yh.ctypes.data, 1, stream) == ERR_INVALID_ARG
    # the reference's own checks still come first and in its order
    with pytest.raises(ggc.InvalidTensorShape):
        ggc._lib.check(call_static(lib, dt, dw, 1, 33, dx, y, stream))
    # a valid call after the refusals still matches the existing entry
    rows = 1000
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    y_ref = torch.zeros(rows, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ggc._lib.check(call_static(lib, dt, dw, rows, cols, dx, y, stream))
    torch.cuda.synchronize()
    ggc._lib.check(lib.ggc_quant_matvec(ctx.h, dt, dw.data_ptr(), dw.numel(), rows, cols, dx.data_ptr(),
                                        dx.numel(), y_ref.data_ptr(), rows))
    ctx.synchronize()
    assert rel_l2(y.cpu().numpy(), y_ref.cpu().numpy()) <= REL_L2

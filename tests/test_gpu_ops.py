"""ops.rs standalone functions on the device (gguf_cuda.ops) against the oracle:
bit-exact where the reference only multiplies and adds (matvec and its
column-major variants, matmul, rmsnorm, layernorm); within a few ulp where it
calls exp / tanh / sin / cos (silu, gelu, softmax, rope).  Plus the reference's
own unit vectors (ops.rs tests) and its size errors."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import ops

REL = 2e-6


def rng(seed):
    return np.random.default_rng(seed)


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(2, 3), (1000, 4096), (37, 11)])
def test_matvec_layouts_bit_exact(orc, ctx, rows, cols):
    r = rng(rows)
    a = r.normal(0, 1, rows * cols).astype(np.float32)
    x = r.normal(0, 1, cols).astype(np.float32)
    b = r.normal(0, 1, rows).astype(np.float32)
    assert bits_equal(ops.matvec(a, rows, cols, x, b, ctx=ctx), orc.matvec(a, rows, cols, x, b))
    assert bits_equal(ops.matvec(a, rows, cols, x, ctx=ctx), orc.matvec(a, rows, cols, x))
    assert bits_equal(ops.linear(a, rows, cols, x, b, ctx=ctx), orc.matvec(a, rows, cols, x, b))
    assert bits_equal(ops.matvec_colmajor(a, rows, cols, x, b, ctx=ctx), orc.matvec_colmajor(a, rows, cols, x, b))
    assert bits_equal(ops.matvec_colmajor_trans(a, cols, rows, x, b, ctx=ctx),
                      orc.matvec_colmajor_trans(a, cols, rows, x, b))


def test_matvec_reference_vectors_and_errors(ggc, ctx):   # ops.rs tests: matvec 2x3 + bias, identity, mismatch
    y = ops.matvec([1, 2, 3, 4, 5, 6], 2, 3, [1, 1, 1], [10, 20], ctx=ctx)
    assert np.allclose(y, [16, 35], atol=1e-6)
    assert np.allclose(ops.matvec([1, 0, 0, 1], 2, 2, [3, 7], ctx=ctx), [3, 7])
    with pytest.raises(ggc.DequantError):
        ops.matvec(np.ones(4), 2, 3, np.ones(3), ctx=ctx)                # a shorter than rows * cols
    with pytest.raises(ggc.DequantError):
        ops.matvec(np.ones(6), 2, 3, np.ones(2), ctx=ctx)                # x length != cols
    with pytest.raises(ggc.DequantError):
        ops.matmul(np.ones(3), 2, 2, np.ones(4), 2, ctx=ctx)


@pytest.mark.parametrize("ra,ca,cb", [(2, 2, 2), (64, 300, 129), (5, 4096, 7)])
def test_matmul_bit_exact(orc, ctx, ra, ca, cb):
    r = rng(ra + cb)
    a = r.normal(0, 1, ra * ca).astype(np.float32)
    b = r.normal(0, 1, ca * cb).astype(np.float32)
    got = ops.matmul(a, ra, ca, b, cb, ctx=ctx)
    assert bits_equal(got, orc.matmul(a, ra, ca, b, cb))
    if (ra, ca, cb) == (2, 2, 2):   # ops.rs test_matmul_2x2
        assert np.allclose(ops.matmul([1, 2, 3, 4], 2, 2, [5, 6, 7, 8], 2, ctx=ctx), [19, 22, 43, 50])


@pytest.mark.parametrize("n", [1, 896, 4096, 10001])
def test_norms_bit_exact(orc, ctx, n):
    r = rng(n)
    x = r.normal(0, 3, n).astype(np.float32)
    w = r.normal(1, 0.1, n).astype(np.float32)
    b = r.normal(0, 0.1, n).astype(np.float32)
    assert bits_equal(ops.rmsnorm(x, w, 1e-6, ctx=ctx), orc.rmsnorm(x, w, 1e-6))
    assert bits_equal(ops.layernorm(x, w, b, 1e-5, ctx=ctx), orc.layernorm(x, w, b, 1e-5))
    # mismatched lengths leave x unchanged, as the reference does
    assert bits_equal(ops.rmsnorm(x, w[:-1] if n > 1 else [], ctx=ctx), x)


def test_transcendental_ops_close(orc, ctx):
    r = rng(9)
    x = r.normal(0, 4, 50000).astype(np.float32)
    for name, got, want in (("silu", ops.silu(x, ctx=ctx), orc.silu(x)), ("gelu", ops.gelu(x, ctx=ctx), orc.gelu(x)),
                            ("softmax", ops.softmax(x, ctx=ctx), orc.softmax(x))):
        assert np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want) <= REL, name
        if name != "gelu":   # gelu's 1 + tanh(t) cancels for x << 0: a few-ulp tanh difference is a large relative one
            err = np.abs(got.astype(np.float64) - want) / np.maximum(np.abs(want), 1e-30)
            assert float(np.max(err[np.abs(want) > 1e-30])) <= 1e-5, name
    hd, n_tok = 128, 9
    xr = r.normal(0, 1, hd * n_tok).astype(np.float32)
    pos = np.array([0, 1, 2, 5, 100, 2047, 7, 3], np.int64)          # one token past the list: position 0
    freqs = orc.build_inv_freq(hd, 1e4)
    got, want = ops.rope(xr, pos, freqs, ctx=ctx), orc.rope(xr, pos, freqs)
    assert np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want) <= 1e-5
    assert bits_equal(ops.softmax(np.zeros(0, np.float32), ctx=ctx), np.zeros(0, np.float32))

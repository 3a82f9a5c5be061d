"""ops.rs on the device (src/infer/ops.rs): the standalone functions with the
reference's argument meaning; numpy (host) arrays in, results in place or
returned.  Size errors raise DequantError as the reference's functions return it."""
from __future__ import annotations

import numpy as np

from ._lib import check, lib
from .api import default_context


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return a.ctypes.data if a is not None and a.size else None


def _mv(fn, a, d0, d1, x, y_len, b, ctx):
    ctx = ctx or default_context()
    a, x = _f32(a), _f32(x)
    y = np.zeros(y_len, np.float32)
    bb = _f32(b) if b is not None else None
    check(fn(ctx.h, _p(a), a.size, d0, d1, _p(x), x.size, _p(y), y.size, _p(bb)))
    return y


def matvec(a, rows, cols, x, b=None, ctx=None):                    # ops.rs:14
    return _mv(lib().ggc_ops_matvec, a, rows, cols, x, rows, b, ctx)


def matvec_colmajor(a, rows, cols, x, b=None, ctx=None):           # ops.rs:121
    return _mv(lib().ggc_ops_matvec_colmajor, a, rows, cols, x, rows, b, ctx)


def matvec_colmajor_trans(a, dim0, dim1, x, b=None, ctx=None):     # ops.rs:172
    return _mv(lib().ggc_ops_matvec_colmajor_trans, a, dim0, dim1, x, dim1, b, ctx)


def linear(a, out_dim, in_dim, x, b=None, ctx=None):               # ops.rs:358
    return matvec(a, out_dim, in_dim, x, b, ctx)


def matmul(a, ra, ca, b, cb, ctx=None):                            # ops.rs:74
    ctx = ctx or default_context()
    a, b = _f32(a), _f32(b)
    c = np.zeros(ra * cb, np.float32)
    check(lib().ggc_ops_matmul(ctx.h, _p(a), a.size, ra, ca, _p(b), b.size, cb, _p(c), c.size))
    return c


def _inplace(fn, x, *rest, ctx=None):
    ctx = ctx or default_context()
    x = _f32(x).copy()
    check(fn(ctx.h, _p(x), x.size, *rest))
    return x


def silu(x, ctx=None):                                             # ops.rs:237
    return _inplace(lib().ggc_ops_silu, x, ctx=ctx)


def gelu(x, ctx=None):                                             # ops.rs:250
    return _inplace(lib().ggc_ops_gelu, x, ctx=ctx)


def softmax(x, ctx=None):                                          # ops.rs:295
    return _inplace(lib().ggc_ops_softmax, x, ctx=ctx)


def rmsnorm(x, w, eps=1e-6, ctx=None):                             # ops.rs:262
    w = _f32(w)
    return _inplace(lib().ggc_ops_rmsnorm, x, _p(w), w.size, float(eps), ctx=ctx)


def layernorm(x, w, b, eps=1e-6, ctx=None):                        # ops.rs:279
    w, b = _f32(w), _f32(b)
    return _inplace(lib().ggc_ops_layernorm, x, _p(w), w.size, _p(b), b.size, float(eps), ctx=ctx)


def rope(x, positions, freqs, ctx=None):                           # ops.rs:318
    pos = np.ascontiguousarray(positions, dtype=np.int64)
    f = _f32(freqs)
    return _inplace(lib().ggc_ops_rope, x, _p(pos), pos.size, _p(f), f.size, ctx=ctx)

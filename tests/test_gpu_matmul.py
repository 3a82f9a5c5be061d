"""ggc_tensor_matmul -- the tensor-core (tcgen05) matrix product of the prefill
path -- against the oracle's bit-exact dequantisation and an f64 product.

Split-bf16 operands (hi + lo) with f32 accumulation: within 1e-4 relative L2
of the f64 reference (the north-star tolerance for matvec / logits), for every
GGUF format, ragged token counts (M not a multiple of 128 or 512), ragged weight
rows (not a multiple of 64) and columns (not a multiple of 64).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import synth
from gguf_cuda._lib import ALL_DTYPES, BLOCK, DTYPE_NAMES

REL_L2 = 1e-4


def rel_l2(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def case(orc, dt, rows, cols, m, seed):
    rng = synth.rng_for(seed, dt, rows, cols)
    w = synth.random_blocks(dt, rows * cols, rng)
    x = rng.normal(0.0, 1.0, size=(m, cols)).astype(np.float32)
    wf = orc.dequantize(w, dt, rows * cols).astype(np.float64).reshape(rows, cols)
    return w, x, x.astype(np.float64) @ wf.T


@pytest.mark.parametrize("dt", ALL_DTYPES, ids=[DTYPE_NAMES[d] for d in ALL_DTYPES])
def test_matmul_every_format(ggc, orc, ctx, dt):
    bs = BLOCK[dt][0]
    cols = max(512, bs)
    rows, m = 192, 130
    w, x, want = case(orc, dt, rows, cols, m, 31)
    t = ggc.Tensor(w, dt, (cols, rows), repack=False, ctx=ctx)
    got = t.matmul(x)
    assert got.shape == (m, rows) and np.all(np.isfinite(got))
    assert rel_l2(got, want) <= REL_L2, (DTYPE_NAMES[dt], rel_l2(got, want))


@pytest.mark.parametrize("rows,cols,m", [(100, 256, 1), (64, 4096, 64), (4096, 512, 600), (37, 40, 515)],
                         ids=["m1-rows100", "k4096", "m600-two-passes", "ragged-f32-cols40"])
def test_matmul_shapes(ggc, orc, ctx, rows, cols, m):
    dt = ggc.Q4_K if cols % 256 == 0 else ggc.F32
    w, x, want = case(orc, dt, rows, cols, m, 32)
    t = ggc.Tensor(w, dt, (cols, rows), repack=False, ctx=ctx)
    got = t.matmul(x)
    assert rel_l2(got, want) <= REL_L2, rel_l2(got, want)
    # row by row it matches the matvec of the same tensor (the decode path's product)
    for r in (0, m - 1):
        assert rel_l2(got[r], t.matvec(x[r])) <= REL_L2


@pytest.mark.parametrize("dtname", ["Q4_K", "Q5_K"])
@pytest.mark.parametrize("rows,cols,m", [(200, 256 * 37, 70), (130, 256, 513), (64, 256 * 5, 1)],
                         ids=["split-k-37-blocks", "one-block-two-passes", "m1"])
def test_matmul_staged_raw_blocks(ggc, orc, ctx, dtname, rows, cols, m):
    """Q4_K / Q5_K stage their raw blocks in shared memory by TMA: ragged rows
    (zero-filled past the matrix), K split in whole blocks, one-block rows."""
    dt = getattr(ggc, dtname)
    w, x, want = case(orc, dt, rows, cols, m, 34)
    t = ggc.Tensor(w, dt, (cols, rows), repack=False, ctx=ctx)
    got = t.matmul(x)
    assert got.shape == (m, rows) and np.all(np.isfinite(got))
    assert rel_l2(got, want) <= REL_L2, rel_l2(got, want)
    assert np.array_equal(got, t.matmul(x))          # deterministic


def test_matmul_device_buffers_and_repeat(ggc, orc, ctx):
    import torch
    dt, rows, cols, m = ggc.Q6_K, 256, 1024, 300
    w, x, want = case(orc, dt, rows, cols, m, 33)
    t = ggc.Tensor(w, dt, (cols, rows), repack=False, ctx=ctx)
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((m, rows), float("nan"), device="cuda")
    torch.cuda.synchronize()
    t.matmul(dx, m=m, y=dy)
    ctx.synchronize()
    a = dy.cpu().numpy()
    t.matmul(dx, m=m, y=dy)
    ctx.synchronize()
    assert np.array_equal(a, dy.cpu().numpy())      # deterministic
    assert rel_l2(a, want) <= REL_L2


def test_matmul_rejects_plane_layout(ggc, ctx):
    w = synth.random_blocks(ggc.Q8_0, 64 * 64, synth.rng_for(1, 8))
    t = ggc.Tensor(w, ggc.Q8_0, (64, 64), repack=True, ctx=ctx)
    with pytest.raises(ggc.InvalidArgument):
        t.matmul(np.zeros((2, 64), np.float32))

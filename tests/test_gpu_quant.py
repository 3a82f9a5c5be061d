"""CUDA dequantisation and matvec against the oracle, through the C ABI.

Dequantisation must be bit-exact (quant.rs:128-345 restated with no FMA);
matvecs must be within 1e-4 relative L2 of the oracle's f32 result.
"""
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import synth
from gguf_cuda._lib import ALL_DTYPES, BLOCK, DTYPE_NAMES

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "dequant_golden.npz")
REL_L2 = 1e-4   # north-star tolerance for matvec / logits


def same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))


def rel_l2(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def edge_blocks(dt, rng):
    """Blocks whose f16 scale fields are +0, -0, max, subnormal, +inf and NaN."""
    bs, bb = BLOCK[dt]
    if bs == 1:
        vals = np.array([0x0000, 0x8000, 0x7BFF, 0x0001, 0x7C00, 0x7E00, 0xFC00, 0xFE01], np.uint16)
        if dt == 0:
            return np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, 3.4e38], np.float32).view(np.uint8)
        return vals.view(np.uint8)
    out = []
    for e in [0x0000, 0x8000, 0x7BFF, 0x0001, 0x7C00, 0x7E00, 0xFE01]:
        b = np.frombuffer(rng.bytes(bb), np.uint8).copy()
        for off in synth._SCALE_FIELDS.get(dt, []):
            b[off:off + 2] = np.array([e], np.uint16).view(np.uint8)
        if dt == 15:   # Q8_K: f32 d
            b[0:4] = np.array([e], np.uint16).view(np.float16).astype(np.float32).view(np.uint8)
        out.append(b)
    return np.concatenate(out)


@pytest.mark.parametrize("dt", ALL_DTYPES, ids=lambda d: DTYPE_NAMES[d])
def test_dequant_bit_exact_small(ggc, orc, ctx, dt):
    rng = synth.rng_for(7, dt)
    bs, bb = BLOCK[dt]
    raw = np.concatenate([synth.random_blocks(dt, bs * 64, rng), edge_blocks(dt, rng)])
    n = raw.size // bb * bs
    assert same_bits(ggc.dequantize(raw, dt, n, ctx=ctx), orc.dequantize(raw, dt, n))


@pytest.mark.parametrize("dt", ALL_DTYPES, ids=lambda d: DTYPE_NAMES[d])
def test_dequant_bit_exact_4096x4096(ggc, orc, ctx, dt):
    """Full 4096 x 4096 weight of each format (the format-sweep shape)."""
    n = 4096 * 4096
    raw = synth.random_blocks(dt, n, synth.rng_for(11, dt))
    assert same_bits(ggc.dequantize(raw, dt, n, ctx=ctx), orc.dequantize(raw, dt, n))


@pytest.mark.parametrize("name", sorted({k[:-4] for k in GOLDEN.files if k.endswith("_raw")}))
def test_dequant_matches_reference_tool_golden(ggc, ctx, name):
    raw, want = GOLDEN[f"{name}_raw"], GOLDEN[f"{name}_out"]
    dt = int(GOLDEN[f"{name}_id"][0])
    assert same_bits(ggc.dequantize(raw, dt, want.size, ctx=ctx), want)


def test_dequant_device_pointers(ggc, orc, ctx):
    import torch
    dt, n = ggc.Q4_K, 256 * 1024
    raw = synth.random_blocks(dt, n, synth.rng_for(3))
    draw = torch.from_numpy(raw.copy()).cuda()
    dout = torch.empty(n, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ggc.dequantize(draw, dt, n, out=dout, ctx=ctx)
    ctx.synchronize()
    assert same_bits(dout.cpu().numpy(), orc.dequantize(raw, dt, n))


def test_dequant_errors_on_device_ctx(ggc, ctx):
    with pytest.raises(ggc.DequantError):
        ggc.dequantize(np.zeros(8, np.uint8), ggc.Q4_0, 32, ctx=ctx)
    with pytest.raises(ggc.InvalidTensorShape):
        ggc.dequantize(np.zeros(36, np.uint8), ggc.Q4_0, 33, ctx=ctx)
    assert ggc.dequantize(np.zeros(0, np.uint8), ggc.Q4_0, 0, ctx=ctx).size == 0


MATVEC_SHAPES = [(64, 1024), (37, 512), (1, 256), (130, 2048)]


@pytest.mark.parametrize("dt", ALL_DTYPES, ids=lambda d: DTYPE_NAMES[d])
@pytest.mark.parametrize("shape", MATVEC_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_quant_matvec_raw(ggc, orc, ctx, dt, shape):
    rows, cols = shape
    rng = synth.rng_for(21, dt, rows, cols)
    w = synth.random_blocks(dt, rows * cols, rng)
    x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
    got = ggc.quant_matvec(w, dt, rows, cols, x, ctx=ctx)
    want = orc.quant_matvec(w, dt, rows, cols, x)
    assert rel_l2(got, want) <= REL_L2


@pytest.mark.parametrize("dt", ALL_DTYPES, ids=lambda d: DTYPE_NAMES[d])
@pytest.mark.parametrize("shape", MATVEC_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_tensor_matvec_planes(ggc, orc, ctx, dt, shape):
    """Repacked (plane layout) decode GEMV."""
    rows, cols = shape
    rng = synth.rng_for(22, dt, rows, cols)
    w = synth.random_blocks(dt, rows * cols, rng)
    x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
    t = ggc.Tensor(w, dt, (cols, rows), repack=True, ctx=ctx)
    got = t.matvec(x)
    want = orc.quant_matvec(w, dt, rows, cols, x)
    assert rel_l2(got, want) <= REL_L2, (rel_l2(got, want), DTYPE_NAMES[dt])


def test_config1_q4_0_4096(ggc, orc, ctx):
    """Q4_0 4096 x 4096: d ~ U[1e-3, 1e-2] (seed 0), x ~ N(0,1) (seed 1); dequant bit-exact, y within 1e-4."""
    rows = cols = 4096
    w = synth.random_blocks(ggc.Q4_0, rows * cols, np.random.default_rng(0))
    x = np.random.default_rng(1).normal(0.0, 1.0, size=cols).astype(np.float32)
    want = orc.quant_matvec(w, ggc.Q4_0, rows, cols, x)
    assert rel_l2(ggc.quant_matvec(w, ggc.Q4_0, rows, cols, x, ctx=ctx), want) <= REL_L2
    t = ggc.Tensor(w, ggc.Q4_0, (cols, rows), repack=True, ctx=ctx)
    assert rel_l2(t.matvec(x), want) <= REL_L2
    assert same_bits(ggc.dequantize(w, ggc.Q4_0, rows * cols, ctx=ctx), orc.dequantize(w, ggc.Q4_0, rows * cols))


SWEEP = [(4096, 4096), (11008, 4096), (4096, 11008)]


@pytest.mark.parametrize("dt", [d for d in ALL_DTYPES if d != 0], ids=lambda d: DTYPE_NAMES[d])
@pytest.mark.parametrize("shape", SWEEP, ids=lambda s: f"{s[0]}x{s[1]}")
def test_format_sweep_full_size(ggc, orc, ctx, dt, shape):
    """Every format at the sweep shapes: plane-layout GEMV within 1e-4 of the oracle."""
    rows, cols = shape
    bs = BLOCK[dt][0]
    if cols % bs:
        pytest.skip("cols not a multiple of the block")
    rng = synth.rng_for(31, dt, rows, cols)
    w = synth.random_blocks(dt, rows * cols, rng)
    x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
    want = orc.quant_matvec(w, dt, rows, cols, x)
    t = ggc.Tensor(w, dt, (cols, rows), repack=True, ctx=ctx)
    assert rel_l2(t.matvec(x), want) <= REL_L2


def test_matvec_linearity_full_size(ggc, ctx):
    """Size-independent property at 11008 x 4096 Q4_K: W(a x + b z) = a Wx + b Wz."""
    rows, cols = 11008, 4096
    rng = synth.rng_for(41)
    w = synth.random_blocks(ggc.Q4_K, rows * cols, rng)
    x = rng.normal(size=cols).astype(np.float32)
    z = rng.normal(size=cols).astype(np.float32)
    t = ggc.Tensor(w, ggc.Q4_K, (cols, rows), ctx=ctx)
    lhs = t.matvec((2.0 * x + 3.0 * z).astype(np.float32))
    rhs = 2.0 * t.matvec(x).astype(np.float64) + 3.0 * t.matvec(z).astype(np.float64)
    assert rel_l2(lhs, rhs) <= 1e-5
    assert np.array_equal(t.matvec(x), t.matvec(x))   # deterministic


@pytest.mark.parametrize("dt", ALL_DTYPES, ids=lambda d: DTYPE_NAMES[d])
def test_device_repack_matches_host_repack(ggc, orc, ctx, dt, monkeypatch):
    """The GPU repack at upload (k_repack) writes the planes the host repack writes:
    the decode GEMV over either gives bit-identical outputs (odd row counts, padded
    spans, several column tiles), within 1e-4 of the oracle."""
    bs = BLOCK[dt][0]
    for rows, cols in [(37, 512), (130, 2048), (50, 11008), (17, 4096 + 256)]:
        if cols % bs:
            continue
        rng = synth.rng_for(23, dt, rows, cols)
        w = synth.random_blocks(dt, rows * cols, rng)
        x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
        monkeypatch.delenv("GGC_REPACK", raising=False)
        dev = ggc.Tensor(w, dt, (cols, rows), repack=True, ctx=ctx).matvec(x)
        monkeypatch.setenv("GGC_REPACK", "host")
        host = ggc.Tensor(w, dt, (cols, rows), repack=True, ctx=ctx).matvec(x)
        monkeypatch.delenv("GGC_REPACK")
        assert same_bits(dev, host), (DTYPE_NAMES[dt], rows, cols)
        assert rel_l2(dev, orc.quant_matvec(w, dt, rows, cols, x)) <= REL_L2


@pytest.mark.parametrize("dt", [12, 112, 1], ids=["Q4_K", "Q3_K_M", "F16"])
def test_repacked_upload_from_device_memory(ggc, ctx, dt):
    """ggc_tensor_upload(repack=1) of raw bytes already in device memory gives the
    same tensor as an upload from host memory (the split runs on the GPU either way)."""
    import torch
    rows, cols = 33, 4096 + 256
    rng = synth.rng_for(24, dt)
    w = synth.random_blocks(dt, rows * cols, rng)
    x = rng.normal(0.0, 1.0, size=cols).astype(np.float32)
    dw = torch.from_numpy(w.copy()).cuda()
    torch.cuda.synchronize()
    from_dev = ggc.Tensor(dw, dt, (cols, rows), repack=True, ctx=ctx).matvec(x)
    from_host = ggc.Tensor(w, dt, (cols, rows), repack=True, ctx=ctx).matvec(x)
    assert same_bits(from_dev, from_host)

"""Pins the CPU oracle to the reference's own unit-test values.

Each test restates one of chaos-asimo/gguf-reader's tests (file:line cited) and
runs it against the oracle, so the oracle is checked before it is trusted as
the parity reference for the CUDA path.
"""
import math
import struct

import numpy as np
import pytest

from tiny_models import min_llama_tensors, min_llama_hp, forward_runs_tensors, forward_runs_hp


def f16b(orc, v):
    return struct.pack("<H", orc.f32_to_f16(v))


# ---- src/infer/quant.rs tests ------------------------------------------------
def test_f16_roundtrip(orc):   # quant.rs:621-627
    for v in [0.0, 1.0, -1.0, 0.5, 3.25, -100.0, 65504.0, 6.1035156e-5]:
        dec = orc.f16_to_f32(orc.f32_to_f16(v))
        assert abs(dec - v) < 1e-5 * max(abs(v), 1.0)


def test_f16_boundaries(orc):   # quant.rs:630-636
    assert orc.f16_to_f32(orc.f32_to_f16(math.inf)) == math.inf
    assert math.isnan(orc.f16_to_f32(orc.f32_to_f16(math.nan)))
    neg0 = orc.f16_to_f32(orc.f32_to_f16(-0.0))
    assert struct.pack("<f", neg0) == struct.pack("<f", -0.0)
    assert orc.f16_to_f32(orc.f32_to_f16(1e30)) == math.inf
    # NaN decodes to the canonical f32 NaN with the sign dropped (quant.rs:26-27)
    nan = np.array([orc.f16_to_f32(0xFE01)], dtype=np.float32)
    assert nan.view(np.uint32)[0] == 0x7FC00000


def test_bf16_roundtrip(orc):   # quant.rs:639-646
    for v in [0.0, 1.0, -2.5, 123.0, -0.25, 1.5e5]:
        bits = np.array([v], dtype=np.float32).view(np.uint32)[0] & 0xFFFF0000
        out = orc.lib().orc_bf16_to_f32(int(bits >> 16))
        assert np.float32(out).view(np.uint32) == bits


def test_q4_0(orc):   # quant.rs:649-664
    block = bytearray(18)
    block[0:2] = f16b(orc, 0.25)
    for i in range(16):
        block[2 + i] = i | (i << 4)
    out = orc.dequantize_block(block, orc.Q4_0, 32)
    for i in range(16):
        assert abs(out[2 * i] - 0.25 * (i - 8)) < 1e-6
        assert abs(out[2 * i + 1] - 0.25 * (i - 8)) < 1e-6


def test_q4_1(orc):   # quant.rs:667-693
    block = bytearray(20)
    block[0:2] = f16b(orc, 0.5)
    block[2:4] = f16b(orc, 0.0)
    for i in range(16):
        block[4 + i] = i | (((i + 1) & 0xF) << 4)
    out = orc.dequantize_block(block, orc.Q4_1, 32)
    for i in range(16):
        assert abs(out[2 * i] - 0.5 * i) < 1e-6
        assert abs(out[2 * i + 1] - 0.5 * ((i + 1) & 0xF)) < 1e-6


def test_q5_0(orc):   # quant.rs:696-732
    block = bytearray(22)
    block[0:2] = f16b(orc, 0.25)
    block[2:6] = bytes([0x11, 0x22, 0, 0])
    for i in range(16):
        block[6 + i] = i | (((i + 1) & 0xF) << 4)
    out = orc.dequantize_block(block, orc.Q5_0, 32)
    qh = struct.unpack("<I", bytes([0x11, 0x22, 0, 0]))[0]
    for i in range(16):
        lo = i | (((qh >> i) << 4) & 0x10)
        hi = ((i + 1) & 0xF) | ((qh >> (i + 12)) & 0x10)
        assert abs(out[i] - 0.25 * (lo - 16)) < 1e-6
        assert abs(out[16 + i] - 0.25 * (hi - 16)) < 1e-6


def test_q5_1(orc):   # quant.rs:735-772
    block = bytearray(24)
    block[0:2] = f16b(orc, 0.25)
    block[2:4] = f16b(orc, 0.0)
    block[4:8] = bytes([0x0F, 0, 0, 0])
    for i in range(16):
        block[8 + i] = i | (((i + 1) & 0xF) << 4)
    out = orc.dequantize_block(block, orc.Q5_1, 32)
    qh = 0x0F
    for i in range(16):
        lo = i | (((qh >> i) << 4) & 0x10)
        hi = ((i + 1) & 0xF) | ((qh >> (i + 12)) & 0x10)
        assert abs(out[i] - 0.25 * lo) < 1e-6
        assert abs(out[16 + i] - 0.25 * hi) < 1e-6


def test_q8_0(orc):   # quant.rs:775-792
    block = bytearray(34)
    block[0:2] = f16b(orc, 0.125)
    for i in range(32):
        block[2 + i] = i % 5
    out = orc.dequantize_block(block, orc.Q8_0, 32)
    for i in range(32):
        assert abs(out[i] - 0.125 * (i % 5)) < 1e-6


def kquant_smoke_block(orc, dt):
    """The block of quant.rs:807-839 (scale fields set, zero bytes filled with i & 0xF)."""
    bb = orc.block_bytes(dt)
    b = bytearray(bb)
    if dt == orc.Q2_K:
        b[80:82] = f16b(orc, 0.5); b[82:84] = f16b(orc, 0.1)
    elif dt in (orc.Q3_K_S, orc.Q3_K_L):
        b[108:110] = f16b(orc, 0.5)
    elif dt == orc.Q3_K_M:
        b[112:114] = f16b(orc, 0.5)
    elif dt in (orc.Q4_K, orc.Q5_K):
        b[0:2] = f16b(orc, 0.5); b[2:4] = f16b(orc, 0.1)
    elif dt == orc.Q6_K:
        b[208:210] = f16b(orc, 0.5)
    elif dt == orc.Q8_K:
        b[0:4] = struct.pack("<f", 0.5)
    for i in range(bb):
        if b[i] == 0:
            b[i] = i & 0x0F
    return bytes(b)


KQUANTS = ["Q2_K", "Q3_K_S", "Q3_K_M", "Q3_K_L", "Q4_K", "Q5_K", "Q6_K", "Q8_K"]


@pytest.mark.parametrize("name", KQUANTS)
def test_kquant_finite_smoke(orc, name):   # quant.rs:795-846
    dt = getattr(orc, name)
    out = orc.dequantize_block(kquant_smoke_block(orc, dt), dt, 256)
    assert np.all(np.isfinite(out))


def test_q4_k(orc):   # quant.rs:849-893
    block = bytearray(144)
    block[0:2] = f16b(orc, 0.5)
    block[2:4] = f16b(orc, 0.1)
    block[4] = 0x02
    block[8] = 0x03
    for i in range(128):
        block[16 + i] = 0x5A
    out = orc.dequantize_block(block, orc.Q4_K, 256)
    for i in range(16):
        assert abs(out[i] - 9.7) < 1e-4
    # sub-blocks 1..7 have zero scale and min in this block
    assert np.all(out[32:] == 0.0)


def test_dequantize_whole(orc):   # quant.rs:896-906
    block = bytearray(18)
    block[0:2] = f16b(orc, 1.0)
    out = orc.dequantize(bytes(block) * 2, orc.Q4_0, 64)
    assert out.size == 64 and np.all(np.isfinite(out))


def test_dequantize_insufficient_bytes(orc):   # quant.rs:909-916
    with pytest.raises(orc.OracleError) as e:
        orc.dequantize(bytes(8), orc.Q4_0, 32)
    assert e.value.status == orc.ERR_DEQUANT and e.value.expected == 18 and e.value.actual == 8


def test_dequantize_unsupported(orc):   # quant.rs:919-925 (Q4_2 = GGUF id 4)
    with pytest.raises(orc.OracleError) as e:
        orc.dequantize_block(bytes(8), 4, 32)
    assert e.value.status == orc.ERR_DEQUANT


def test_dequantize_shape_error(orc):   # quant.rs:409-415
    with pytest.raises(orc.OracleError) as e:
        orc.dequantize(bytes(36), orc.Q4_0, 33)
    assert e.value.status == orc.ERR_INVALID_TENSOR_SHAPE and e.value.elements == 33 and e.value.block == 32


def q4k_matvec_case(orc):
    """quant.rs:929-969: 8 x 512 Q4_K, d = 0.5, scale j=0 = (r%5)+1, qs 0x5A, x = i%3."""
    rows, cols = 8, 512
    w = bytearray()
    for r in range(rows):
        for _ in range(cols // 256):
            b = bytearray(144)
            b[0:2] = f16b(orc, 0.5)
            b[4] = (r % 5) + 1
            b[16:144] = bytes([0x5A]) * 128
            w += b
    x = np.array([i % 3 for i in range(cols)], dtype=np.float32)
    return bytes(w), rows, cols, x


def test_quant_matvec_matches_dequant(orc):   # quant.rs:928-969
    w, rows, cols, x = q4k_matvec_case(orc)
    wd = orc.dequantize(w, orc.Q4_K, rows * cols).reshape(rows, cols)
    y_ref = np.zeros(rows, dtype=np.float32)
    for r in range(rows):
        acc = np.float32(0)
        for c in range(cols):
            acc = np.float32(acc + np.float32(wd[r, c] * x[c]))
        y_ref[r] = acc
    y = orc.quant_matvec(w, orc.Q4_K, rows, cols, x)
    assert np.all(np.abs(y - y_ref) < 1e-3 * np.maximum(np.abs(y_ref), 1.0))
    # the oracle accumulates exactly like dot_row (serial f32): bit-identical here
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))


def test_quant_matvec_f32(orc):   # quant.rs:972-988
    rows, cols = 4, 8
    w = np.arange(rows * cols, dtype=np.float32)
    y = orc.quant_matvec(w.view(np.uint8), orc.F32, rows, cols, np.ones(cols, np.float32))
    for r in range(rows):
        assert abs(y[r] - sum(range(r * cols, (r + 1) * cols))) < 1e-4


def test_quant_matvec_f16(orc):   # quant.rs:991-1010
    rows, cols = 2, 4
    w = b"".join(f16b(orc, float(i)) for i in range(rows * cols))
    y = orc.quant_matvec(w, orc.F16, rows, cols, np.full(cols, 2.0, np.float32))
    for r in range(rows):
        assert abs(y[r] - sum(2.0 * i for i in range(r * cols, (r + 1) * cols))) < 1e-4


def test_quant_matvec_dim_mismatch(orc):   # quant.rs:1013-1022
    with pytest.raises(orc.OracleError) as e:
        orc.quant_matvec(bytes(16), orc.Q4_0, 1, 32, np.ones(16, np.float32), y_len=1)
    assert e.value.status == orc.ERR_DEQUANT and e.value.expected == 32 and e.value.actual == 16


# ---- src/infer/ops.rs tests ----------------------------------------------------
def test_matvec(orc):   # ops.rs:376-404
    y = orc.matvec([1, 2, 3, 4, 5, 6], 2, 3, [1, 1, 1], b=[10, 20])
    assert abs(y[0] - 16) < 1e-6 and abs(y[1] - 35) < 1e-6
    y = orc.matvec([1, 0, 0, 1], 2, 2, [3, 7])
    assert abs(y[0] - 3) < 1e-6 and abs(y[1] - 7) < 1e-6
    with pytest.raises(orc.OracleError):
        orc.matvec([1.0] * 4, 2, 3, [1, 1, 1])


def test_matmul(orc):   # ops.rs:406-417, :566-581
    c = orc.matmul([1, 2, 3, 4], 2, 2, [5, 6, 7, 8], 2)
    assert np.allclose(c, [19, 22, 43, 50], atol=1e-5)
    c = orc.matmul([1, 2, 3, 4, 5, 6], 3, 2, [7, 8, 9, 10, 11, 12], 3)
    assert np.allclose(c, [27, 30, 33, 61, 68, 75, 95, 106, 117], atol=1e-5)


def test_silu(orc):   # ops.rs:419-442
    x = orc.silu([0.0, 1.0, -1.0, 10.0])
    e = np.float32(math.exp(-1.0))
    assert abs(x[0]) < 1e-6
    assert abs(x[1] - 1.0 / (1.0 + e)) < 1e-5
    assert abs(x[2] - (-1.0) / (1.0 + math.exp(1.0))) < 1e-5
    assert abs(x[3] - 10.0 / (1.0 + math.exp(-10.0))) < 1e-5
    x = orc.silu([100.0, -100.0, 1000.0, -1000.0, -1e10])
    assert np.all(np.isfinite(x)) and abs(x[1]) < 1e-30 and abs(x[0] - 100.0) < 1e-3


def test_gelu(orc):   # ops.rs:444-450
    x = orc.gelu([0.0, 1.0])
    assert abs(x[0]) < 1e-6 and abs(x[1] - 0.8413) < 1e-3


def test_rmsnorm(orc):   # ops.rs:452-473
    scale = np.float32(math.sqrt(1.0 / (7.5 + 1e-6)))
    x = orc.rmsnorm([1, 2, 3, 4], [1, 1, 1, 1])
    assert abs(x[0] - scale) < 1e-6 and abs(x[3] - 4 * scale) < 1e-6
    x = orc.rmsnorm([1, 2, 3, 4], [2, 1, 1, 1])
    assert abs(x[0] - 2 * scale) < 1e-6 and abs(x[1] - 2 * scale) < 1e-6


def test_layernorm(orc):   # ops.rs:475-489
    x = orc.layernorm([1, 2, 3, 4], [1] * 4, [0] * 4)
    inv = 1.0 / math.sqrt(1.25 + 1e-6)
    assert abs(x[0] - (1 - 2.5) * inv) < 1e-5 and abs(x[3] - (4 - 2.5) * inv) < 1e-5


def test_softmax(orc):   # ops.rs:491-507, :583-591
    x = orc.softmax([1.0, 2.0, 3.0])
    assert abs(float(x.sum()) - 1.0) < 1e-6 and x[2] > x[1] > x[0]
    e = [math.exp(v - 3.0) for v in (1.0, 2.0, 3.0)]
    assert abs(x[0] - e[0] / sum(e)) < 1e-6 and abs(x[2] - e[2] / sum(e)) < 1e-6
    x = orc.softmax([1000.0, 1001.0, 1002.0])
    assert abs(float(x.sum()) - 1.0) < 1e-6 and np.all(np.isfinite(x))


def test_rope_basic(orc):   # ops.rs:509-539
    x = orc.rope([1, 0, 0, 1, 1, 0, 0, 1], [0, 1], [1.0, 0.001])
    assert np.allclose(x[:4], [1, 0, 0, 1], atol=1e-6)
    s0, c0 = math.sin(1.0), math.cos(1.0)
    s1, c1 = math.sin(0.001), math.cos(0.001)
    assert abs(x[4] - c0) < 1e-6 and abs(x[5] + s1) < 1e-6
    assert abs(x[6] - s0) < 1e-6 and abs(x[7] - c1) < 1e-6


def test_rope_freqs(orc):   # ops.rs:541-553
    f = orc.rope_freqs(8, 10000.0, 5)
    assert f.shape == (5, 4) and np.all(np.abs(f[0]) < 1e-6)
    assert abs(f[1][0] - 1.0) < 1e-6 and abs(f[1][1] - 1.0 / 10000.0 ** 0.25) < 1e-6


# ---- src/infer/model/llama.rs and src/infer/cache.rs tests --------------------
def test_inv_freq(orc):   # llama.rs:909-915
    inv = orc.build_inv_freq(8, 10000.0)
    assert inv.size == 4 and abs(inv[0] - 1.0) < 1e-6


def test_forward_runs(orc):   # llama.rs:788-899
    m = orc.Model(forward_runs_hp(), forward_runs_tensors())
    logits = m.forward([1, 0], [0, 1])
    assert logits.size == 8 and np.all(np.isfinite(logits))


def test_cache_semantics(orc):   # cache.rs:148-238 through the model's cache
    m = orc.Model(forward_runs_hp(), forward_runs_tensors())
    assert m.cache_len() == 0
    m.cache_append(0, np.full(2, 0.1), np.full(2, 0.2))
    m.cache_append(0, np.full(2, 0.3), np.full(2, 0.4))
    assert m.cache_len() == 2
    k, v = m.cache_read(0)
    assert np.allclose(k, [0.1, 0.1, 0.3, 0.3]) and np.allclose(v, [0.2, 0.2, 0.4, 0.4])
    m.truncate(1)
    assert m.cache_len() == 1
    m.truncate(5)   # truncate never grows
    assert m.cache_len() == 1
    m.reset_cache()
    assert m.cache_len() == 0


def test_forward_appends_cache(orc):   # llama.rs:473-475: one K/V row per token and layer
    m = orc.Model(forward_runs_hp(), forward_runs_tensors())
    m.forward([1, 0], [0, 1])
    assert m.cache_len() == 2
    m.forward([2], [2])
    assert m.cache_len() == 3


def test_empty_input(orc):   # llama.rs:277-280
    m = orc.Model(forward_runs_hp(), forward_runs_tensors())
    with pytest.raises(orc.OracleError) as e:
        m.forward([], [])
    assert e.value.status == orc.ERR_INFERENCE


# ---- tests/inference.rs --------------------------------------------------------
def test_min_llama_generates_max_tokens(orc):   # inference.rs:275-296 (eos outside the vocabulary)
    m = orc.Model(min_llama_hp(), min_llama_tensors())
    ids = m.generate_greedy([0, 0, 1], 5, eos=255)
    assert len(ids) == 5 and all(i < 8 for i in ids)
    # all logits tie at 0.0 in this model; the greedy sampler keeps the LAST maximum
    assert ids == [7, 7, 7, 7, 7]


def test_min_llama_eos_stops(orc):   # inference.rs:229-272 (eos = 7 is sampled first)
    m = orc.Model(min_llama_hp(), min_llama_tensors())
    assert m.generate_greedy([0, 0, 1], 4, eos=7) == []
    assert m.cache_len() == 3


def test_min_llama_reproducible(orc):   # inference.rs:299-308
    a = orc.Model(min_llama_hp(), min_llama_tensors()).generate_greedy([0], 8, eos=255)
    b = orc.Model(min_llama_hp(), min_llama_tensors()).generate_greedy([0], 8, eos=255)
    assert a == b


def test_q4_0_roundtrip(orc):   # inference.rs:311-357
    d = orc.f32_to_f16(0.5)
    b1 = bytearray(18); b1[0:2] = struct.pack("<H", d); b1[2:] = bytes([0x88]) * 16
    out1 = orc.dequantize(bytes(b1), orc.Q4_0, 32)
    assert np.all(out1 == 0.0)
    b2 = bytearray(18); b2[0:2] = struct.pack("<H", d)
    for i in range(16):
        b2[2 + i] = 0x00 if i % 2 == 0 else 0xFF
    out2 = orc.dequantize(bytes(b2), orc.Q4_0, 32)
    for i, v in enumerate(out2):
        q = -8.0 if (i // 2) % 2 == 0 else 7.0
        assert abs(v - 0.5 * q) < 1e-5
    out3 = orc.dequantize(bytes(b1) + bytes(b2), orc.Q4_0, 64)
    assert out3.size == 64 and np.all(out3[:32] == 0.0) and np.all(np.isfinite(out3))


# ---- model/llama.rs:656-710 physical-span re-inference ----------------------------
def test_infer_k_quant_dtype(orc):
    n = 4096 * 4096
    # padded Q4_0 (18 B / 32) re-read as Q4_K because 18 * 8 = 144
    assert orc.infer_k_quant_dtype(n // 32 * 18, n, orc.Q4_0) == orc.Q4_K
    assert orc.infer_k_quant_dtype(n // 256 * 176, n, orc.Q4_K) == orc.Q5_K
    assert orc.infer_k_quant_dtype(n // 256 * 114, n, orc.Q3_K_S) == orc.Q3_K_M
    # marked Q5_1 holding 210 B / 256: re-read as Q6_K only while span % blocks <= 256
    assert orc.infer_k_quant_dtype(210, 256, orc.Q5_1) == orc.Q6_K
    assert orc.infer_k_quant_dtype(n // 256 * 210, n, orc.Q5_1) is None
    assert orc.infer_k_quant_dtype(123, n, orc.F32) is None
    assert orc.infer_k_quant_dtype(n // 32 * 20, n, orc.Q4_1) is None   # 160 B / 256 not in the table


# ---- sampler.rs:86-186 restatement (orc_sample), checked on CPU --------------
def test_oracle_sampler_basics(orc):
    import numpy as np
    lg = np.array([1.0, 3.0, 2.0, 3.0, -1.0], np.float32)
    assert orc.sample(lg, dict(temperature=0.0, repeat_penalty=1.0)) == 3          # greedy: the last maximum
    assert orc.sample(lg, dict(temperature=1.0, top_k=1, repeat_penalty=1.0), u=0.99) == 1   # stable sort: index 1 first
    # the penalty divides a positive logit: 3 / 2 < 2, so index 2 leads
    assert orc.sample(lg, dict(temperature=0.0, repeat_penalty=2.0), seen=[1, 3]) == 2
    # u walks the sorted candidates: small u -> the most probable, u near 1 -> the last kept
    cfg = dict(temperature=1.0, top_k=3, top_p=1.0, repeat_penalty=1.0)
    assert orc.sample(lg, cfg, u=0.0) == 1 and orc.sample(lg, cfg, u=0.999) == 2
    ids = [orc.sample(lg, cfg, u=u) for u in np.linspace(0, 0.999, 200)]
    assert ids == sorted(ids, key=[1, 3, 2].index)                                 # monotone in u
    # top-p 0.5 keeps the top two (equal mass 0.42 each): never index 2
    assert all(orc.sample(lg, dict(top_k=0, top_p=0.5, repeat_penalty=1.0), u=u) in (1, 3) for u in np.linspace(0, 0.99, 50))
    # min-p 0.9 keeps only probabilities within 90 % of the top: indices 1 and 3
    assert all(orc.sample(lg, dict(top_k=0, top_p=1.0, min_p=0.9, repeat_penalty=1.0), u=u) in (1, 3)
               for u in np.linspace(0, 0.99, 50))


def test_oracle_sampler_reference_unit_tests(orc):   # sampler.rs:230-327, over a sweep of uniform draws
    import numpy as np
    us = [float(u) for u in np.linspace(0.0, 0.999, 41)]
    greedy = dict(temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.0)
    assert orc.sample(np.array([1.0, 5.0, 3.0, 2.0], np.float32), greedy) == 1          # test_greedy / temperature 0
    top_k2 = dict(temperature=1.0, top_k=2, top_p=1.0, repeat_penalty=1.0)
    lg = np.array([9.0, 10.0, -100.0, -100.0], np.float32)
    assert {orc.sample(lg, top_k2, u=u) for u in us} <= {0, 1}                         # test_top_k
    top_p = dict(temperature=1.0, top_k=100, top_p=0.5, repeat_penalty=1.0)
    assert {orc.sample(np.array([10.0, 9.0, -100.0, -100.0], np.float32), top_p, u=u) for u in us} <= {0, 1}   # test_top_p
    pen = dict(temperature=0.0, top_k=40, top_p=1.0, min_p=0.0, repeat_penalty=10.0)
    assert orc.sample(np.array([5.0, 5.0], np.float32), pen, seen=[0]) == 1            # test_repeat_penalty
    min_p = dict(temperature=1.0, top_k=100, top_p=1.0, min_p=0.5, repeat_penalty=1.0)
    assert {orc.sample(np.array([10.0, 0.0, -100.0], np.float32), min_p, u=u) for u in us} == {0}   # test_min_p
    ramp = (np.arange(100) * 0.1).astype(np.float32)
    cfg = dict(temperature=1.0, top_k=40, top_p=0.95, repeat_penalty=1.0)
    assert all(orc.sample(ramp, cfg, u=u) == orc.sample(ramp, cfg, u=u) for u in us)  # test_deterministic_with_seed
    lg50 = (np.arange(50) * 0.5 - 12.0).astype(np.float32)
    cfg = dict(temperature=0.8, top_k=20, top_p=0.9, repeat_penalty=1.0)
    seen = []
    for u in us[:20]:                                                                 # test_sample_valid_range
        tid = orc.sample(lg50, cfg, seen, u=u)
        assert 0 <= tid < 50
        seen.append(tid)

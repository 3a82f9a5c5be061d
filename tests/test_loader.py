"""The GGUF loader (host side, CPU): header / KV / tensor-info parsing, alignment,
tensor bytes, physical spans, HParams, tensor-name resolution and the
physical-span dtype re-inference of dequant_tensor_physical (llama.rs:719-768),
checked against the oracle's restatement of infer_k_quant_dtype."""
import struct

import numpy as np
import pytest

import gguf_cuda as ggc
from gguf_cuda import loader, synth
from gguf_cuda.loader import (T_ARR, T_BOOL, T_F32, T_F64, T_I8, T_I16, T_I32, T_I64, T_STR, T_U8, T_U16, T_U32,
                              T_U64)

Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K, F32 = 2, 6, 8, 12, 13, 14, 0
TINY = dict(vocab_size=100, embed_dim=64, n_heads=4, n_kv_heads=2, ffn_dim=128, n_layers=2, rope_freq_base=1e4,
            qkv_bias=True, weights="q8_0_normal")


def blocks(dt, n, seed=0):
    return synth.random_blocks(dt, n, synth.rng_for(seed, dt, n))


def test_round_trip_kv_types_tensors_and_alignment(tmp_path):
    kv = [("general.architecture", T_STR, "llama"), ("a.u8", T_U8, 200), ("a.i8", T_I8, -5), ("a.u16", T_U16, 65000),
          ("a.i16", T_I16, -300), ("a.u32", T_U32, 4_000_000_000), ("a.i32", T_I32, -7), ("a.f32", T_F32, 0.5),
          ("a.bool", T_BOOL, True), ("a.u64", T_U64, 2**40), ("a.i64", T_I64, -2**40), ("a.f64", T_F64, 1e-300),
          ("a.arr", T_ARR, (T_I32, [1, -2, 3])), ("a.strs", T_ARR, (T_STR, ["x", "yz"])),
          ("general.alignment", T_U32, 64)]
    t1 = blocks(Q4_K, 512)
    t2 = np.arange(10, dtype=np.float32)
    p = tmp_path / "m.gguf"
    loader.write_gguf(p, kv, [("w", [256, 2], Q4_K, t1), ("b", [10], F32, t2)], alignment=64)
    f = loader.GgufFile.open(p)
    assert f.version == 3 and f.alignment == 64 and f.data_offset % 64 == 0
    for key, ty, val in kv:
        want = list(val[1]) if ty == T_ARR else val
        assert f.kv[key] == pytest.approx(want) if ty in (T_F32, T_F64) else f.kv[key] == want, key
    w, b = f.find_tensor("w"), f.find_tensor("b")
    assert w.shape == [256, 2] and w.dtype == Q4_K and w.offset == 0 and b.offset % 64 == 0
    assert np.array_equal(f.tensor_data(w), t1) and np.array_equal(f.tensor_data(b).view(np.float32), t2)
    assert f.tensor_physical_span(w) == b.offset                       # to the next tensor
    assert f.tensor_physical_span(b) == f.file_size - f.data_offset - b.offset   # last: to the file end


def test_format_errors(tmp_path):
    p = tmp_path / "m.gguf"
    loader.write_gguf(p, [("general.architecture", T_STR, "llama")], [("b", [4], F32, np.zeros(4, np.float32))])
    raw = bytearray(p.read_bytes())
    bad = bytearray(raw)
    bad[0] = ord("X")
    with pytest.raises(loader.GgufFormatError, match="magic"):
        loader.GgufFile(memoryview(bytes(bad)))
    bad = bytearray(raw)
    bad[4:8] = struct.pack("<I", 2)
    with pytest.raises(loader.GgufFormatError, match="version"):
        loader.GgufFile(memoryview(bytes(bad)))
    full = loader.GgufFile(memoryview(bytes(raw)))
    f = loader.GgufFile(memoryview(bytes(raw[: full.data_offset + 8])))   # data cut short
    with pytest.raises(loader.GgufFormatError, match="past the end"):
        f.tensor_data(f.find_tensor("b"))
    with pytest.raises(loader.GgufFormatError):
        loader.GgufFile(memoryview(bytes(raw[:20])))                 # header cut short


def _header(n_tensors, n_kv):
    return struct.pack("<IIqq", loader.GGUF_MAGIC, 3, n_tensors, n_kv)


def _gstr(b):
    return struct.pack("<Q", len(b)) + b


def _open(raw):
    return loader.GgufFile(memoryview(bytes(raw)))


def test_reader_edge_cases():
    """The reader cases of the reference's tests/parse_buffer.rs, on byte buffers."""
    for raw in (b"", b"\x47"):                                           # empty, one byte
        with pytest.raises(loader.GgufFormatError):
            _open(raw)
    f = _open(_header(0, 0))                                              # header only parses
    assert f.kv == {} and f.tensors == []
    with pytest.raises(loader.GgufFormatError, match="past the end"):      # 1 KV claimed, none there
        _open(_header(0, 1))
    big = _gstr(b"big") + struct.pack("<iiQ", T_ARR, T_U8, 1000) + bytes([1, 2, 3, 4])
    with pytest.raises(loader.GgufFormatError, match="past the end"):      # array count past the data
        _open(_header(0, 1) + big)
    nested = _gstr(b"nested") + struct.pack("<iiQ", T_ARR, T_ARR, 0)
    with pytest.raises(loader.GgufFormatError, match="element type 9"):    # arrays of arrays
        _open(_header(0, 1) + nested)
    bad = _gstr(b"bad") + struct.pack("<i", T_STR) + _gstr(bytes([0xFF, 0xFE, 0xFD]))
    with pytest.raises(loader.GgufFormatError, match="UTF-8"):
        _open(_header(0, 1) + bad)

    def tensor(name, dims, dtype, offset=0):
        return _gstr(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}q", *dims) + \
            struct.pack("<iQ", dtype, offset)

    with pytest.raises(loader.GgufFormatError, match="negative"):
        _open(_header(1, 0) + tensor(b"neg", [-5, 3], F32))
    f = _open(_header(1, 0) + tensor(b"z", [2, 2], 99))                  # unknown dtype: parses ...
    assert f.tensors[0].dtype == 99
    with pytest.raises(ggc.InferenceError, match="unknown dtype 99"):    # ... and fails when sized (tensor.rs:64-80)
        f.tensors[0].data_size()
    kvs = b"".join(_gstr(k) + struct.pack("<iI", T_U32, i) for i, k in enumerate([b"first", b"second", b"third"]))
    assert list(_open(_header(0, 3) + kvs).kv) == ["first", "second", "third"]   # KV order kept
    one = tensor(b"a", [10], F32)
    assert _open(_header(1, 0) + one + bytes(64)).alignment == 32        # default alignment
    al = _gstr(b"general.alignment") + struct.pack("<iI", T_U32, 16)
    f = _open(_header(1, 1) + al + one + bytes(64))
    assert f.alignment == 16 and f.data_offset % 16 == 0 and f.data_offset <= f.file_size


def test_reader_counts_dims_and_alignment():
    """The parser cases of src/file.rs tests: counts, dimension limits, alignment 0."""
    for nt, nk in ((0, -1), (-5, 0), (0, 1_000_000)):                    # negative, or beyond the file size
        with pytest.raises(loader.GgufFormatError, match="count"):
            _open(_header(nt, nk))

    def tensor(name, dims, dtype=F32):
        return _gstr(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}q", *dims) + \
            struct.pack("<iQ", dtype, 0)

    with pytest.raises(loader.GgufFormatError, match="9 dims"):
        _open(_header(1, 0) + tensor(b"t", [1] * 9))
    f = _open(_header(1, 0) + tensor(b"s", []))                          # a scalar: no dims, one element
    assert f.tensors[0].shape == [] and f.tensors[0].num_elements() == 1
    f = _open(_header(2, 0) + tensor(b"a", [2, 3, 4, 5, 6]) + tensor(b"b", list(range(1, 9))))
    assert f.tensors[0].shape == [2, 3, 4, 5, 6] and f.tensors[1].shape == list(range(1, 9))
    zero = _gstr(b"general.alignment") + struct.pack("<iI", T_U32, 0)
    assert _open(_header(0, 1) + zero).alignment == 32                   # alignment 0 falls back


def test_alignment_only_from_u32_and_first_occurrence_wins():
    """file.rs:166-174 takes general.alignment only from a U32 value and stops at
    the first such key; get / find_tensor return the first occurrence (file.rs:367-374)."""
    def tensor(name, dims, offset):
        return _gstr(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}q", *dims) + \
            struct.pack("<iQ", F32, offset)

    one = tensor(b"a", [10], 0)
    u64 = _gstr(b"general.alignment") + struct.pack("<iQ", T_U64, 64)
    assert _open(_header(1, 1) + u64 + one + bytes(128)).alignment == 32          # U64: ignored
    st = _gstr(b"general.alignment") + struct.pack("<i", T_STR) + _gstr(b"64")
    assert _open(_header(1, 1) + st + one + bytes(128)).alignment == 32           # string: ignored
    u32 = _gstr(b"general.alignment") + struct.pack("<iI", T_U32, 16)
    f = _open(_header(0, 2) + u64 + u32)                                           # the first key decides
    assert f.alignment == 32 and f.kv["general.alignment"] == 64
    dup = _gstr(b"k") + struct.pack("<iI", T_U32, 1) + _gstr(b"k") + struct.pack("<iI", T_U32, 2)
    assert _open(_header(0, 2) + dup).kv["k"] == 1
    f = _open(_header(2, 0) + tensor(b"w", [8], 0) + tensor(b"w", [8], 32) + bytes(128))
    assert f.find_tensor("w").offset == 0


def test_tensor_sizes():   # src/tensor.rs tests: element counts (saturating) and block data sizes
    T = loader.TensorInfo
    assert T("t", [0, 5], F32, 0).num_elements() == 0 and T("s", [], F32, 0).num_elements() == 1
    assert T("h", [loader.U64_MAX, 2], F32, 0).num_elements() == loader.U64_MAX
    assert T("h", [loader.U64_MAX // 2] * 2, F32, 0).num_elements() == loader.U64_MAX
    assert T("t", [4096], Q4_0, 0).data_size() == 128 * 18
    assert T("t", [1024], Q8_0, 0).data_size() == 32 * 34
    assert T("t", [4096, 4096], Q4_K, 0).data_size() == 65536 * 144
    assert T("t", [256], 15, 0).data_size() == 292                       # Q8_K
    with pytest.raises(ggc.InvalidTensorShape, match="multiple") as e:   # InvalidTensorShape {name, elements, block}
        T("bad", [33], Q4_0, 0).data_size()
    assert e.value.elements == 33 and e.value.block == 32


def test_open_errors_and_missing_ffn_length(tmp_path):
    """tests/from_reader_path.rs (missing path, empty file) and the missing-KV
    case of tests/inference.rs (no ffn_length: an error, not a crash)."""
    with pytest.raises(OSError):
        loader.GgufFile.open(tmp_path / "does-not-exist.gguf")
    empty = tmp_path / "empty.gguf"
    empty.write_bytes(b"")
    with pytest.raises(loader.GgufFormatError, match="empty"):
        loader.GgufFile.open(empty)
    p = tmp_path / "noffn.gguf"
    kv = [("general.architecture", T_STR, "llama"), ("general.alignment", T_U32, 32), ("llama.vocab_size", T_U32, 8),
          ("llama.embedding_length", T_U32, 4), ("llama.attention.head_count", T_U32, 2), ("llama.block_count", T_U32, 1)]
    loader.write_gguf(p, kv, [])
    with pytest.raises(loader.GgufFormatError, match="feed_forward_length"):
        loader.hparams(loader.GgufFile.open(p))


def test_hparams_keys_and_defaults(tmp_path):
    p = tmp_path / "q.gguf"
    kv = [("general.architecture", T_STR, "qwen2"), ("qwen2.embedding_length", T_U32, 64),
          ("qwen2.attention.head_count", T_U32, 4), ("qwen2.feed_forward_length", T_U32, 128),
          ("qwen2.block_count", T_U32, 1), ("qwen2.rope.freq_base", T_F32, 1e6)]
    loader.write_gguf(p, kv, [("token_embd.weight", [64, 77], F32, np.zeros(64 * 77, np.float32))])
    hp = loader.hparams(loader.GgufFile.open(p))
    assert hp == dict(arch="qwen2", vocab_size=77, embed_dim=64, n_heads=4, n_kv_heads=4, ffn_dim=128, n_layers=1,
                      rope_freq_base=1e6)
    p2 = tmp_path / "l.gguf"
    kv = [("general.architecture", T_STR, "llama"), ("llama.vocab_size", T_U32, 9), ("llama.embedding_length", T_U32, 8),
          ("llama.attention.head_count", T_U32, 2), ("llama.attention.head_count_kv", T_U32, 1),
          ("llama.ffn_length", T_U32, 16), ("llama.block_count", T_U32, 3)]
    loader.write_gguf(p2, kv, [("x", [1], F32, np.zeros(1, np.float32))])
    hp = loader.hparams(loader.GgufFile.open(p2))
    assert (hp["vocab_size"], hp["n_kv_heads"], hp["ffn_dim"], hp["rope_freq_base"]) == (9, 1, 16, 10000.0)
    p3 = tmp_path / "g.gguf"
    loader.write_gguf(p3, [("general.architecture", T_STR, "gpt2")], [("x", [1], F32, np.zeros(1, np.float32))])
    with pytest.raises(loader.GgufFormatError, match="unsupported architecture"):
        loader.hparams(loader.GgufFile.open(p3))


@pytest.mark.parametrize("marked,phys,pad,want", [
    (Q4_K, Q5_K, 0, Q5_K),     # marked Q4_K, 176 bytes / 256 elements: Q5_K (llama.rs:648-651)
    (Q4_0, Q4_0, 16, Q4_K),    # padded Q4_0: 18*8 = 144 bytes / 256 -> read as Q4_K (the reference's trap)
    (Q5_0, Q5_0, 16, Q5_K),    # padded Q5_0: 22*8 = 176 -> Q5_K
    (Q6_K, Q6_K, 0, Q6_K),     # consistent: kept
    (Q8_0, Q8_0, 0, Q8_0),
], ids=["q4k-marked-q5k-bytes", "q4_0-padded", "q5_0-padded", "q6k", "q8_0"])
def test_physical_dtype_reinference(ggc, orc, tmp_path, marked, phys, pad, want):
    n = 256 * 160                                   # 1280 32-blocks: padding < 1 byte per 8 blocks
    raw = blocks(phys, n, 3)
    p = tmp_path / "p.gguf"
    loader.write_gguf(p, [("general.architecture", T_STR, "llama")],
                      [("w", [256, 160], marked, raw), ("next", [8], F32, np.zeros(8, np.float32))], pad={"w": pad})
    f = loader.GgufFile.open(p)
    t = f.find_tensor("w")
    span = f.tensor_physical_span(t)
    got = loader.physical_tensor(f, t)
    assert got["dtype"] == want
    oracle_dt = orc.infer_k_quant_dtype(span, n, marked)
    if span != n // ggc.block_size(marked) * ggc.block_bytes(marked):
        assert (oracle_dt if oracle_dt is not None else marked) == want   # the oracle restatement agrees
    assert got["raw"].size == n // ggc.block_size(want) * ggc.block_bytes(want)
    assert np.array_equal(got["raw"], np.frombuffer(raw.tobytes()[: got["raw"].size], np.uint8)) or pad


def test_model_tensors_role_order_and_names(tmp_path):
    hp, ts = synth.make_model(TINY, seed=0)
    p = tmp_path / "m.gguf"
    loader.write_model_gguf(p, hp, ts)
    f = loader.GgufFile.open(p)
    hp2, ts2 = loader.model_tensors(f)
    for k in ("vocab_size", "embed_dim", "n_heads", "n_kv_heads", "ffn_dim", "n_layers"):
        assert hp2[k] == hp[k]
    assert len(ts2) == 3 + 12 * hp["n_layers"]
    assert ts2[3 + 1]["name"] == "blk.0.attn_q.weight" and ts2[3 + 12 + 11]["name"] == "blk.1.ffn_down.weight"
    for a, b in zip(ts, ts2):
        assert (a is None) == (b is None)
        if a is not None:
            assert a["dtype"] == b["dtype"] and np.array_equal(np.asarray(a["raw"]).view(np.uint8).ravel(), b["raw"])
    # optional biases absent -> None; a missing weight -> MissingTensor
    hp3, ts3 = synth.make_model(dict(TINY, qkv_bias=False), seed=0)
    loader.write_model_gguf(tmp_path / "nb.gguf", hp3, ts3)
    _, tb = loader.model_tensors(loader.GgufFile.open(tmp_path / "nb.gguf"))
    assert tb[3 + 2] is None and tb[3 + 4] is None and tb[3 + 6] is None
    ts3[3 + 12 + 7] = None                          # blk.1.attn_output
    loader.write_model_gguf(tmp_path / "miss.gguf", hp3, ts3)
    with pytest.raises(loader.MissingTensorError, match="llama.1.attn.wo"):
        loader.model_tensors(loader.GgufFile.open(tmp_path / "miss.gguf"))


def test_old_style_names_take_precedence(tmp_path):
    """LlamaModel::new tries `{arch}.N.attn.wq` before `blk.N.attn_q.weight`."""
    hp, ts = synth.make_model(dict(TINY, n_layers=1), seed=1)
    p = tmp_path / "m.gguf"
    loader.write_model_gguf(p, hp, ts)
    f = loader.GgufFile.open(p)
    old = f.find_tensor("blk.0.attn_q.weight")
    f._by_name["llama.0.attn.wq"] = f.find_tensor("blk.0.attn_k.weight")   # an old-style alias
    _, t2 = loader.model_tensors(f)
    assert t2[3 + 1]["name"] == "blk.0.attn_k.weight" and old is not None

"""GGUF files -> LlamaModel: the host side of the loader.

Mirrors the reference's file and model set-up path so that a real ``.gguf``
drops in:
  * ``GgufFile``: header, metadata KVs, tensor infos, ``general.alignment`` and
    the data offset (src/file.rs:72-190, version 3 only, magic "GGUF");
    ``tensor_data`` (file.rs:205-228) and ``tensor_physical_span`` (file.rs:242-268:
    the distance to the next tensor in offset order, the last one to file end).
  * ``hparams``: HParams::parse / parse_generic (src/infer/model/hparams.rs:47-142):
    ``{arch}.*`` keys, vocab from ``{arch}.vocab_size`` or token_embd's shape,
    ``ffn_length`` or ``feed_forward_length``, head_count_kv defaulting to
    head_count, ``attention.rope_freq_base`` or ``rope.freq_base`` (10000 default).
  * ``model_tensors``: the role order of ``ggc_model_create``, names resolved as
    LlamaModel::new does (old ``{arch}.N.attn.wq`` style first, then
    ``blk.N.attn_q.weight``; llama.rs:135-157), each tensor's bytes and dtype as
    dequant_tensor_physical chooses them (llama.rs:719-768): when the physical
    span differs from the marked dtype's size, the dtype is re-inferred from bytes
    per 256 elements (``ggc_infer_k_quant_dtype``, llama.rs:656-710) and the exact
    block bytes are taken from the physical span.
The file is memory-mapped; tensor bytes are views into the map.
"""
from __future__ import annotations

import mmap
import os
import struct
from pathlib import Path

import numpy as np

from . import _lib as L

GGUF_MAGIC = 0x46554747            # "GGUF", little-endian
GGUF_VERSION = 3
GGUF_DEFAULT_ALIGNMENT = 32
U64_MAX = (1 << 64) - 1

# metadata value types (src/types.rs:7-21)
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}


class GgufFormatError(ValueError):
    """A malformed or unsupported file (the reference's InvalidMagic /
    UnsupportedVersion / OutOfBounds / InvalidGgufType variants)."""


class MissingTensorError(GgufFormatError):
    """MissingTensor { name, kind: tensor } of LlamaModel::new (llama.rs:621-632)."""

    def __init__(self, name: str):
        super().__init__(f"MissingTensor {{ name: {name}, kind: tensor }}")
        self.name = name


class TensorInfo:
    __slots__ = ("name", "shape", "dtype", "offset")

    def __init__(self, name: str, shape: list, dtype: int, offset: int):
        self.name, self.shape, self.dtype, self.offset = name, shape, dtype, offset

    def num_elements(self) -> int:
        """Product of the dims, saturating at 2^64 - 1 (src/tensor.rs:18-22)."""
        n = 1
        for d in self.shape:
            n = min(n * d, U64_MAX)
        return n

    def data_size(self) -> int:
        """Bytes by the marked dtype's block structure (src/tensor.rs:64-80):
        InferenceError for an unknown dtype, InvalidTensorShape {name, elements,
        block} when the element count is not a multiple of the block size."""
        if self.dtype not in L.BLOCK:
            raise L.host_error(L.InferenceError, f"tensor {self.name}: unknown dtype {self.dtype}")
        bs, bb = L.BLOCK[self.dtype]
        n = self.num_elements()
        if n % bs:
            raise L.host_error(L.InvalidTensorShape, f"tensor {self.name}: {n} elements not a multiple of block {bs}",
                               elements=n, block=bs)
        return n // bs * bb


class _Cursor:
    def __init__(self, buf, pos: int = 0):
        self.buf, self.pos = buf, pos

    def take(self, fmt: str):
        size = struct.calcsize(fmt)
        if self.pos + size > len(self.buf):
            raise GgufFormatError(f"read of {size} bytes at {self.pos} past the end ({len(self.buf)})")
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += size
        return v

    def string(self) -> str:
        n = self.take("<Q")
        if self.pos + n > len(self.buf):
            raise GgufFormatError(f"string of {n} bytes at {self.pos} past the end")
        try:   # the reader rejects a string that is not UTF-8 (InvalidStringLength)
            s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8")
        except UnicodeDecodeError as e:
            raise GgufFormatError(f"invalid UTF-8 in the string of {n} bytes at {self.pos}") from e
        self.pos += n
        return s

    def value(self, ty: int):
        if ty in _SCALAR:
            return self.take(_SCALAR[ty])
        if ty == T_STR:
            return self.string()
        if ty == T_ARR:
            ety = self.take("<i")
            if ety not in _SCALAR and ety != T_STR:   # nested arrays and unknown types (InvalidArrayElemType)
                raise GgufFormatError(f"invalid array element type {ety}")
            n = self.take("<Q")
            # every element takes at least its scalar size (a string its 8-byte length)
            least = struct.calcsize(_SCALAR[ety]) if ety in _SCALAR else 8
            if n * least > len(self.buf) - self.pos:
                raise GgufFormatError(f"array of {n} elements at {self.pos} past the end ({len(self.buf)})")
            return [self.value(ety) for _ in range(n)]
        raise GgufFormatError(f"invalid metadata type {ty}")


def _align_up(v: int, a: int) -> int:
    return (v + a - 1) // a * a


class GgufFile:
    """A parsed GGUF file (memory-mapped)."""

    def __init__(self, buf, owner=None):
        self._buf = buf
        self._owner = owner
        c = _Cursor(buf)
        magic = c.take("<I")
        if magic != GGUF_MAGIC:
            raise GgufFormatError(f"invalid magic 0x{magic:08x}")
        self.version = c.take("<I")
        if self.version != GGUF_VERSION:
            raise GgufFormatError(f"unsupported version {self.version}")
        n_tensors = c.take("<q")
        n_kv = c.take("<q")
        if n_tensors < 0 or n_kv < 0:
            raise GgufFormatError("negative tensor or KV count")
        if n_kv > len(buf) or n_tensors > len(buf):   # every entry takes bytes: a corrupt count (InvalidCount)
            raise GgufFormatError(f"tensor count {n_tensors} or KV count {n_kv} exceeds the file size {len(buf)}")
        # lookups return the first occurrence of a key or tensor name, as
        # GgufFile::get / find_tensor do (file.rs:367-374)
        self.kv, self.kv_types = {}, {}
        for _ in range(n_kv):
            key = c.string()
            ty = c.take("<i")
            val = c.value(ty)
            if key not in self.kv:
                self.kv[key], self.kv_types[key] = val, ty
        self.tensors = []
        for _ in range(n_tensors):
            name = c.string()
            n_dims = c.take("<I")
            if n_dims > 8:
                raise GgufFormatError(f"tensor {name}: {n_dims} dims")
            shape = [c.take("<q") for _ in range(n_dims)]
            if any(d < 0 for d in shape):   # InvalidTensorDim
                raise GgufFormatError(f"tensor {name}: negative dimension in {shape}")
            dtype = c.take("<i")
            offset = c.take("<Q")
            self.tensors.append(TensorInfo(name, shape, dtype, offset))
        # general.alignment counts only as a U32 value, 0 meaning the default
        # (file.rs:166-174); any other type keeps the default
        self.alignment = GGUF_DEFAULT_ALIGNMENT
        if self.kv_types.get("general.alignment") == T_U32 and self.kv["general.alignment"]:
            self.alignment = int(self.kv["general.alignment"])
        self.data_offset = _align_up(c.pos, self.alignment)
        self.file_size = len(buf)
        self._by_name = {}
        for t in self.tensors:
            self._by_name.setdefault(t.name, t)
        self._sorted = sorted(t.offset for t in self.tensors)

    @classmethod
    def open(cls, path) -> "GgufFile":
        f = open(Path(path), "rb")
        try:
            if os.fstat(f.fileno()).st_size == 0:   # (mmap refuses an empty file)
                raise GgufFormatError(f"{path}: empty file")
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        finally:
            f.close()
        return cls(memoryview(mm), owner=mm)

    def find_tensor(self, name: str):
        return self._by_name.get(name)

    def architecture(self):
        return self.kv.get("general.architecture")

    def _slice(self, start: int, n: int) -> np.ndarray:
        end = start + n
        if end > self.file_size:
            raise GgufFormatError(f"tensor data [{start}, {end}) past the end of the file ({self.file_size})")
        return np.frombuffer(self._buf, dtype=np.uint8, count=n, offset=start)

    def tensor_data(self, t: TensorInfo) -> np.ndarray:
        return self._slice(self.data_offset + t.offset, t.data_size())

    def tensor_physical_span(self, t: TensorInfo) -> int:
        if not self.tensors:
            raise GgufFormatError("no tensors")
        i = int(np.searchsorted(self._sorted, t.offset))
        if i >= len(self._sorted) or self._sorted[i] != t.offset:
            raise GgufFormatError(f"tensor offset {t.offset} not found")
        if i + 1 < len(self._sorted):
            end = self._sorted[i + 1]
        else:
            end = max(self.file_size - self.data_offset, t.offset)
        return max(end - t.offset, 0)

    def tensor_data_physical(self, t: TensorInfo) -> np.ndarray:
        return self._slice(self.data_offset + t.offset, self.tensor_physical_span(t))


# ---- model set-up ---------------------------------------------------------------
def _u32_at(f: GgufFile, key: str) -> int:
    v = f.kv.get(key)
    if v is None or isinstance(v, (str, list)):
        raise GgufFormatError(f"missing or non-integer key {key}")
    return int(v)


def hparams(f: GgufFile) -> dict:
    """HParams::parse (hparams.rs:47-142) as the dict LlamaModel takes."""
    arch = f.architecture()
    if arch is None:
        raise GgufFormatError("missing general.architecture")
    if not (arch in ("llama", "qwen2", "mistral") or arch.startswith(("llama", "qwen2", "qwen3", "mistral"))):
        raise GgufFormatError(f"unsupported architecture {arch}")
    k = lambda s: f"{arch}.{s}"
    if k("vocab_size") in f.kv:
        vocab = _u32_at(f, k("vocab_size"))
    else:
        emb = f.find_tensor(f"{arch}.token_embd") or f.find_tensor("token_embd.weight")
        if emb is None:
            raise GgufFormatError("vocab_size: no KV and no token_embd tensor")
        if len(emb.shape) != 2:
            raise GgufFormatError(f"vocab_size: token_embd shape {emb.shape} is not [D, V]")
        vocab = int(emb.shape[1])
    embed = _u32_at(f, k("embedding_length"))
    heads = _u32_at(f, k("attention.head_count"))
    ffn = _u32_at(f, k("ffn_length")) if k("ffn_length") in f.kv else _u32_at(f, k("feed_forward_length"))
    layers = _u32_at(f, k("block_count"))
    kvh = f.kv.get(k("attention.head_count_kv"))
    kvh = int(kvh) if isinstance(kvh, (int, float)) and not isinstance(kvh, bool) else heads
    base = f.kv.get(k("attention.rope_freq_base"))
    if not isinstance(base, (int, float)) or isinstance(base, bool):
        base = f.kv.get(k("rope.freq_base"))
    if not isinstance(base, (int, float)) or isinstance(base, bool):
        base = 10000.0
    return dict(arch=arch, vocab_size=vocab, embed_dim=embed, n_heads=heads, n_kv_heads=kvh, ffn_dim=ffn,
                n_layers=layers, rope_freq_base=float(base))


def physical_tensor(f: GgufFile, t: TensorInfo) -> dict:
    """The bytes and dtype dequant_tensor_physical (llama.rs:719-768) would read."""
    n = t.num_elements()
    if t.dtype not in L.BLOCK:
        raise GgufFormatError(f"tensor {t.name}: unsupported dtype {t.dtype}")
    bs, bb = L.BLOCK[t.dtype]
    span = f.tensor_physical_span(t)
    expected = n // bs * bb
    dtype, physical = t.dtype, False
    if span != expected:
        inferred = L.lib().ggc_infer_k_quant_dtype(span, n, t.dtype)
        if inferred >= 0:
            dtype, physical = inferred, True
    if physical:
        dbs, dbb = L.BLOCK[dtype]
        raw = f.tensor_data_physical(t)[: n // dbs * dbb]
    else:
        raw = f.tensor_data(t)
    return {"raw": raw, "dtype": dtype, "n_elements": n, "name": t.name}


def _resolve(f: GgufFile, primary: str, fallback: str, required: bool = True):
    for name in (primary, fallback):
        t = f.find_tensor(name)
        if t is not None:
            return t
    if required:
        raise MissingTensorError(primary)
    return None


def model_tensors(f: GgufFile) -> tuple:
    """(hparams dict, tensors in ggc_model_create's role order)."""
    hp = hparams(f)
    p = hp["arch"]
    top = [_resolve(f, f"{p}.token_embd", "token_embd.weight"),
           _resolve(f, f"{p}.output_norm", "output_norm.weight"),
           _resolve(f, f"{p}.output", "output.weight")]
    out = [physical_tensor(f, t) for t in top]
    for l in range(hp["n_layers"]):
        names = [
            (f"{p}.{l}.attn_norm", f"blk.{l}.attn_norm.weight", True),
            (f"{p}.{l}.attn.wq", f"blk.{l}.attn_q.weight", True),
            (f"{p}.{l}.attn.b_q", f"blk.{l}.attn_q.bias", False),
            (f"{p}.{l}.attn.wk", f"blk.{l}.attn_k.weight", True),
            (f"{p}.{l}.attn.b_k", f"blk.{l}.attn_k.bias", False),
            (f"{p}.{l}.attn.wv", f"blk.{l}.attn_v.weight", True),
            (f"{p}.{l}.attn.b_v", f"blk.{l}.attn_v.bias", False),
            (f"{p}.{l}.attn.wo", f"blk.{l}.attn_output.weight", True),
            (f"{p}.{l}.ffn_norm", f"blk.{l}.ffn_norm.weight", True),
            (f"{p}.{l}.ffn.w1", f"blk.{l}.ffn_up.weight", True),
            (f"{p}.{l}.ffn.w2", f"blk.{l}.ffn_gate.weight", True),
            (f"{p}.{l}.ffn.w3", f"blk.{l}.ffn_down.weight", True),
        ]
        for primary, fallback, req in names:
            t = _resolve(f, primary, fallback, req)
            out.append(physical_tensor(f, t) if t is not None else None)
    return hp, out


# ---- writer (synthetic models, tests) -----------------------------------------------
def _pack_value(v, ty: int) -> bytes:
    if ty in _SCALAR:
        return struct.pack(_SCALAR[ty], v)
    if ty == T_STR:
        b = v.encode("utf-8")
        return struct.pack("<Q", len(b)) + b
    raise GgufFormatError(f"cannot write type {ty}")


def write_gguf(path, kv: list, tensors: list, alignment: int = GGUF_DEFAULT_ALIGNMENT, pad: dict | None = None):
    """Writes a version-3 GGUF file.  kv: [(key, type, value)] (arrays as
    (key, T_ARR, (elem_type, [values]))); tensors: [(name, shape, dtype, raw
    bytes)] in file order, each data start aligned; pad: {name: extra bytes}
    inserted after a tensor's data (as some files carry)."""
    pad = pad or {}
    head = bytearray()
    head += struct.pack("<IIqq", GGUF_MAGIC, GGUF_VERSION, len(tensors), len(kv))
    for key, ty, val in kv:
        head += _pack_value(key, T_STR) + struct.pack("<i", ty)
        if ty == T_ARR:
            ety, vals = val
            head += struct.pack("<iQ", ety, len(vals)) + b"".join(_pack_value(x, ety) for x in vals)
        else:
            head += _pack_value(val, ty)
    offsets, off = [], 0
    for name, shape, dtype, raw in tensors:
        offsets.append(off)
        off = _align_up(off + len(raw) + pad.get(name, 0), alignment)
    for (name, shape, dtype, raw), o in zip(tensors, offsets):
        head += _pack_value(name, T_STR) + struct.pack("<I", len(shape))
        head += b"".join(struct.pack("<q", d) for d in shape) + struct.pack("<iQ", dtype, o)
    data_offset = _align_up(len(head), alignment)
    with open(path, "wb") as fh:
        fh.write(head)
        fh.write(b"\0" * (data_offset - len(head)))
        pos = 0
        for (name, shape, dtype, raw), o in zip(tensors, offsets):
            fh.write(b"\0" * (o - pos))
            b = bytes(np.ascontiguousarray(raw).view(np.uint8))
            fh.write(b)
            pos = o + len(b)
        fh.write(b"\0" * (off - pos))


def write_model_gguf(path, hp: dict, tensors: list, alignment: int = GGUF_DEFAULT_ALIGNMENT, arch: str = "llama"):
    """A llama-architecture GGUF file from (hparams, tensors in ggc_model_create's
    role order), with the usual tensor names and `{arch}.*` keys (synthetic
    models as files)."""
    d, f_, v = hp["embed_dim"], hp["ffn_dim"], hp["vocab_size"]
    hd = d // hp["n_heads"]
    qd, kvd = hp["n_heads"] * hd, hp["n_kv_heads"] * hd
    kv = [("general.architecture", T_STR, arch),
          (f"{arch}.vocab_size", T_U32, v),
          (f"{arch}.embedding_length", T_U32, d),
          (f"{arch}.attention.head_count", T_U32, hp["n_heads"]),
          (f"{arch}.attention.head_count_kv", T_U32, hp["n_kv_heads"]),
          (f"{arch}.feed_forward_length", T_U32, f_),
          (f"{arch}.block_count", T_U32, hp["n_layers"]),
          (f"{arch}.rope.freq_base", T_F32, float(hp["rope_freq_base"]))]
    if alignment != GGUF_DEFAULT_ALIGNMENT:
        kv.append(("general.alignment", T_U32, alignment))
    layer_roles = [("attn_norm.weight", [d]), ("attn_q.weight", [d, qd]), ("attn_q.bias", [qd]),
                   ("attn_k.weight", [d, kvd]), ("attn_k.bias", [kvd]), ("attn_v.weight", [d, kvd]),
                   ("attn_v.bias", [kvd]), ("attn_output.weight", [qd, d]), ("ffn_norm.weight", [d]),
                   ("ffn_up.weight", [d, f_]), ("ffn_gate.weight", [d, f_]), ("ffn_down.weight", [f_, d])]
    names = [("token_embd.weight", [d, v]), ("output_norm.weight", [d]), ("output.weight", [d, v])]
    for l in range(hp["n_layers"]):
        names += [(f"blk.{l}.{r}", s) for r, s in layer_roles]
    out = []
    for (name, shape), t in zip(names, tensors):
        if t is not None:
            out.append((name, shape, int(t["dtype"]), np.asarray(t["raw"])))
    write_gguf(path, kv, out, alignment=alignment)

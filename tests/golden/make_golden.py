"""Generates tests/golden/dequant_golden.npz from the reference's own Python
dequantisers (tools/gguf_forward_check.py in chaos-asimo/gguf-reader).

Run in a container where the reference is mounted (it is read, never copied):
    python tests/golden/make_golden.py /path/to/reference

That script computes each element in double precision from the exact f16/int
operands and rounds once to f32, which equals the Rust f32 result for Q5_0,
Q5_1, Q8_0, Q4_K, Q5_K, Q6_K and Q8_K (every product there is exact in f32 and
only the final add/sub rounds).  Its deq_q4_0 uses a wrong 6-byte block and is
not used; Q4_0/Q4_1/Q2_K/Q3_K are pinned by the reference's unit-test values in
tests/test_oracle_known_answers.py instead.

Block bytes are seeded random, with edge blocks appended: scale fields set to
+0, -0, the largest f16, an f16 subnormal, +inf and NaN.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if len(sys.argv) != 2:
    sys.exit("usage: make_golden.py /path/to/reference  (the gguf-reader checkout to read the tool from)")
REF = Path(sys.argv[1])

# GGUF ids and block geometry (src/types.rs)
FORMATS = {  # name: (gguf id, block elems, block bytes, f16 scale offsets, tool function)
    "Q5_0": (6, 32, 22, [0], "deq_q5_0"),
    "Q5_1": (7, 32, 24, [0, 2], "deq_q5_1"),
    "Q8_0": (8, 32, 34, [0], "deq_q8_0"),
    "Q4_K": (12, 256, 144, [0, 2], "deq_q4_k"),
    "Q5_K": (13, 256, 176, [0, 2], "deq_q5_k"),
    "Q6_K": (14, 256, 210, [208], "deq_q6_k"),
    "Q8_K": (15, 256, 292, [], "deq_q8_k"),
}
EDGE_F16 = [0x0000, 0x8000, 0x7BFF, 0x0001, 0x7C00, 0x7E00]


def load_tool():
    path = REF / "tools" / "gguf_forward_check.py"
    spec = importlib.util.spec_from_file_location("gguf_forward_check", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def blocks_for(name, rng, n_random=48):
    gid, bs, bb, offs, _ = FORMATS[name]
    raw = np.frombuffer(rng.bytes(n_random * bb), dtype=np.uint8).copy().reshape(n_random, bb)
    lo, hi = (1e-3, 1e-2) if bs == 32 else (1e-4, 1e-3)
    for off in offs:
        raw[:, off:off + 2] = rng.uniform(lo, hi, size=n_random).astype(np.float16).view(np.uint8).reshape(-1, 2)
    if name == "Q8_K":
        raw[:, 0:4] = rng.uniform(1e-4, 1e-3, size=n_random).astype(np.float32).view(np.uint8).reshape(-1, 4)
    edges = []
    for e in EDGE_F16:
        b = np.frombuffer(rng.bytes(bb), dtype=np.uint8).copy()
        if name == "Q8_K":
            b[0:4] = np.array([e], dtype=np.uint16).view(np.float16).astype(np.float32).view(np.uint8)
        for off in offs:
            b[off:off + 2] = np.array([e], dtype=np.uint16).view(np.uint8)
        edges.append(b)
    return np.concatenate([raw.reshape(-1), np.concatenate(edges)])


def main():
    tool = load_tool()
    rng = np.random.default_rng(20261201)
    out = {}
    for name, (gid, bs, bb, offs, fn) in FORMATS.items():
        raw = blocks_for(name, rng)
        with np.errstate(all="ignore"):
            vals = getattr(tool, fn)(bytes(raw))
        vals = np.asarray(vals, dtype=np.float32)
        assert vals.size == raw.size // bb * bs
        out[f"{name}_raw"] = raw
        out[f"{name}_out"] = vals
        out[f"{name}_id"] = np.array([gid])
    np.savez_compressed(HERE / "dequant_golden.npz", **out)
    print("wrote", HERE / "dequant_golden.npz", {k: v.shape for k, v in out.items() if k.endswith("_out")})


if __name__ == "__main__":
    main()

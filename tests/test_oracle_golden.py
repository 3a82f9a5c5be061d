"""The oracle against golden vectors made by the reference's own Python
dequantisers (tests/golden/make_golden.py): bit-exact, NaN matching NaN."""
from pathlib import Path

import numpy as np
import pytest

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "dequant_golden.npz")
NAMES = sorted({k[:-4] for k in GOLDEN.files if k.endswith("_raw")})


def same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return np.all(nan | (a.view(np.uint32) == b.view(np.uint32)))


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_tool(orc, name):
    raw = GOLDEN[f"{name}_raw"]
    want = GOLDEN[f"{name}_out"]
    dt = int(GOLDEN[f"{name}_id"][0])
    got = orc.dequantize(raw, dt, want.size)
    assert same_bits(got, want)

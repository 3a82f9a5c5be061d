"""The bench's CPU-side legs on small cases (no GPU): the oracle's format sweep
that sits beside the GPU sweep in cpu_baseline, and the decode positions the
timed steps use."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import bench


def test_cpu_matvec_sweep_small():
    r = bench.cpu_matvec_sweep([2, 12, 1], [(64, 512), (16, 1024)], reps=1)
    assert r["threads"] >= 1 and r["seconds"] > 0
    assert set(r["entries"]) == {"Q4_0_64x512", "Q4_0_16x1024", "Q4_K_64x512", "Q4_K_16x1024",
                                 "F16_64x512", "F16_16x1024"}
    for e in r["entries"].values():
        assert e["ms"] > 0 and e["gbs"] > 0


def test_decode_bench_ends_at_the_context():
    """Planted rows P, one forward at position P, max(W - 1, 0) warm-up steps and
    K timed steps fill the cache to exactly C, so the last step attends to C rows."""
    for C, W, K in [(2048, 8, 128), (2048, 0, 16), (512, 1, 64), (2048, 5, 20)]:
        P = bench.planted_rows(C, W, K)
        assert P >= 1 and P + 1 + max(W - 1, 0) + K == C

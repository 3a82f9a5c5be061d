"""Tensor-parallel shard plan (ggc_tp_plan) on the CPU: the Megatron split of
one layer -- q/k/v rows by head, ffn rows on ffn_down block boundaries with the
remainder on the lowest ranks -- and, with two gloo ranks, that the column
slices of attn_output / ffn_down give partial matvecs (oracle) whose all-reduced
sum is the full product.
"""
import os
import socket

import numpy as np
import pytest

from gguf_cuda import synth

LLAMA2 = dict(vocab_size=32000, embed_dim=4096, n_heads=32, n_kv_heads=32, ffn_dim=11008, n_layers=32,
              rope_freq_base=1e4)
LLAMA3 = dict(LLAMA2, n_kv_heads=8, ffn_dim=14336, vocab_size=128256, rope_freq_base=5e5)
QWEN = dict(vocab_size=151936, embed_dim=896, n_heads=14, n_kv_heads=2, ffn_dim=4864, n_layers=24,
            rope_freq_base=1e6)
Q4_0, Q8_0, Q4_K, Q6_K, F32 = 2, 8, 12, 14, 0


def plans(ggc, hp, wo, down, world):
    return [ggc.tp_plan(hp, wo, down, r, world) for r in range(world)]


def assert_partition(ranges, total):
    pos = 0
    for first, count in ranges:
        assert first == pos and count > 0
        pos += count
    assert pos == total


@pytest.mark.parametrize("hp,wo,down", [(LLAMA2, Q4_K, Q6_K), (LLAMA2, Q4_K, Q4_K), (LLAMA3, Q4_0, Q4_0),
                                        (LLAMA3, Q8_0, Q8_0)], ids=["llama2-q6k-down", "llama2-q4k", "llama3-q4_0",
                                                                     "llama3-q8_0"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_partitions_every_dimension(ggc, hp, wo, down, world):
    ps = plans(ggc, hp, wo, down, world)
    assert_partition([p["heads"] for p in ps], hp["n_heads"])
    assert_partition([p["kv_heads"] for p in ps], hp["n_kv_heads"])
    assert_partition([p["ffn"] for p in ps], hp["ffn_dim"])
    bs = ggc.block_size(down)
    for p in ps:
        first, count = p["ffn"]
        assert first % bs == 0 and count % bs == 0
        assert p["heads"][1] == hp["n_heads"] // world
        # GQA: the rank's q heads map onto its own kv heads
        g = hp["n_heads"] // hp["n_kv_heads"]
        assert p["heads"][0] // g == p["kv_heads"][0]


def test_llama2_ffn_split_is_uneven_in_super_blocks(ggc):
    # 11008 = 43 super-blocks of 256: 22/21, 11/11/11/10, 6,6,6,5,5,5,5,5
    for world, want in [(2, [22, 21]), (4, [11, 11, 11, 10]), (8, [6, 6, 6, 5, 5, 5, 5, 5])]:
        got = [p["ffn"][1] // 256 for p in plans(ggc, LLAMA2, Q4_K, Q6_K, world)]
        assert got == want


def test_plan_errors(ggc):
    with pytest.raises(ggc.InvalidArgument, match="does not divide"):
        ggc.tp_plan(LLAMA2, Q4_K, Q4_K, 0, 3)
    with pytest.raises(ggc.InvalidArgument, match="does not divide"):
        ggc.tp_plan(QWEN, Q8_0, Q8_0, 0, 4)              # 2 kv heads
    assert ggc.tp_plan(QWEN, Q8_0, Q8_0, 1, 2)["heads"] == (7, 7)
    with pytest.raises(ggc.InvalidArgument, match="whole"):
        # 7 heads x 64 = 448 attn_output columns per rank: not whole 256-element super-blocks
        ggc.tp_plan(QWEN, Q4_K, Q8_0, 0, 2)
    with pytest.raises(ggc.InvalidArgument, match="rank"):
        ggc.tp_plan(LLAMA2, Q4_K, Q4_K, 2, 2)
    tiny = dict(LLAMA2, ffn_dim=512)                     # 2 super-blocks for 4 ranks
    with pytest.raises(ggc.InvalidArgument, match="blocks for 4 ranks"):
        ggc.tp_plan(tiny, Q4_K, Q4_K, 0, 4)
    with pytest.raises(ggc.InvalidTensorShape):
        ggc.tp_plan(dict(LLAMA2, ffn_dim=11000), Q4_K, Q4_K, 0, 2)


# ---- two gloo ranks: partial products of the column shards sum to the full one
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cols(raw, dtype, rows, cols, c0, n, bs, bb):
    """Columns [c0, c0 + n) of a raw block matrix (whole blocks)."""
    return np.ascontiguousarray(raw.reshape(rows, cols // bs * bb)[:, c0 // bs * bb:(c0 + n) // bs * bb]).ravel()


def _gloo_rank(rank, world, port, out_q):
    import torch.distributed as dist
    import gguf_cuda as ggc
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch
        hp = dict(LLAMA2, embed_dim=1024, n_heads=8, n_kv_heads=8, ffn_dim=2816)   # 11 super-blocks: 6 + 5
        hd = hp["embed_dim"] // hp["n_heads"]
        errs = {}
        for name, dtype, rows, cols in [("attn_output", Q4_K, hp["embed_dim"], hp["embed_dim"]),
                                        ("ffn_down", Q6_K, hp["embed_dim"], hp["ffn_dim"])]:
            p = ggc.tp_plan(hp, Q4_K, dtype, rank, world)
            c0, n = (p["heads"][0] * hd, p["heads"][1] * hd) if name == "attn_output" else p["ffn"]
            rng = synth.rng_for(7, dtype, rows, cols)
            w = synth.random_blocks(dtype, rows * cols, rng)            # same bytes on every rank
            x = np.random.default_rng(1).normal(0, 1, cols).astype(np.float32)
            bs, bb = ggc.block_size(dtype), ggc.block_bytes(dtype)
            part = oracle.quant_matvec(_cols(w, dtype, rows, cols, c0, n, bs, bb), dtype, rows, n, x[c0:c0 + n])
            t = torch.from_numpy(part.astype(np.float64))
            dist.all_reduce(t)                                             # the exchange step
            spans = [None] * world
            dist.all_gather_object(spans, (int(c0), int(n)))
            if rank == 0:
                full = oracle.quant_matvec(w, dtype, rows, cols, x).astype(np.float64)
                rel = float(np.linalg.norm(t.numpy() - full) / np.linalg.norm(full))
                errs[name] = (rel, spans)
        out_q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_partial_sums_equal_full_product(ggc, orc):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=240) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    errs = res[0]
    for name, (rel, spans) in errs.items():
        assert rel <= 1e-6, (name, rel)
        total = 1024 if name == "attn_output" else 2816
        assert_partition(spans, total)
    assert errs["ffn_down"][1] == [(0, 1536), (1536, 1280)]


def _gloo_withholding_rank(rank, world, port, out_q):
    """Rank 1 computes its shard but never joins the all-reduce (a rank lost
    between steps); rank 0's collective must end with an error after the short
    process-group timeout instead of waiting forever."""
    import os
    import time
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    partial = torch.ones(64)
    if rank == 1:
        time.sleep(8)          # alive, but withholding its partial sum
        out_q.put((rank, "withheld"))
        return
    t0 = time.perf_counter()
    try:
        dist.all_reduce(partial)
        out_q.put((rank, "completed"))
    except Exception as e:   # the timeout surfaces as an exception on the waiting rank
        out_q.put((rank, f"error after {time.perf_counter() - t0:.1f} s: {type(e).__name__}"))


def test_gloo_rank_withholding_its_partial_ends_the_others_collective_with_an_error():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_withholding_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=60) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res[1] == "withheld"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2]) < 8.0

#!/usr/bin/env python3
"""Benchmark of the quantized decode hot path on B200.

Metric: decode tokens/s of a Llama-2-7B-shaped model in the Q4_K_M mix (Q4_K,
Q6_K for the output head and attn_v / ffn_down of even layers, f32 norms), batch
1, at context 2048 (the KV cache is prefilled with planted K/V rows so the K
timed steps end at 2048), f32 KV cache as the reference keeps it.  Weights are
seeded synthetic blocks.

One step = one token through all 32 layers (greedy sample -> forward), run by the
device-side decode loop (one CUDA graph per token).  `value` is timed with CUDA
events on the library's stream with the weights resident in HBM; `e2e` times the
reference-facing C-ABI call LlamaModel::forward(host token) -> host logits per
token.  Per-step HBM traffic (~6 GB) is far above L2, so no explicit L2 flush.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) the ranks run ONE model tensor-parallel (default,
`--parallel tp`: q/k/v/up/gate rows and attn_output/ffn_down columns sharded,
NCCL all-reduce of the hidden state after attn_output and ffn_down; strong
scaling: `value` is that model's tokens/s) or, with `--parallel replicas`, one
independent replica per rank (weak scaling: `value` sums the replicas).
`--impl reference` times the CPU restatement of the reference's rayon path.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gguf-reader_b200"))

MODEL = "llama2-7b-q4_k_m"
METRIC = "decode tokens/s, Llama-7B-shape Q4_K; quant matvec HBM GB/s vs B200 peak"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=None, help="fewer layers (small profiling cases only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", choices=["tp", "replicas"], default="tp", help="multi-GPU mode (N > 1)")
    ap.add_argument("--prefill", type=int, default=512, help="prompt tokens of the prefill measurement (0: skip)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return FALLBACK_HBM_GBS, "fallback"


def traffic_record():
    p = ROOT / "profiles" / "roofline_traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def record(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (C++ restatement of the reference's rayon CPU path)
# ---------------------------------------------------------------------------
def cpu_decode_sample(hp, ts, ctx_len, steps, layer_counts=(2, 4)):
    """Per-token decode time of the oracle at context ctx_len, extrapolated to all
    layers from models holding the first 2 and 4 layers (same tensors)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    oracle.build()
    threads = oracle.get_threads()
    n_layers = hp["n_layers"]
    kvd = hp["n_kv_heads"] * (hp["embed_dim"] // hp["n_heads"])
    rng = np.random.default_rng(0)
    times = {}
    for L in layer_counts:
        h = dict(hp, n_layers=L)
        m = oracle.Model(h, ts[:3 + 12 * L])
        k = rng.normal(size=(ctx_len - 1) * kvd).astype(np.float32)
        for l in range(L):
            m.cache_append(l, k, k)
        m.forward([1], [ctx_len - 1])          # warm-up token (materialised weights are cached)
        m.truncate(ctx_len - 1)
        t = []
        for s in range(steps):
            t0 = time.perf_counter()
            m.forward([2 + s], [ctx_len - 1])
            t.append(time.perf_counter() - t0)
            m.truncate(ctx_len - 1)
        times[L] = statistics.median(t)
        del m
    a, b = layer_counts
    per_layer = (times[b] - times[a]) / (b - a)
    fixed = times[a] - a * per_layer
    t_full = fixed + n_layers * per_layer
    return {"value": 1.0 / t_full, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"oracle decode of 1 token at ctx {ctx_len} on {a}- and {b}-layer prefixes of the model "
                      f"(median of {steps}), extrapolated to {n_layers} layers: "
                      f"{times[a]*1e3:.1f} ms / {times[b]*1e3:.1f} ms -> {t_full*1e3:.1f} ms per token"}


def run_reference(args, rank, world):
    from gguf_cuda import synth
    if rank != 0:
        return
    hp, ts = synth.make_model(MODEL, n_layers=4, seed=0)
    hp["n_layers"] = synth.CONFIGS[MODEL]["n_layers"]
    cb = cpu_decode_sample(hp, ts, args.ctx, steps=max(1, min(args.steps, 8)))
    v = cb["value"]
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / v, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args), "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def config_block(args):
    layers = "" if args.layers is None else f", first {args.layers} layers only (profiling case)"
    return {"workload": f"{MODEL} decode, batch 1, context {args.ctx} (cache prefilled with planted K/V rows so the "
                        f"timed steps end at {args.ctx}), f32 KV cache{layers}", "global_batch": 1, "seq_len": args.ctx,
            "parallelism": parallelism(args), "l2": "per-step traffic ~6 GB >> 126 MB L2 (no flush needed)"}


def parallelism(args):
    if args.gpus <= 1:
        return "single GPU"
    if args.parallel == "tp":
        return f"tp{args.gpus} (NCCL all-reduce after attn_output and ffn_down)"
    return f"replicas x{args.gpus}"


def tp_mode(args, world):
    return world > 1 and args.parallel == "tp"


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def gemv_roofline(ggc, ctx, torch, stream, peak_gbs):
    """Dominant kernel (k_gemv<Q4_K>, the 11008 x 4096 ffn shape) timed live with
    CUDA events over back-to-back launches on rotating weight copies (> 2x L2)."""
    from gguf_cuda import synth
    out = {}
    rows, cols = 11008, 4096
    shapes = {"Q4_K_11008x4096": (ggc.Q4_K, 11008, 4096), "Q6_K_4096x11008": (ggc.Q6_K, 4096, 11008),
              "Q4_0_4096x4096": (ggc.Q4_0, 4096, 4096), "Q4_K_4096x4096": (ggc.Q4_K, 4096, 4096),
              "Q8_0_4096x4096": (ggc.Q8_0, 4096, 4096)}
    for name, (dt, rows, cols) in shapes.items():
        raw = synth.random_blocks(dt, rows * cols, synth.rng_for(77, dt))
        wbytes = raw.nbytes
        copies = max(2, int(np.ceil(2 * 126e6 / wbytes)) + 1)
        tensors = [ggc.Tensor(raw, dt, (cols, rows), ctx=ctx) for _ in range(copies)]
        x = torch.randn(cols, device="cuda", dtype=torch.float32)
        y = torch.empty(rows, device="cuda", dtype=torch.float32)
        torch.cuda.synchronize()
        for t in tensors:
            t.matvec(x, y)
        ctx.synchronize()
        reps = max(3, 200 // copies) * copies
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        seq = [tensors[i % copies] for i in range(reps)]
        torch.cuda.nvtx.range_push(f"matvec_{name}")   # ncu --nvtx-include "matvec_<name>/" picks these launches
        with torch.cuda.stream(stream):
            e0.record(stream)
            ggc.Tensor.matvec_batch(seq, x, y)           # back to back from C: no host call per launch
            e1.record(stream)
        torch.cuda.nvtx.range_pop()
        e1.synchronize()
        per = e0.elapsed_time(e1) / 1e3 / reps
        alg = wbytes + 4 * cols + 4 * rows
        out[name] = {"us_per_launch": per * 1e6, "algorithmic_bytes": alg, "gbs": alg / per / 1e9,
                     "frac_of_peak": alg / per / 1e9 / peak_gbs}
        del tensors
    return out


def prefill_measure(args, model, hp, ts, stream, torch, barrier, max_over_ranks, world):
    """A seeded prompt of args.prefill tokens through LlamaModel::forward on an
    empty cache: its first n-1 tokens run through the batched tensor-core path
    (k_mm_tc), the last through the decode step.  FLOPs: 2 x (layer weight
    parameters) per token for the projections of every layer but the last (which
    stops after K/V), plus attention 4 x hd x visible keys per head."""
    n = args.prefill
    L, d, f = hp["n_layers"], hp["embed_dim"], hp["ffn_dim"]
    hd = d // hp["n_heads"]
    kv = hp["n_kv_heads"] * hd
    per_tok_full = 2 * (d * d + 2 * d * kv + d * d + 3 * d * f)
    per_tok_last = 2 * (2 * d * kv)
    attn = sum(4 * hd * (t + 1) * hp["n_heads"] for t in range(n - 1)) * (L - 1)
    flops = (per_tok_full * (L - 1) + per_tok_last) * (n - 1) + attn
    prompt = np.random.default_rng(21).integers(0, hp["vocab_size"], size=n).astype(np.uint32)
    pos = np.arange(n, dtype=np.int64)
    logits = np.zeros(hp["vocab_size"], dtype=np.float32)
    times = []
    for it in range(4):   # 1 warm-up + 3 timed
        model.reset_cache()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if it == 3:
            torch.cuda.nvtx.range_push("prefill")   # ncu --nvtx-include "prefill/" picks the last timed pass
        model.forward(prompt, pos, logits=logits)
        if it == 3:
            torch.cuda.nvtx.range_pop()
        e1.record(stream)
        e1.synchronize()
        if it:
            times.append(max_over_ranks(e0.elapsed_time(e1) / 1e3))
    t = float(np.median(times))
    return {"tokens": n, "ms": t * 1e3, "tokens_per_s": n / t, "model_tflops": flops / t / 1e12,
            "flops": flops, "n_gpus": world,
            "api": "ggc_model_forward(n host tokens) on an empty cache -> host logits",
            "path": "n-1 tokens batched (k_mm_tc tcgen05 split-bf16 products, k_attn_prefill), last token decode step"}


def run_ours(args, rank, world, local_rank):
    import torch
    import gguf_cuda as ggc
    from gguf_cuda import synth
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local_rank))
    tp = tp_mode(args, world)
    if tp:   # one communicator of the library's own, from rank 0's unique id
        nid = [ggc.Context.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        ctx = ggc.Context(local_rank, rank=rank, world=world, nccl_id=nid[0])
    else:
        ctx = ggc.Context(local_rank)
    stream = torch.cuda.ExternalStream(ctx.stream)
    peak_gbs, peak_src = peaks()

    hp, ts = synth.make_model(MODEL, seed=0, n_layers=args.layers)
    W, K, C = args.warmup, args.steps, args.ctx
    P = C - W - K
    assert P >= 1, "context too small for warmup + steps"
    model = ggc.LlamaModel(hp, ts, max_ctx=C, ctx=ctx)
    w_bytes = synth.weight_bytes_per_token(ts)
    # prefill: P seeded K/V rows planted in every layer (a decode step's cost does
    # not depend on the cached values)
    rng = np.random.default_rng(1)
    for l in range(hp["n_layers"]):
        kv = rng.normal(size=(P, model.kv_dim)).astype(np.float32)
        model.cache_append(l, kv, kv)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(local_rank)
    with sampler:
        model.decode(W)                                   # warm-up steps
        barrier()
        l0 = ctx.kernel_launches()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        e0.record(stream)
        model.decode(K, sync=False)
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        e1.synchronize()
        launches = ctx.kernel_launches() - l0
        ids = model.wait(K)
        barrier()
    elapsed = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    assert len(ids) == K and model.cache_len() == C
    streams = 1 if tp else world   # token streams the job decodes
    value = streams * K / elapsed

    # e2e: reference-facing forward(host token) -> host logits, per token
    model.truncate(P + W)
    tok = np.array([ids[0]], dtype=np.uint32)
    pos = np.array([P + W], dtype=np.int64)
    logits = np.zeros(hp["vocab_size"], dtype=np.float32)
    model.forward(tok, pos, logits=logits)   # first call outside timing
    model.truncate(P + W)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for s in range(K):
        pos[0] = P + W + s
        model.forward(tok, pos, logits=logits)
        tok[0] = model.last_argmax
    f1.record(stream)
    f1.synchronize()
    e2e_elapsed = max_over_ranks(f0.elapsed_time(f1) / 1e3)
    barrier()

    prefill = prefill_measure(args, model, hp, ts, stream, torch, barrier, max_over_ranks, world) \
        if args.prefill > 0 else None

    result = None
    if rank == 0:
        kv_bytes = synth.kv_bytes_per_token(hp, C - K // 2)
        step_bytes = w_bytes + kv_bytes
        # HBM bytes one GPU moves per token: its shard of the layers and the KV
        # cache, plus the replicated output head (tensor parallel)
        lm_bytes = int(ts[2]["raw"].nbytes)
        gpu_bytes = (w_bytes - lm_bytes + kv_bytes) / world + lm_bytes if tp else step_bytes
        model_gbs = gpu_bytes * (K / elapsed) / 1e9   # per GPU
        rl = gemv_roofline(ggc, ctx, torch, stream, peak_gbs)
        dom = rl["Q4_K_11008x4096"]
        tr = traffic_record().get("k_gemv_span<Q4_K> 11008x4096")
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            hp4, ts4 = hp, ts
            cpu = cpu_decode_sample(hp4, ts4, C, steps=4)
        result = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": elapsed / K * 1e3, "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded Q4_K_M blocks)",
            "config": config_block(args),
            "e2e": {"value": streams * K / e2e_elapsed, "unit": "tokens/s", "h2d_bytes_per_step": 4 + 8,
                    "d2h_bytes_per_step": 4 * hp["vocab_size"] + 4,
                    "api": "ggc_model_forward(1 host token) -> host logits + argmax, per token"},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "achieved": dom["gbs"], "peak": peak_gbs, "unit": "GB/s",
                         "frac": dom["gbs"] / peak_gbs, "traffic": tr,
                         "kernel": "k_gemv_span<Q4_K> 11008x4096 (ffn_up/gate shape), back-to-back launches",
                         "peak_source": peak_src},
            "model_roofline": {"bytes_per_step": step_bytes, "weight_bytes": w_bytes, "kv_bytes": kv_bytes,
                               "bytes_per_step_per_gpu": gpu_bytes, "achieved_gbs_per_gpu": model_gbs,
                               "frac": model_gbs / peak_gbs, "bound_tokens_s": peak_gbs * 1e9 / gpu_bytes * streams},
            "matvec": rl,
            "prefill": prefill,
            "clocks": sampler.record(),
            "cpu_baseline": cpu,
        }
    if dist is not None:
        dist.barrier()
    del model
    if rank == 0:
        print(json.dumps(result), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    lib = ROOT / "gguf-reader_b200" / "lib" / "libgguf_cuda.so"
    if not lib.exists():
        import __graft_entry__
        __graft_entry__.build()
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()

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
the hidden state all-reduced after attn_output and ffn_down -- fused into those
GEMVs over NVLink peer memory, or NCCL; `allreduce` says which; strong scaling:
`value` is that model's tokens/s) or, with `--parallel replicas`, one
independent replica per rank (weak scaling: `value` sums the replicas).

Before the timing every rank runs a parity probe (`tp_parity`: a 2-layer prefix
of the model, 8-token prompt, 32 greedy ids, checked on rank 0 against the
oracle).  `configs` adds the other named workloads: Qwen2-0.5B Q8_0 (32-token
prompt + 128 greedy steps, 1 GPU) and Llama-3-8B Q4_0 (2048-token prefill;
256 decode steps ending at context 8192, f16 KV; tensor parallel at N > 1).
`cpu_baseline` and `--impl reference` run one procedure: the oracle (C++
restatement of the reference's rayon CPU path) decoding whole tokens of the
full model at the same context on the host cores (extrapolated from layer
prefixes only when the host RAM cannot hold the f32 model; it says so).
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
    ap.add_argument("--no-configs", dest="configs", action="store_false",
                    help="skip the Qwen2-0.5B and Llama-3-8B workloads")
    ap.add_argument("--no-matvec-sweep", dest="sweep", action="store_false",
                    help="time only the roofline matvec, not the 15-format x 3-shape sweep")
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
def oracle_bytes(hp, ts, ctx_len):
    """Host bytes the oracle holds for a model: every tensor materialised as f32
    (the reference's materialize, llama.rs:183-204) plus the f32 KV cache."""
    kvd = hp["n_kv_heads"] * (hp["embed_dim"] // hp["n_heads"])
    return 4 * sum(int(t["n_elements"]) for t in ts if t is not None) + 8 * hp["n_layers"] * ctx_len * kvd


def _oracle_token_times(oracle, hp, ts, ctx_len, tokens, warmup):
    """Per-token times of the oracle decoding at context ctx_len: the cache holds
    ctx_len - 1 planted rows, each token is forwarded at position ctx_len - 1 and
    the cache is truncated back after it."""
    kvd = hp["n_kv_heads"] * (hp["embed_dim"] // hp["n_heads"])
    m = oracle.Model(hp, ts)
    kv = np.random.default_rng(0).normal(size=(ctx_len - 1) * kvd).astype(np.float32)
    for l in range(hp["n_layers"]):
        m.cache_append(l, kv, kv)
    t = []
    for s in range(warmup + tokens):
        t0 = time.perf_counter()
        m.forward([2 + s], [ctx_len - 1])
        if s >= warmup:
            t.append(time.perf_counter() - t0)
        m.truncate(ctx_len - 1)
    del m
    return t


def cpu_decode(hp, ts, ctx_len, tokens, warmup=1):
    """Decode tokens/s of the oracle on this host's cores, one procedure for both
    CPU legs (our arm's cpu_baseline and the reference arm).  The whole model when
    the host's free RAM holds its f32 materialisation; otherwise a least-squares
    line through 2/4/8/16-layer prefixes of the model, reported as an extrapolation
    with its residual."""
    import psutil
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    oracle.build()
    threads = oracle.get_threads()
    L = hp["n_layers"]
    need = oracle_bytes(hp, ts, ctx_len)
    avail = psutil.virtual_memory().available
    base = {"unit": "tokens/s", "cores": threads, "kind": "port", "tokens_timed": tokens}
    if avail > 1.25 * need + 4e9:
        t0 = time.perf_counter()
        t = _oracle_token_times(oracle, hp, ts, ctx_len, tokens, warmup)
        wall = time.perf_counter() - t0
        total = float(sum(t))
        return dict(base, value=tokens / total, seconds=total, wall_seconds=wall, method="full model",
                    sample=f"oracle decoding {tokens} tokens (after {warmup} warm-up) at context {ctx_len} through all "
                           f"{L} layers: {need / 1e9:.1f} GB of f32 weights and KV on the host, {threads} threads, "
                           f"{total / tokens * 1e3:.1f} ms per token (median {statistics.median(t) * 1e3:.1f})")
    counts = [c for c in (2, 4, 8, 16) if c <= L] or [L]
    per = {}
    for c in counts:
        h = dict(hp, n_layers=c)
        per[c] = statistics.median(_oracle_token_times(oracle, h, ts[:3 + 12 * c], ctx_len, tokens, warmup))
    xs = np.array(counts, float)
    ys = np.array([per[c] for c in counts])
    b, a = np.polyfit(xs, ys, 1) if len(counts) > 1 else (ys[0] / xs[0], 0.0)
    resid = float(np.sqrt(np.mean((a + b * xs - ys) ** 2)))
    t_full = float(a + b * L)
    return dict(base, value=1.0 / t_full, seconds=float(sum(per.values())) * tokens, method="extrapolated",
                fit={"layers": counts, "ms_per_token": [per[c] * 1e3 for c in counts], "rms_residual_ms": resid * 1e3},
                sample=f"EXTRAPOLATED: the host's free RAM ({avail / 1e9:.0f} GB) does not hold the {need / 1e9:.0f} GB "
                       f"f32 model; oracle decode at context {ctx_len} on {counts}-layer prefixes (median of {tokens} "
                       f"tokens each), least-squares line to {L} layers: {t_full * 1e3:.1f} ms per token, "
                       f"rms residual {resid * 1e3:.2f} ms")


def cpu_matvec_sweep(dtypes, shapes, seed=77, reps=2):
    """quant_matvec of the oracle (the reference's quant.rs:526-570 restated: block
    dequant, then one serial multiply-add per element, rows split over the host
    threads) for every format and sweep shape: the same seeded weights as the GPU
    sweep, x ~ N(0, 1) seed 1, median of `reps` after a warm-up; GB/s of the same
    algorithmic bytes (W + 4 cols + 4 rows)."""
    from gguf_cuda import synth
    from gguf_cuda._lib import DTYPE_NAMES
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    oracle.build()
    out = {}
    t_all = time.perf_counter()
    for dt in dtypes:
        for rows, cols in shapes:
            raw = synth.random_blocks(dt, rows * cols, synth.rng_for(seed, dt, rows, cols))
            x = np.random.default_rng(1).normal(size=cols).astype(np.float32)
            oracle.quant_matvec(raw, dt, rows, cols, x)
            t = []
            for _ in range(reps):
                t0 = time.perf_counter()
                oracle.quant_matvec(raw, dt, rows, cols, x)
                t.append(time.perf_counter() - t0)
            per = statistics.median(t)
            alg = raw.nbytes + 4 * cols + 4 * rows
            out[f"{DTYPE_NAMES[dt]}_{rows}x{cols}"] = {"ms": per * 1e3, "gbs": alg / per / 1e9}
    return {"threads": oracle.get_threads(), "seconds": time.perf_counter() - t_all,
            "what": "oracle quant_matvec (reference quant.rs:526-570 restated), all host threads, "
                    f"median of {reps} after a warm-up, GB/s of W + 4 cols + 4 rows", "entries": out}


def planted_rows(C, W, K):
    """K/V rows planted before the decode timing: one forward at position P, then
    max(W - 1, 0) warm-up steps and K timed steps end at context C."""
    return C - max(W, 1) - K


def run_reference(args, rank, world):
    """The reference's CPU path (the oracle port; the Rust crate cannot be built
    here) on the host cores: W warm-up tokens, then K timed tokens, each one
    decode step of the whole model at context args.ctx.  Rank 0 only."""
    from gguf_cuda import synth
    if rank != 0:
        return
    hp, ts = synth.make_model(MODEL, seed=0)
    cb = cpu_decode(hp, ts, args.ctx, tokens=args.steps, warmup=args.warmup)
    v = cb["value"]
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / v, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args), "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def config_block(args, allreduce=None):
    layers = "" if args.layers is None else f", first {args.layers} layers only (profiling case)"
    return {"workload": f"{MODEL} decode, batch 1, context {args.ctx} (K/V rows planted at positions 0..P-1, one "
                        f"token forwarded at position P, then warm-up and timed steps at positions P+1..{args.ctx - 1}, "
                        f"each attending to every earlier row), f32 KV cache{layers}", "global_batch": 1,
            "seq_len": args.ctx,
            "parallelism": parallelism(args, allreduce), "l2": "per-step traffic ~6 GB >> 126 MB L2 (no flush needed)"}


ALLREDUCE_NAMES = {"peer": "all-reduce fused into the attn_output / ffn_down GEMVs over NVLink peer memory",
                   "nccl": "NCCL all-reduce after attn_output and ffn_down"}


def parallelism(args, allreduce=None):
    if args.gpus <= 1:
        return "single GPU"
    if args.parallel == "tp":
        return f"tp{args.gpus} ({ALLREDUCE_NAMES.get(allreduce, 'all-reduce after attn_output and ffn_down')})"
    return f"replicas x{args.gpus}"


def tp_mode(args, world):
    return world > 1 and args.parallel == "tp"


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def time_matvec(ggc, ctx, torch, stream, dt, rows, cols, peak_gbs, seed=77, min_reps=200):
    """One weight shape timed live with CUDA events over back-to-back launches
    (ggc_tensor_matvec_batch: no host call per launch) on rotating copies of the
    weight whose total exceeds 2x L2, so every launch streams from HBM."""
    from gguf_cuda import synth
    raw = synth.random_blocks(dt, rows * cols, synth.rng_for(seed, dt, rows, cols))
    wbytes = raw.nbytes
    copies = max(2, int(np.ceil(2 * 126e6 / wbytes)) + 1)
    tensors = [ggc.Tensor(raw, dt, (cols, rows), ctx=ctx) for _ in range(copies)]
    x = torch.from_numpy(np.random.default_rng(1).normal(size=cols).astype(np.float32)).cuda()   # x ~ N(0, 1), seed 1
    y = torch.empty(rows, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    for t in tensors:
        t.matvec(x, y)
    ctx.synchronize()
    reps = max(3, min_reps // copies) * copies
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    seq = [tensors[i % copies] for i in range(reps)]
    name = f"{ggc.DTYPE_NAMES[dt]}_{rows}x{cols}"
    torch.cuda.nvtx.range_push(f"matvec_{name}")   # ncu --nvtx-include "matvec_<name>/" picks these launches
    with torch.cuda.stream(stream):
        e0.record(stream)
        ggc.Tensor.matvec_batch(seq, x, y)
        e1.record(stream)
    torch.cuda.nvtx.range_pop()
    e1.synchronize()
    per = e0.elapsed_time(e1) / 1e3 / reps
    alg = wbytes + 4 * cols + 4 * rows
    del tensors
    return name, {"us_per_launch": per * 1e6, "algorithmic_bytes": alg, "gbs": alg / per / 1e9,
                  "frac_of_peak": alg / per / 1e9 / peak_gbs,
                  "kernel": "k_gemv" if dt in (ggc.F16, ggc.BF16, ggc.F32) else "k_gemv_span"}


SWEEP_SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008)]


def gemv_roofline(ggc, ctx, torch, stream, peak_gbs, sweep=True):
    """The dominant kernel (k_gemv_span<Q4_K> at the 11008 x 4096 ffn shape) and the
    format sweep: the 15 quantized and half formats at 4096 x 4096, 11008 x 4096 and
    4096 x 11008 (rows x cols), each timed as time_matvec does."""
    out = {}
    for dt in [d for d in ggc.ALL_DTYPES if d != ggc.F32] if sweep else []:
        for rows, cols in SWEEP_SHAPES:
            name, rec = time_matvec(ggc, ctx, torch, stream, dt, rows, cols, peak_gbs, min_reps=60)
            out[name] = rec
    name, rec = time_matvec(ggc, ctx, torch, stream, ggc.Q4_K, 11008, 4096, peak_gbs)   # the roofline line: more reps
    out[name] = rec
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


def rel_l2(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def parity_probe(ggc, ctx, rank, barrier):
    """The checker before the timing: a 2-layer prefix of the benchmark model (the
    rank's shard of it under tensor parallelism), an 8-token prompt and 32 greedy
    ids, against the oracle on rank 0 (logits within 1e-4 relative L2, ids equal)."""
    from gguf_cuda import synth
    hp, ts = synth.make_model(MODEL, n_layers=2, seed=0)
    prompt = np.random.default_rng(5).integers(0, hp["vocab_size"], size=8).astype(np.uint32)
    pos = np.arange(8, dtype=np.int64)
    m = ggc.LlamaModel(hp, ts, max_ctx=64, ctx=ctx)
    logits = m.forward(prompt, pos)
    ids = m.decode(32)
    kind = m.allreduce
    m.close()
    barrier()
    if rank != 0:
        return None
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    o = oracle.Model(hp, ts)
    want = o.forward(prompt, pos)
    want_ids, lg, p = [], want, 8
    for _ in range(32):
        want_ids.append(oracle.greedy(lg))
        lg = o.forward([want_ids[-1]], [p])
        p += 1
    err = rel_l2(logits, want)
    return {"model": f"{MODEL}, first 2 layers", "prompt_tokens": 8, "greedy_ids": 32, "rel_l2": err,
            "ids_match": ids == want_ids, "pass": err <= 1e-4 and ids == want_ids, "allreduce": kind}


def time_decode(model, stream, torch, steps, barrier, max_over_ranks):
    """Device-timed greedy decode of `steps` tokens (CUDA events on the library stream)."""
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    model.decode(steps, sync=False)
    e1.record(stream)
    e1.synchronize()
    ids = model.wait(steps)
    return max_over_ranks(e0.elapsed_time(e1) / 1e3), ids


def qwen2_arm(ggc, ctx, stream, torch, peak_gbs, barrier, max_over_ranks):
    """Qwen2-0.5B shape, Q8_0, 24 layers, 1 GPU: a 32-token prompt of seeded
    uniform ids, then 128 greedy decode steps on the f32 KV cache."""
    from gguf_cuda import synth
    name = "qwen2-0.5b-q8_0"
    hp, ts = synth.make_model(name, seed=0)
    m = ggc.LlamaModel(hp, ts, max_ctx=32 + 128 + 8, ctx=ctx)
    prompt = np.random.default_rng(31).integers(0, hp["vocab_size"], size=32).astype(np.uint32)
    pos = np.arange(32, dtype=np.int64)
    runs = []
    for it in range(4):   # 1 warm-up + 3 timed
        m.reset_cache()
        barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        m.forward(prompt, pos, want_logits=False)
        p1.record(stream)
        t, ids = time_decode(m, stream, torch, 128, barrier, max_over_ranks)
        p1.synchronize()
        if it:
            runs.append((t, p0.elapsed_time(p1) / 1e3, len(ids)))
    m.close()
    t, tp, nids = sorted(runs)[1]
    w_bytes = synth.weight_bytes_per_token(ts)
    kv = synth.kv_bytes_per_token(hp, 32 + 64)
    gbs = (w_bytes + kv) * 128 / t / 1e9
    return {"workload": f"{name}: 24 layers, 32-token prompt then 128 greedy decode steps, f32 KV cache, 1 GPU",
            "decode_tokens_per_s": 128 / t, "ms_per_token": t / 128 * 1e3, "prompt_ms": tp * 1e3,
            "bytes_per_token": w_bytes + kv, "achieved_gbs": gbs, "frac_of_hbm": gbs / peak_gbs,
            "ids": nids, "timed": "median of 3 after 1 warm-up, CUDA events"}


def llama3_arm(ggc, ctx, stream, torch, peak_gbs, barrier, max_over_ranks, world, tflops_peak):
    """Llama-3-8B shape (GQA 32/8, ffn 14336, vocab 128256), Q4_0, f16 KV cache:
    a 2048-token prefill of seeded uniform ids on an empty cache, and 256 greedy
    decode steps whose context ends at 8192 (earlier rows planted); one model,
    tensor parallel over the ranks."""
    from gguf_cuda import synth
    name = "llama3-8b-q4_0"
    hp, ts = synth.make_model(name, seed=0)
    C, K, W = 8192, 256, 8
    m = ggc.LlamaModel(hp, ts, max_ctx=C, kv_f16=True, ctx=ctx)
    L, d, f = hp["n_layers"], hp["embed_dim"], hp["ffn_dim"]
    hd = d // hp["n_heads"]
    kvd = hp["n_kv_heads"] * hd
    n = 2048
    prompt = np.random.default_rng(41).integers(0, hp["vocab_size"], size=n).astype(np.uint32)
    pos = np.arange(n, dtype=np.int64)
    per_tok = 2 * (2 * d * d + 2 * d * kvd + 3 * d * f)
    flops = (per_tok * (L - 1) + 2 * 2 * d * kvd) * (n - 1) + \
        sum(4 * hd * (t + 1) * hp["n_heads"] for t in range(n - 1)) * (L - 1)
    times = []
    for it in range(3):   # 1 warm-up + 2 timed
        m.reset_cache()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        m.forward(prompt, pos, want_logits=False)
        e1.record(stream)
        e1.synchronize()
        if it:
            times.append(max_over_ranks(e0.elapsed_time(e1) / 1e3))
    tpf = min(times)
    # decode ending at context C: plant C - K - W rows, W warm-up steps, K timed
    m.reset_cache()
    P = C - K - W
    rows = np.random.default_rng(2).normal(size=(P, m.kv_dim)).astype(np.float32)
    for l in range(L):
        m.cache_append(l, rows, rows)
    m.forward([1], [P], want_logits=False)
    m.decode(W - 1)
    t, ids = time_decode(m, stream, torch, K, barrier, max_over_ranks)
    assert m.cache_len() == C
    kind = m.allreduce
    m.close()
    w_bytes = synth.weight_bytes_per_token(ts)
    lm = int(ts[2]["raw"].nbytes)
    kv = synth.kv_bytes_per_token(hp, C - K // 2, 2)
    gpu_bytes = (w_bytes - lm + kv) / world + lm
    gbs = gpu_bytes * K / t / 1e9
    return {"workload": f"{name}: 32 layers, 2048-token prefill on an empty cache; {K} greedy decode steps ending at "
                        f"context {C} (earlier rows planted), f16 KV cache, tp{world}",
            "allreduce": kind if world > 1 else "none",
            "prefill": {"tokens": n, "ms": tpf * 1e3, "tokens_per_s": n / tpf, "model_tflops": flops / tpf / 1e12,
                        "frac_of_bf16_sustained": flops / tpf / 1e12 / tflops_peak,
                        "frac_of_bf16_sustained_issued": 3 * flops / tpf / 1e12 / tflops_peak,
                        "note": "3 bf16 MMAs issued per product (split operands); min of 2 after 1 warm-up"},
            "decode_tokens_per_s": K / t, "ms_per_token": t / K * 1e3, "bytes_per_token_per_gpu": gpu_bytes,
            "achieved_gbs_per_gpu": gbs, "frac_of_hbm": gbs / peak_gbs, "ids": len(ids)}


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
    tflops_peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops_sustained"] \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1400.0

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

    parity = parity_probe(ggc, ctx, rank, barrier) if args.layers is None else None

    hp, ts = synth.make_model(MODEL, seed=0, n_layers=args.layers)
    W, K, C = args.warmup, args.steps, args.ctx
    P = planted_rows(C, W, K)
    assert P >= 1, "context too small for warmup + steps"
    t_load = time.perf_counter()
    model = ggc.LlamaModel(hp, ts, max_ctx=C, ctx=ctx)   # raw rows uploaded, split into planes on the GPU
    t_load = time.perf_counter() - t_load
    allreduce = model.allreduce if tp else "none"
    w_bytes = synth.weight_bytes_per_token(ts)
    # prefill: P seeded K/V rows planted in every layer (a decode step's cost does
    # not depend on the cached values), then one token forwarded at position P so
    # the decode steps continue at positions P + 1 .. C - 1 and attend to every
    # cached row (planting advances the cache slot, not the position)
    rng = np.random.default_rng(1)
    for l in range(hp["n_layers"]):
        kv = rng.normal(size=(P, model.kv_dim)).astype(np.float32)
        model.cache_append(l, kv, kv)
    model.forward(np.array([1], np.uint32), np.array([P], np.int64), want_logits=False)

    sampler = ClockSampler(local_rank)
    with sampler:
        model.decode(max(W - 1, 0))                       # warm-up steps (the forward above was the first)
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
    if prefill:
        prefill["frac_of_bf16_sustained"] = prefill["model_tflops"] / tflops_peak
        prefill["frac_of_bf16_sustained_issued"] = 3 * prefill["model_tflops"] / tflops_peak
    model.close()
    del model

    configs = {}
    if args.layers is None and args.configs:
        if world == 1:
            configs["qwen2-0.5b-q8_0"] = qwen2_arm(ggc, ctx, stream, torch, peak_gbs, barrier, max_over_ranks)
        if tp or world == 1:
            configs["llama3-8b-q4_0"] = llama3_arm(ggc, ctx, stream, torch, peak_gbs, barrier, max_over_ranks,
                                                   world if tp else 1, tflops_peak)

    result = None
    if rank == 0:
        kv_bytes = synth.kv_bytes_per_token(hp, C - K // 2)
        step_bytes = w_bytes + kv_bytes
        # HBM bytes one GPU moves per token: its shard of the layers and the KV
        # cache, plus the replicated output head (tensor parallel)
        lm_bytes = int(ts[2]["raw"].nbytes)
        gpu_bytes = (w_bytes - lm_bytes + kv_bytes) / world + lm_bytes if tp else step_bytes
        model_gbs = gpu_bytes * (K / elapsed) / 1e9   # per GPU
        rl = gemv_roofline(ggc, ctx, torch, stream, peak_gbs, sweep=args.sweep)
        dom = rl["Q4_K_11008x4096"]
        sweep_fracs = {k: round(v["frac_of_peak"], 3) for k, v in rl.items()}
        tr = traffic_record().get("k_gemv_span<Q4_K> 11008x4096")
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_decode(hp, ts, C, tokens=8, warmup=1)
            if args.sweep:   # the format sweep on the host cores, beside the GPU's
                cpu["matvec"] = cpu_matvec_sweep([d for d in ggc.ALL_DTYPES if d != ggc.F32], SWEEP_SHAPES)
        result = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": elapsed / K * 1e3, "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded Q4_K_M blocks)",
            "config": config_block(args, allreduce),
            "allreduce": allreduce,
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
            "tp_parity": parity,
            "load": {"s": t_load, "weight_bytes": int(sum(int(t["raw"].nbytes) for t in ts if t is not None
                                                           and t.get("raw") is not None)),
                     "what": "ggc_model_create wall time (rank 0): raw weight rows to HBM, plane split by "
                             "k_repack on the GPU, prefill raw copies, KV cache and RoPE table"},
            "matvec": rl,
            "matvec_frac_summary": sweep_fracs,
            "prefill": prefill,
            "configs": configs,
            "clocks": sampler.record(),
            "cpu_baseline": cpu,
        }
    if dist is not None:
        dist.barrier()
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

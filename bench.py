"""Benchmark: batch-1 greedy decode tokens/s of the Llama-3-8B-shaped Q4_0 model
(config 3: KV cache pre-filled to 4096 positions) on B200, plus % of the HBM
roofline, the end-to-end rate through the C ABI, and the CPU oracle baseline.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                [--workload 8b|1b|70b] [--no-prefill] [--no-cpu]

On one GPU the line also carries "prefill": config 4 (the 8B shape with Q8_0
linears), a 512-token prompt through the tensor-core prefill path, timed with
CUDA events over back-to-back prefills (ids resident), plus its end-to-end
rate through llmrs_prefill and the CPU oracle's prefill rate.

One "step" = one greedy decode token through every layer + LM head.  Inputs
(weights 4.2 GB, KV 1.1 GB) are far larger than the 126 MB L2, so no flush is
needed between steps.  Synthetic seeded weights stand in for checkpoints.
With N > 1 (torchrun, one rank per GPU) the model is tensor parallel over the N
GPUs: one sequence, the same total work (strong scaling); the roofline's peak
is then the N GPUs' aggregate HBM bandwidth.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "8b": dict(cfg=dict(n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336,
                        vocab=128256, max_seq=4608, rms_eps=1e-5, rope_theta=500000.0, weight_format=0,
                        tied_embeddings=0),
               kv=4096, name="llama3-8b-shaped Q4_0 decode, KV pre-filled to 4096 (config 3)"),
    "1b": dict(cfg=dict(n_layers=16, hidden=2048, n_heads=32, n_kv_heads=8, head_dim=64, ffn=8192,
                        vocab=128256, max_seq=256, rms_eps=1e-5, rope_theta=500000.0, weight_format=0,
                        tied_embeddings=1),
               kv=32, name="llama3.2-1b-shaped Q4_0 decode after a 32-token prompt (config 1)"),
    "70b": dict(cfg=dict(n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672,
                         vocab=128256, max_seq=2176, rms_eps=1e-5, rope_theta=500000.0, weight_format=0,
                         tied_embeddings=0),
                kv=2048, name="llama3-70b-shaped Q4_0 decode, KV pre-filled to 2048 (config 5)"),
}
SEED = 0x5EED

# config 4: the 8B shape with Q8_0 linears, prefill of a 512-token prompt
PREFILL = dict(cfg=dict(n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
                        max_seq=576, rms_eps=1e-5, rope_theta=500000.0, weight_format=1, tied_embeddings=0),
               n=512, name="llama3-8b-shaped Q8_0 prefill of a 512-token prompt (config 4)")

# DRAM bytes per launch of each decode-step GEMV of the 8B shape, from one ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum; profiles/
# decode_step_8b_kv4096_launches.md has the command and the table).
MEASURED_GEMV_DRAM_8B = {"qkv_gemv": 14.27e6, "o_gemv": 9.54e6, "gate_up_gemv": 66.18e6, "down_gemv": 33.18e6,
                         "lm_head_gemv": 296.07e6}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def load_pkg():
    import importlib.util
    if "llmrs_b200" in sys.modules:
        return sys.modules["llmrs_b200"]
    pkg = os.path.join(ROOT, "llm.rs_b200")
    spec = importlib.util.spec_from_file_location("llmrs_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llmrs_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


# ----------------------------------------------------------- byte accounting
def linear_shapes(c):
    """(N, K) of every quantised linear read per decode token (native GQA)."""
    D, H, F = c["head_dim"], c["hidden"], c["ffn"]
    qkv = ((c["n_heads"] + 2 * c["n_kv_heads"]) * D, H)
    per_layer = [qkv, (H, c["n_heads"] * D), (2 * F, H), (H, F)]
    return per_layer * c["n_layers"] + [(c["vocab"], H)]


def q_bytes(n, k, c):
    # Q4: nibbles + fp16 scale = 18 B per 32 weights (Q8_0: 34 B); the tied 1B head has f32 scales (20 B)
    if c["weight_format"] == 1:
        return n * k * 34 // 32
    return n * k * 18 // 32


def algo_bytes_per_token(c, S):
    w = sum(q_bytes(n, k, c) for n, k in linear_shapes(c))
    if c["tied_embeddings"]:
        w += c["vocab"] * c["hidden"] // 16  # f32 instead of f16 scales on the tied head
    kv = 2 * c["n_layers"] * c["n_kv_heads"] * c["head_dim"] * S * 4
    norms = (2 * c["n_layers"] + 1) * c["hidden"] * 4
    emb = c["hidden"] * 4
    return w + kv + norms + emb, w, kv


def gemv_bytes(kind, c):
    D, H, F, V = c["head_dim"], c["hidden"], c["ffn"], c["vocab"]
    n, k = {"qkv_gemv": ((c["n_heads"] + 2 * c["n_kv_heads"]) * D, H), "o_gemv": (H, c["n_heads"] * D),
            "gate_up_gemv": (2 * F, H), "down_gemv": (H, F), "lm_head_gemv": (V, H)}[kind]
    b = q_bytes(n, k, c) + k * 4 + n * 4
    if kind == "lm_head_gemv" and c["tied_embeddings"]:
        b += n * k // 16
    return b


def prefill_ops(c, n):
    """Integer MACs x 2 of the linears for n rows (the LM head for the last row
    only, the row llmrs_prefill returns) and f32 attention FLOPs (QK and PV
    over the causal triangle)."""
    lin = sum(2 * nn * k for nn, k in linear_shapes(c)[:-1]) * n + 2 * c["vocab"] * c["hidden"]
    att = 4 * c["n_layers"] * c["n_heads"] * c["head_dim"] * n * (n + 1) // 2
    return lin, att


def prefill_prompt(c, n):
    return [(SEED * 31 + 7919 * i) % c["vocab"] for i in range(n)]


# ----------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), "--query-gpu=" + q,
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # start timing only once the sampler is producing (startup takes ~0.1-1 s)
            t_end = time.time() + 5.0
            while not self.lines and time.time() < t_end:
                time.sleep(0.01)
            self.lines.clear()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- CPU baseline
def cpu_baseline(wl, n_tokens, threads=None):
    """The reference CPU path restated in C (oracle/), expanded GQA exactly as
    src/core/loader.rs:62-98 builds it, timed on this host's cores."""
    from oracle import oracle as O
    if threads:
        O.set_threads(threads)
    c = dict(wl["cfg"])
    m = O.Model(c, expand_gqa=True)
    m.init_synthetic(SEED)
    m.kv_fill_synthetic(SEED, wl["kv"])
    tok = O.synth_token(SEED, 0, c["vocab"])
    m.forward([tok], wl["kv"])  # warm-up token (page faults, thread start-up)
    times = []
    pos = wl["kv"] + 1
    for i in range(n_tokens):
        t0 = time.perf_counter()
        logits = m.forward([tok], pos)
        times.append(time.perf_counter() - t0)
        tok = O.argmax(logits)
        pos += 1
    m.close()
    return 1.0 / statistics.median(times), O.get_threads(), times


def cpu_prefill_baseline(threads=None):
    """The oracle's prefill (the reference's m > 1 path) of a 32-token prompt
    through 2 layers of the config-4 model, scaled to 32 layers."""
    from oracle import oracle as O
    if threads:
        O.set_threads(threads)
    c = dict(PREFILL["cfg"], n_layers=2)
    m = O.Model(c, expand_gqa=True)
    m.init_synthetic(SEED)
    ids = prefill_prompt(c, 32)
    m.forward(ids[:4], 0)  # warm-up
    t0 = time.perf_counter()
    m.forward(ids, 0)
    t = (time.perf_counter() - t0) * PREFILL["cfg"]["n_layers"] / c["n_layers"]
    m.close()
    return 32 / t, O.get_threads(), t


def int8_peak_tops():
    """cuBLASLt int8 GEMM throughput (torch._int_mm, 8192^3), the measured
    int8 tensor peak the prefill is compared with."""
    import torch
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        torch._int_mm(a, b)
    e1.record()
    torch.cuda.synchronize()
    return 2.0 * n ** 3 / (e0.elapsed_time(e1) / 10 / 1000.0) / 1e12


def run_prefill(L, ctx, args):
    c = dict(PREFILL["cfg"])
    if args.layers:
        c["n_layers"] = args.layers
    n = PREFILL["n"]
    m = L.Model(ctx, dict(c, scale_dtype=L.F16))
    m.init_synthetic(SEED)
    ids = prefill_prompt(c, n)
    m.time_prefill(ids, 0, args.warmup)  # warm-up
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        ms = m.time_prefill(ids, 0, max(1, min(args.steps, 10)))
    e2e = []
    for _ in range(3):
        t0 = time.perf_counter()
        m.prefill(ids, 0, want_logits=True)
        e2e.append(time.perf_counter() - t0)
    m.close()
    lin, att = prefill_ops(c, n)
    try:
        peak = int8_peak_tops()
    except Exception:
        peak = None
    tops = (lin + att) / (ms / 1000.0) / 1e12
    out = {"metric": "prefill tokens/s", "value": round(n / (ms / 1000.0), 1), "unit": "tokens/s",
           "ms": round(ms, 3), "workload": PREFILL["name"], "prompt_tokens": n,
           "dtype": "q8_0 x q8_0 (exact integer block dots on tcgen05 with bf16 operands, f32 block sums)",
           "e2e": {"value": round(n / statistics.median(e2e), 1), "unit": "tokens/s",
                   "h2d_bytes_per_step": 4 * n, "d2h_bytes_per_step": 4 * c["vocab"] + 8},
           "ops_per_prefill": {"linear_int_ops": lin, "attention_f32_flops": att},
           "achieved_tops": round(tops, 1), "clocks": clk.summary()}
    if peak:
        out["roofline"] = {"bound": "tensor", "achieved": round(tops, 1), "peak": round(peak, 1), "unit": "TOP/s",
                           "frac": round(tops / peak, 4),
                           "peak_source": "measured here: cuBLASLt int8 GEMM 8192^3 (torch._int_mm)",
                           "note": "the exact per-32-block f32 epilogue (3 f32 ops per block and output) bounds the "
                                   "GEMM, not the tensor pipe"}
    if not args.no_cpu:
        v, cores, t = cpu_prefill_baseline()
        out["cpu_baseline"] = {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                               "sample": "32-token prompt through 2 of the 32 layers (%.1f s scaled to 32 layers)" % t}
    return out


# ------------------------------------------------------------------ our arm
def run_ours(args, rank, world):
    L = load_pkg()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    wl = WORKLOADS[args.workload]
    c = dict(wl["cfg"])
    if args.layers:
        c["n_layers"] = args.layers
    ctx = L.Context(local)
    # N > 1: tensor parallel over the N GPUs (one sequence, strong scaling)
    m = L.Model(ctx, dict(c, tp_rank=rank, tp_size=world))
    m.init_synthetic(SEED)
    m.kv_fill_synthetic(SEED, wl["kv"])
    if world > 1:
        L.connect_tensor_parallel(m)
    kv0 = wl["kv"]
    tok0 = 1234 % c["vocab"]
    K, W = args.steps, args.warmup
    assert kv0 + max(K, W) + 1 <= c["max_seq"], "steps exceed the KV capacity"
    # warm-up (also captures the step graph)
    m.time_decode(tok0, kv0, W)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    with ClockSampler(local) as clk:
        ms = m.time_decode(tok0, kv0, K)
    if dist is not None:
        import torch
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / K
    value = K / (ms / 1000.0)  # one sequence decoded by all ranks together
    # per-kernel durations (kernel by kernel, events around each launch)
    prof = [m.profile_decode(tok0, kv0 + i) for i in range(3)]
    per_kind = {}
    for run in prof:
        agg = {}
        for kind, t in run:
            agg.setdefault(kind, []).append(t)
        for kind, ts in agg.items():
            per_kind.setdefault(kind, []).append(sum(ts))
    kind_ms = {k: statistics.median(v) for k, v in per_kind.items()}
    kind_count = {}
    for kind, _ in prof[0]:
        kind_count[kind] = kind_count.get(kind, 0) + 1
    if world > 1:  # the slowest rank sets the pace
        import torch
        import torch.distributed as dist
        names = sorted(kind_ms)
        t = torch.tensor([kind_ms[k] for k in names], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        kind_ms = {k: float(v) for k, v in zip(names, t.tolist())}
    gemv_kinds = [k for k in kind_ms if k.endswith("_gemv")]
    gemv_bytes_step = sum(gemv_bytes(k, c) * kind_count[k] for k in gemv_kinds)
    gemv_ms_step = sum(kind_ms[k] for k in gemv_kinds)
    gemv_launches = sum(kind_count[k] for k in gemv_kinds)
    traffic = None
    if args.workload == "8b" and not args.layers and world == 1:
        traffic = round(sum(MEASURED_GEMV_DRAM_8B[k] * kind_count[k] for k in gemv_kinds) / gemv_launches)
    peak, peak_src = load_peaks()
    peak *= world  # aggregate HBM bandwidth of the N GPUs
    achieved = gemv_bytes_step / (gemv_ms_step / 1000.0) / 1e9
    S_mid = kv0 + K // 2
    tot_bytes, w_bytes, kv_bytes = algo_bytes_per_token(c, S_mid)
    step_gbs = tot_bytes / (ms_per_step / 1000.0) / 1e9
    # end to end through the C ABI: token in from host memory, argmax (+err word) back
    E = min(K, 64)
    m.decode_step(tok0, kv0, want_logits=False)
    t0 = time.perf_counter()
    tok = tok0
    for i in range(E):
        tok, _ = m.decode_step(tok, kv0 + i, want_logits=False)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        import torch
        import torch.distributed as dist
        t = torch.tensor([e2e_s], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_val = E / e2e_s
    kernels_step = m.decode_kernel_count()
    out = {
        "metric": "batch-1 greedy decode tokens/s (Llama-3-8B-shaped Q4_0, KV 4096)" if args.workload == "8b"
        else "batch-1 greedy decode tokens/s (%s)" % wl["name"],
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "q4_0 x q8_0 (int8 dot, f32 accumulate), f32 KV",
        "data": "synthetic (seeded random-init weights of the named shape; KV pre-filled N(0,1))",
        "config": {"workload": wl["name"], "model": args.workload, "global_batch": 1, "seq_len": S_mid,
                   "kv_prefill": kv0, "parallelism": "tp%d" % world,
                   "l2": "inputs larger than L2 (weights %.2f GB + KV %.2f GB per token)" % (w_bytes / 1e9,
                                                                                              kv_bytes / 1e9)},
        "roofline": {"bound": "hbm", "kernel": "gemv_tma_kernel (all Q4 GEMVs of one decode step)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_unit": "bytes per launch",
                     "algorithmic_bytes_per_launch": round(gemv_bytes_step / gemv_launches), "peak_source": peak_src,
                     "gemv_launches_per_step": gemv_launches, "gemv_bytes_per_step": gemv_bytes_step,
                     "per_kernel_ms": {k: round(v, 4) for k, v in kind_ms.items()},
                     "step_algorithmic_bytes": tot_bytes, "step_achieved_gbs": round(step_gbs, 1),
                     "step_frac": round(step_gbs / peak, 4)},
        "e2e": {"value": round(e2e_val, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 8},
        "gpu_launches": world * kernels_step * K,
        "clocks": clk.summary(),
    }
    if world == 1 and args.workload == "8b" and not args.layers and not args.no_prefill:
        m.close()
        out["prefill"] = run_prefill(L, ctx, args)
        m = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n_cpu = 2 if args.workload != "70b" else 1
        v, cores, times = cpu_baseline(wl, n_cpu)
        out["cpu_baseline"] = {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                               "sample": "%d decode tokens of the same model at KV %d (median of %s s)" %
                                         (n_cpu, kv0 + 1, [round(t, 2) for t in times])}
    if m is not None:
        m.close()
    ctx.close()
    return out


def prefill_reference(args):
    if args.workload != "8b" or args.no_prefill:
        return None
    v, cores, t = cpu_prefill_baseline()
    return {"metric": "prefill tokens/s", "value": round(v, 3), "unit": "tokens/s", "workload": PREFILL["name"],
            "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": "32-token prompt through 2 of the 32 layers (%.1f s scaled to 32 layers)" % t}}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    wl = WORKLOADS[args.workload]
    n = max(1, min(args.steps, 4 if args.workload != "70b" else 2))
    v, cores, times = cpu_baseline(wl, n)
    return {
        "impl": "reference",
        "metric": "batch-1 greedy decode tokens/s (Llama-3-8B-shaped Q4_0, KV 4096)" if args.workload == "8b"
        else "batch-1 greedy decode tokens/s (%s)" % wl["name"],
        "value": round(v, 3), "unit": "tokens/s", "n_gpus": world, "steps": n, "warmup": 1,
        "ms_per_step": round(1000.0 / v, 2), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4_0 x q8_0 (int8 dot, f32 accumulate), f32 KV",
        "data": "synthetic (seeded random-init weights; KV pre-filled N(0,1))",
        "config": {"workload": wl["name"], "model": args.workload, "kv_prefill": wl["kv"],
                   "parallelism": "cpu (rayon-equivalent OpenMP over 512-row chunks)"},
        "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": "%d decode tokens at KV %d; reference CPU path restated in C (oracle/), "
                                   "Rust reference not buildable here" % (n, wl["kv"] + 1)},
        "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "prefill": prefill_reference(args),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="8b")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill leg")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the config-4 prefill leg (with --layers: a small case for ncu; not a bench line)")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (small cases for ncu captures; not a bench line)")
    args = ap.parse_args()
    assert args.warmup >= 3, "at least 3 warm-up steps"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    if args.prefill_only:
        L = load_pkg()
        ctx = L.Context(int(os.environ.get("LOCAL_RANK", "0")))
        out = run_prefill(L, ctx, args)
        ctx.close()
    elif args.impl == "reference":
        out = run_reference(args, rank, world)
    else:
        out = run_ours(args, rank, world)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and out is not None:
        print(json.dumps(out))


if __name__ == "__main__":
    main()

"""Benchmark: batch-1 greedy decode tokens/s of the Llama-3-8B-shaped Q4_0 model
(config 3: KV cache pre-filled to 4096 positions) on B200, plus % of the HBM
roofline, the end-to-end rate through the C ABI, and the CPU oracle baseline.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                [--workload 8b|1b|70b] [--no-extra] [--no-prefill] [--no-cpu]

One "step" = one greedy decode token through every layer + LM head.  Inputs
(weights 4.2 GB, KV 1.1 GB) are far larger than the 126 MB L2, so no flush is
needed between steps.  Synthetic seeded weights stand in for checkpoints.

On one GPU the line also carries, each as its own record:
  "gemv_sweep"  config 2: GB/s of the batch-1 Q4_0 GEMV on the six sweep
                shapes, back-to-back launches in one CUDA graph over weight
                copies that together exceed the L2 (every launch streams from HBM);
  "configs"     config 1 (1B shape, 32-token prompt + 128 greedy steps) and
                config 5 (70B shape, KV 2048, 128 greedy steps) on this GPU;
  "prefill"     config 4 (8B shape, Q8_0 linears), a 512-token prompt through
                the tensor-core prefill path, then 64 decode steps.
With N > 1 (torchrun, one rank per GPU) the model is tensor parallel over the N
GPUs: one sequence, the same total work (strong scaling); the roofline's peak
is then the N GPUs' aggregate HBM bandwidth.

Roofline.  "frac" is the dominant kernel family's (the Q4 GEMVs, ~3/4 of the
step): their algorithmic bytes per step / their summed in-graph durations,
taken from the device timeline of graph-launched steps (each kernel's share =
last-CTA end minus the previous kernel's last-CTA end, so the shares add up to
the step).  "step_frac" is the north-star figure: weight + KV bytes per token
/ the step time / the aggregate HBM bandwidth.
"""
import argparse
import json
import os
import platform
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
               kv=4096, steps=256, name="llama3-8b-shaped Q4_0 decode, KV pre-filled to 4096 (config 3)"),
    "1b": dict(cfg=dict(n_layers=16, hidden=2048, n_heads=32, n_kv_heads=8, head_dim=64, ffn=8192,
                        vocab=128256, max_seq=256, rms_eps=1e-5, rope_theta=500000.0, weight_format=0,
                        tied_embeddings=1),
               kv=32, steps=128, name="llama3.2-1b-shaped Q4_0 decode after a 32-token prompt (config 1)"),
    "70b": dict(cfg=dict(n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672,
                         vocab=128256, max_seq=2304, rms_eps=1e-5, rope_theta=500000.0, weight_format=0,
                         tied_embeddings=0),
                kv=2048, steps=128, name="llama3-70b-shaped Q4_0 decode, KV pre-filled to 2048 (config 5)"),
}
SEED = 0x5EED

# config 4: the 8B shape with Q8_0 linears, prefill of a 512-token prompt + 64 decode steps
PREFILL = dict(cfg=dict(n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
                        max_seq=640, rms_eps=1e-5, rope_theta=500000.0, weight_format=1, tied_embeddings=0),
               n=512, decode=64, name="llama3-8b-shaped Q8_0 prefill of a 512-token prompt + 64 decode steps (config 4)")

# config 2: the GEMV sweep (out x in)
SWEEP = [(2048, 2048), (8192, 2048), (2048, 8192), (14336, 4096), (4096, 14336), (128256, 4096)]

# DRAM bytes per launch of each decode-step GEMV of the 8B shape, from one ncu
# capture of a 2-layer model (dram__bytes_read.sum + dram__bytes_write.sum).
MEASURED_GEMV_DRAM_8B = {"qkv_gemv": 14.27e6, "o_gemv": 9.54e6, "gate_up_gemv": 66.18e6, "down_gemv": 33.18e6,
                         "lm_head_gemv": 296.07e6}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", 6650.0)), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback (6.65 TB/s)"


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


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


# ----------------------------------------------------------- byte accounting
def linear_shapes(c, tp=1):
    """(N, K) of every quantised linear read per decode token by one rank (native GQA)."""
    D, H, F = c["head_dim"], c["hidden"], c["ffn"] // tp
    hq, hkv = c["n_heads"] // tp, c["n_kv_heads"] // tp
    qkv = ((hq + 2 * hkv) * D, H)
    per_layer = [qkv, (H, hq * D), (2 * F, H), (H, F)]
    return per_layer * c["n_layers"] + [(c["vocab"] // tp, H)]


def q_bytes(n, k, c):
    # Q4: nibbles + fp16 scale = 18 B per 32 weights (Q8_0: 34 B)
    if c["weight_format"] == 1:
        return n * k * 34 // 32
    return n * k * 18 // 32


def algo_bytes_per_token(c, S, tp=1):
    """Weight + KV (+ norms, embedding row) bytes of one decode token over all ranks."""
    w = sum(q_bytes(n, k, c) for n, k in linear_shapes(c, tp)) * tp
    if c["tied_embeddings"]:
        w += c["vocab"] * c["hidden"] // 16  # f32 instead of f16 scales on the tied head
    kv = 2 * c["n_layers"] * c["n_kv_heads"] * c["head_dim"] * S * 4
    norms = (2 * c["n_layers"] + 1) * c["hidden"] * 4
    emb = c["hidden"] * 4
    return w + kv + norms + emb, w, kv


def gemv_bytes(kind, c, tp=1):
    """Algorithmic bytes of one launch of a decode-step GEMV on one rank."""
    D, H, F, V = c["head_dim"], c["hidden"], c["ffn"] // tp, c["vocab"] // tp
    hq, hkv = c["n_heads"] // tp, c["n_kv_heads"] // tp
    n, k = {"qkv_gemv": ((hq + 2 * hkv) * D, H), "o_gemv": (H, hq * D),
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
_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown"}


class ClockSampler:
    """SM clock and clock-event reasons of this process's GPU, sampled every
    ~1 ms through NVML (the source nvidia-smi reads) while the timed region
    runs; falls back to `nvidia-smi -lms 50` without NVML."""

    def __init__(self, cuda_device):
        self.cuda_device = cuda_device
        self.sm, self.reasons, self.power = [], set(), []
        self.max_mhz = None
        self.source = None
        self._stop = threading.Event()
        self._t = None
        self._proc = None
        self._lines = []

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:  # NVML numbers GPUs without CUDA_VISIBLE_DEVICES: go by PCI bus id
            import torch
            pr = torch.cuda.get_device_properties(self.cuda_device)
            bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.cuda_device)

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            get_r = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons

            def run():
                while not self._stop.is_set():
                    try:
                        self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                        r = int(get_r(h))
                        for bit, name in _REASONS.items():
                            if r & bit:
                                self.reasons.add(name)
                    except Exception:
                        pass
                    time.sleep(0.001)

            self._t = threading.Thread(target=run, daemon=True)
            self._t.start()
            self.source = "nvml, ~1 ms"
            t_end = time.time() + 2.0
            while not self.sm and time.time() < t_end:
                time.sleep(0.001)
            self.sm.clear()
            self.reasons.clear()
        except Exception:
            self._smi_start()
        return self

    def _smi_start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self._proc = subprocess.Popen(["nvidia-smi", "-i", str(self.cuda_device), "--query-gpu=" + q,
                                           "--format=csv,noheader,nounits", "-lms", "50"],
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)

            def read():
                for line in self._proc.stdout:
                    self._lines.append(line.strip())

            self._t = threading.Thread(target=read, daemon=True)
            self._t.start()
            t_end = time.time() + 5.0
            while not self._lines and time.time() < t_end:
                time.sleep(0.01)
            self._lines.clear()
            self.source = "nvidia-smi -lms 50"
        except Exception:
            self._proc = None

    def __exit__(self, *a):
        self._stop.set()
        if self._proc:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except Exception:
                self._proc.kill()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for ln in self._lines:
                f = [x.strip() for x in ln.split(",")]
                if len(f) < 9:
                    continue
                try:
                    self.sm.append(float(f[1]))
                    self.max_mhz = float(f[2])
                except ValueError:
                    continue
                for name, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        self.reasons.add(name)
        elif self._t:
            self._t.join(timeout=1.0)

    def summary(self):
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": self.source}


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


# ------------------------------------------------------------ in-graph shares
def in_graph_ms(m, tok, pos, reps=3):
    """Per kernel kind: summed in-graph duration (ms) per step and launches per
    step, from the device timeline of `reps` traced, graph-launched steps."""
    acc, counts = {}, {}
    for r in range(reps):
        tr = m.trace_decode(tok, pos + r)
        prev = tr[0][1]
        per = {}
        for (kind, start, go, ready, end) in tr:
            per[kind] = per.get(kind, 0) + (end - prev)
            prev = end
            if r == 0:
                counts[kind] = counts.get(kind, 0) + 1
        for k, v in per.items():
            acc.setdefault(k, []).append(v / 1e6)
    return {k: statistics.median(v) for k, v in acc.items()}, counts


def decode_record(L, ctx, wl, c, rank, world, K, W, clock_device, with_trace=True, prompt=False):
    """Time K graph-launched decode steps of workload `wl` (after W warm-up
    steps), plus the in-graph kernel shares and the roofline fractions.  The
    KV cache holds wl["kv"] positions: pre-filled with N(0,1) rows, or (prompt)
    written by a prefill of a wl["kv"]-token prompt."""
    m = L.Model(ctx, dict(c, tp_rank=rank, tp_size=world))
    m.init_synthetic(SEED)
    if world > 1:
        L.connect_tensor_parallel(m)
    kv0 = wl["kv"]
    if prompt:
        tok0, _ = m.prefill(prefill_prompt(c, kv0), 0, want_logits=False)
    else:
        m.kv_fill_synthetic(SEED, kv0)
        tok0 = 1234 % c["vocab"]
    assert kv0 + max(K, W) + 8 <= c["max_seq"], "steps exceed the KV capacity"
    m.time_decode(tok0, kv0, W)  # warm-up (also captures the step graph)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    with ClockSampler(clock_device) as clk:
        ms = m.time_decode(tok0, kv0, K)
    if dist is not None:
        import torch
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    rec = {"m": m, "ms": ms, "kv0": kv0, "tok0": tok0, "clocks": clk.summary()}
    if with_trace:
        kind_ms, counts = in_graph_ms(m, tok0, kv0)
        if world > 1:
            import torch
            names = sorted(kind_ms)
            t = torch.tensor([kind_ms[k] for k in names], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            kind_ms = {k: float(v) for k, v in zip(names, t.tolist())}
        rec["kind_ms"], rec["counts"] = kind_ms, counts
    return rec


def roofline(c, wl, rec, K, world, peak_gbs, peak_src, traffic=None):
    ms_per_step = rec["ms"] / K
    S_mid = rec["kv0"] + K // 2
    tot_bytes, w_bytes, kv_bytes = algo_bytes_per_token(c, S_mid, world)
    step_gbs = tot_bytes / (ms_per_step / 1000.0) / 1e9
    peak = peak_gbs * world
    out = {"bound": "hbm", "unit": "GB/s", "peak": round(peak, 1), "peak_source": peak_src,
           "step_algorithmic_bytes": tot_bytes, "step_achieved_gbs": round(step_gbs, 1),
           "step_frac": round(step_gbs / peak, 4),
           "step_frac_definition": "weight + KV (+ norms, embedding row) bytes per token / ms_per_step / "
                                   "aggregate HBM bandwidth of the n_gpus"}
    if "kind_ms" in rec:
        kind_ms, counts = rec["kind_ms"], rec["counts"]
        gemv = [k for k in kind_ms if k.endswith("_gemv")]
        g_bytes = sum(gemv_bytes(k, c, world) * counts[k] for k in gemv) * world
        g_ms = sum(kind_ms[k] for k in gemv)
        launches = sum(counts[k] for k in gemv)
        achieved = g_bytes / (g_ms / 1000.0) / 1e9
        att_bytes = 2 * c["n_layers"] * c["n_kv_heads"] * c["head_dim"] * (rec["kv0"] + 1) * 4
        out.update({
            "kernel": "gemv_tma_kernel (every Q4 GEMV of a decode step)",
            "achieved": round(achieved, 1), "frac": round(achieved / peak, 4),
            "frac_definition": "GEMV algorithmic bytes per step / the GEMVs' summed in-graph durations "
                               "(device timeline of graph-launched steps) / aggregate HBM bandwidth",
            "traffic": traffic, "traffic_unit": "DRAM bytes per GEMV launch (ncu)",
            "algorithmic_bytes_per_launch": round(g_bytes / world / launches),
            "gemv_launches_per_step": launches, "gemv_bytes_per_step": g_bytes,
            "in_graph_ms_per_step": {k: round(v, 4) for k, v in sorted(kind_ms.items())},
            "in_graph_sum_ms": round(sum(kind_ms.values()), 4),
            "attention_achieved_gbs": round(att_bytes / (kind_ms["attention"] / 1000.0) / 1e9, 1)
            if "attention" in kind_ms else None,
        })
    return out


def run_gemv_sweep(L, ctx, reps=20):
    """Config 2: device us per launch and GB/s of the Q4_0 x Q8_0 GEMV, every
    launch streaming its own weight copy from HBM (copies >= 2x the L2)."""
    import torch
    dev = torch.device("cuda", ctx.device)
    peak, _ = load_peaks()
    out = {}
    for n, k in SWEEP:
        wb = n * k // 2 + n * (k // 32) * 2
        copies = max(2, min(256, -(-(256 << 20) // wb)))
        codes = [torch.randint(0, 256, (n * k // 2,), dtype=torch.uint8, device=dev) for _ in range(copies)]
        scl = [(torch.rand(n * (k // 32), device=dev) * 0.004 + 1e-4).half() for _ in range(copies)]
        x = torch.randn(k, device=dev)
        y = torch.empty(n, device=dev)
        us = L.time_gemv(ctx, [t.data_ptr() for t in codes], [t.data_ptr() for t in scl], x.data_ptr(),
                         y.data_ptr(), n, k, reps)
        by = n * k * 18 // 32 + 4 * k + 4 * n
        out["%dx%d" % (n, k)] = {"us_per_launch": round(us, 3), "algorithmic_bytes": by,
                                 "gbs": round(by / (us * 1e-6) / 1e9, 1), "frac": round(by / (us * 1e-6) / 1e9 / peak, 4),
                                 "weight_copies": copies}
        del codes, scl
        torch.cuda.empty_cache()
    return {"metric": "batch-1 Q4_0 GEMV effective GB/s (config 2)",
            "method": "llmrs_time_gemv: back-to-back launches in one CUDA graph with programmatic overlap, each "
                      "on its own weight copy (copies together >= 256 MB > L2), %d graph replays" % reps,
            "peak_gbs": peak, "shapes": out}


def run_prefill(L, ctx, args):
    c = dict(PREFILL["cfg"])
    if args.layers:
        c["n_layers"] = args.layers
    n = PREFILL["n"]
    m = L.Model(ctx, dict(c, scale_dtype=L.F16))
    m.init_synthetic(SEED)
    ids = prefill_prompt(c, n)
    m.time_prefill(ids, 0, args.warmup)  # warm-up
    with ClockSampler(ctx.device) as clk:
        ms = m.time_prefill(ids, 0, max(1, min(args.steps, 10)))
    e2e = []
    for _ in range(3):
        t0 = time.perf_counter()
        m.prefill(ids, 0, want_logits=True)
        e2e.append(time.perf_counter() - t0)
    # the 64 decode steps that follow the prompt (config 4), device-timed
    tok, _ = m.prefill(ids, 0, want_logits=False)
    dms = m.time_decode(tok, n, PREFILL["decode"])
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
           "decode_after_prompt": {"steps": PREFILL["decode"], "tokens_per_s": round(PREFILL["decode"] / (dms / 1000.0), 1)},
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
                               "cpu": cpu_model(),
                               "sample": "32-token prompt through 2 of the 32 layers (%.1f s scaled to 32 layers)" % t}
    return out


def run_config(L, ctx, name, peak, peak_src, args):
    """One N=1 sub-record: decode tokens/s of another config on this GPU."""
    wl = WORKLOADS[name]
    c = dict(wl["cfg"])
    K = wl["steps"]
    rec = decode_record(L, ctx, wl, c, 0, 1, K, max(3, args.warmup), ctx.device, prompt=name == "1b")
    m = rec["m"]
    toks = m.generate(rec["tok0"], rec["kv0"], 8)  # the greedy loop on the device
    m.close()
    return {"metric": "batch-1 greedy decode tokens/s", "workload": wl["name"], "value": round(K / (rec["ms"] / 1000.0), 2),
            "unit": "tokens/s", "steps": K, "ms_per_step": round(rec["ms"] / K, 4),
            "roofline": roofline(c, wl, rec, K, 1, peak, peak_src), "clocks": rec["clocks"],
            "greedy_tokens_sample": [int(t) for t in toks]}


# ------------------------------------------------------------------ our arm
def run_ours(args, rank, world):
    L = load_pkg()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    wl = WORKLOADS[args.workload]
    c = dict(wl["cfg"])
    if args.layers:
        c["n_layers"] = args.layers
    ctx = L.Context(local)
    K, W = args.steps, args.warmup
    rec = decode_record(L, ctx, wl, c, rank, world, K, W, local)
    m = rec["m"]
    ms = rec["ms"]
    ms_per_step = ms / K
    value = K / (ms / 1000.0)  # one sequence decoded by all ranks together
    traffic = None
    if args.workload == "8b" and not args.layers and world == 1:
        counts = rec["counts"]
        gk = [k for k in counts if k.endswith("_gemv")]
        traffic = round(sum(MEASURED_GEMV_DRAM_8B[k] * counts[k] for k in gk) / sum(counts[k] for k in gk))
    peak, peak_src = load_peaks()
    roof = roofline(c, wl, rec, K, world, peak, peak_src, traffic)
    # end to end through the C ABI: token in from host memory, argmax (+err word) back
    kv0, tok0 = rec["kv0"], rec["tok0"]
    E = min(K, 64)
    m.decode_step(tok0, kv0, want_logits=False)
    t0 = time.perf_counter()
    tok = tok0
    for i in range(E):
        tok, _ = m.decode_step(tok, kv0 + i, want_logits=False)
    e2e_s = time.perf_counter() - t0
    ranks = [{"rank": rank, "local_rank": local, "device": local}]
    if world > 1:
        import torch
        import torch.distributed as dist
        t = torch.tensor([e2e_s], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
        try:
            name = torch.cuda.get_device_properties(local).name
            pr = torch.cuda.get_device_properties(local)
            bus = "%04x:%02x:%02x" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        except Exception:
            name, bus = None, None
        mine = {"rank": rank, "local_rank": local, "device": local, "gpu": name, "pci": bus,
                "tp_connected": True, "host": platform.node()}
        ranks = [None] * world
        dist.all_gather_object(ranks, mine)
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
        "config": {"workload": wl["name"], "model": args.workload, "global_batch": 1,
                   "seq_len": kv0 + K // 2, "kv_prefill": kv0, "parallelism": "tp%d" % world,
                   "l2": "inputs larger than L2, no flush (%.2f GB read per token)" % (roof["step_algorithmic_bytes"] / 1e9)},
        "roofline": roof,
        "e2e": {"value": round(e2e_val, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 8, "api": "llmrs_decode_step (token in, argmax + error word out)"},
        "gpu_launches": world * kernels_step * K,
        "kernels_per_step_per_rank": kernels_step,
        "ranks": ranks,
        "clocks": rec["clocks"],
    }
    m.close()
    if world == 1 and not args.layers and not args.no_extra and args.workload == "8b":
        out["gemv_sweep"] = run_gemv_sweep(L, ctx)
        out["configs"] = {"config1_1b": run_config(L, ctx, "1b", peak, peak_src, args),
                          "config5_70b": run_config(L, ctx, "70b", peak, peak_src, args)}
        if not args.no_prefill:
            out["prefill"] = run_prefill(L, ctx, args)
    if rank == 0 and world == 1 and not args.no_cpu:
        n_cpu = 24 if args.workload != "70b" else 2
        v, cores, times = cpu_baseline(wl, n_cpu)
        out["cpu_baseline"] = {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                               "cpu": cpu_model(),
                               "sample": "%d decode tokens of the same model at KV %d.. (median of %.1f s of work)" %
                                         (n_cpu, kv0 + 1, sum(times))}
    ctx.close()
    return out


def prefill_reference(args):
    if args.workload != "8b" or args.no_prefill:
        return None
    v, cores, t = cpu_prefill_baseline()
    return {"metric": "prefill tokens/s", "value": round(v, 3), "unit": "tokens/s", "workload": PREFILL["name"],
            "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "cpu": cpu_model(),
                             "sample": "32-token prompt through 2 of the 32 layers (%.1f s scaled to 32 layers)" % t}}


def run_reference(args, rank, world):
    """The reference's CPU path (restated in C, oracle/) on the host cores:
    the Rust reference cannot be built here (no Rust toolchain)."""
    if rank != 0:
        return None
    wl = WORKLOADS[args.workload]
    n = max(1, min(args.steps, 32 if args.workload != "70b" else 2))
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
        "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
                         "sample": "%d decode tokens at KV %d..; reference CPU path restated in C (oracle/), "
                                   "Rust reference not buildable here (%.1f s of work)" % (n, wl["kv"] + 1, sum(times))},
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
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill record")
    ap.add_argument("--no-extra", action="store_true", help="skip the sweep, config-1/5 and prefill records")
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

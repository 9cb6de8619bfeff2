#!/usr/bin/env python
"""Benchmark of the FP8 block-scaled matmul path (qwen35-c's q35_mm.c) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (``value``): benchmark configuration 3 -- one full
64-layer FP8 decode weight stream (48 Gated-DeltaNet + 16 GQA layers, the
configuration-2 projection shapes plus the MLP in every layer, 24.33 GB of
FP8 weights), one token, tensor-parallel over the N GPUs (column-parallel +
all-gather, row-parallel + all-reduce), captured in one CUDA graph (or run as
one cooperative launch) per rank.  ``value`` = weight bytes streamed by all
ranks / step time (GB/s), ``ms_per_step`` = ms per decode token.  Inputs are
resident in HBM; the weights (24.33 GB / N per GPU) are far larger than L2,
so every step reads them from DRAM.

Also on the same line: the live roofline of the dominant kernel; the
end-to-end figure through the reference-facing C-ABI with host buffers; and,
each measured in a child process of its own so that a failure there cannot
take the headline with it (its key then holds {"error": ...}):
configuration 0 (the isolated decode GEMV), the configuration-1 sweep, the
bf16 lm_head matvec, configuration 2 (one layer's prefill GEMMs at M=2048),
configuration 4 (M=8192 prefill through the projection set, under TP at
N>1) and the CPU baseline (the reference's own q35_mm.c on the host cores,
the full 64-layer stream).

``--impl reference`` runs the reference's CPU implementation
(oracle/_ref/libq35ref.so, qwen35-c/src/q35_mm.c compiled unmodified) over
the same 64-layer stream, K timed steps after W warm-up steps.

For N > 1 launch with torchrun (one process per GPU, rendezvous on
127.0.0.1); rank 0 prints the single JSON line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "qwen38-in-c_b200"))

METRIC = "FP8 decode GEMV HBM GB/s (% peak); prefill GEMM TFLOP/s; 64-layer ms/token"
HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0
EXTRAS = ("c0", "c1", "lm_head", "c2", "c4", "cpu", "out_batch")


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=64, help="decode-stack depth (64 = configuration 3)")
    ap.add_argument("--no-extras", action="store_true", help="skip the extras, e2e and the CPU baseline")
    ap.add_argument("--extra", choices=EXTRAS, default=None,
                    help="run one extra measurement and print its JSON (the child-process mode)")
    ap.add_argument("--cpu-steps", type=int, default=3, help="timed steps of the CPU baseline (our arm)")
    ap.add_argument("--profile-c0", action="store_true",
                    help="only the isolated configuration-0 GEMV (a small command for ncu captures)")
    ap.add_argument("--profile-c2", action="store_true",
                    help="only the configuration-2 gate projection at M=2048 through the GEMM (for ncu captures)")
    ap.add_argument("--profile-c1-tc", type=int, default=0, metavar="M",
                    help="only one projection (--profile-shape, default 17408x5120) at M tokens through the "
                         "tensor cores on exact activations (q35cu_gemv_fp8_tc), --steps calls (for ncu captures)")
    ap.add_argument("--profile-shape", default="17408x5120", metavar="ROWSxCOLS",
                    help="the projection shape of --profile-c1-tc")
    ap.add_argument("--profile-lm-head", type=int, default=0, metavar="ROWS",
                    help="only the bf16 lm_head matvec on ROWS x 5120, --steps calls (for ncu captures)")
    return ap.parse_args(argv)


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", HBM_FALLBACK_GBS), d.get("bf16_tflops", BF16_FALLBACK_TFLOPS), d.get(
            "bf16_tflops_sustained", BF16_FALLBACK_TFLOPS), "measured"
    return HBM_FALLBACK_GBS, BF16_FALLBACK_TFLOPS, BF16_FALLBACK_TFLOPS, "fallback"


class Clocks:
    """SM clock, power and clock-event reasons of one GPU, sampled every 10 ms
    by NVML in a thread while the timed region runs (nvidia-smi -lms 200 as a
    fallback when NVML is unavailable).  Only reads the settings."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.thread = None
        self.samples = []
        self.stop_ev = threading.Event()
        self.nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            h = None
            try:
                import torch

                bus = torch.cuda.get_device_properties(index).pci_bus_id
                h = pynvml.nvmlDeviceGetHandleByPciBusId(("%08x:%02x:%02x.0" % (
                    torch.cuda.get_device_properties(index).pci_domain_id, bus,
                    torch.cuda.get_device_properties(index).pci_device_id)).encode())
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.nvml = (pynvml, h)
        except Exception:
            self.nvml = None

    def _poll(self):
        nv, h = self.nvml
        while not self.stop_ev.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((sm, mx, pw, rs))
            except Exception:
                pass
            self.stop_ev.wait(0.01)

    def start(self):
        if self.nvml:
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.thread:
            self.stop_ev.set()
            self.thread.join(timeout=5)
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "source": "nvml"}
            reasons = sorted({n for _, _, _, r in self.samples for n, bit in self.REASONS if r & bit})
            return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                    "sm_max_mhz": max(s[1] for s in self.samples), "reasons": reasons,
                    "samples": len(self.samples), "power_w_max": round(max(s[2] for s in self.samples), 1),
                    "source": "nvml, every 10 ms during the timed region"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons, pw = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [t.strip() for t in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                pw.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(pw) if pw else None, "source": "nvidia-smi -lms 200"}


# ---------------------------------------------------------------------------
# the reference arm / CPU baseline: qwen35-c's q35_mm.c on the host cores
# ---------------------------------------------------------------------------
def cpu_info() -> dict:
    """The host CPU as this process sees it: model, the logical CPUs it may
    run on, and how many physical cores those are (SMT siblings counted once;
    the reference's own thread heuristic is 5/3 x physical cores,
    qwen35-c/src/cli/cli_common.c:98-104)."""
    allowed = os.sched_getaffinity(0)
    model, phys, per_core = None, set(), {}
    try:
        with open("/proc/cpuinfo") as f:
            for rec in f.read().split("\n\n"):
                d = {}
                for line in rec.splitlines():
                    if ":" in line:
                        k, v = line.split(":", 1)
                        d[k.strip()] = v.strip()
                if "processor" not in d or int(d["processor"]) not in allowed:
                    continue
                model = model or d.get("model name")
                key = (d.get("physical id"), d.get("core id"))
                phys.add(key)
                per_core[key] = per_core.get(key, 0) + 1
    except OSError:
        pass
    n_phys = len(phys) or None
    return {"model": model, "logical_cpus": len(allowed), "physical_cores": n_phys,
            "smt": bool(per_core) and max(per_core.values()) > 1,
            "heuristic_threads_5_3": (min(len(allowed), n_phys * 5 // 3) if n_phys else None)}


class CpuStream:
    """The 64-layer decode weight stream (configuration 3) in host memory, for
    the reference's CPU matmul.  Layers 0 (DeltaNet) and 3 (GQA) are
    generated with the seeded generator the GPU stack uses (same seeds, same
    N(0, 0.02) 128x128 block quantisation); every other layer holds a
    byte-rotated copy of the weights of its kind (a different rotation per
    layer), so each layer is distinct memory with the same value distribution
    -- the reference's converter speed depends on the bytes, not on which
    values sit where.  24.33 GB of FP8 weights in all."""

    def __init__(self, n_layers: int = 64):
        import numpy as np

        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle  # noqa: F401  (test infrastructure: the CPU baseline / reference arm only)
        import stack

        self.orc = oracle.Oracle()
        base = {}
        for layer, kind in ((0, "dn"), (3, "gqa")):
            ws = {}
            for name, rows in (stack.DN_COL if kind == "dn" else stack.GQA_COL):
                ws[name] = self.orc.synth_fp8(stack.seed_of(layer, name), rows, stack.HIDDEN)
            ao = "out" if kind == "dn" else "o"
            ws[ao] = self.orc.synth_fp8(stack.seed_of(layer, ao), stack.HIDDEN, stack.OUT_K)
            ws["gate"] = self.orc.synth_fp8(stack.seed_of(layer, "gate"), stack.MLP, stack.HIDDEN)
            ws["up"] = self.orc.synth_fp8(stack.seed_of(layer, "up"), stack.MLP, stack.HIDDEN)
            ws["down"] = self.orc.synth_fp8(stack.seed_of(layer, "down"), stack.HIDDEN, stack.MLP)
            base[kind] = ws
        self.layers = []
        for i, kind in enumerate(stack.layer_kinds(n_layers)):
            if i in (0, 3):
                self.layers.append((kind, base[kind]))
                continue
            rot = {}
            for j, (name, (W, sc)) in enumerate(base[kind].items()):
                shift = (i * 7919 + j * 104729) % W.size
                rot[name] = (np.roll(W.reshape(-1), shift).reshape(W.shape), sc)
            self.layers.append((kind, rot))
        self.x = self.orc.synth_act(77, (n_layers, stack.HIDDEN))
        self.weight_bytes = sum(W.nbytes for _, ws in self.layers for W, _ in ws.values())

    def step(self, mm_fp8, mm_multi4) -> None:
        """One decode step: every layer's projections in the engine's order
        (q35_deltanet.c:329,360 / q35_attn.c:273-275,262 / q35_model.c:934,937)."""
        import stack

        for i, (kind, ws) in enumerate(self.layers):
            names = [n for n, _ in (stack.DN_COL if kind == "dn" else stack.GQA_COL)]
            outs = mm_multi4([ws[n][0] for n in names], [ws[n][1] for n in names], self.x[i])[: len(names)]
            src = outs[-1] if kind == "dn" else outs[0]
            ao = ws["out" if kind == "dn" else "o"]
            o = mm_fp8(ao[0], ao[1], src[: stack.OUT_K].copy())
            g, _ = mm_multi4([ws["gate"][0], ws["up"][0]], [ws["gate"][1], ws["up"][1]], o)[:2]
            mm_fp8(ws["down"][0], ws["down"][1], g)


def time_cpu_stream(steps: int, warmup: int) -> dict:
    """The reference q35_mm.c (oracle/_ref, AVX2 + FMA + OpenMP, every host
    CPU this process may use; the oracle port if _ref was not built) over
    the full 64-layer stream: `warmup` untimed steps, then `steps` timed ones
    (wall clock, their mean)."""
    import stack

    t_setup = time.perf_counter()
    cs = CpuStream()
    setup_s = time.perf_counter() - t_setup
    import oracle

    if oracle.Reference.available():
        R = oracle.Reference()
        kind = "reference"
        mm_fp8, mm_multi4 = R.mm_fp8, R.mm_fp8_multi4
    else:
        kind = "port"
        mm_fp8 = cs.orc.mm_fp8

        def mm_multi4(Ws, Ss, xx):
            return [cs.orc.mm_fp8(w, s, xx) for w, s in zip(Ws, Ss)]
    for _ in range(warmup):
        cs.step(mm_fp8, mm_multi4)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        cs.step(mm_fp8, mm_multi4)
        times.append(time.perf_counter() - t0)
    step_s = sum(times) / len(times)
    info = cpu_info()
    return {
        "value": stack.weight_bytes() / step_s / 1e9, "unit": "GB/s", "cores": cs.orc.threads(), "kind": kind,
        "ms_per_step": step_s * 1e3, "ms_per_step_min": min(times) * 1e3, "steps": steps, "warmup": warmup,
        "sample": f"the full {len(cs.layers)}-layer decode weight stream per step ({cs.weight_bytes / 1e9:.2f} GB "
                  f"FP8, 256 q35_mm_fp8 / q35_mm_fp8_multi4 calls), mean of {steps} timed steps after {warmup} "
                  f"warm-up; {cs.orc.threads()} OpenMP threads",
        "impl": "q35_mm.c compiled -O2 -mavx2 -mfma -fopenmp" if kind == "reference" else "oracle C port",
        "cpu": info, "setup_s": round(setup_s, 1),
    }


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cb = time_cpu_stream(args.steps, args.warmup)
    line = {
        "metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": cb["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (FP8 e4m3 weights, bf16 scales)",
        "data": "synthetic (seeded N(0,0.02) weights, 128x128 block-quantised; N(0,1) activations)",
        "config": {"workload": "configuration 3: 64-layer FP8 decode weight stream, M=1",
                   "weight_bytes_per_step": __import__("stack").weight_bytes()},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "cpu": cb["cpu"],
        "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def gemv_bytes(rows, cols, m=1):
    return rows * cols + 4 * ((rows + 127) // 128) * ((cols + 127) // 128) + 4 * m * (rows + cols)


def time_gemv_rotating(q35cu, torch, rows, cols, m, copies=5, rounds=20, path="gemv", graph=False):
    """Isolated GEMV: `copies` distinct weights cycled so none is L2-resident.
    path "gemv": the CUDA-core decode GEMV (q35cu_gemv_fp8); "tc": the tensor
    cores with exact fp32 activations (q35cu_gemv_fp8_tc, the path
    q35_mm_fp8_batch takes for 16..127 tokens).  graph: one call per weight
    captured in a CUDA graph and replayed (device time without the Python
    and launch overhead of eager calls)."""
    ws = [q35cu.Weight.synth_fp8(1000 + i, rows, cols) for i in range(copies)]
    try:
        X = torch.randn((m, cols), device="cuda")
        Y = torch.empty((m, rows), device="cuda")
        work = torch.empty(q35cu.load().q35cu_gemv_fp8_tc_workspace_bytes(m, cols), dtype=torch.uint8, device="cuda")

        def call(w, stream=None):
            if path == "tc":
                q35cu.gemv_tc(w, X, Y, work, stream)
            else:
                q35cu.gemv(w, X, Y, m, stream)

        for w in ws:
            call(w)  # eager first: the multi-token path allocates its split scratch here
        torch.cuda.synchronize()
        g = None
        if graph:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    for w in ws:
                        call(w, s)
            torch.cuda.current_stream().wait_stream(s)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(rounds):
            if g is not None:
                g.replay()
            else:
                for w in ws:
                    call(w)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (rounds * copies)
        del g
    finally:
        for w in ws:
            w.free()
    b = gemv_bytes(rows, cols, m)
    return {"rows": rows, "cols": cols, "m": m, "path": path, "timing": "cuda graph" if graph else "eager",
            "us": round(us, 2), "GBps": round(b / us / 1e3, 1), "TFLOPs": round(2 * m * rows * cols / us / 1e6, 3)}


def bf16_weight(q35cu, torch, rows, cols, seed=4242):
    """A bf16 [rows, cols] weight of N(0, 0.02) values, uploaded through
    q35cu_weight_upload_bf16 (the lm_head operand of q35_mm_bf16)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = (torch.randn((rows, cols), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    host = dev.view(torch.int16).cpu().numpy().view("uint16")
    del dev
    return q35cu.Weight.upload_bf16(host)


def time_lm_head(q35cu, torch, hbm_peak, rows=248320, cols=5120, reps=20):
    """The bf16 lm_head matvec (q35_mm_bf16 on a device-resident weight,
    q35cu_gemv_bf16): 2.5 GB per call, larger than L2; CUDA events per call."""
    w = bf16_weight(q35cu, torch, rows, cols)
    try:
        x = torch.randn(cols, device="cuda")
        y = torch.empty(rows, device="cuda")
        for _ in range(3):
            q35cu.gemv_bf16(w, x, y)
        torch.cuda.synchronize()
        us = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            q35cu.gemv_bf16(w, x, y)
            b.record()
            torch.cuda.synchronize()
            us.append(a.elapsed_time(b) * 1e3)
    finally:
        w.free()
    us.sort()
    med = us[len(us) // 2]
    by = 2 * rows * cols + 4 * cols + 4 * rows  # weight + x + y
    return {"rows": rows, "cols": cols, "kernel": "gemv_tma_kernel<bf16>", "us_median": round(med, 2),
            "us_min": round(us[0], 2), "GBps": round(by / med / 1e3, 1), "frac_of_measured_hbm": round(by / med / 1e3 / hbm_peak, 4)}


def kernel_roofline(q35cu, torch, st, hbm_peak, reps=3):
    """Per-launch CUDA-event timing of every GEMV launch of one step (no
    collectives), on the stream they run on; sum of algorithmic bytes / sum of
    launch durations."""
    stream = torch.cuda.current_stream()
    launches, labels = [], []
    for L in st.layers:
        launches.append(("multi", [p.w for p in L.col_in]))
        labels.append("qkv+z" if L.kind == "dn" else "q+k+v")
        launches.append(("gemv", L.attn_out.w))
        labels.append("out" if L.kind == "dn" else "o")
        launches.append(("multi", [L.gate.w, L.up.w]))
        labels.append("gate+up")
        launches.append(("gemv", L.down.w))
        labels.append("down")
    total_bytes = 0
    for kind, w in launches:
        ws = w if kind == "multi" else [w]
        for ww in ws:
            total_bytes += gemv_bytes(ww.rows, ww.cols)
    xs = torch.randn((stack_max_cols(st),), device="cuda")
    ybuf = torch.empty((40000,), device="cuda")
    durs = []
    per = {}
    for _ in range(reps):
        evs = []
        for kind, w in launches:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            if kind == "multi":
                outs, off = [], 0
                for ww in w:
                    outs.append(ybuf[off:off + ww.rows])
                    off += ww.rows
                q35cu.multi(w, xs[: w[0].cols], outs, 1)
            else:
                q35cu.gemv(w, xs[: w.cols], ybuf[: w.rows], 1)
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
        ts = [a.elapsed_time(b) * 1e-3 for a, b in evs]
        durs.append(sum(ts))
        for (kind, w), lab, dt in zip(launches, labels, ts):
            ws = w if kind == "multi" else [w]
            by = sum(gemv_bytes(ww.rows, ww.cols) for ww in ws)
            e = per.setdefault(lab, [0, 0.0, 0])
            e[0] += by
            e[1] += dt
            e[2] += 1
    t = statistics.median(durs)
    ach = total_bytes / t / 1e9
    breakdown = {lab: {"launches_per_step": e[2] // reps, "us": round(e[1] / e[2] * 1e6, 2),
                       "GBps": round(e[0] / e[1] / 1e9, 1)} for lab, e in per.items()}
    return ach, total_bytes / len(launches), t / len(launches), len(launches), breakdown


C2_SHAPES = [("qkv", 10240, 5120), ("z", 6144, 5120), ("out", 5120, 6144), ("q", 12288, 5120),
             ("k", 1024, 5120), ("v", 1024, 5120), ("o", 5120, 6144), ("gate", 17408, 5120),
             ("up", 17408, 5120), ("down", 5120, 17408)]


# projections of one layer that multiply the same activations (DeltaNet
# input, attention input, MLP input); out, o and down each read their own
C2_GROUPS = [("qkv", "z"), ("q", "k", "v"), ("gate", "up"), ("out",), ("o",), ("down",)]


def time_prefill_c2(q35cu, torch, bf16_peak, m=2048, reps=5):
    """Configuration 2: one decoder layer's projections at M=2048 tokens through
    the tensor-core GEMM (device API, bf16-rounded activations resident in HBM)."""
    ws = [(n, q35cu.Weight.synth_fp8(9000 + i, r, c)) for i, (n, r, c) in enumerate(C2_SHAPES)]
    try:
        kmax = max(w.cols for _, w in ws)
        X = torch.randn((m, kmax), device="cuda").to(torch.bfloat16)
        xs = {w.cols: X[:, : w.cols].contiguous() for _, w in ws}
        work = torch.empty(q35cu.gemm_workspace_bytes(m, kmax), dtype=torch.uint8, device="cuda")
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > L2 (126 MB)
        per, tot_f, tot_t = {}, 0.0, 0.0
        for n, w in ws:
            yv = torch.empty((m, w.rows), device="cuda")
            for _ in range(3):  # warm-up
                q35cu.gemm(w, xs[w.cols].view(torch.int16), yv, work)
            torch.cuda.synchronize()
            evs = []
            for _ in range(reps):
                flush.zero_()  # L2 flushed between timed calls
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                q35cu.gemm(w, xs[w.cols].view(torch.int16), yv, work)
                e1.record()
                evs.append((e0, e1))
            torch.cuda.synchronize()
            dt = sum(a.elapsed_time(b) for a, b in evs) * 1e-3 / reps
            fl = 2.0 * m * w.rows * w.cols
            per[n] = {"rows": w.rows, "cols": w.cols, "us": round(dt * 1e6, 1), "TFLOPs": round(fl / dt / 1e12, 1)}
            tot_f += fl
            tot_t += dt
        # the projections that read one input, as one q35cu_gemm_fp8_multi call each
        byname = dict(ws)
        fused, fz_t = {}, 0.0
        for grp in C2_GROUPS:
            gw = [byname[n] for n in grp]
            ys = [torch.empty((m, w.rows), device="cuda") for w in gw]
            x = xs[gw[0].cols].view(torch.int16)
            for _ in range(3):
                q35cu.gemm_multi(gw, x, ys, work)
            torch.cuda.synchronize()
            evs = []
            for _ in range(reps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                q35cu.gemm_multi(gw, x, ys, work)
                e1.record()
                evs.append((e0, e1))
            torch.cuda.synchronize()
            dt = sum(a.elapsed_time(b) for a, b in evs) * 1e-3 / reps
            fl = sum(2.0 * m * w.rows * w.cols for w in gw)
            fused["|".join(grp)] = {"us": round(dt * 1e6, 1), "TFLOPs": round(fl / dt / 1e12, 1)}
            fz_t += dt
        q35cu.check_device_status()
    finally:
        for _, w in ws:
            w.free()
    ach = tot_f / tot_t / 1e12
    fz = tot_f / fz_t / 1e12
    return {"m": m, "flops": tot_f, "ms": round(tot_t * 1e3, 3), "TFLOPs": round(ach, 1),
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": bf16_peak, "unit": "TFLOP/s",
                         "frac": round(ach / bf16_peak, 4),
                         "kernel": ("gemm_prep_kernel + gemm_fp8_tc_kernel (f16 operands)" if os.environ.get("Q35CU_GEMM_F16")
                                    else "gemm_prep_e4m3_kernel + gemm_e4m3_tc_kernel (e4m3 operands)")
                         + " -- one q35cu_gemm_fp8 call, L2 flushed before each",
                         "peak_source": "measured bf16_tflops (burst, MEASURED_PEAKS.json)"},
            "by_projection": per,
            "fused_by_input": {"ms": round(fz_t * 1e3, 3), "TFLOPs": round(fz, 1),
                               "frac": round(fz / bf16_peak, 4),
                               "note": "projections that read the same input in one q35cu_gemm_fp8_multi call "
                                       "(one preparation, one launch over their row blocks); L2 flushed before each",
                               "by_group": fused}}


# ---------------------------------------------------------------------------
# process setup shared by the main run and the child processes
# ---------------------------------------------------------------------------
class Dist:
    """One process per GPU: torch.distributed (NCCL; gloo for host objects),
    the library's NCCL communicator and its NVLink exchange areas."""

    def __init__(self, want_p2p: bool = True):
        import torch
        import torch.distributed as dist

        import q35cu

        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.p2p = False
        torch.cuda.set_device(self.local)
        q35cu.load()
        q35cu.check(q35cu.load().q35cu_set_device(self.local))
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.cpu_group = dist.new_group(backend="gloo")
            uid = [q35cu.nccl_unique_id() if self.rank == 0 else None]
            dist.broadcast_object_list(uid, src=0, group=self.cpu_group)
            q35cu.tp_init(self.rank, self.world, uid[0])
            if want_p2p:
                # the one-shot NVLink collectives: every rank's exchange-area handle
                hs = [None] * self.world
                dist.all_gather_object(hs, q35cu.p2p_handle(), group=self.cpu_group)
                q35cu.p2p_open(self.rank, self.world, hs)
                self.p2p = True

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        import q35cu

        if self.world > 1:
            self.torch.cuda.synchronize()
            self.dist.barrier()
            if self.p2p:
                q35cu.p2p_close()
            q35cu.tp_finalize()
            self.dist.barrier()
            self.dist.destroy_process_group()


def time_config4(d: Dist, bf16_peak, m=8192, reps=3, scheme="literal"):
    """Configuration 4: long prefill (M=8192 tokens) through the 64-layer
    projection set under tensor parallelism, on this rank's shards of a
    4-layer stack (layers 0-2 DeltaNet, layer 3 GQA; every layer of a kind has
    the same shapes).  One DeltaNet and one GQA layer (prefill.PrefillLayers:
    the engine's batch-prefill projection order, every GEMM through
    q35cu_gemm_fp8) are timed with CUDA events (median of `reps`, max over
    ranks) and extrapolated x48 / x16.  The device status word is read after
    the warm-up and after the timed runs, so a wait that gave up is reported
    as such rather than as a wrong number."""
    import q35cu
    import prefill
    import stack

    torch = d.torch
    st = stack.Stack(d.rank, d.world, n_layers=4)
    try:
        pf = prefill.PrefillLayers(st, m=m, scheme=scheme)
        out = {}
        for name, L in (("dn", pf.dn), ("gqa", pf.gqa)):
            pf.layer_reserved(L)  # warm-up
            torch.cuda.synchronize()
            q35cu.check_device_status()
            d.barrier()
            ts = []
            for _ in range(reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                pf.layer_reserved(L)
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            q35cu.check_device_status()
            d.barrier()
            out[name] = d.max_over_ranks(statistics.median(ts))
            out[name + "_flops_rank"] = pf.flops(L)
    finally:
        st.free()
    kinds = stack.layer_kinds()
    n_dn = sum(1 for k in kinds if k == "dn")
    n_gqa = len(kinds) - n_dn
    ms = n_dn * out["dn"] + n_gqa * out["gqa"]
    total_flops = 2.0 * m * stack.weight_bytes()  # every rank's shards: the whole model
    rank_flops = n_dn * out["dn_flops_rank"] + n_gqa * out["gqa_flops_rank"]
    literal = scheme == "literal"
    return {"m": m, "ms_per_pass_extrapolated": round(ms, 2), "tflop_per_pass": round(total_flops / 1e12, 1),
            "TFLOPs": round(total_flops / (ms * 1e-3) / 1e12, 1),
            "per_gpu_TFLOPs": round(rank_flops / (ms * 1e-3) / 1e12, 1),
            "frac_per_gpu": round(rank_flops / (ms * 1e-3) / 1e12 / bf16_peak, 4),
            "ms_per_layer": {"deltanet": round(out["dn"], 3), "gqa": round(out["gqa"], 3)},
            "sample": "one DeltaNet + one GQA layer timed (median of %d, max over ranks), x%d / x%d"
                      % (reps, n_dn, n_gqa),
            "device_status": "clean after warm-up and timed runs",
            "collectives": ("none" if d.world == 1 else
                            "NCCL all-gather after column-parallel, all-reduce after row-parallel" if literal else
                            "NCCL all-reduce after row-parallel (Megatron pairing: no all-gather)")}


def time_out_batching(q35cu, torch, lengths=(512, 2048)):
    """The prefill caller change (oracle/prefill_batch.py) measured through
    the reference-facing C-ABI with host buffers: the DeltaNet out_proj
    (5120 x 6144) of an L-token prefill as L q35_mm_fp8 calls -- the engine's
    loop, qwen35-c/src/q35_deltanet.c:491-499 -- against one
    q35_mm_fp8_batch call (the patched engine; the tensor-core GEMM on
    bf16-rounded activations).  Wall clock of the calls themselves (their
    arguments prepared beforehand, as a C caller holds them)."""
    import ctypes as C

    import numpy as np

    sys.path.insert(0, os.path.join(REPO, "tests"))
    from parity import rel_l2

    w = q35cu.Weight.synth_fp8(4711, 5120, 6144)
    W, sc = w.download_fp8()
    w.free()
    L_ = q35cu.load()
    wp, sp = W.ctypes.data_as(q35cu._u8p), sc.ctypes.data_as(q35cu._u16p)
    out = {}
    for L in lengths:
        g = torch.Generator().manual_seed(L)
        X = torch.randn((L, 6144), generator=g).to(torch.bfloat16).float().numpy()
        Y1 = np.empty((L, 5120), np.float32)
        xs = [X[t].ctypes.data_as(q35cu._f32p) for t in range(L)]
        ys = [Y1[t].ctypes.data_as(q35cu._f32p) for t in range(L)]
        L_.q35_mm_fp8(wp, sp, 5120, 6144, xs[0], ys[0])  # uploads the weight (first touch)
        t0 = time.perf_counter()
        for t in range(L):
            L_.q35_mm_fp8(wp, sp, 5120, 6144, xs[t], ys[t])
        t_tok = time.perf_counter() - t0
        Y2 = np.empty((L, 5120), np.float32)
        L_.q35_mm_fp8_batch(wp, sp, 5120, 6144, L, X.ctypes.data_as(q35cu._f32p), Y2.ctypes.data_as(q35cu._f32p))
        t0 = time.perf_counter()
        L_.q35_mm_fp8_batch(wp, sp, 5120, 6144, L, X.ctypes.data_as(q35cu._f32p), Y2.ctypes.data_as(q35cu._f32p))
        t_b = time.perf_counter() - t0
        out[str(L)] = {"per_token_ms": round(t_tok * 1e3, 2), "batched_ms": round(t_b * 1e3, 2),
                       "speedup": round(t_tok / t_b, 1), "rel_l2_batched_vs_per_token": rel_l2(Y2, Y1)}
    L_.q35cu_release_all()
    return {"projection": "DeltaNet out_proj 5120x6144", "by_tokens": out,
            "path": "q35_mm_fp8 x L (host buffers) vs one q35_mm_fp8_batch (host buffers)"}


def run_extra(args) -> int:
    """Child-process mode: one extra measurement, printed as one JSON line."""
    if args.extra == "cpu":
        r = time_cpu_stream(args.cpu_steps, 1)
        print(json.dumps(r), flush=True)
        return 0
    import q35cu

    hbm_peak, bf16_peak, _, _ = peaks()
    d = Dist(want_p2p=False)
    torch = d.torch
    r = None
    try:
        if args.extra == "c0":
            r = time_gemv_rotating(q35cu, torch, 17408, 5120, 1)
        elif args.extra == "c1":
            r = []
            for rows, cols in ((17408, 5120), (5120, 17408)):
                for m in (1, 4, 16, 32, 48, 64):
                    if m < 16 or m == 64:
                        r.append(time_gemv_rotating(q35cu, torch, rows, cols, m, copies=3, rounds=10))
                    if m >= 16:  # what q35_mm_fp8_batch runs at this size
                        r.append(time_gemv_rotating(q35cu, torch, rows, cols, m, copies=3, rounds=10, path="tc",
                                                    graph=True))
        elif args.extra == "lm_head":
            r = time_lm_head(q35cu, torch, hbm_peak)
        elif args.extra == "c2":
            r = time_prefill_c2(q35cu, torch, bf16_peak)
        elif args.extra == "out_batch":
            r = time_out_batching(q35cu, torch)
        elif args.extra == "c4":
            r = time_config4(d, bf16_peak)
            if d.world > 1:
                r["paired"] = time_config4(d, bf16_peak, scheme="paired")
        torch.cuda.synchronize()
        q35cu.check_device_status()
    finally:
        d.close()
    if d.rank == 0:
        print(json.dumps(r), flush=True)
    return 0


def run_child(name: str, args, timeout: float = 900.0):
    """Run `bench.py --extra name` in a child process (under the same
    rank/world environment; a child process group of its own on another
    port when N > 1) and return its JSON, or {"error": ...} if it failed."""
    env = dict(os.environ)
    if "MASTER_PORT" in env:
        env["MASTER_PORT"] = str(int(env["MASTER_PORT"]) + 1 + EXTRAS.index(name))
        # the child group's rank 0 hosts its own store (torchrun's agent store
        # serves the parent group only)
        env.pop("TORCHELASTIC_USE_AGENT_STORE", None)
    cmd = [sys.executable, os.path.abspath(__file__), "--extra", name, "--gpus", str(args.gpus),
           "--cpu-steps", str(args.cpu_steps)]
    t0 = time.time()
    try:
        p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout)
    except subprocess.TimeoutExpired:
        return {"error": f"timed out after {timeout:.0f} s"}
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{") or ln.startswith("[")]
    if p.returncode != 0 or (int(os.environ.get("RANK", "0")) == 0 and not lines):
        tail = (p.stderr or p.stdout).strip().splitlines()[-6:]
        return {"error": f"rc={p.returncode}: " + " | ".join(tail)}
    if not lines:
        return None
    r = json.loads(lines[-1])
    if isinstance(r, dict):
        r["child_wall_s"] = round(time.time() - t0, 1)
    return r


def stack_max_cols(st):
    return max(max(p.w.cols for p in L.col_in + [L.attn_out, L.gate, L.up, L.down]) for L in st.layers)


def e2e_c_abi(q35cu, st, steps, warmup):
    """configuration 3 through the reference-facing q35_mm_* entry points with
    HOST buffers (N=1): every call copies its input in and its output out."""
    import numpy as np

    import stack

    # host keys bound to the device-resident weights (a loader that streamed
    # the tensors to HBM itself; see q35cu_weight_bind)
    keys = []
    hostw = {}
    for i, L in enumerate(st.layers):
        for p in L.col_in + [L.attn_out, L.gate, L.up, L.down]:
            kw = np.zeros(16, np.uint8)
            ks = np.zeros(16, np.uint16)
            p.w.bind(kw, ks)
            keys.append((kw, ks))
            hostw[(i, p.name)] = (kw, ks, p.w.rows, p.w.cols)
    lib = q35cu.load()
    import ctypes as C

    # Every buffer and ctypes argument is built once, as a C engine would hold
    # its scratch buffers (qwen35-c/src/q35_model.c:603-608): the timed loop is
    # only the 256 q35_mm_* calls and the copy of each layer's fresh input.
    f32p = q35cu._f32p
    rng = np.random.default_rng(5)
    xs = rng.standard_normal((len(st.layers), stack.HIDDEN)).astype(np.float32)
    x_in = np.empty(stack.HIDDEN, np.float32)
    calls = []  # (function, args)
    keep = []
    h2d_step = d2h_step = 0

    def multi_call(keys4, x):
        n = len(keys4)
        outs = [np.empty(k[2], np.float32) for k in keys4]
        rows = (C.c_uint32 * 4)(*([k[2] for k in keys4] + [0] * (4 - n)))
        wp = (q35cu._u8p * 4)(*([k[0].ctypes.data_as(q35cu._u8p) for k in keys4] + [q35cu._u8p()] * (4 - n)))
        sp = (q35cu._u16p * 4)(*([k[1].ctypes.data_as(q35cu._u16p) for k in keys4] + [q35cu._u16p()] * (4 - n)))
        yp = (f32p * 4)(*([o.ctypes.data_as(f32p) for o in outs] + [f32p()] * (4 - n)))
        keep.extend([outs, rows, wp, sp, yp])
        calls.append((lib.q35_mm_fp8_multi4, (wp, sp, rows, keys4[0][3], x.ctypes.data_as(f32p), yp)))
        return outs

    def single_call(key, x, y):
        kw, ks, r, c = key
        calls.append((lib.q35_mm_fp8, (kw.ctypes.data_as(q35cu._u8p), ks.ctypes.data_as(q35cu._u16p), r, c,
                                       x.ctypes.data_as(f32p), y.ctypes.data_as(f32p))))

    layer_calls = []
    for i, L in enumerate(st.layers):
        start = len(calls)
        cols = [hostw[(i, p.name)] for p in L.col_in]
        outs = multi_call(cols, x_in)
        h2d_step += 4 * stack.HIDDEN
        d2h_step += 4 * sum(k[2] for k in cols)
        src = outs[-1] if L.kind == "dn" else outs[0]  # out / o read the first OUT_K values (a prefix)
        o = np.empty(stack.HIDDEN, np.float32)
        keep.append(o)
        single_call(hostw[(i, L.attn_out.name)], src, o)
        h2d_step += 4 * stack.OUT_K
        d2h_step += 4 * stack.HIDDEN
        g, u = multi_call([hostw[(i, "gate")], hostw[(i, "up")]], o)
        h2d_step += 4 * stack.HIDDEN
        d2h_step += 8 * stack.MLP
        y = np.empty(stack.HIDDEN, np.float32)
        keep.append(y)
        single_call(hostw[(i, "down")], g, y)
        h2d_step += 4 * stack.MLP
        d2h_step += 4 * stack.HIDDEN
        layer_calls.append(calls[start:])
    for s in range(warmup + steps):
        if s == warmup:
            t0 = time.perf_counter()
        for i, lc in enumerate(layer_calls):
            x_in[:] = xs[i]
            for f, a in lc:
                f(*a)
    dt = (time.perf_counter() - t0) / steps
    lib.q35cu_release_all()  # drop the bindings (the weights stay owned by the stack)
    return {"value": round(stack.weight_bytes(st.n_layers) / dt / 1e9, 1), "unit": "GB/s",
            "ms_per_step": round(dt * 1e3, 3), "h2d_bytes_per_step": h2d_step,
            "d2h_bytes_per_step": d2h_step,
            "path": "q35_mm_fp8_multi4 / q35_mm_fp8 (host pointers, synchronous) per projection"}


def traffic_ratio():
    """DRAM bytes (read + write) per algorithmic byte of the decode GEMV, from
    the committed ncu capture (profiles/gemv_fp8_c0.json; the command that
    made it is in the file)."""
    p = os.path.join(REPO, "profiles", "gemv_fp8_c0.json")
    if not os.path.exists(p):
        return None, None
    with open(p) as f:
        d = json.load(f)
    return d.get("traffic_per_algorithmic_byte"), d.get("kernel")


def run_ours(args):
    import q35cu
    import stack

    d = Dist(want_p2p=True)
    torch, world, rank = d.torch, d.world, d.rank
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}; using WORLD_SIZE", file=sys.stderr)

    hbm_peak, bf16_peak, bf16_sus, peak_src = peaks()
    st = stack.Stack(rank, world, n_layers=args.layers, scheme="literal")
    st.x.copy_(torch.randn(st.x.shape, generator=torch.Generator().manual_seed(1234)).cuda())
    torch.cuda.synchronize()

    results = {}
    graphs = []
    # "chain" = the step as one cooperative launch (q35cu_chain_*, TP exchanges
    # fused); "graph" variants = one launch per projection captured in a CUDA
    # graph with the named collective backend
    variants = [("chain", "literal"), ("chain", "paired"), ("fused", "literal"), ("fused", "paired"),
                ("p2p", "literal"), ("p2p", "paired"), ("nccl", "literal"), ("nccl", "paired")] if world > 1 \
        else [("chain", "literal"), ("graph", "literal")]
    for coll, scheme in variants:
        st.scheme, st.coll = scheme, ("fused" if coll in ("chain", "graph") else coll)
        run_step = st.step_chain if coll == "chain" else st.step
        # eager warm-up (the chain's first run uploads its op table), then
        # capture one step in a CUDA graph
        for _ in range(2):
            run_step()
        torch.cuda.synchronize()
        q35cu.check_device_status()
        d.barrier()
        n0 = q35cu.load().q35cu_launch_count()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                run_step(s) if coll == "chain" else run_step()
        torch.cuda.current_stream().wait_stream(s)
        kernels_per_step = q35cu.load().q35cu_launch_count() - n0
        graphs.append(g)
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        d.barrier()
        clk = Clocks(d.local)
        clk.start()
        time.sleep(0.3)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        clocks = clk.stop()
        q35cu.check_device_status()
        d.barrier()
        ms = d.max_over_ranks(e0.elapsed_time(e1) / args.steps)
        results[(coll, scheme)] = {"ms": ms, "clocks": clocks, "kernels_per_step": kernels_per_step}

    # the headline is the fastest variant of the literal scheme (every variant is listed)
    main_key = min((k for k in results if k[1] == "literal"), key=lambda k: results[k]["ms"])
    main = results[main_key]
    total_bytes = stack.weight_bytes(args.layers)
    value = total_bytes / (main["ms"] * 1e-3) / 1e9

    # e2e through the public API with host buffers
    e2e = None
    if world == 1 and not args.no_extras:
        e2e = e2e_c_abi(q35cu, st, steps=max(2, args.steps // 4), warmup=2)
    else:
        # TP: H2D of the step's inputs from pinned memory, the step, D2H of its outputs
        hx = torch.randn(st.x.shape).pin_memory()
        hy = torch.empty(st.y.shape).pin_memory()
        g = graphs[variants.index(main_key)]
        for _ in range(2):
            st.x.copy_(hx, non_blocking=True)
            g.replay()
            hy.copy_(st.y, non_blocking=True)
        torch.cuda.synchronize()
        d.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            st.x.copy_(hx, non_blocking=True)
            g.replay()
            hy.copy_(st.y, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        ms_e2e = d.max_over_ranks(e0.elapsed_time(e1) / args.steps)
        e2e = {"value": round(total_bytes / (ms_e2e * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms_e2e, 3),
               "h2d_bytes_per_step": hx.numel() * 4, "d2h_bytes_per_step": hy.numel() * 4,
               "path": "pinned H2D of the 64 layer inputs + graphed TP step + D2H of the 64 layer outputs"}

    # live roofline of the dominant kernel, this rank.  Every kernel of the
    # timed step is the decode GEMV (256 PDL-chained launches of
    # gemv_mma_kernel in the graph, or the one gemv_chain_kernel launch), so
    # its achieved bandwidth is the step's algorithmic bytes (this rank's
    # weights + scales + activations) over the step's event time, i.e. the
    # average launch duration inside the timed region.  The per-projection
    # standalone launches, each timed alone with events (no PDL overlap), are
    # listed as a breakdown.
    ach_p, bytes_per_launch_p, s_per_launch_p, nl_p, breakdown = kernel_roofline(q35cu, torch, st, hbm_peak)
    bytes_step = bytes_per_launch_p * nl_p
    s_step = main["ms"] * 1e-3
    ach = bytes_step / s_step / 1e9
    if main_key[0] == "chain":
        bytes_per_launch, s_per_launch, nl = bytes_step, s_step, args.steps
        kernel_name = "gemv_chain_kernel (the whole step: one cooperative launch)"
    else:
        bytes_per_launch, s_per_launch, nl = bytes_step / nl_p, s_step / nl_p, nl_p * args.steps
        kernel_name = "gemv_mma_kernel (decode GEMV): the step's %d launches, PDL-chained in one CUDA graph" % nl_p
    ach = d.max_over_ranks(-ach) * -1 if world > 1 else ach  # slowest rank
    ratio, ratio_kernel = traffic_ratio()
    traffic = round(ratio * bytes_per_launch) if ratio else None
    st_free_bytes = st.local_weight_bytes

    for g in graphs:
        del g
    graphs.clear()
    st.free()
    torch.cuda.synchronize()

    # extras, each in a child process of its own (rank 0 at N=1; configuration
    # 4 on every rank).  The decode configurations first: the tensor-core GEMMs
    # of configurations 2 and 4 run at the power cap, and the clocks take a
    # while to come back.
    extras = {}
    if not args.no_extras:
        if world == 1:
            extras["config0_gemv"] = run_child("c0", args)
            extras["config1_sweep"] = run_child("c1", args)
            extras["lm_head_bf16"] = run_child("lm_head", args)
            extras["config2_prefill"] = run_child("c2", args)
            extras["prefill_out_batching"] = run_child("out_batch", args)
        c4 = run_child("c4", args)
        if rank == 0:
            extras["config4_prefill"] = c4
    cpu = None
    if rank == 0 and world == 1 and not args.no_extras:
        cpu = run_child("cpu", args)

    kernels, colls = st.launches_per_step()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(main["ms"], 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (FP8 e4m3 weights x fp32 activations)",
            "data": "synthetic (seeded N(0,0.02) weights, 128x128 block-quantised in HBM; N(0,1) activations)",
            "config": {"workload": f"configuration 3: {args.layers}-layer FP8 decode weight stream, M=1, "
                                   f"48 DeltaNet + 16 GQA layers",
                       "weight_bytes_per_step": total_bytes, "weight_bytes_per_gpu": st_free_bytes,
                       "parallelism": f"tp{world}",
                       "tp_scheme": "literal (all-gather after column-parallel, all-reduce after row-parallel)",
                       "launch": ("one cooperative launch per step (q35cu_chain_run)" if main_key[0] == "chain"
                                  else "one launch per projection, CUDA graph"),
                       "collectives": ("fused into the GEMV epilogues over NVLink peer memory" if
                                       main_key[0] in ("chain", "fused") and world > 1 else
                                       ("none" if world == 1 else main_key[0])),
                       "l2": "inputs larger than L2 (weights per GPU per step >> 126 MB)", "cuda_graph": True},
            "gpu_launches": main["kernels_per_step"] * args.steps,
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(ach / hbm_peak, 4), "traffic": traffic,
                         "traffic_basis": (f"ncu dram read+write per algorithmic byte of {ratio_kernel} "
                                           f"(profiles/gemv_fp8_c0.json) x this launch's algorithmic bytes"
                                           if ratio else None),
                         "kernel": kernel_name,
                         "peak_source": f"{peak_src} hbm_gbs (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback",
                         "launches_timed": nl, "algorithmic_bytes_per_launch": round(bytes_per_launch),
                         "us_per_launch": round(s_per_launch * 1e6, 2),
                         "standalone_gemv": {"GBps": round(ach_p, 1), "us_per_launch": round(s_per_launch_p * 1e6, 2),
                                             "by_projection": breakdown}},
            "clocks": main["clocks"],
            "e2e": e2e,
        }
        line["variants"] = {f"{c}_{sc}": {"ms_per_step": round(r["ms"], 4),
                                          "value": round(total_bytes / (r["ms"] * 1e-3) / 1e9, 1)}
                            for (c, sc), r in results.items()}
        if world > 1:
            line["variants_note"] = ("chain = one cooperative launch per step with the exchange fused, fused = one "
                                     "launch per projection with the exchange in the GEMV epilogue (no collective "
                                     "kernel), p2p = libq35cuda "
                                     "one-shot NVLink collective kernels, nccl = NCCL; literal = all-gather "
                                     "after column-parallel + all-reduce after row-parallel, paired = Megatron pairing "
                                     "(no all-gather, the row-parallel projection consumes the local shard)")
            line["collectives_per_step"] = colls
        if cpu is not None:
            if "error" in cpu:
                line["cpu_baseline"] = cpu
            else:
                line["cpu_baseline"] = {k: cpu.get(k) for k in ("value", "unit", "cores", "kind", "sample")}
                line["cpu_baseline"]["ms_per_step"] = cpu.get("ms_per_step")
                line["cpu_baseline"]["cpu"] = cpu.get("cpu")
        line.update(extras)
        print(json.dumps(line), flush=True)

    d.close()
    return 0


def run_profile_c0(args):
    import torch

    import q35cu

    torch.cuda.set_device(0)
    q35cu.check(q35cu.load().q35cu_set_device(0))
    r = time_gemv_rotating(q35cu, torch, 17408, 5120, 1, copies=5, rounds=max(1, args.steps))
    print(json.dumps({"config0_gemv": r}), flush=True)
    return 0


def run_profile_c2(args):
    import torch

    import q35cu

    torch.cuda.set_device(0)
    q35cu.check(q35cu.load().q35cu_set_device(0))
    w = q35cu.Weight.synth_fp8(9007, 17408, 5120)
    try:
        X = torch.randn((2048, 5120), device="cuda").to(torch.bfloat16)
        Y = torch.empty((2048, 17408), device="cuda")
        work = torch.empty(q35cu.gemm_workspace_bytes(2048, 5120), dtype=torch.uint8, device="cuda")
        for _ in range(max(1, args.steps)):
            q35cu.gemm(w, X.view(torch.int16), Y, work)
        torch.cuda.synchronize()
    finally:
        w.free()
    print(json.dumps({"config2_gate_gemm": "ok", "launches": max(1, args.steps)}), flush=True)
    return 0


def run_profile_c1_tc(args):
    import torch

    import q35cu

    torch.cuda.set_device(0)
    L = q35cu.load()
    q35cu.check(L.q35cu_set_device(0))
    m = args.profile_c1_tc
    rows, cols = (int(v) for v in args.profile_shape.lower().split("x"))
    w = q35cu.Weight.synth_fp8(1000, rows, cols)
    try:
        X = torch.randn((m, cols), device="cuda")
        Y = torch.empty((m, rows), device="cuda")
        work = torch.empty(L.q35cu_gemv_fp8_tc_workspace_bytes(m, cols), dtype=torch.uint8, device="cuda")
        for _ in range(max(1, args.steps)):
            q35cu.gemv_tc(w, X, Y, work)
        torch.cuda.synchronize()
        q35cu.check_device_status()
        ok = bool(torch.isfinite(Y).all())
    finally:
        w.free()
    print(json.dumps({"config1_tc": "ok" if ok else "non-finite", "m": m, "shape": [rows, cols],
                      "launches": max(1, args.steps)}), flush=True)
    return 0 if ok else 1


def run_profile_lm_head(args):
    import torch

    import q35cu

    torch.cuda.set_device(0)
    q35cu.check(q35cu.load().q35cu_set_device(0))
    w = bf16_weight(q35cu, torch, args.profile_lm_head, 5120)
    try:
        x = torch.randn(5120, device="cuda")
        y = torch.empty(args.profile_lm_head, device="cuda")
        for _ in range(max(1, args.steps)):
            q35cu.gemv_bf16(w, x, y)
        torch.cuda.synchronize()
        ok = bool(torch.isfinite(y).all())
    finally:
        w.free()
    print(json.dumps({"lm_head_bf16": "ok" if ok else "non-finite", "rows": args.profile_lm_head,
                      "launches": max(1, args.steps)}), flush=True)
    return 0 if ok else 1


def main():
    args = parse()
    if args.extra:
        return run_extra(args)
    if args.profile_c0:
        return run_profile_c0(args)
    if args.profile_c2:
        return run_profile_c2(args)
    if args.profile_lm_head:
        return run_profile_lm_head(args)
    if args.profile_c1_tc:
        return run_profile_c1_tc(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

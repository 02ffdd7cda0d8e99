"""Benchmark of the int4 decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload spec|gemm] [--impl vella|reference]

Prints ONE JSON line on rank 0.  Workloads:
  gemm  the small-M MLX-affine GEMM sweep: M in {1,2,4,5,8,9,16} x (N,K) in
        {(5120,5120),(1024,5120),(25600,5120),(5120,25600),(151936,5120)} x int4/int8,
        weights ~N(0,0.02) quantized group 64 with bf16 scale/bias, x ~N(0,1) bf16.
        A step is one pass over the whole sweep; every call reads a different copy of its
        weights (copies > 3x the 126 MB L2), so the weights stream from HBM.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GEMM_SHAPES = [(5120, 5120), (1024, 5120), (25600, 5120), (5120, 25600), (151936, 5120)]
GEMM_MS = [1, 2, 4, 5, 8, 9, 16]
L2_BYTES = 126 * 2 ** 20


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def gemm_bytes(m, n, k, bits):
    return n * k * bits // 8 + n * (k // 64) * 4 + m * k * 2 + m * n * 2


class ClockSampler:
    """nvidia-smi clocks during the timed region (median SM MHz under load, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["unsampled"]}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# GEMM sweep
# ---------------------------------------------------------------------------------------

def quantize_gpu(w, bits):
    """MLX affine quantize on the GPU with torch ops (bench input preparation only)."""
    import torch
    n, k = w.shape
    wg = w.float().reshape(n, k // 64, 64)
    n_bins = float((1 << bits) - 1)
    w_max = wg.amax(dim=2)
    w_min = wg.amin(dim=2)
    side = w_min.abs() > w_max.abs()
    scale = torch.clamp((w_max - w_min) / n_bins, min=1e-7)
    scale = torch.where(side, scale, -scale)
    edge = torch.where(side, w_min, w_max)
    q0 = torch.sign(edge / scale) * torch.floor((edge / scale).abs() + 0.5)
    at_zero = q0 == 0
    scale = torch.where(at_zero, scale, edge / torch.where(at_zero, torch.ones_like(q0), q0))
    bias = torch.where(at_zero, torch.zeros_like(edge), edge)
    q = (wg - bias[..., None]) / scale[..., None]
    q = torch.clamp(torch.sign(q) * torch.floor(q.abs() + 0.5), 0, n_bins).to(torch.int64).reshape(n, k)
    per = 32 // bits
    q = q.reshape(n, k // per, per)
    shifts = (torch.arange(per, device=w.device) * bits)
    packed = (q << shifts).sum(dim=2)
    packed = torch.where(packed >= 2 ** 31, packed - 2 ** 32, packed).to(torch.int32)
    return packed.contiguous(), scale.to(torch.bfloat16).contiguous(), bias.to(torch.bfloat16).contiguous()


def run_gemm(args, rank, world):
    import torch
    from vella_b200 import smallm as S
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    hbm, _, peak_kind = peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    stream = torch.cuda.Stream(device=dev)
    plans = []  # (bits, n, k, m, copies, x, out, graph_calls)
    with torch.cuda.stream(stream):
        for bits in (4, 8):
            for (n, k) in GEMM_SHAPES:
                w = torch.randn(n, k, generator=g, device=dev) * 0.02
                packed, sc, bi = quantize_gpu(w, bits)
                del w
                wbytes = gemm_bytes(0, n, k, bits)
                copies = max(2, -(-3 * L2_BYTES // wbytes))
                ws = [S.Weights(packed, sc, bi, bits)] + [
                    S.Weights(packed.clone(), sc.clone(), bi.clone(), bits) for _ in range(copies - 1)]
                for m in GEMM_MS:
                    x = (torch.randn(m, k, generator=g, device=dev)).to(torch.bfloat16)
                    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
                    plans.append((bits, n, k, m, ws, x, out))
    torch.cuda.synchronize()
    # one workspace for every graph (they replay one after another on one stream)
    ws_bytes = max(S.workspace_size(m, n, k, torch.bfloat16, bits) for bits, n, k, m, *_ in plans)
    workspace = torch.zeros(max(ws_bytes, 256) // 4 + 64, dtype=torch.int32, device=dev)
    # one CUDA graph per (bits, shape, M): `reps` calls cycling through the weight copies
    reps = 8
    graphs = []
    for bits, n, k, m, ws, x, out in plans:
        with torch.cuda.stream(stream):
            S.matmul(x, ws[0], out=out, workspace=workspace)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for i in range(reps):
                S.matmul(x, ws[i % len(ws)], out=out, workspace=workspace)
        graphs.append(gr)
    torch.cuda.synchronize()

    def step():
        for gr in graphs:
            gr.replay()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # per-config timing with events (for the sweep table and the roofline)
    per = []
    for (bits, n, k, m, ws, x, out), gr in zip(plans, graphs):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record()
            for _ in range(4):
                gr.replay()
            e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1000 / (4 * reps)
        per.append({"bits": bits, "n": n, "k": k, "m": m, "us": round(us, 3),
                    "gbs": round(gemm_bytes(m, n, k, bits) / us / 1e3, 1)})
    with ClockSampler(dev.index) as clk:
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record()
            for _ in range(args.steps):
                step()
            e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1)
    total_bytes = sum(gemm_bytes(m, n, k, bits) for bits, n, k, m, *_ in plans) * reps * args.steps
    value = total_bytes / (ms / 1e3) / 1e9
    m8 = [p for p in per if p["bits"] == 4 and p["m"] <= 8]
    m8_bytes = sum(gemm_bytes(p["m"], p["n"], p["k"], 4) for p in m8)
    m8_us = sum(p["us"] for p in m8)
    dominant = m8_bytes / m8_us / 1e3
    line = {
        "metric": "small-M int4/int8 GEMM HBM GB/s (sweep aggregate)",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u4/u8 x bf16", "data": "synthetic",
        "config": {"workload": "gemm sweep M{1,2,4,5,8,9,16} x 5 (N,K) x int4/int8, group 64, bf16",
                   "l2": "weights rotate over copies > 3x L2"},
        "roofline": {"bound": "hbm", "achieved": round(dominant, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(dominant / hbm, 3), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "qgemm int4 M<=8 (sweep subset)"},
        "clocks": clk.summary(),
        "gpu_launches": len(plans) * reps * args.steps,
        "sweep": per,
    }
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="gemm", choices=["gemm"])
    ap.add_argument("--impl", default="vella", choices=["vella", "reference"])
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "reference arm not wired yet"}))
        return
    line = run_gemm(args, rank, world)
    if rank == 0:
        print(json.dumps(line))


if __name__ == "__main__":
    main()

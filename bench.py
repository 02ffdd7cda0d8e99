"""Benchmark of the int4 draft-and-verify decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload spec|gemm|whisper] [--impl vella|reference]

Prints ONE JSON line on rank 0.  Workloads:
  spec  (default) the 30B-class int4 draft-and-verify decode: tokens/s/GPU at K=4, p=0.7 with
        the K in {4,8} x p in {.5,.7,.9} sweep in the same line.
  whisper  the Whisper decoder step at large-v3-turbo shapes (fp16, one stream, 224 greedy
        tokens after a 4-token prompt, encoder included per step), with the Whisper-tiny
        (config 1) GPU rate beside its CPU oracle rate.
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
# DRAM bytes per algorithmic byte of the small-M int4 GEMM, from one ncu capture of
# qgemm_stream_kernel at M=5, N=25600, K=5120 (75.04 MB read+write for 74.04 MB algorithmic;
# profiles/qgemm_stream_int4_25600x5120_m5.txt).  Traffic scales with the weights read, so the
# verify pass's average launch is reported as its algorithmic bytes times this ratio.
STREAM_TRAFFIC_RATIO = 75.04 / 74.04


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def gemm_bytes(m, n, k, bits):
    """Algorithmic bytes of one call: weights (+ bf16 scales/biases when quantized), x, out."""
    wbytes = n * k * bits // 8 + n * (k // 64) * 4 if bits else n * k * 2
    return wbytes + m * k * 2 + m * n * 2


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


def gemm_plans(cases, dev, stream):
    """Weights (copies rotating over > 3x L2), inputs and outputs of every (bits, N, K, M) case;
    cases are (bits, n, k, [m, ..]).  Returns the plans and one shared workspace."""
    import torch
    from vella_b200 import smallm as S
    g = torch.Generator(device=dev).manual_seed(0)
    plans = []  # (bits, n, k, m, weight copies, x, out)
    with torch.cuda.stream(stream):
        for bits, n, k, ms in cases:
            w = torch.randn(n, k, generator=g, device=dev) * 0.02
            wbytes = gemm_bytes(0, n, k, bits)
            copies = max(2, -(-3 * L2_BYTES // wbytes))
            if bits:
                packed, sc, bi = quantize_gpu(w, bits)
                ws = [S.Weights(packed, sc, bi, bits)] + [
                    S.Weights(packed.clone(), sc.clone(), bi.clone(), bits) for _ in range(copies - 1)]
            else:
                wd = w.to(torch.bfloat16)
                ws = [S.Weights(wd, bits=0)] + [S.Weights(wd.clone(), bits=0) for _ in range(copies - 1)]
            del w
            for m in ms:
                x = (torch.randn(m, k, generator=g, device=dev)).to(torch.bfloat16)
                out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
                plans.append((bits, n, k, m, ws, x, out))
    torch.cuda.synchronize()
    ws_bytes = max(S.workspace_size(m, n, k, torch.bfloat16, bits) for bits, n, k, m, *_ in plans)
    workspace = torch.zeros(max(ws_bytes, 256) // 4 + 64, dtype=torch.int32, device=dev)
    return plans, workspace


def gemm_graphs(plans, workspace, stream, reps):
    """One CUDA graph per case: `reps` calls cycling through its weight copies."""
    import torch
    from vella_b200 import smallm as S
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
    return graphs


def gemm_time_each(plans, graphs, stream, reps, hbm, iters=4):
    """Per case: mean call time from CUDA events on the launching stream (after a warm replay)."""
    import torch
    per = []
    for (bits, n, k, m, ws, x, out), gr in zip(plans, graphs):
        with torch.cuda.stream(stream):
            gr.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                gr.replay()
            e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1000 / (iters * reps)
        gbs = gemm_bytes(m, n, k, bits) / us / 1e3
        per.append({"bits": bits, "n": n, "k": k, "m": m, "us": round(us, 3), "gbs": round(gbs, 1),
                    "frac": round(gbs / hbm, 3), "tflops": round(2.0 * m * n * k / us / 1e6, 1)})
    return per


def m8_aggregate(per):
    """Bytes-weighted HBM rate of the int4 calls of at most 8 rows."""
    sel = [p for p in per if p["bits"] == 4 and p["m"] <= 8] or per
    return sum(gemm_bytes(p["m"], p["n"], p["k"], p["bits"]) for p in sel) / sum(p["us"] for p in sel) / 1e3


def run_gemm(args, rank, world):
    import torch
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    hbm, _, peak_kind = peaks()
    stream = torch.cuda.Stream(device=dev)
    cases = [(b, n, k, GEMM_MS) for b in (4, 8) for (n, k) in GEMM_SHAPES]
    if args.shape:  # one (bits, N, K, M) case, e.g. a small capture for a profiler
        b, n, k, m = (int(v) for v in args.shape.split(","))
        cases = [(b, n, k, [m])]
    plans, workspace = gemm_plans(cases, dev, stream)
    reps = 8
    graphs = gemm_graphs(plans, workspace, stream, reps)

    def step():
        for gr in graphs:
            gr.replay()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    per = gemm_time_each(plans, graphs, stream, reps, hbm)
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
    dominant = m8_aggregate(per)
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


def gemm_subline(dev, hbm, peak_kind):
    """The config-2 GEMM shapes inside the default bench line: int4 at M in {1, 5, 8} and int8 at
    M = 1 for every (N, K), each call timed alone (CUDA graph of 8 calls over rotating weight
    copies, CUDA events), with its HBM fraction."""
    import torch
    stream = torch.cuda.Stream(device=dev)
    cases = [(4, n, k, [1, 5, 8]) for (n, k) in GEMM_SHAPES] + [(8, n, k, [1]) for (n, k) in GEMM_SHAPES]
    plans, workspace = gemm_plans(cases, dev, stream)
    reps = 8
    graphs = gemm_graphs(plans, workspace, stream, reps)
    with torch.cuda.stream(stream):
        for gr in graphs:
            gr.replay()
    per = gemm_time_each(plans, graphs, stream, reps, hbm)
    agg = m8_aggregate(per)
    del graphs, plans, workspace
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {"unit": "GB/s", "peak": hbm, "peak_kind": peak_kind,
            "int4_m_le_8_gbs": round(agg, 1), "int4_m_le_8_frac": round(agg / hbm, 3),
            "note": "each call alone, weights rotated over copies > 3x L2; bytes = N*K*bits/8 + N*K/64*4 + M*K*2 + M*N*2",
            "cases": per}


# ---------------------------------------------------------------------------------------
# 30B-class int4 draft-and-verify (the headline)
# ---------------------------------------------------------------------------------------

TARGET = dict(n_layers=64, d_model=5120, n_heads=40, n_kv_heads=8, head_dim=128, ffn=25600, vocab=151936, bits=4)
DRAFT = dict(n_layers=28, d_model=2048, n_heads=16, n_kv_heads=8, head_dim=128, ffn=6144, vocab=151936, bits=0)
PREFIX, NEW_TOKENS = 750, 448
SWEEP = [(4, 0.5), (4, 0.7), (4, 0.9), (8, 0.5), (8, 0.7), (8, 0.9)]
HEADLINE = (4, 0.7)
BATCH_STREAMS = 32  # streams per GPU of the batched measurement
# Tree verification with stochastic acceptance: 256 streams over the box's 8 GPUs, i.e. 32 per
# GPU; branching 3 at depth 1, then 2, 2, 1 (33 draft nodes + the root = 34 verify rows per
# stream); temperature 0.7; the real (random-init) draft model proposes.
TREE_STREAMS, TREE_BRANCHING, TREE_TEMPERATURE, TREE_TOKENS = 32, (3, 2, 2, 1), 0.7, NEW_TOKENS


def expected_tokens_per_pass(k, p):
    return (1 - p ** (k + 1)) / (1 - p)


def dist_setup(world, backend="nccl"):
    """One process per GPU; the process group only carries the barrier and the max-over-ranks
    of the timings (the decode path itself has no collective: every GPU owns whole streams)."""
    if world <= 1:
        return None
    import datetime
    import torch.distributed as dist
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return dist


def dist_max(dist, value, dev):
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def weak_scaling_value(units_per_rank, world, seconds_max):
    """Whole-job throughput: the units all ranks processed over the slowest rank's time."""
    return units_per_rank * world / seconds_max


def verify_gemm_roofline(target, k, dev, reps=3):
    """Replays the target's verify GEMMs (all 64 layers + LM head, M = k+1) in a CUDA graph on
    one stream and times them with CUDA events: the dominant kernel's achieved HBM rate."""
    import torch
    from vella_b200 import smallm as S
    from vella_b200 import _lib as L

    class Dev:
        def __init__(self, ptr, n):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i4", "data": (ptr, False), "version": 3}

    def view(name, layer, dtype, shape):
        ptr, nbytes = target.tensor(name, layer)
        t = torch.as_tensor(Dev(ptr, nbytes // 4), device=dev)
        return t.view(dtype).view(*shape)

    c = TARGET
    d, H, KV, hd, F, V = c["d_model"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["ffn"], c["vocab"]
    m = k + 1

    def qw(name, layer, n, kk):
        return S.Weights(view(f"{name}.w", layer, torch.int32, (n, kk // 8)),
                         view(f"{name}.s", layer, torch.bfloat16, (n, kk // 64)),
                         view(f"{name}.b", layer, torch.bfloat16, (n, kk // 64)), 4)

    calls, nbytes = [], 0
    xs = {kk: torch.randn(m, kk, device=dev).to(torch.bfloat16) for kk in (d, H * hd, F)}
    outs = {n: torch.empty(m, n, device=dev, dtype=torch.bfloat16) for n in (d, (H + 2 * KV) * hd, F, V)}
    for layer in range(c["n_layers"]):
        for name, n, kk, epi in (("qkv", (H + 2 * KV) * hd, d, "none"), ("o", d, H * hd, "residual"),
                                 ("gate", F, d, "siluGate"), ("down", d, F, "residual")):
            w = qw(name, layer, n, kk)
            up = qw("up", layer, F, d) if epi == "siluGate" else None
            calls.append((w, kk, n, epi, up))
            nbytes += gemm_bytes(m, n, kk, 4) * (2 if up is not None else 1)
    calls.append((qw("lm_head", -1, V, d), d, V, "none", None))
    nbytes += gemm_bytes(m, V, d, 4)
    ws_bytes = max(S.workspace_size(m, n, kk, torch.bfloat16, 4, epi) for _, kk, n, epi, _ in calls)
    ws = torch.zeros(max(ws_bytes, 256) // 4 + 64, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def run():
        for w, kk, n, epi, up in calls:
            res = outs[n] if epi == "residual" else None
            S.matmul(xs[kk], w, epilogue=epi, residual=res, up=up, out=outs[n], workspace=ws)

    with torch.cuda.stream(stream):
        run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        run()
    with torch.cuda.stream(stream):
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    return {"bytes_per_pass": nbytes, "ms_per_pass": ms, "gbs": nbytes / ms / 1e6, "launches": len(calls)}


def run_spec(args, rank, world):
    import torch
    from vella_b200 import _lib as L
    from vella_b200 import decode as VD
    dist = dist_setup(world)
    local = int(os.environ.get("LOCAL_RANK", 0))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hbm, _, peak_kind = peaks()
    max_seq = PREFIX + NEW_TOKENS + 64
    tc = VD.ModelConfig(**TARGET, max_seq=max_seq, max_prefix=PREFIX, rope_theta=1e6)
    dc = VD.ModelConfig(**DRAFT, max_seq=max_seq, max_prefix=PREFIX, rope_theta=1e6)
    t0 = time.time()
    target = VD.Model(tc, local)
    target.init_random(1, 0.02)   # the same random-init replica on every GPU
    draft = VD.Model(dc, local)
    draft.init_random(2, 0.02)
    init_s = time.time() - t0
    # each GPU decodes its own stream: prefix embeddings ~N(0, 1) seeded by rank
    fill = L.lib().vella_fill_normal
    for m, dd, tid in ((target, TARGET["d_model"], 11), (draft, DRAFT["d_model"], 12)):
        ptr, _ = m.tensor("prefix")
        L.check(fill(ptr, PREFIX * dd, L.BF16, 3 + rank, tid, 0.0, 1.0, None))
    torch.cuda.synchronize()

    # plain greedy decode: the reference continuation of the oracle draft, and the baseline
    sd = VD.SpecDecoder(target, draft, k=HEADLINE[0], mode=VD.DRAFT_ORACLE, oracle_p=HEADLINE[1], seed=7 + rank)
    sd.set_prefix(None, None, PREFIX)
    greedy = sd.decode_greedy(NEW_TOKENS + 16)
    ref = greedy.tokens
    greedy_tps = (len(ref) - 1) / (greedy.ms / 1e3)  # the first token comes from the prefill
    sweep = []
    for (k, p) in SWEEP:
        s2 = VD.SpecDecoder(target, draft, k=k, mode=VD.DRAFT_ORACLE, oracle_p=p, seed=7 + rank)
        s2.set_prefix(None, None, PREFIX)
        s2.set_reference(ref)
        r = s2.decode_mtp(NEW_TOKENS)
        exact = r.tokens == ref[:NEW_TOKENS]
        st = r.stats
        sweep.append({"k": k, "p": p, "tokens_per_s": round((len(r.tokens) - 1) / (r.ms / 1e3), 1),
                      "passes": st["passes"], "tokens_per_pass": round((len(r.tokens) - 1) / max(st["passes"], 1), 3),
                      "expected_tokens_per_pass": round(expected_tokens_per_pass(k, p), 3),
                      "accepted_hist": st["accepted"][:k + 1], "bit_exact_vs_greedy": exact,
                      "decode_ms": round(r.ms, 2), "prefill_ms": round(st["last_prefill_ms"], 2)})
        s2.close()

    # headline: K=4, p=0.7, timed `steps` decodes after `warmup`
    k, p = HEADLINE
    sd.close()
    sd = VD.SpecDecoder(target, draft, k=k, mode=VD.DRAFT_ORACLE, oracle_p=p, seed=7 + rank)
    sd.set_prefix(None, None, PREFIX)
    sd.set_reference(ref)
    for _ in range(args.warmup):
        sd.decode_mtp(NEW_TOKENS)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    decode_ms, tokens, passes = 0.0, 0, 0
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            r = sd.decode_mtp(NEW_TOKENS)
            decode_ms += r.ms
            tokens += len(r.tokens) - 1
            passes += r.stats["passes"]
            exact = r.tokens == ref[:NEW_TOKENS]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    decode_ms = dist_max(dist, decode_ms, dev)
    value = weak_scaling_value(tokens, world, decode_ms / 1e3)

    # end to end through the public API: host (pinned) prefix -> device, prefill, decode, tokens -> host
    # (the host copy holds the same prefix, so the reference continuation still applies)
    class DevView:
        def __init__(self, ptr, n):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i2", "data": (ptr, False), "version": 3}

    def host_prefix(model, dd):
        ptr, _ = model.tensor("prefix")
        return torch.as_tensor(DevView(ptr, PREFIX * dd), device=dev).cpu().pin_memory()

    pin_t, pin_d = host_prefix(target, TARGET["d_model"]), host_prefix(draft, DRAFT["d_model"])
    se = VD.SpecDecoder(target, draft, k=k, mode=VD.DRAFT_ORACLE, oracle_p=p, seed=7 + rank)
    se.set_reference(ref)
    e2e_s, e2e_tokens = 0.0, 0
    for it in range(max(1, args.steps)):
        w0 = time.perf_counter()
        L.check(L.lib().vella_spec_set_prefix(se.handle, pin_t.data_ptr(), pin_d.data_ptr(), PREFIX, 1))
        r = se.decode(NEW_TOKENS, VD.DECODE_SPEC)
        e2e_s += time.perf_counter() - w0
        e2e_tokens += len(r.tokens)
    e2e_s = dist_max(dist, e2e_s, dev)
    h2d = PREFIX * (TARGET["d_model"] + DRAFT["d_model"]) * 2
    d2h = NEW_TOKENS * 4

    roof = verify_gemm_roofline(target, k, dev)
    launches_per_pass = k * (1 + 8 * DRAFT["n_layers"] + 3 + 1) + (1 + 8 * TARGET["n_layers"] + 3) + 1
    weights_gb = (target.weight_bytes() + draft.weight_bytes()) / 1e9
    line = {
        "metric": "int4 draft-verify tokens/s/GPU (30B-class target, K=4, acceptance p=0.7)",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(decode_ms / args.steps, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u4 weights x bf16 activations (draft bf16)", "data": "synthetic",
        "config": {"workload": "30B-class int4 target (64L d5120 GQA40/8x128 FFN25600 V151936, g64 bf16 scale/bias) "
                               "+ bf16 draft (28L d2048 16/8x128 FFN6144); 750-position ~N(0,1) prefix; 448 tokens; "
                               "oracle draft; 1 stream per GPU; step = one 448-token decode after the prefill",
                   "k": k, "p": p, "streams_per_gpu": 1, "l2": f"weights {weights_gb:.1f} GB >> 126 MB L2"},
        "bit_exact_vs_greedy": exact,
        "greedy_tokens_per_s": round(greedy_tps, 1),
        "tokens_per_pass": round(tokens / max(passes, 1), 3),
        "sweep": sweep,
        "e2e": {"value": round(e2e_tokens * world / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "includes": "prefix H2D from pinned memory, prefill, decode, token D2H"},
        "roofline": {"bound": "hbm", "achieved": round(roof["gbs"], 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(roof["gbs"] / hbm, 3),
                     "traffic": int(roof["bytes_per_pass"] / roof["launches"] * STREAM_TRAFFIC_RATIO),
                     "traffic_unit": "bytes per launch (scaled from the M=5 25600x5120 ncu capture)",
                     "peak_kind": peak_kind,
                     "kernel": f"qgemm int4 at M={k + 1}: the verify pass's {roof['launches']} GEMM launches "
                               f"({roof['bytes_per_pass'] / 1e9:.2f} GB algorithmic) replayed in a graph",
                     "verify_gemm_ms": round(roof["ms_per_pass"], 3)},
        "clocks": clk.summary(),
        "gpu_launches": passes * launches_per_pass,
        "init_s": round(init_s, 1),
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(k, p, tokens / max(passes, 1))
    for x in (sd, se):
        x.close()
    target.close()
    draft.close()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if not args.no_gemm:
        line["gemm"] = gemm_subline(dev, hbm, peak_kind)
    if not args.no_batched:
        line["batched"] = run_spec_batched(rank, local, BATCH_STREAMS, k, p)
        line["batched"]["tokens_per_s_all_gpus"] = round(
            world * BATCH_STREAMS * (NEW_TOKENS - 1) / dist_max(dist, line["batched"]["decode_ms"] / 1e3, dev), 1)
    if not args.no_tree:
        line["tree"] = run_spec_tree(rank, local, TREE_STREAMS, TREE_BRANCHING, TREE_TEMPERATURE, TREE_TOKENS)
        line["tree"]["tokens_per_s_all_gpus"] = round(
            world * line["tree"]["tokens"] / dist_max(dist, line["tree"]["decode_ms"] / 1e3, dev), 1)
    if not args.no_whisper:
        line["whisper"] = whisper_subline(rank, local, hbm, peak_kind)
        for key, n in (("tokens_per_s_all_gpus", 1), ("streams_tokens_per_s_all_gpus", WHISPER_STREAMS)):
            ms = line["whisper"]["decode_ms"] if n == 1 else line["whisper"]["streams"]["decode_ms"]
            line["whisper"][key] = round(world * n * WHISPER_TOKENS / dist_max(dist, ms / 1e3, dev), 1)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


def whisper_subline(rank, local, hbm, peak_kind):
    """Config 3 beside the headline: the Whisper decoder at large-v3-turbo shapes (fp16), one
    stream (encode one 30 s window, 224 greedy tokens; one warm-up then one timed window) and
    WHISPER_STREAMS streams in one handle.  Device times from the library's CUDA events."""
    import numpy as np
    from vella_b200 import whisper as VW
    c = VW.TURBO
    m = VW.Whisper(c, local)
    m.init_random(1 + rank, 0.02)
    mel = np.random.default_rng(2 + rank).standard_normal((c.n_mels, 2 * c.n_audio)).astype(np.float32)
    m.encode(mel)
    m.decode(WHISPER_PROMPT, WHISPER_TOKENS)
    m.encode(mel)
    enc_ms = m.stats()["encode_ms"]
    r = m.decode(WHISPER_PROMPT, WHISPER_TOKENS)
    m.close()
    step_us = r.decode_ms / (WHISPER_TOKENS - 1) * 1e3
    achieved = whisper_step_bytes(c) / (step_us * 1e-6) / 1e9
    out = {"workload": "config 3: Whisper large-v3-turbo shapes (32 enc / 4 dec layers, d 1280, 20x64 heads, FFN 5120, "
                       "V 51866), fp16 random weights ~N(0,0.02), 4-token prompt, 224 greedy tokens per window",
           "tokens_per_s": round(WHISPER_TOKENS / ((r.prefill_ms + r.decode_ms) / 1e3), 1),
           "decode_ms": round(r.prefill_ms + r.decode_ms, 2), "step_us": round(step_us, 1),
           "encode_ms": round(enc_ms, 2),
           "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(achieved / hbm, 3), "peak_kind": peak_kind,
                        "kernel": "decoder step (algorithmic bytes / measured step time)"}}
    out["streams"] = run_whisper_streams(rank, local, WHISPER_STREAMS)
    return out


def run_spec_batched(rank, local, S, k, p):
    """S independent streams per GPU decoded as one batch: every draft step and every verify
    runs all streams' rows together (verify M = S * (k + 1), the tensor-core GEMM path).
    Same weights as the single-stream run, S different prefixes; the oracle draft follows
    each stream's own greedy continuation (the batched greedy decode, same GEMM path)."""
    import numpy as np
    import torch
    from vella_b200 import _lib as L
    from vella_b200 import decode as VD
    max_seq = PREFIX + NEW_TOKENS + 64
    tc = VD.ModelConfig(**TARGET, max_seq=max_seq, max_prefix=PREFIX, rope_theta=1e6, streams=S)
    dc = VD.ModelConfig(**DRAFT, max_seq=max_seq, max_prefix=PREFIX, rope_theta=1e6, streams=S)
    target = VD.Model(tc, local)
    target.init_random(1, 0.02)
    draft = VD.Model(dc, local)
    draft.init_random(2, 0.02)
    fill = L.lib().vella_fill_normal
    for m, dd, tid in ((target, TARGET["d_model"], 21), (draft, DRAFT["d_model"], 22)):
        ptr, _ = m.tensor("prefix")
        L.check(fill(ptr, S * PREFIX * dd, L.BF16, 3 + rank, tid, 0.0, 1.0, None))
    torch.cuda.synchronize()
    sd = VD.SpecDecoder(target, draft, k=k, mode=VD.DRAFT_ORACLE, oracle_p=p, seed=7 + rank)
    sd.set_prefix(None, None, PREFIX)
    greedy = sd.decode_batch(NEW_TOKENS, VD.DECODE_GREEDY)
    g = sd.stats()
    sd.set_reference(greedy)
    sd.decode_batch(NEW_TOKENS, VD.DECODE_SPEC)  # warm-up (captures the pass graph)
    p0 = sd.stats()["passes"]
    spec = sd.decode_batch(NEW_TOKENS, VD.DECODE_SPEC)
    st = sd.stats()
    tokens = S * (NEW_TOKENS - 1)  # each stream's first token comes from its prefill
    out = {"streams_per_gpu": S, "k": k, "p": p,
           "tokens_per_s": round(tokens / (st["last_decode_ms"] / 1e3), 1),
           "greedy_tokens_per_s": round(tokens / (g["last_decode_ms"] / 1e3), 1),
           "passes": st["passes"] - p0, "decode_ms": round(st["last_decode_ms"], 1),
           "prefill_ms_all_streams": round(st["last_prefill_ms"], 1),
           "bit_exact_vs_batched_greedy": bool(np.array_equal(spec, greedy)),
           "note": "decode-only device time; verify rows per pass = streams x (k+1) on the tensor cores"}
    sd.close()
    target.close()
    draft.close()
    return out


def run_spec_tree(rank, local, S, branching, temperature, new_tokens):
    """S streams per GPU decoded with tree verification and stochastic acceptance: per pass
    the draft expands the tree depth by depth (one batched draft forward per depth, children
    sampled from the draft's softmax at `temperature`), the target verifies every stream's
    whole tree in one forward (S x (nodes + 1) rows, tree-attention masks), and each stream
    accepts along the tree by rejection sampling against the running residual (Philox
    uniforms per pass/node/stream).  Random-init weights: the acceptance rate is whatever the
    two random models' softmaxes give, reported beside the throughput."""
    import torch
    from vella_b200 import _lib as L
    from vella_b200 import decode as VD
    nodes = 0
    width = 1
    for b in branching:
        width *= b
        nodes += width
    rows = nodes + 1
    max_seq = PREFIX + new_tokens + 2 * rows + 16
    tc = VD.ModelConfig(**TARGET, max_seq=max_seq, max_prefix=PREFIX, rope_theta=1e6, streams=S,
                        rows_per_stream=rows)
    dc = VD.ModelConfig(**DRAFT, max_seq=max_seq, max_prefix=PREFIX, rope_theta=1e6, streams=S)
    target = VD.Model(tc, local)
    target.init_random(1, 0.02)
    draft = VD.Model(dc, local)
    draft.init_random(2, 0.02)
    fill = L.lib().vella_fill_normal
    for m, dd, tid in ((target, TARGET["d_model"], 31), (draft, DRAFT["d_model"], 32)):
        ptr, _ = m.tensor("prefix")
        L.check(fill(ptr, S * PREFIX * dd, L.BF16, 5 + rank, tid, 0.0, 1.0, None))
    torch.cuda.synchronize()
    sd = VD.SpecDecoder(target, draft, k=len(branching), mode=VD.DRAFT_MODEL, seed=11 + rank,
                        temperature=temperature, tree=branching)
    sd.set_prefix(None, None, PREFIX)
    sd.decode_batch(16, VD.DECODE_SPEC)  # warm-up: prefill, graph capture
    st0 = sd.stats()
    out_toks = sd.decode_batch(new_tokens, VD.DECODE_SPEC)
    st = sd.stats()
    passes = st["passes"] - st0["passes"]
    hist = [a - b for a, b in zip(st["accepted"], st0["accepted"])]
    tokens = S * (new_tokens - 1)  # each stream's first token comes from its prefill
    sampled = int(out_toks.size)
    out = {"streams_per_gpu": S, "streams_all_gpus_at_8": 8 * S, "branching": list(branching),
           "draft_nodes": nodes, "verify_rows_per_pass": S * rows, "temperature": temperature,
           "draft": "bf16 draft model, random init (children sampled from its softmax)",
           "new_tokens_per_stream": new_tokens, "tokens": tokens,
           "tokens_per_s": round(tokens / (st["last_decode_ms"] / 1e3), 1),
           "passes": passes, "tokens_per_stream_pass": round(tokens / max(passes * S, 1), 3),
           "accepted_hist": hist[:len(branching) + 1], "decode_ms": round(st["last_decode_ms"], 1),
           "prefill_ms_all_streams": round(st["last_prefill_ms"], 1), "tokens_checked": sampled,
           "note": "decode-only device time; 32 streams per GPU is the 8-GPU share of 256 streams"}
    sd.close()
    target.close()
    draft.close()
    return out


# ---------------------------------------------------------------------------------------
# CPU baseline: the oracle's C restatement of the same pass, timed on the host cores
# ---------------------------------------------------------------------------------------

def cpu_pass_seconds(k, layers_sampled=1):
    """Times one target layer's verify GEMMs (M=k+1), one draft layer step (M=1) and both LM
    heads with the oracle's C GEMM (OpenMP); extrapolates a whole pass."""
    import numpy as np
    from oracle import cgemm as C
    rng = np.random.default_rng(0)
    m = k + 1

    def q(n, kk):
        return (rng.integers(0, 2 ** 32, size=(n, kk // 8), dtype=np.uint32),
                np.full((n, kk // 64), 0x3C00, np.uint16), np.full((n, kk // 64), 0xBC00, np.uint16))

    c, d = TARGET, DRAFT
    t_shapes = [((c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"], c["d_model"]), (c["d_model"], c["n_heads"] * c["head_dim"]),
                (c["ffn"], c["d_model"]), (c["ffn"], c["d_model"]), (c["d_model"], c["ffn"])]
    t_layer = 0.0
    for n, kk in t_shapes:
        w = q(n, kk)
        x = rng.standard_normal((m, kk)).astype(np.float32)
        s0 = time.perf_counter()
        C.qgemm(x, *w, 4)
        t_layer += time.perf_counter() - s0
    wl = q(c["vocab"] // 8, c["d_model"])
    s0 = time.perf_counter()
    C.qgemm(rng.standard_normal((m, c["d_model"])).astype(np.float32), *wl, 4)
    t_lm = (time.perf_counter() - s0) * 8
    d_shapes = [((d["n_heads"] + 2 * d["n_kv_heads"]) * d["head_dim"], d["d_model"]), (d["d_model"], d["n_heads"] * d["head_dim"]),
                (d["ffn"], d["d_model"]), (d["ffn"], d["d_model"]), (d["d_model"], d["ffn"])]
    d_layer = 0.0
    for n, kk in d_shapes:
        w = (rng.integers(0, 2 ** 16, size=(n, kk), dtype=np.uint16) & 0x3FFF)
        x = rng.standard_normal((1, kk)).astype(np.float32)
        s0 = time.perf_counter()
        C.gemm_dense(x, w)
        d_layer += time.perf_counter() - s0
    wd = rng.integers(0, 2 ** 16, size=(d["vocab"] // 8, d["d_model"]), dtype=np.uint16) & 0x3FFF
    s0 = time.perf_counter()
    C.gemm_dense(rng.standard_normal((1, d["d_model"])).astype(np.float32), wd)
    d_lm = (time.perf_counter() - s0) * 8
    t_rows, d_rows = cpu_row_ops_seconds(c, k + 1), cpu_row_ops_seconds(d, 1)
    per_pass = c["n_layers"] * (t_layer + t_rows) + t_lm + k * (d["n_layers"] * (d_layer + d_rows) + d_lm)
    return per_pass, C.threads()


CPU_CACHE = PREFIX + NEW_TOKENS // 2  # mean cache length over a 448-token decode after the prefix


def cpu_row_ops_seconds(c, rows):
    """One layer's row work in the numpy oracle: the two RMSNorms, RoPE of q and the new keys,
    and causal GQA attention of `rows` query rows over a CPU_CACHE-position cache."""
    import math

    import numpy as np
    from oracle import decoder as D
    rng = np.random.default_rng(1)
    d, H, KV, hd = c["d_model"], c["n_heads"], c["n_kv_heads"], c["head_dim"]
    T = CPU_CACHE
    x = rng.standard_normal((rows, d)).astype(np.float32)
    w = np.ones(d, np.float32)
    q = rng.standard_normal((rows, H, hd)).astype(np.float32)
    kc = rng.standard_normal((T, KV, hd)).astype(np.float32)
    vc = rng.standard_normal((T, KV, hd)).astype(np.float32)
    pos = np.arange(T - rows, T)
    table = np.zeros((T, hd // 2, 2), np.float32)
    table[:, :, 0] = 1.0
    s0 = time.perf_counter()
    D.rmsnorm(x, w, 1e-6, "bf16")
    D.rmsnorm(x, w, 1e-6, "bf16")
    D.rope(q, pos, table, "bf16")
    D.rope(kc[T - rows:], pos, table, "bf16")
    D.attention(q, kc, vc, pos, 1.0 / math.sqrt(hd), "bf16")
    return time.perf_counter() - s0


def cpu_baseline(k, p, tokens_per_pass=None):
    """The oracle's CPU restatement of one pass, on the host cores; tokens per pass from the GPU
    run when given (else the oracle draft's expectation)."""
    per_pass, threads = cpu_pass_seconds(k)
    tpp = tokens_per_pass if tokens_per_pass else expected_tokens_per_pass(k, p)
    tps = tpp / per_pass
    return {"value": round(tps, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"C/OpenMP oracle GEMMs of 1 target layer (M={k + 1}), 1 draft layer (M=1) and 1/8 of each "
                      f"LM head, plus the numpy oracle's RMSNorms, RoPE and attention of one layer of each over a "
                      f"{CPU_CACHE}-position cache, timed once and extrapolated to one pass (64+{k}x28 layers, both "
                      f"heads) at {tpp:.2f} tokens per pass "
                      f"({'measured on the GPU' if tokens_per_pass else 'expected'})"}


def run_reference(args, rank, world):
    """The reference's own CPU path cannot run here (Swift + MLX on Apple Silicon); its CPU
    restatement (the oracle's C GEMMs) is timed instead on the same config."""
    k, p = HEADLINE
    for _ in range(args.warmup):
        cpu_pass_seconds(k)
    total, threads = 0.0, 1
    w0 = time.perf_counter()
    for _ in range(args.steps):
        s, threads = cpu_pass_seconds(k)
        total += s
    wall_ms = (time.perf_counter() - w0) * 1e3 / max(args.steps, 1)
    per_pass = total / max(args.steps, 1)
    tps = expected_tokens_per_pass(k, p) / per_pass
    sample = (f"one draft-and-verify pass per step (64 target layers at M={k + 1}, {k} draft steps of 28 layers, "
              f"both LM heads) extrapolated from 1 timed layer each: C/OpenMP oracle GEMMs and the numpy oracle's "
              f"norms, RoPE and attention over a {CPU_CACHE}-position cache; E[tokens/pass] "
              f"{expected_tokens_per_pass(k, p):.2f}; ms_per_step is the wall time of one step's timed sample")
    return {"impl": "reference", "metric": "int4 draft-verify tokens/s/GPU (30B-class target, K=4, acceptance p=0.7)",
            "value": round(tps, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(wall_ms, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4 x fp32 (CPU)",
            "data": "synthetic", "config": {"workload": "30B-class int4 target + bf16 draft, K=4, p=0.7 (CPU restatement)"},
            "cpu_baseline": {"value": round(tps, 3), "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": round(tps, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------------------
# Whisper decoder step (config 3: large-v3-turbo shapes, fp16) and the tiny-shaped config 1
# ---------------------------------------------------------------------------------------

WHISPER_PROMPT = [50258, 50259, 50359, 50363]  # <|startoftranscript|> <|en|> <|transcribe|> <|notimestamps|>
WHISPER_TOKENS = 224
WHISPER_STREAMS = 64  # independent windows per GPU decoded together (config 3, batched form)


def whisper_step_bytes(c):
    """Algorithmic HBM bytes of one decoder step: the decoder Linears (cross k|v excluded:
    projected once per window), the vocabulary projection, the cross K/V of every layer and
    the self K/V up to the mean position."""
    d, F, V, A = c.d_model, c.ffn, c.vocab, c.n_audio
    wb = (c.bits / 8) if c.bits else 2
    sb = (4 / 64) if c.bits else 0
    per_layer = (3 * d * d + d * d + d * d + d * d + 2 * d * F) * (wb + sb)
    vocab = V * d * (wb + sb)
    cross = c.dec_layers * A * 2 * d * 2
    self_kv = c.dec_layers * 2 * (len(WHISPER_PROMPT) + WHISPER_TOKENS // 2) * d * 2
    return c.dec_layers * per_layer + vocab + cross + self_kv


def whisper_encoder_flops(c):
    d, F, A = c.d_model, c.ffn, c.n_audio
    kp1 = (3 * c.n_mels + 63) // 64 * 64
    conv = 2 * (2 * A) * d * kp1 + 2 * A * d * 3 * d
    layer = 2 * A * (3 * d * d + d * d + 2 * d * F) + 2 * 2 * A * A * d
    return conv + c.enc_layers * layer + 2 * A * 2 * d * d * c.dec_layers


def whisper_oracle_tokens_per_s(seconds_budget=6.0):
    """The oracle's greedy decode of the tiny config on this host's cores (numpy), a bounded
    sample: the encoder once, then greedy steps until the budget is spent."""
    import numpy as np
    from oracle import affine as A
    from oracle import whisper as Wh
    c = Wh.WhisperConfig()  # Whisper-tiny shapes, int4 decoder
    rng = np.random.default_rng(0)
    d, F = c.d_model, c.ffn

    def dense(n, k):
        return {"w": A.to_storage(rng.standard_normal((n, k)).astype(np.float32) * 0.02, "f16")}

    def qnt(n, k):
        p, s_, b_ = A.quantize(rng.standard_normal((n, k)).astype(np.float32) * 0.02, 4, "f16")
        return {"w": p, "s": s_, "b": b_}

    def vec(n, mean=0.0, sd=0.02):
        return A.from_storage(A.to_storage((mean + sd * rng.standard_normal(n)).astype(np.float32), "f16"), "f16")

    W = {"conv1": dense(d, 256), "conv1_b": vec(d), "conv2": dense(d, 3 * d), "conv2_b": vec(d),
         "enc_pos": Wh.sinusoids(c.n_audio, d), "enc_ln_w": vec(d, 1, .1), "enc_ln_b": vec(d),
         "dec_ln_w": vec(d, 1, .1), "dec_ln_b": vec(d), "embed": qnt(c.vocab, d),
         "dec_pos": vec((c.max_target, d)), "enc": [], "dec": []}
    for _ in range(c.enc_layers):
        W["enc"].append({"ln1_w": vec(d, 1, .1), "ln1_b": vec(d), "qkv": dense(3 * d, d), "qkv_b": vec(3 * d),
                         "o": dense(d, d), "o_b": vec(d), "ln2_w": vec(d, 1, .1), "ln2_b": vec(d),
                         "fc1": dense(F, d), "fc1_b": vec(F), "fc2": dense(d, F), "fc2_b": vec(d)})
    for _ in range(c.dec_layers):
        L = {f"{n}_{x}": vec(d, 1, .1) if x == "w" else vec(d) for n in ("ln1", "ln2", "ln3") for x in ("w", "b")}
        for name, n, k in (("qkv", 3 * d, d), ("o", d, d), ("cq", d, d), ("ckv", 2 * d, d), ("co", d, d),
                           ("fc1", F, d), ("fc2", d, F)):
            L[name], L[name + "_b"] = qnt(n, k), vec(n)
        W["dec"].append(L)
    mel = rng.standard_normal((c.n_mels, 2 * c.n_audio)).astype(np.float32)
    enc = Wh.encoder(c, W, mel)
    xkv = Wh.cross_kv(c, W, enc)
    cache = [[None, None] for _ in W["dec"]]
    Wh.decoder_forward(c, W, xkv, WHISPER_PROMPT, 0, cache)
    t0, n, pos, tok = time.perf_counter(), 0, len(WHISPER_PROMPT), 0
    while time.perf_counter() - t0 < seconds_budget and pos < c.max_target:
        hid = Wh.decoder_forward(c, W, xkv, [tok], pos, cache)
        tok = int(np.argmax(Wh.logits(c, W, hid)[0]))
        pos += 1
        n += 1
    return n / (time.perf_counter() - t0), n


def run_whisper(args, rank, world):
    import numpy as np
    import torch
    from vella_b200 import whisper as VW
    dist = dist_setup(world)
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    hbm, tflops, peak_kind = peaks()
    c = VW.TURBO
    m = VW.Whisper(c, local)
    m.init_random(1 + rank, 0.02)
    mel = torch.from_numpy(np.random.default_rng(2 + rank).standard_normal((c.n_mels, 2 * c.n_audio))
                           .astype(np.float32)).pin_memory()
    for _ in range(args.warmup):
        m.encode(mel.numpy())
        m.decode(WHISPER_PROMPT, WHISPER_TOKENS)
    enc_ms, dec_ms, pre_ms, wall = [], [], [], []
    with ClockSampler(local) as clk:
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        for _ in range(args.steps):
            t0 = time.perf_counter()
            m.encode(mel.numpy())        # host mel -> device inside the call
            r = m.decode(WHISPER_PROMPT, WHISPER_TOKENS)
            wall.append(time.perf_counter() - t0)
            st = m.stats()
            enc_ms.append(st["encode_ms"])
            pre_ms.append(r.prefill_ms)
            dec_ms.append(r.decode_ms)
            assert len(r.tokens) == WHISPER_TOKENS
        torch.cuda.synchronize()
    dec_s = sum(pre_ms + dec_ms) / 1e3
    tokens = WHISPER_TOKENS * args.steps
    dec_s = dist_max(dist, dec_s, f"cuda:{local}") if dist else dec_s
    wall_s = dist_max(dist, sum(wall), f"cuda:{local}") if dist else sum(wall)
    value = weak_scaling_value(tokens, world, dec_s)
    step_us = sum(dec_ms) / (args.steps * (WHISPER_TOKENS - 1)) * 1e3
    sbytes = whisper_step_bytes(c)
    achieved = sbytes / (step_us * 1e-6) / 1e9
    enc_tflops = whisper_encoder_flops(c) / (sum(enc_ms) / args.steps * 1e-3) / 1e12
    line = {
        "metric": "Whisper decoder tokens/s/GPU (large-v3-turbo shapes, fp16, 1 stream, greedy 224 tokens)",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dec_s * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "Whisper large-v3-turbo shapes (32 enc / 4 dec layers, d 1280, 20x64 heads, FFN 5120, "
                               "128 mels, 1500 frames, V 51866), fp16 random weights ~N(0,0.02); mel 128x3000 ~N(0,1); "
                               "4-token prompt, 224 greedy tokens; step = encode + decode of one 30 s window",
                   "streams_per_gpu": 1, "l2": "decoder weights 316 MB + cross K/V 31 MB per step > 126 MB L2"},
        "step_us": round(step_us, 2),
        "encode_ms": round(sum(enc_ms) / args.steps, 3),
        "encoder_tflops": round(enc_tflops, 1),
        "e2e": {"value": round(tokens / wall_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": c.n_mels * 2 * c.n_audio * 4, "d2h_bytes_per_step": WHISPER_TOKENS * 4,
                "includes": "host mel -> device, encoder, cross K/V, prefill, 224 steps, token read-back"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 3), "traffic": None, "peak_kind": peak_kind,
                     "kernel": f"decoder step ({sbytes / 1e6:.1f} MB algorithmic: weights, vocabulary, cross and self "
                               f"K/V) / measured step time"},
        "clocks": clk.summary(),
        "gpu_launches": args.steps * (WHISPER_TOKENS * (2 + 12 * c.dec_layers + 4)
                                      + 4 + c.enc_layers * 8 + c.dec_layers),
    }
    if rank == 0 and not args.no_cpu_baseline:
        # config 1 (Whisper-tiny shapes, int4 decoder) on both sides
        t = VW.Whisper(VW.TINY, local)
        t.init_random(3, 0.02)
        tmel = np.random.default_rng(4).standard_normal((VW.TINY.n_mels, 2 * VW.TINY.n_audio)).astype(np.float32)
        t.encode(tmel)
        t.decode(WHISPER_PROMPT, 64)
        r = t.decode(WHISPER_PROMPT, 64)
        gpu_tiny = 64 / ((r.prefill_ms + r.decode_ms) / 1e3)
        t.close()
        cpu_tps, n = whisper_oracle_tokens_per_s()
        line["cpu_baseline"] = {"value": round(cpu_tps, 2), "unit": "tokens/s", "cores": os.cpu_count(),
                                "kind": "port",
                                "sample": f"numpy oracle, Whisper-tiny shapes (config 1), int4 decoder: {n} greedy "
                                          f"steps after the prompt, encoder not timed"}
        line["config1_gpu_tokens_per_s"] = round(gpu_tiny, 1)
    m.close()
    if not args.no_batched:
        line["streams"] = run_whisper_streams(rank, local, WHISPER_STREAMS)
        line["streams"]["tokens_per_s_all_gpus"] = round(
            world * line["streams"]["tokens"] / dist_max(dist, line["streams"]["decode_ms"] / 1e3, f"cuda:{local}"), 1)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


def run_whisper_streams(rank, local, S):
    """S independent 30 s windows per GPU in one handle: S encoder passes, then one decoder
    forward of S rows per token (one CUDA graph per step), 224 greedy tokens per stream."""
    import numpy as np
    from dataclasses import replace
    from vella_b200 import whisper as VW
    c = replace(VW.TURBO, streams=S)
    m = VW.Whisper(c, local)
    m.init_random(1 + rank, 0.02)
    mels = np.random.default_rng(20 + rank).standard_normal((S, c.n_mels, 2 * c.n_audio)).astype(np.float32)
    m.encode(mels)
    enc_ms = m.stats()["encode_ms"]
    m.decode_batch(WHISPER_PROMPT, 8)  # warm-up: eager step, then the captured step graph
    toks = m.decode_batch(WHISPER_PROMPT, WHISPER_TOKENS)
    st = m.stats()
    m.close()
    dec_ms = st["prefill_ms"] + st["decode_ms"]
    tokens = S * WHISPER_TOKENS
    return {"streams_per_gpu": S, "tokens": tokens, "tokens_per_s": round(tokens / (dec_ms / 1e3), 1),
            "decode_ms": round(dec_ms, 2), "step_us": round(st["decode_ms"] / (WHISPER_TOKENS - 1) * 1e3, 1),
            "encode_ms_all_streams": round(enc_ms, 1), "distinct_sequences": int(len({tuple(r) for r in toks.tolist()})),
            "note": "prompt forward + 224 steps of S rows each (device time); encoder not in the rate"}


def run_profile_pass(args):
    """A short run for an ncu launch list: the headline models, a 16-position prefix, the
    prefill and two draft-and-verify passes (one eager, one graph replay)."""
    import torch
    from vella_b200 import _lib as L
    from vella_b200 import decode as VD
    dev = torch.device("cuda", 0)
    P = 16
    target = VD.Model(VD.ModelConfig(**TARGET, max_seq=128, max_prefix=P, rope_theta=1e6), 0)
    target.init_random(1, 0.02)
    draft = VD.Model(VD.ModelConfig(**DRAFT, max_seq=128, max_prefix=P, rope_theta=1e6), 0)
    draft.init_random(2, 0.02)
    for m, dd, tid in ((target, TARGET["d_model"], 11), (draft, DRAFT["d_model"], 12)):
        ptr, _ = m.tensor("prefix")
        L.check(L.lib().vella_fill_normal(ptr, P * dd, L.BF16, 3, tid, 0.0, 1.0, None))
    torch.cuda.synchronize()
    sd = VD.SpecDecoder(target, draft, k=HEADLINE[0], mode=VD.DRAFT_ORACLE, oracle_p=HEADLINE[1], seed=7)
    sd.set_prefix(None, None, P)
    sd.prefill()
    sd.step()
    sd.step()
    torch.cuda.synchronize()
    return {"profile": "prefill(16) + 2 passes", "passes": sd.stats()["passes"]}


def run_profile_tree(args):
    """A short tree-verification run for an ncu launch list: the headline shapes cut to 4
    target and 2 draft layers (per-layer kernels are what the list is for), 32 streams, a
    64-position prefix, branching 3,2,2,1 at temperature 0.7, 4 tokens per stream after a
    2-token warm-up decode."""
    global PREFIX, TARGET, DRAFT
    saved = PREFIX, TARGET, DRAFT
    PREFIX = 64
    TARGET = dict(TARGET, n_layers=4)
    DRAFT = dict(DRAFT, n_layers=2)
    try:
        r = run_spec_tree(0, 0, TREE_STREAMS, TREE_BRANCHING, TREE_TEMPERATURE, 4)
    finally:
        PREFIX, TARGET, DRAFT = saved
    return {"profile": "tree verification, 4+2 layers, 32 streams", "passes": r["passes"]}


def run_profile_whisper(args):
    """A short Whisper run for an ncu launch list: large-v3-turbo shapes, one 30 s window
    encoded, the 4-token prompt, then 6 single decoder steps (the steps are what the list is for)."""
    import numpy as np
    import torch
    from vella_b200 import whisper as VW
    c = VW.TURBO
    m = VW.Whisper(c, 0)
    m.init_random(1, 0.02)
    m.encode(np.random.default_rng(2).standard_normal((c.n_mels, 2 * c.n_audio)).astype(np.float32))
    t = m.begin(WHISPER_PROMPT)
    for _ in range(6):
        t = m.step()
    torch.cuda.synchronize()
    m.close()
    return {"profile": "Whisper turbo: encode + prompt + 6 decoder steps", "last_token": t}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="spec", choices=["spec", "gemm", "whisper"])
    ap.add_argument("--impl", default="vella", choices=["vella", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="spec workload: skip the multi-stream measurement")
    ap.add_argument("--no-tree", action="store_true", help="spec workload: skip the tree + sampling measurement")
    ap.add_argument("--no-gemm", action="store_true", help="spec workload: skip the config-2 GEMM sub-line")
    ap.add_argument("--no-whisper", action="store_true", help="spec workload: skip the config-3 Whisper sub-line")
    ap.add_argument("--shape", default="", help="gemm workload: one case 'bits,N,K,M' instead of the sweep")
    ap.add_argument("--profile-pass", action="store_true", help="short run for an ncu launch list")
    ap.add_argument("--profile-tree", action="store_true", help="short tree-verification run for an ncu launch list")
    ap.add_argument("--profile-whisper", action="store_true", help="short Whisper decoder run for an ncu launch list")
    args = ap.parse_args()
    if args.profile_whisper:
        print(json.dumps(run_profile_whisper(args)))
        return
    if args.profile_pass:
        print(json.dumps(run_profile_pass(args)))
        return
    if args.profile_tree:
        print(json.dumps(run_profile_tree(args)))
        return
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, rank, world)))
        return
    run = {"gemm": run_gemm, "whisper": run_whisper, "spec": run_spec}[args.workload]
    line = run(args, rank, world)
    if rank == 0:
        print(json.dumps(line))


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Benchmark of the block-scaled GEMM hot path (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload mxfp8|mxfp4|fp8block|e8m0block] [--layout tn|nn|tt|nt]
                    [--b-format raw|shuffle16]
    python bench.py --sweep | --quant | --grouped | --tune CSV     (one JSON line each)

Default workload (the headline metric): MXFP8 GEMM M=N=K=8192, layout
tn, E4M3 with E8M0 scales per 32 K, bf16 out, fp32 accumulation.  One step is
one GEMM over the whole problem.  For N > 1 GPUs (torchrun, one process per
GPU) the GEMM is partitioned along N with weights pre-sharded: every rank
computes its own M x 8192 x K column shard (weak scaling, no collective in the
timed region; configs[4]).  --workload mxfp4 reads B in the preshuffled
shuffle_weight(16,16) layout unless --b-format raw; e8m0block is
the reference's own launcher, launch_blockscale_bpreshuffle (E8M0 1x128 /
128x128 scales, shuffled B).

Printed JSON line: value = TFLOPS of the whole job from device-side CUDA
events (max over ranks).  Calls whose inputs fit in L2 (or, for skinny M <= 128
calls, in twice the L2) are preceded by a 256 MiB read that flushes L2, and the
flushes are excluded; calls shorter than 0.25 ms are timed as one CUDA-graph
replay of the K steps so that host launch overhead stays out (config.l2 and
config.timing say which).  e2e = the same GEMM through the public C-ABI call
with pinned host buffers (inputs H2D + output D2H inside the timed region),
roofline of the GEMM kernel, cpu_baseline = the reference's CPU verification
GEMM (oracle/_ref, "reference", or its restatement in oracle/, "port") on a
row sample, and sampled clocks.

--impl reference times the reference's CPU verification GEMM on the same
metric: its own CPU functions compiled from its sources (oracle/_ref) when that
library is built, else their restatement in oracle/ (its GPU kernels are
HIP/gfx950-only).
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


L2_BYTES = 126 * 1024 * 1024


def l2_policy(m, in_bytes):
    """(flush L2 before every timed call, the call is bound by the weight
    stream).  Inputs that fit in L2 are flushed.  Skinny calls (M <= 128)
    stream their weights from HBM, so their roofline is bandwidth, and their
    inputs are flushed unless they exceed twice the L2: weights left in L2 by
    the previous call would otherwise inflate the bandwidth."""
    hbm_bound = m <= 128
    return in_bytes < (2 * L2_BYTES if hbm_bound else L2_BYTES), hbm_bound


def load_traffic(workload, m, n, k, b_format):
    """DRAM bytes (read + write) of one launch of the workload's dominant
    kernel from the committed ncu capture (profiles/dram_traffic.json), when
    that capture was taken on this very shape; else None."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.exists():
        return None, None
    e = json.loads(p.read_text()).get(workload)
    if not e or e["shape"] != [m, n, k] or (b_format is not None and e["b_format"] != b_format):
        return None, None
    return e["read_bytes"] + e["write_bytes"], f"ncu capture, profiles/{e['summary']}"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000,
                    help="timed GEMM launches (the default keeps the timed region near 1 s so the "
                         "100 ms clock samples cover it)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="mxfp8", choices=["mxfp8", "mxfp4", "fp8block", "e8m0block"])
    ap.add_argument("--b-format", default=None, choices=["raw", "shuffle16"],
                    help="B layout for the MX workloads (default: shuffle16 for mxfp4, raw for mxfp8)")
    ap.add_argument("--layout", default="tn", choices=["tn", "nn", "tt", "nt"])
    ap.add_argument("--kernel", default="auto", choices=["auto", "1cta", "pair", "swap", "wide"],
                    help="kernel: auto, single-CTA tiles, CTA pairs (cta_group::2), the transposed decode "
                         "kernel (M <= 64), or the wide single-CTA 128x256 kernel (fp8block only)")
    ap.add_argument("--split-k", type=int, default=0,
                    help="split_k of the timed call for the mxfp8, mxfp4 and fp8block workloads "
                         "(0 = the library's choice; 1 keeps every unit whole)")
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192, help="per-rank N")
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--shape", default=None,
                    help="M,N,K (N per rank); same as --m/--n/--k, which torchrun's own parser "
                         "would take as abbreviations of its options")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tune", default=None, metavar="CSV",
                    help="tune kernel / split-K per shape (fp8 block-scale sweep shapes and skinny MX "
                         "shapes) and write the tuned table (aiter CSV schema) to CSV")
    ap.add_argument("--tuned", default=None, metavar="CSV",
                    help="use a tuned table for the library's auto calls (--sweep)")
    ap.add_argument("--quant", action="store_true",
                    help="activation quantise+pack bandwidth (bf16 -> mxfp8/mxfp4/fp8_block), one JSON line")
    ap.add_argument("--quant-m", type=int, default=None, help="--quant: only this row count")
    ap.add_argument("--quant-fmt", default=None, choices=["mxfp8", "mxfp4", "fp8_block"],
                    help="--quant: only this format")
    ap.add_argument("--sweep", action="store_true",
                    help="fp8 block-scale sweep, M in {1,16,64,128,1024,8192} x 4 (N,K) shapes, one JSON line")
    ap.add_argument("--chain", action="store_true",
                    help="decode chain: the four configs[1] (N,K) GEMMs at M=16 back to back (one L2 flush "
                         "before the chain) against the same calls one at a time, one JSON line")
    ap.add_argument("--grouped", action="store_true",
                    help="grouped (MoE) GEMMs of the three families on decode and prefill expert mixes, one JSON line")
    ap.add_argument("--families", default="fp8block,mxfp8,mxfp4",
                    help="comma-separated families for --grouped")
    ap.add_argument("--no-configs4", action="store_true",
                    help="skip the configs[4] sub-record (N-sharded M=16384 N=57344 K=8192 MXFP4 and "
                         "fp32 block-scale, GEMM and GEMM + all-gather)")
    ap.add_argument("--c4-steps", type=int, default=8)
    ap.add_argument("--c4-strips", type=int, default=4, help="M strips of the overlapped GEMM + all-gather")
    ap.add_argument("--c4-grid", type=int, default=0,
                    help="CTA cap of the overlapped configs[4] strip GEMMs (0 = one per SM; a cap leaves "
                         "SMs to NCCL's kernels)")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the N=1 mxfp4 and sustained sub-records")
    args = ap.parse_args()
    if args.shape:
        args.m, args.n, args.k = (int(v) for v in args.shape.split(","))
    return args


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        # raw samples go to $BENCH_CLOCKS_DIR (kept) or a temporary directory
        out_dir = Path(os.environ.get("BENCH_CLOCKS_DIR") or tempfile.mkdtemp(prefix="bench_clocks_"))
        out_dir.mkdir(parents=True, exist_ok=True)
        self.path = out_dir / f"clocks_rank{self.gpu}.csv"
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


# ---------------------------------------------------------------------------
# synthetic inputs on the device (torch ops; not the measured path)
# ---------------------------------------------------------------------------
def quant_mx_torch(x, qmax, fp4):
    """Per-32 power-of-two scales 2^ceil(log2(amax/qmax)) and RNE-quantised
    elements, computed with torch on the device."""
    import torch
    rows, k = x.shape
    g = x.view(rows, k // 32, 32).float()
    amax = g.abs().amax(dim=2)
    mant, ex = torch.frexp((amax / qmax).clamp_min(1e-30))
    e = torch.where(mant == 0.5, ex - 1, ex).clamp(-127, 127)
    e = torch.where(amax > 0, e, torch.zeros_like(e))
    sf = (e + 127).to(torch.uint8)
    scaled = torch.ldexp(g, (-e).unsqueeze(-1).float()).view(rows, k)
    if not fp4:
        return scaled.to(torch.float8_e4m3fn), sf
    # E2M1 RNE by thresholds on |v|: codes 0..7 <-> {0,.5,1,1.5,2,3,4,6}
    a = scaled.abs()
    thr = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=x.device)
    code = torch.bucketize(a, thr, right=False).to(torch.uint8)   # ties go low...
    ties_up = torch.isin(a, torch.tensor([0.75, 1.75, 3.5], device=x.device))  # ...except to even codes
    code = code + ties_up.to(torch.uint8)
    code = code | ((scaled < 0).to(torch.uint8) << 3)
    packed = code[:, 0::2] | (code[:, 1::2] << 4)
    return packed.contiguous(), sf


def make_mx_inputs(bs, m, n, k, fp4, layout, device, seed):
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    x = torch.randn(m, k, device=device, generator=gen)
    w = torch.randn(n, k, device=device, generator=gen)
    qmax = 6.0 if fp4 else 448.0
    qa, sa = quant_mx_torch(x, qmax, fp4)
    qb, sb = quant_mx_torch(w, qmax, fp4)
    del x, w
    if not fp4:
        if layout[0] == "n":
            qa = qa.view(torch.uint8).t().contiguous().view(torch.float8_e4m3fn)
        if layout[1] == "t":
            qb = qb.view(torch.uint8).t().contiguous().view(torch.float8_e4m3fn)
    return qa, qb, sa, sb


def make_e8m0block_inputs(bs, m, n, k, device, seed):
    """E4M3 A [M,K] and shuffle_weight(16,16) B, E8M0 scale bytes 124..130
    (the reference's fill_scales range): SFA column-major [M,K/128] (bytes
    [K/128][M]), SFB [N/128,K/128]."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    qa = (torch.randn(m, k, device=device, generator=gen) * 64).to(torch.float8_e4m3fn)
    qb = (torch.randn(n, k, device=device, generator=gen) * 64).to(torch.float8_e4m3fn)
    qb_sh = bs.pack_b(qb.view(torch.uint8), "shuffle16", unpack=True).view(torch.float8_e4m3fn)
    sfa_t = torch.randint(124, 131, (k // 128, m), device=device, generator=gen, dtype=torch.uint8)
    sfb = torch.randint(124, 131, (n // 128, k // 128), device=device, generator=gen, dtype=torch.uint8)
    return qa, qb_sh, sfa_t, sfb


def make_fp8block_inputs(m, n, k, device, seed):
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    x = torch.randn(m, k, device=device, generator=gen)
    w = torch.randn(n, k, device=device, generator=gen)
    xa = x.view(m, k // 128, 128).abs().amax(dim=2).clamp_min(1e-30) / 448.0
    qa = (x.view(m, k // 128, 128) / xa.unsqueeze(-1)).view(m, k).to(torch.float8_e4m3fn)
    wb = w.view(n // 128, 128, k // 128, 128).abs().amax(dim=(1, 3)).clamp_min(1e-30) / 448.0
    qb = (w.view(n // 128, 128, k // 128, 128) / wb[:, None, :, None]).view(n, k).to(torch.float8_e4m3fn)
    # K-panel preshuffle B'[K/128][N][128]
    qb_kp = qb.view(torch.uint8).view(n, k // 128, 128).permute(1, 0, 2).contiguous().view(torch.float8_e4m3fn)
    return qa, qb_kp, xa.contiguous(), wb.contiguous()


# ---------------------------------------------------------------------------
# CPU baseline (the reference's CPU GEMM restated in oracle/, "port")
# ---------------------------------------------------------------------------
def use_all_host_cores():
    """The CPU legs run on every core this process may use (torchrun sets
    OMP_NUM_THREADS=1 for its workers); must run before the OpenMP library
    of the oracle is loaded."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(n)
    return n


def cpu_gemm(workload, rows, n, k, seed=0):
    """One CPU verification GEMM of `rows` activation rows against the whole
    N x K weight matrix, ready to time: returns (fn, kind, module).  The
    reference's own CPU functions (oracle/_ref, compiled from its host
    drivers) are used when that library is built ("reference"); otherwise the
    restatement in oracle/ ("port").  Inputs are quantised by the oracle."""
    import numpy as np
    from oracle import oracle as orc
    from oracle import ref as rlib
    orc.build()
    use_ref = rlib.available()
    g = rlib if use_ref else orc
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    if workload == "mxfp8":
        (qa, sa), (qb, sb) = orc.quant_mxfp8(x), orc.quant_mxfp8(w)
        fn = lambda: g.gemm_mxfp8(qa, qb, sa, sb)
    elif workload == "mxfp4":
        (qa, sa), (qb, sb) = orc.quant_mxfp4(x), orc.quant_mxfp4(w)
        fn = lambda: g.gemm_mxfp4(qa, qb, sa, sb)
    elif workload == "e8m0block":
        qa, qb = orc.quant_mxfp8(x)[0], orc.quant_mxfp8(w)[0]
        sfa_t = rng.integers(124, 131, size=(k // 128, rows)).astype(np.uint8)
        sfb = rng.integers(124, 131, size=(n // 128, k // 128)).astype(np.uint8)
        fn = lambda: g.gemm_e8m0_block(qa, qb, sfa_t, sfb)
    else:
        (qa, sa), (qb, sb) = orc.quant_fp8_block(x, 1), orc.quant_fp8_block(w, 128)
        fn = lambda: g.gemm_fp8_block(qa, qb, sa, sb)
    return fn, ("reference" if use_ref else "port"), g


CPU_KIND_NOTE = {
    "reference": "the reference's own CPU verification GEMM (compiled from its host-driver sources into "
                 "oracle/_ref with g++ -O3 -fopenmp)",
    "port": "the reference's CPU verification GEMM restated in oracle/ (oracle/_ref not built)",
}


def cpu_baseline(workload, m, n, k, target_s=12.0, max_rows=None):
    use_all_host_cores()
    fn1, kind, g = cpu_gemm(workload, 1, n, k)
    t0 = time.perf_counter()
    fn1()
    t1 = time.perf_counter() - t0
    rows = max(1, min(int(target_s / max(t1, 1e-6)), max_rows or m, m))
    t = t1
    if rows > 1:
        fn, _, _ = cpu_gemm(workload, rows, n, k)
        t0 = time.perf_counter()
        fn()
        t = time.perf_counter() - t0
    tflops = 2.0 * rows * n * k / t / 1e12
    return {"value": tflops, "unit": "TFLOPS", "cores": g.num_threads(), "kind": kind,
            "sample": f"{rows} of {m} rows x N={n} x K={k} ({t:.1f} s, extrapolated to TFLOPS); "
                      f"{CPU_KIND_NOTE[kind]}"}


def metric_name(workload):
    return {"mxfp8": "MXFP8 block-scaled GEMM TFLOPS (8192^3)",
            "mxfp4": "MXFP4 block-scaled GEMM TFLOPS (8192^3)",
            "fp8block": "FP8 fp32-block-scale GEMM TFLOPS",
            "e8m0block": "FP8 E8M0-block-scale GEMM TFLOPS (launch_blockscale_bpreshuffle)"}[workload]


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    use_all_host_cores()
    m, n, k = args.m, args.n * world, args.k
    rows = 1
    fn, kind, g = cpu_gemm(args.workload, rows, n, k)
    # bound the whole run to a few minutes
    t0 = time.perf_counter()
    fn()
    t_one = time.perf_counter() - t0
    budget = 150.0
    steps = max(1, min(args.steps, int(budget / max(t_one, 1e-6))))
    for _ in range(min(args.warmup, 2)):
        fn()
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    dt = (time.perf_counter() - t0) / steps
    value = 2.0 * rows * n * k / dt / 1e12
    cores = g.num_threads()
    line = {
        "impl": "reference", "metric": metric_name(args.workload), "value": value, "unit": "TFLOPS",
        "n_gpus": world, "steps": steps, "warmup": min(args.warmup, 2), "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {"mxfp8": "mxfp8", "mxfp4": "mxfp4"}.get(args.workload, "fp8-e4m3"),
        "data": "synthetic",
        "config": {"workload": f"{args.workload} M={m} N={n} K={k} layout={args.layout}",
                   "sample_rows_per_step": rows},
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": cores, "kind": kind,
                         "sample": f"{rows} row x N={n} x K={k} per step, {steps} steps"},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": CPU_KIND_NOTE[kind] + "; the reference's GPU kernels are HIP/gfx950-only",
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    bs = importlib.import_module("355_1_trans_b200")
    peaks, peak_kind = load_peaks()

    m, n, k = args.m, args.n, args.k
    wl = args.workload
    fp4 = wl == "mxfp4"
    b_format = args.b_format or ("shuffle16" if fp4 else "raw")
    if wl in ("mxfp8", "mxfp4"):
        qa, qb, sa, sb = make_mx_inputs(bs, m, n, k, fp4, args.layout if not fp4 else "tn", dev, 1234 + rank)
        if b_format == "shuffle16":
            if not fp4 and args.layout[1] != "n":
                raise SystemExit("--b-format shuffle16 needs a K-major B (layout tn or nn)")
            qb = bs.pack_b(qb.view(torch.uint8), "shuffle16", unpack=True).view(qb.dtype)
        if world > 1:
            # the replicated activation A (and its scales) is broadcast once from rank 0
            dist.broadcast(qa.view(torch.uint8), 0)
            dist.broadcast(sa, 0)
        sa_n = bs.pack_scales(sa)   # weights' and activations' scales in the native atom layout
        sb_n = bs.pack_scales(sb)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        if fp4:
            call = lambda: bs.gemm_a4w4_mxfp4(qa, qb, sa_n, sb_n, out=out, scale_format="native",
                                              kernel=args.kernel, b_format=b_format, split_k=args.split_k)
            a_bytes, b_bytes = m * k // 2, n * k // 2
        else:
            call = lambda: bs.gemm_a8w8_mxfp8(qa, qb, sa_n, sb_n, layout=args.layout, out=out,
                                              scale_format="native", kernel=args.kernel, b_format=b_format,
                                              split_k=args.split_k)
            a_bytes, b_bytes = m * k, n * k
        sf_bytes = (m + n) * k // 32
    elif wl == "e8m0block":
        qa, qb, sa, sb = make_e8m0block_inputs(bs, m, n, k, dev, 1234 + rank)
        if world > 1:
            dist.broadcast(qa.view(torch.uint8), 0)
            dist.broadcast(sa, 0)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        call = lambda: bs.gemm_a8w8_blockscale_bpreshuffle(qa, qb, sa.t(), sb, torch.bfloat16, out)
        a_bytes, b_bytes = m * k, n * k
        sf_bytes = m * (k // 128) + (n // 128) * (k // 128)
    else:
        qa, qb, sa, sb = make_fp8block_inputs(m, n, k, dev, 1234 + rank)
        if world > 1:
            dist.broadcast(qa.view(torch.uint8), 0)
            dist.broadcast(sa, 0)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        call = lambda: bs.gemm_a8w8_bpreshuffle(qa, qb, sa, sb, torch.bfloat16, preshuffled=True, out=out,
                                                kernel=args.kernel, split_k=args.split_k)
        a_bytes, b_bytes = m * k, n * k
        sf_bytes = 4 * m * (k // 128) + 4 * (n // 128) * (k // 128)
    flops = 2.0 * m * n * k
    alg_bytes = a_bytes + b_bytes + sf_bytes + 2 * m * n
    # When the inputs fit in the 126 MB L2, a 256 MiB read evicts them before
    # every timed call, and the value comes from the per-call events around
    # the GEMM alone (the flush also lets the host enqueue the next call, so a
    # short kernel is not timed behind its own launch).  Larger inputs stream
    # from HBM on every call anyway.
    in_bytes = a_bytes + b_bytes + sf_bytes
    flush_l2, hbm_bound = l2_policy(m, in_bytes)
    if flush_l2:
        flush_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)   # 256 MiB
        flush_sink = torch.empty((), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()

    # The clock sampler starts (and takes its first readings) before the
    # warm-up, so the timed steps follow the warm-up without an idle gap in
    # which the SM clock could fall back.
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0

    stream = torch.cuda.current_stream(dev)
    # A call shorter than the host's launch path (decode shapes) is timed as
    # one CUDA-graph replay of the K steps, so host overhead stays out of the
    # device time; with the L2 flush in the steps, a graph of the K flushes
    # alone is timed too and subtracted.
    e_a, e_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_a.record(stream)
    for _ in range(5):
        call()
    e_b.record(stream)
    torch.cuda.synchronize()
    use_graph = e_a.elapsed_time(e_b) / 5 < 0.25
    graph_main = graph_flush = None
    if use_graph:
        graph_main = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_main):
            for _ in range(args.steps):
                if flush_l2:
                    torch.sum(flush_buf, dim=0, out=flush_sink)
                call()
        if flush_l2:
            graph_flush = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph_flush):
                for _ in range(args.steps):
                    torch.sum(flush_buf, dim=0, out=flush_sink)
        graph_main.replay()
        if graph_flush is not None:
            graph_flush.replay()
        torch.cuda.synchronize()
        assert bs.check_device_error() == 0
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    torch.cuda.nvtx.range_push(f"bsgemm {wl} timed x{args.steps}")   # one range per timed region
    if use_graph:
        graph_main.replay()
    else:
        for i in range(args.steps):
            if flush_l2:
                torch.sum(flush_buf, dim=0, out=flush_sink)
            starts[i].record(stream)
            call()
            ends[i].record(stream)
    torch.cuda.nvtx.range_pop()
    t_end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    if use_graph:
        flush_ms = 0.0
        if graph_flush is not None:
            f_a, f_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f_a.record(stream)
            graph_flush.replay()
            f_b.record(stream)
            torch.cuda.synchronize()
            flush_ms = f_a.elapsed_time(f_b)
        kern_ms = max(total_ms - flush_ms, 1e-6) / args.steps
    else:
        kern_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    tm = torch.tensor([total_ms, kern_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    total_ms, kern_ms = float(tm[0]), float(tm[1])
    # with the flush in the loop the wall time between steps holds the flush
    # kernels, so the per-call GEMM time is the step time
    ms_per_step = kern_ms if (flush_l2 or use_graph) else total_ms / args.steps
    value = world * flops / (ms_per_step * 1e-3) / 1e12
    assert bs.check_device_error() == 0

    # optional all-gather of the bf16 column shards (reported, not in value)
    allgather_ms = None
    if world > 1:
        gathered = torch.empty(world, m, n, dtype=torch.bfloat16, device=dev)
        for _ in range(2):
            dist.all_gather_into_tensor(gathered, out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            dist.all_gather_into_tensor(gathered, out)
        e1.record(stream)
        torch.cuda.synchronize()
        ag = torch.tensor([e0.elapsed_time(e1) / 5], dtype=torch.float64, device=dev)
        dist.all_reduce(ag, op=dist.ReduceOp.MAX)
        allgather_ms = float(ag[0])
        del gathered

    # e2e through the public API with pinned host buffers (reference-facing
    # row-major scales, packed inside the library call)
    e2e = None
    h_a = qa.view(torch.uint8).cpu().pin_memory()
    h_b = qb.view(torch.uint8).cpu().pin_memory()
    h_sa = sa.cpu().pin_memory()
    h_sb = sb.cpu().pin_memory()
    h_out = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
    d_a, d_b = torch.empty_like(qa.view(torch.uint8)), torch.empty_like(qb.view(torch.uint8))
    d_sa, d_sb = torch.empty_like(sa), torch.empty_like(sb)
    # MX, layout tn: the host-staged entry point pipelines the copies with the
    # GEMM blocks (bsgemm_mx_host_gemm); the other workloads copy, call, copy back
    host_staged = wl in ("mxfp8", "mxfp4") and args.layout == "tn" and world == 1
    if host_staged:
        del d_a, d_b, d_sa, d_sb
        fdt = torch.uint8 if fp4 else torch.float8_e4m3fn
        h_a8, h_b8 = h_a.view(fdt), h_b.view(fdt)
        probe = bs.Args()
        bs.lib().bsgemm_args_init(ctypes.byref(probe))
        probe.m, probe.n, probe.k = m, n, k
        fam = bs.FAMILY_MXFP4 if fp4 else bs.FAMILY_MXFP8
        host_ws = torch.empty(int(bs.lib().bsgemm_mx_host_workspace_size(fam, ctypes.byref(probe))),
                              dtype=torch.uint8, device=dev)

    def e2e_step():
        if host_staged:
            bs.gemm_mx_from_host(h_a8, h_b8, h_sa, h_sb, fp4=fp4, out=h_out, b_format=b_format,
                                 workspace=host_ws)
            return
        d_b.copy_(h_b, non_blocking=True)
        d_sb.copy_(h_sb, non_blocking=True)
        if world == 1 or rank == 0:
            d_a.copy_(h_a, non_blocking=True)
            d_sa.copy_(h_sa, non_blocking=True)
        if world > 1:
            # the replicated activations cross the host link once (rank 0) and
            # reach the other ranks over NVLink
            dist.broadcast(d_a, 0)
            dist.broadcast(d_sa, 0)
        if wl == "mxfp8":
            r = bs.gemm_a8w8_mxfp8(d_a.view(torch.float8_e4m3fn), d_b.view(torch.float8_e4m3fn), d_sa, d_sb,
                                   layout=args.layout, out=out, b_format=b_format)
        elif wl == "mxfp4":
            r = bs.gemm_a4w4_mxfp4(d_a, d_b, d_sa, d_sb, out=out, b_format=b_format)
        elif wl == "e8m0block":
            r = bs.gemm_a8w8_blockscale_bpreshuffle(d_a.view(torch.float8_e4m3fn), d_b.view(torch.float8_e4m3fn),
                                                    d_sa.t(), d_sb, torch.bfloat16, out)
        else:
            r = bs.gemm_a8w8_bpreshuffle(d_a.view(torch.float8_e4m3fn), d_b.view(torch.float8_e4m3fn),
                                         d_sa, d_sb, torch.bfloat16, preshuffled=True, out=out)
        h_out.copy_(r, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    et = torch.tensor([e0.elapsed_time(e1) / args.e2e_steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_ms = float(et[0])
    a_host = h_a.numel() + h_sa.numel() * h_sa.element_size()
    b_host = h_b.numel() + h_sb.numel() * h_sb.element_size()
    h2d = a_host + world * b_host          # the whole job: A once, every rank its own B
    e2e = {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(world * m * n * 2),
           "host_bytes_per_rank": {"rank0_h2d": int(a_host + b_host), "other_h2d": int(b_host) if world > 1 else None,
                                   "d2h": int(m * n * 2)},
           "path": ("bsgemm_mx_host_gemm (host-staged C-ABI call: pinned host A, B, row-major scales and C; "
                    "H2D chunks, GEMM blocks and D2H blocks pipelined, result complete on return)"
                    if host_staged else
                    "C-ABI call with pinned host buffers, reference-facing row-major scales" +
                    ("; A and its scales copied to rank 0 only and NCCL-broadcast, each rank copies its own "
                     "B shard and reads back its own C shard" if world > 1 else ""))}

    # roofline of the GEMM kernel
    if hbm_bound:
        bound, unit = "hbm", "GB/s"
        achieved = alg_bytes / (kern_ms * 1e-3) / 1e9
        peak = peaks.get("hbm_gbs")
        basis = f"hbm_gbs ({peak_kind})"
    else:
        bound, unit = "tensor", "TFLOP/s"
        achieved = flops / (kern_ms * 1e-3) / 1e12
        # the timed loop is long enough to reach the 1 kW power cap: when the
        # sampled clocks show sw_power_cap, compare against the measured
        # sustained GEMM peak (same regime), else against the burst peak
        mult = 4.0 if fp4 else 2.0
        burst = peaks.get("bf16_tflops") * mult
        sustained = (peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")) * mult
        capped = bool(clk) and "sw_power_cap" in clk.get("reasons", [])
        peak = sustained if capped else burst
        basis = (f"{mult:.0f} x bf16_tflops_{'sustained' if capped else 'burst'} ({peak_kind}): dense "
                 f"{'MXFP4' if fp4 else 'FP8/MXFP8'} tensor rate is {mult:.0f}x bf16 on B200; "
                 f"{'sw_power_cap was active during the timed region' if capped else 'no power cap seen'}")
    traffic, traffic_src = load_traffic(wl, m, n, k, b_format if wl in ("mxfp8", "mxfp4") else None)
    roofline = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                "frac": achieved / peak if peak else None, "traffic": traffic, "traffic_source": traffic_src,
                "peak_basis": basis,
                "algorithmic_bytes_per_launch": alg_bytes, "flops_per_launch": flops,
                "kernel_ms": kern_ms}
    if bound == "tensor":
        roofline["frac_of_burst_peak"] = achieved / burst
        roofline["frac_of_sustained_peak"] = achieved / sustained

    extra = {}
    if world == 1 and not args.no_extra and wl == "mxfp8" and (m, n, k) == (8192, 8192, 8192):
        extra["sustained"] = sustained_record(call, kern_ms, stream, local, flops, peaks, peak_kind)
    # free the headline's device buffers before the other sub-records
    out = qa = qb = sa = sb = call = None
    sa_n = sb_n = flush_buf = host_ws = d_a = d_b = d_sa = d_sb = None
    graph_main = graph_flush = None
    torch.cuda.empty_cache()
    if world == 1 and not args.no_extra and wl == "mxfp8" and (m, n, k) == (8192, 8192, 8192):
        extra["mxfp4"] = mxfp4_record(bs, dev, stream, peaks, peak_kind, args.layout)
    if not args.no_configs4:
        import bench_configs4
        c4 = bench_configs4.run(sys.modules[__name__], bs, dev, world, rank, dist if world > 1 else None, peaks,
                                steps=args.c4_steps, strips=args.c4_strips, overlap_grid=args.c4_grid)
        if c4 is not None:
            extra["configs4"] = c4

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl, m, n, k)

    if rank == 0:
        line = {
            "metric": metric_name(wl), "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": {"mxfp8": "mxfp8", "mxfp4": "mxfp4", "fp8block": "fp8-e4m3", "e8m0block": "fp8-e4m3"}[wl],
            "data": "synthetic (seeded torch.randn, quantised on device)",
            "config": {"workload": f"{wl} M={m} N={n}/rank K={k} layout={args.layout if wl == 'mxfp8' else 'tn'}",
                       "b_format": b_format if wl in ("mxfp8", "mxfp4") else
                       ("shuffle16" if wl == "e8m0block" else "kpanel128"),
                       "out": "bf16", "accum": "fp32",
                       "scales": {"fp8block": "fp32 1x128 / 128x128",
                                  "e8m0block": "E8M0 1x128 / 128x128 (reference launcher layout)"}.get(
                                      wl, "native tcgen05 atoms (pre-packed)"),
                       "parallelism": f"N-sharded x{world}" if world > 1 else "single GPU",
                       "l2": (f"inputs ({in_bytes / 1e6:.0f} MB) below "
                              f"{'twice ' if hbm_bound else ''}the 126 MB L2: a 256 MiB read flushes L2 before "
                              "every timed call; value and ms_per_step exclude the flushes")
                             if flush_l2 else
                             f"inputs ({in_bytes / 1e6:.0f} MB) exceed the 126 MB L2 (and each step writes a C "
                             "larger than L2); no flush",
                       "timing": ("one CUDA-graph replay of the K steps (minus a graph of the K flushes)"
                                  if use_graph else "CUDA events around each of the K calls on the launching stream")},
            "gpu_launches": args.steps,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
        }
        if allgather_ms is not None:
            line["allgather_ms"] = allgather_ms
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def sustained_record(call, kern_ms, stream, local, flops, peaks, peak_kind, seconds=2.5):
    """The headline GEMM back to back for a timed region of `seconds` (long
    enough to reach the 1 kW power cap), with its own clock samples; compared
    with the measured sustained GEMM peak."""
    import torch
    steps = max(1, int(seconds * 1e3 / max(kern_ms, 1e-3)))
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    for _ in range(20):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        call()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / steps
    tflops = flops / (ms * 1e-3) / 1e12
    sustained = 2.0 * (peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops"))
    return {"steps": steps, "timed_s": ms * steps / 1e3, "ms_per_step": ms, "tflops": tflops,
            "peak": sustained, "frac": tflops / sustained, "frac_of_burst_peak": tflops / (2.0 * peaks["bf16_tflops"]),
            "peak_basis": f"2 x bf16_tflops_sustained ({peak_kind})", "clocks": clk}


def mxfp4_record(bs, dev, stream, peaks, peak_kind, layout, steps=20):
    """configs[3]'s 8192^3 MXFP4 GEMM (B in shuffle_weight(16,16), native
    scales): its 71 MB of inputs fit in L2, so a 256 MiB read flushes L2
    before every call and the per-call events exclude the flushes."""
    import torch
    m = n = k = 8192
    qa, qb, sa, sb = make_mx_inputs(bs, m, n, k, True, "tn", dev, 4321)
    qb = bs.pack_b(qb, "shuffle16", unpack=True)
    sa_n, sb_n = bs.pack_scales(sa), bs.pack_scales(sb)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    call = lambda: bs.gemm_a4w4_mxfp4(qa, qb, sa_n, sb_n, out=out, scale_format="native", b_format="shuffle16")
    flush_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)
    for _ in range(5):
        call()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        torch.sum(flush_buf, dim=0, out=sink)
        a.record(stream)
        call()
        b.record(stream)
    torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    flops = 2.0 * m * n * k
    tflops = flops / (ms * 1e-3) / 1e12
    peak = 4.0 * peaks["bf16_tflops"]
    return {"workload": "mxfp4 M=N=K=8192 layout=tn, B shuffle_weight(16,16) read in place, native scales, bf16 out",
            "steps": steps, "ms_per_step": ms, "tflops": tflops, "peak": peak, "frac": tflops / peak,
            "peak_basis": f"4 x bf16_tflops burst ({peak_kind}): dense MXFP4 tensor rate is 4x bf16 on B200",
            "l2": "256 MiB read flushes L2 before every call; excluded", "target_frac": 0.60}


def run_sweep(args):
    """Decode/prefill sweep: M in {1,16,64,128,1024,8192} x (N,K) in {(7168,2048),
    (4096,7168), (24576,1536), (7168,18432)}, fp32 block scales, K-panel B,
    bf16 out.

    Device time per GEMM call with cold L2: one CUDA graph replays R times
    (L2 flush, GEMM call) and a second graph replays the R flushes alone; the
    difference of the two CUDA-event times, divided by R, is the time of one
    call including its launch gap behind the flush.  (Events on this GPU tick
    in 2.048 us steps, too coarse to time one decode-sized call; over R calls
    the step is R times smaller.)  The flush READS a 256 MiB buffer: a
    write-based flush would leave ~126 MB of dirty lines whose write-back
    would be charged to the GEMM.  The call's kernels (GEMM and, when K is
    split, the reduce) are all captured.  Also reports the host time of one
    eager call."""
    import torch
    dev = torch.device("cuda", 0)
    bs = importlib.import_module("355_1_trans_b200")
    peaks, peak_kind = load_peaks()
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)   # 256 MiB
    sink = torch.empty((), dtype=torch.float32, device=dev)
    reps = 20

    def graph_time(fn, rounds):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(rounds):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        del g
        return statistics.median(ts)

    def flushes():
        for _ in range(reps):
            torch.sum(flush, dim=0, out=sink)

    rows = []
    for (n, k) in ((7168, 2048), (4096, 7168), (24576, 1536), (7168, 18432)):
        qa_full, qb, sa_full, sb = make_fp8block_inputs(8192, n, k, dev, 7)
        for m in (1, 16, 64, 128, 1024, 8192):
            qa, sa = qa_full[:m].contiguous(), sa_full[:m].contiguous()
            out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            call = lambda: bs.gemm_a8w8_bpreshuffle(qa, qb, sa, sb, torch.bfloat16, preshuffled=True, out=out)

            def flush_and_gemm():
                for _ in range(reps):
                    torch.sum(flush, dim=0, out=sink)
                    call()

            for _ in range(3):
                call()
            torch.cuda.synchronize()
            rounds = max(3, args.steps)
            t_both = graph_time(flush_and_gemm, rounds)
            t_flush = graph_time(flushes, rounds)
            ms = max(t_both - t_flush, 1e-6) / reps
            host_us = []
            for _ in range(rounds):
                t0 = time.perf_counter()
                call()
                host_us.append((time.perf_counter() - t0) * 1e6)
                torch.cuda.synchronize()
            byts = m * k + n * k + 4 * m * (k // 128) + 4 * (n // 128) * (k // 128) + 2 * m * n
            rows.append({"m": m, "n": n, "k": k, "us": ms * 1e3, "host_call_us": statistics.median(host_us),
                         "tflops": 2.0 * m * n * k / ms / 1e9,
                         "gbs": byts / ms / 1e6, "hbm_frac": byts / ms / 1e6 / peaks["hbm_gbs"]})
    assert bs.check_device_error() == 0
    print(json.dumps({"sweep": "fp8 block-scale, M x (N,K) grid", "hbm_peak_gbs": peaks["hbm_gbs"],
                      "peak_kind": peak_kind, "l2": "flushed (256 MiB read) before every timed call",
                      "timing": f"graph of {reps} x (flush, call) minus graph of {reps} flushes",
                      "rows": rows}), flush=True)
    return 0


def run_chain(args):
    """Decode chain: the fp32 block-scale GEMMs of BASELINE configs[1]'s four
    (N, K) groups at M=16 (K-panel B, bf16 out, the library's automatic
    kernel and split), issued back to back as one serving step would.  One
    CUDA graph replays R x (256 MiB L2-flushing read, the four GEMMs); a
    second replays the flushes alone; the difference / R is the chain's time.
    Each GEMM launches with programmatic dependent launch, so its prologue
    and L2 prefetch of weights overlap the GEMM before it.  Compared with the
    sum of the four calls timed one at a time (a flush before each)."""
    import torch
    dev = torch.device("cuda", 0)
    bs = importlib.import_module("355_1_trans_b200")
    peaks, peak_kind = load_peaks()
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)
    reps = 10

    def graph_time(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(max(3, min(args.steps, 10))):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        del g
        return statistics.median(ts)

    m = 16
    calls, wbytes = [], 0
    for i, (n, k) in enumerate(((7168, 2048), (4096, 7168), (24576, 1536), (7168, 18432))):
        qa, qb, sa, sb = make_fp8block_inputs(m, n, k, dev, 20 + i)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        calls.append((lambda qa=qa, qb=qb, sa=sa, sb=sb, out=out:
                      bs.gemm_a8w8_bpreshuffle(qa, qb, sa, sb, torch.bfloat16, preshuffled=True, out=out)))
        wbytes += n * k + 4 * (n // 128) * (k // 128)
    for c in calls:
        c()
    torch.cuda.synchronize()

    def flushes():
        for _ in range(reps):
            torch.sum(flush, dim=0, out=sink)

    def chain():
        for _ in range(reps):
            torch.sum(flush, dim=0, out=sink)
            for c in calls:
                c()

    t_flush = graph_time(flushes)
    chain_us = (graph_time(chain) - t_flush) / reps * 1e3
    single_us = []
    for c in calls:
        def one(c=c):
            for _ in range(reps):
                torch.sum(flush, dim=0, out=sink)
                c()
        single_us.append((graph_time(one) - t_flush) / reps * 1e3)
    assert bs.check_device_error() == 0
    hbm = peaks["hbm_gbs"]
    print(json.dumps({"chain": "fp32 block-scale decode, M=16, (N,K) = (7168,2048), (4096,7168), (24576,1536), "
                               "(7168,18432), K-panel B, bf16 out, automatic kernel and split",
                      "l2": "flushed (256 MiB read) once before the chain / before each single call",
                      "chain_us": chain_us, "single_us": single_us, "sum_single_us": sum(single_us),
                      "weight_bytes": wbytes, "chain_hbm_frac": wbytes / chain_us / 1e3 / hbm,
                      "single_hbm_frac": wbytes / sum(single_us) / 1e3 / hbm,
                      "hbm_peak_gbs": hbm, "peak_kind": peak_kind}), flush=True)
    return 0


def run_quant(args):
    """bsgemm_quantize bandwidth: bf16 activations [M, 7168] -> each format with
    its default scale layout, L2 flushed before every call, graph-difference
    timing as in the sweep.  Bytes = bf16 read + elements + scales written."""
    import torch
    dev = torch.device("cuda", 0)
    bs = importlib.import_module("355_1_trans_b200")
    peaks, peak_kind = load_peaks()
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)
    reps = 20

    def graph_time(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(max(3, min(args.steps, 10))):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        del g
        return statistics.median(ts)

    def flushes():
        for _ in range(reps):
            torch.sum(flush, dim=0, out=sink)

    t_flush = graph_time(flushes)
    rows = []
    k = 7168
    for m in ((args.quant_m,) if args.quant_m else (16, 128, 1024, 8192, 32768)):
        x = torch.randn(m, k, device=dev).to(torch.bfloat16)
        for fmt in ((args.quant_fmt,) if args.quant_fmt else ("mxfp8", "mxfp4", "fp8_block")):
            call = lambda: bs.quantize(x, fmt)
            call()

            def both():
                for _ in range(reps):
                    torch.sum(flush, dim=0, out=sink)
                    call()

            ms = max(graph_time(both) - t_flush, 1e-6) / reps
            out_bytes = m * k // (2 if fmt == "mxfp4" else 1) + (m * k // 32 if fmt != "fp8_block" else 4 * m * k // 128)
            byts = 2 * m * k + out_bytes
            rows.append({"m": m, "k": k, "format": fmt, "us": ms * 1e3, "gbs": byts / ms / 1e6,
                         "hbm_frac": byts / ms / 1e6 / peaks["hbm_gbs"]})
    assert bs.check_device_error() == 0
    print(json.dumps({"quantize": "bf16 [M, 7168] -> format, default scale layout", "hbm_peak_gbs": peaks["hbm_gbs"],
                      "peak_kind": peak_kind, "l2": "flushed before every call",
                      "timing": f"graph of {reps} x (flush, call) minus graph of {reps} flushes", "rows": rows}),
          flush=True)
    return 0


def run_grouped(args):
    """Grouped (MoE) GEMMs: fp32 block-scale (K-panel B), MXFP8 (raw B) and
    MXFP4 (shuffle_weight(16,16) B), native expert scales for MX, on
    (experts x tokens, N, K) mixes: decode (32 x 4), prefill (8 x 512) and
    ragged prefill (4096 tokens over 32 experts, multinomial, seed 0).
    Every expert has its own weights in HBM.  L2 flushed before every call,
    graph-difference timing as in the sweep; one call includes the scale
    packing the grouped entry point does.  Bytes = weights + activations +
    scales + bf16 C; hbm_frac relates them to the measured copy bandwidth."""
    import numpy as np
    import torch
    dev = torch.device("cuda", 0)
    bs = importlib.import_module("355_1_trans_b200")
    peaks, peak_kind = load_peaks()
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)
    reps = 10

    def graph_time(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(max(3, min(args.steps, 10))):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        del g
        return statistics.median(ts)

    def flushes():
        for _ in range(reps):
            torch.sum(flush, dim=0, out=sink)

    t_flush = graph_time(flushes)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    ragged = np.random.default_rng(0).multinomial(4096, np.ones(32) / 32)
    mixes = (("decode", [4] * 32, 4096, 7168), ("decode", [4] * 32, 7168, 2048),
             ("prefill", [512] * 8, 4096, 7168), ("ragged prefill", list(ragged), 4096, 7168))
    rows = []
    for family in args.families.split(","):
        if family not in ("fp8block", "mxfp8", "mxfp4"):
            raise SystemExit(f"unknown family {family}")
        for label, sizes, n, k in mixes:
            e, t = len(sizes), int(sum(sizes))
            offs = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32), device=dev)
            out = torch.empty(t, n, dtype=torch.bfloat16, device=dev)
            fp4 = family == "mxfp4"
            kb = k // 2 if fp4 else k
            if family == "fp8block":
                qa, _, sa, _ = make_fp8block_inputs(t, 128, k, dev, 1)
                _, qb1, _, sb1 = make_fp8block_inputs(1, n, k, dev, 2)
                B = qb1.view(torch.uint8).reshape(1, -1).repeat(e, 1).view(torch.float8_e4m3fn)
                B = B.reshape(e, k // 128, n, 128)
                SB = sb1.unsqueeze(0).repeat(e, 1, 1).contiguous()
                calls = [("auto", lambda: bs.gemm_a8w8_blockscale_grouped(qa, B, sa, SB, offs, max(sizes), out=out))]
                if "prefill" in label:   # CTA pairs, on request for grouped calls
                    calls.append(("pair", lambda: bs.gemm_a8w8_blockscale_grouped(qa, B, sa, SB, offs, max(sizes),
                                                                                  out=out, kernel="pair")))
                sf_bytes = 4 * t * (k // 128) + 4 * e * (n // 128) * (k // 128)
            else:
                hi = 256 if fp4 else 0x70   # any packed E2M1 byte; E4M3 bytes below the NaN codes
                qa = torch.randint(0, hi, (t, kb), device=dev, generator=gen, dtype=torch.uint8)
                B = torch.randint(0, hi, (e, n, kb), device=dev, generator=gen, dtype=torch.uint8)
                if not fp4:
                    qa, B = qa.view(torch.float8_e4m3fn), B.view(torch.float8_e4m3fn)
                else:
                    B = torch.stack([bs.pack_b(B[i], "shuffle16", unpack=True) for i in range(e)])
                sa = torch.randint(120, 134, (t, k // 32), device=dev, generator=gen, dtype=torch.uint8)
                sb1 = torch.randint(120, 134, (n, k // 32), device=dev, generator=gen, dtype=torch.uint8)
                SB = torch.stack([bs.pack_scales(sb1)] * e)
                ws = torch.empty(1 << 26, dtype=torch.uint8, device=dev)
                fn = bs.gemm_a4w4_mxfp4_grouped if fp4 else bs.gemm_a8w8_mxfp8_grouped
                bfmt = "shuffle16" if fp4 else "raw"
                calls = [("auto", lambda: fn(qa, B, sa, SB, offs, max(sizes), out=out, b_format=bfmt,
                                             b_scale_format="native", workspace=ws))]
                sf_bytes = t * (k // 32) + e * n * (k // 32)
            for kern, call in calls:
                for _ in range(3):
                    call()
                torch.cuda.synchronize()

                def both(call=call):
                    for _ in range(reps):
                        torch.sum(flush, dim=0, out=sink)
                        call()

                ms = max(graph_time(both) - t_flush, 1e-6) / reps
                byts = e * n * kb + t * kb + sf_bytes + 2 * t * n
                rows.append({"family": family, "mix": label, "kernel": kern, "experts": e, "tokens": t, "n": n,
                             "k": k, "us": ms * 1e3, "tflops": 2.0 * t * n * k / ms / 1e9, "gbs": byts / ms / 1e6,
                             "hbm_frac": byts / ms / 1e6 / peaks["hbm_gbs"]})
            del B, SB, qa, sa, out
    assert bs.check_device_error() == 0
    print(json.dumps({"grouped": "MoE GEMMs, experts x tokens, each expert its own weights",
                      "hbm_peak_gbs": peaks["hbm_gbs"], "peak_kind": peak_kind,
                      "l2": "flushed (256 MiB read) before every call",
                      "timing": f"graph of {reps} x (flush, call) minus graph of {reps} flushes", "rows": rows}),
          flush=True)
    return 0


# (N, K) groups of the reference's traced DeepSeek-V4 a8w8 deployment shapes
# (dsv4_a8w8_all_traced_shapes.csv: 125 rows, M from 6 to 16384), tuned at
# power-of-two M buckets: a call takes the row of the smallest tuned M >= its M.
DSV4_NK = ((1536, 7168), (2048, 7168), (6144, 7168), (7168, 3072), (7168, 7168), (7168, 16384), (7168, 21504),
           (8192, 1536), (65536, 1536))
DSV4_M = (1, 16, 64, 128, 256, 512, 1024, 2048, 4096)


def run_tune(args):
    """Tuned table for the fp8 block-scale sweep shapes (M <= 1024 of the
    decode/prefill grid), the DeepSeek-V4 (N, K) groups at power-of-two M
    buckets, and the skinny MX shapes M in {1, 16, 64, 128, 1024}, N = K = 8192;
    written in the aiter tuned-CSV schema."""
    import torch
    dev = torch.device("cuda", 0)
    bs = importlib.import_module("355_1_trans_b200")
    tuning = importlib.import_module("355_1_trans_b200.tuning")
    rows = []
    groups = [((n, k), (1, 16, 64, 128, 1024)) for (n, k) in ((7168, 2048), (4096, 7168), (24576, 1536), (7168, 18432))]
    groups += [((n, k), DSV4_M + ((8192, 16384) if (n, k) == (7168, 7168) else ())) for (n, k) in DSV4_NK
               if (n, k) not in {g[0] for g in groups}]
    for (n, k), ms in groups:
        qa_full, qb, sa_full, sb = make_fp8block_inputs(max(ms), n, k, dev, 7)

        def make_call(m, n_, k_, kernel, split, qa_full=qa_full, qb=qb, sa_full=sa_full, sb=sb):
            qa, sa = qa_full[:m].contiguous(), sa_full[:m].contiguous()
            out = torch.empty(m, n_, dtype=torch.bfloat16, device=dev)
            return lambda: bs.gemm_a8w8_bpreshuffle(qa, qb, sa, sb, torch.bfloat16, preshuffled=True, out=out,
                                                    kernel=kernel, split_k=split)

        rows += tuning.tune("fp8_block", [(m, n, k) for m in ms], make_call)
        del qa_full, qb, sa_full, sb
        torch.cuda.empty_cache()
    for fp4 in (False, True):
        n = k = 8192
        qa_full, qb, sa_full, sb = make_mx_inputs(bs, 1024, n, k, fp4, "tn", dev, 3)
        sb_n = bs.pack_scales(sb)
        if fp4:
            qb = bs.pack_b(qb.view(torch.uint8), "shuffle16", unpack=True)

        def make_call(m, n_, k_, kernel, split, fp4=fp4, qa_full=qa_full, sa_full=sa_full, qb=qb, sb_n=sb_n):
            qa = qa_full[:m].contiguous()
            sa_n = bs.pack_scales(sa_full[:m].contiguous())
            out = torch.empty(m, n_, dtype=torch.bfloat16, device=dev)
            if fp4:
                return lambda: bs.gemm_a4w4_mxfp4(qa, qb, sa_n, sb_n, out=out, scale_format="native",
                                                  b_format="shuffle16", kernel=kernel, split_k=split)
            return lambda: bs.gemm_a8w8_mxfp8(qa, qb, sa_n, sb_n, out=out, scale_format="native",
                                              kernel=kernel, split_k=split)

        rows += tuning.tune("mxfp4" if fp4 else "mxfp8", [(m, n, k) for m in (1, 16, 64, 128, 1024)], make_call)
    with open(args.tune, "w", newline="", encoding="utf-8") as f:
        import csv
        w = csv.DictWriter(f, fieldnames=tuning.TUNED_HEADER)
        w.writeheader()
        w.writerows(rows)
    print(json.dumps({"tuned_rows": len(rows), "csv": args.tune}), flush=True)
    return 0


def main():
    args = parse()
    if args.tuned:
        importlib.import_module("355_1_trans_b200.tuning").use_tuned(args.tuned)
    if args.impl == "reference":
        return run_reference(args)
    if args.tune:
        return run_tune(args)
    if args.sweep:
        return run_sweep(args)
    if args.quant:
        return run_quant(args)
    if args.chain:
        return run_chain(args)
    if args.grouped:
        return run_grouped(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

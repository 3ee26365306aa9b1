"""Per-shape kernel / split-K selection from a tuned table (aiter CSV schema).

The reference's tuning flow keeps one CSV row per (M, N, K) with the chosen
kernel and split-K (schema checked by the reference's analyze_gemm_config.py:23,
TUNED_HEADER).  This module keeps that schema:

    gfx,cu_num,M,N,K,bias,dtype,outdtype,scaleAB,bpreshuffle,libtype,solidx,splitK,us,kernelName,err_ratio,tflops,bw

with gfx = "sm_100a", libtype = "bsgemm", solidx = the bsgemm_args.kernel value
(0 auto, 1 single-CTA tiles, 2 CTA pairs, 3 transposed decode kernel, 4 wide
single-CTA 128x256 tiles), and
dtype naming the family ("fp8_block", "mxfp8", "mxfp4").

`tune()` times every candidate (kernel, split-K) of each shape on the current
GPU -- cold L2, CUDA-graph difference timing as in bench.py --sweep -- and
writes the fastest, with err_ratio = the fraction of its outputs that differ
from the unsplit result by more than 2^-7 |ref| + 1e-3.  `TunedTable.lookup()`
returns the row for an exact M, else for the smallest tuned M above it (the
CUDA-graph batch bucket), else for the largest tuned M.  `use_tuned()`
installs a table that the "auto" calls of this package consult.

tuned/b200_sm100a.csv (next to this module) was produced on a B200 by
`python bench.py --tune <csv>`: the fp8 block-scale decode/prefill shapes
M in {1, 16, 64, 128, 1024} x (N, K) in {(7168, 2048), (4096, 7168),
(24576, 1536), (7168, 18432)}; the (N, K) groups of the reference's traced
DeepSeek-V4 a8w8 shapes (dsv4_a8w8_all_traced_shapes.csv) at M in {1, 16,
64, 128, 256, 512, 1024, 2048, 4096} (and 8192, 16384 for (7168, 7168)); and
the skinny MX shapes M in {1, 16, 64, 128, 1024} x N = K = 8192.  It is
opt-in: `use_tuned(DEFAULT_TABLE)`.
"""
from __future__ import annotations

import bisect
import csv
import statistics
from pathlib import Path

TUNED_HEADER = ["gfx", "cu_num", "M", "N", "K", "bias", "dtype", "outdtype", "scaleAB", "bpreshuffle",
                "libtype", "solidx", "splitK", "us", "kernelName", "err_ratio", "tflops", "bw"]
KERNEL_NAMES = {0: "auto", 1: "1cta", 2: "pair", 3: "swap", 4: "wide"}
DEFAULT_TABLE = Path(__file__).resolve().parent / "tuned" / "b200_sm100a.csv"


class TunedTable:
    def __init__(self, rows: list[dict]):
        self._by_nk: dict[tuple, list[tuple[int, dict]]] = {}
        for r in rows:
            key = (r["dtype"], int(r["N"]), int(r["K"]))
            self._by_nk.setdefault(key, []).append((int(r["M"]), r))
        for v in self._by_nk.values():
            v.sort(key=lambda t: t[0])

    @classmethod
    def load(cls, path) -> "TunedTable":
        with open(path, newline="", encoding="utf-8") as f:
            rows = list(csv.DictReader(f))
        missing = [c for c in TUNED_HEADER if rows and c not in rows[0]]
        if missing:
            raise ValueError(f"{path}: missing columns {missing}")
        return cls(rows)

    def lookup(self, family: str, m: int, n: int, k: int):
        """(kernel name, split_k) for the shape, or None when (N, K) is not tuned."""
        lst = self._by_nk.get((family, n, k))
        if not lst:
            return None
        ms = [t[0] for t in lst]
        i = bisect.bisect_left(ms, m)
        row = lst[min(i, len(lst) - 1)][1]
        return KERNEL_NAMES[int(row["solidx"])], int(row["splitK"])


_ACTIVE: TunedTable | None = None


def use_tuned(table) -> None:
    """Install a TunedTable (or a CSV path) for the package's "auto" calls;
    None removes it."""
    global _ACTIVE
    _ACTIVE = TunedTable.load(table) if isinstance(table, (str, Path)) else table


def active() -> TunedTable | None:
    return _ACTIVE


def _graph_time(fn, reps, rounds):
    import torch
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


def candidates(family: str, m: int, k: int, n: int | None = None, sms: int = 148):
    """(kernel, split_k) pairs worth timing for a shape.  Split-K is tried
    only while a kernel's output tiles leave SMs idle (with n unknown, always)."""
    num_kb = k // (256 if family == "mxfp4" else 128)
    splits = [s for s in (1, 2, 3, 4, 6, 8, 12, 16) if s <= num_kb]
    out = [("auto", 0)]
    kernels = ["1cta"]
    if m <= 64:
        kernels.append("swap")
    if m >= 256 or (family == "fp8_block" and m > 128):
        kernels.append("pair")
    for kern in kernels:
        tiles = None
        if n is not None:
            tiles = -(-n // 128) * (1 if kern == "swap" else -(-m // 128))
        if kern == "pair" and family == "fp8_block":
            out.append((kern, 0))   # the pair kernel's partial last wave as K slices
        for s in splits:
            if kern == "pair" and s > 1:
                continue
            if s > 1 and tiles is not None and tiles >= sms:
                continue
            out.append((kern, s))
    return out


def tune(family: str, shapes, make_call, *, reps: int = 10, rounds: int = 5, gfx: str = "sm_100a",
         cu_num: int = 148, out_csv=None) -> list[dict]:
    """Time every candidate of every shape and return (and optionally write)
    the tuned rows.  make_call(m, n, k, kernel, split_k) must return a
    zero-argument function that runs one GEMM and returns its output tensor."""
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)   # 256 MiB, read to evict L2
    sink = torch.empty((), dtype=torch.float32, device=dev)

    def flushes():
        for _ in range(reps):
            torch.sum(flush, dim=0, out=sink)

    t_flush = _graph_time(flushes, reps, rounds)
    rows = []
    for (m, n, k) in shapes:
        ref = make_call(m, n, k, "1cta", 1)().float()
        best = None
        for kern, split in candidates(family, m, k, n, cu_num):
            call = make_call(m, n, k, kern, split)
            try:
                out = call()
            except RuntimeError:
                continue   # the combination is not supported for this shape
            torch.cuda.synchronize()

            def both():
                for _ in range(reps):
                    torch.sum(flush, dim=0, out=sink)
                    call()

            us = max(_graph_time(both, reps, rounds) - t_flush, 1e-6) / reps * 1e3
            if best is None or us < best[0]:
                err = (out.float() - ref).abs() > (2.0 ** -7) * ref.abs() + 1e-3
                best = (us, kern, split, float(err.float().mean().item()))
        us, kern, split, err_ratio = best
        solidx = {v: k for k, v in KERNEL_NAMES.items()}[kern]
        if family == "mxfp4":
            byts = (m * k + n * k) // 2 + (m + n) * k // 32 + 2 * m * n
        elif family == "mxfp8":
            byts = m * k + n * k + (m + n) * k // 32 + 2 * m * n
        else:
            byts = m * k + n * k + 4 * m * (k // 128) + 4 * (n // 128) * (k // 128) + 2 * m * n
        rows.append({"gfx": gfx, "cu_num": cu_num, "M": m, "N": n, "K": k, "bias": False, "dtype": family,
                     "outdtype": "bf16", "scaleAB": True, "bpreshuffle": True, "libtype": "bsgemm",
                     "solidx": solidx, "splitK": split, "us": round(us, 3),
                     "kernelName": f"bsgemm_{family}_{kern}_ks{split}", "err_ratio": err_ratio,
                     "tflops": round(2.0 * m * n * k / us / 1e6, 2), "bw": round(byts / us / 1e3, 2)})
    if out_csv is not None:
        with open(out_csv, "w", newline="", encoding="utf-8") as f:
            w = csv.DictWriter(f, fieldnames=TUNED_HEADER)
            w.writeheader()
            w.writerows(rows)
    return rows

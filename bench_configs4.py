"""BASELINE configs[4] inside bench.py: the N-sharded multi-GPU GEMM.

M=16384, N=57344, K=8192 for MXFP4 (B in shuffle_weight(16,16), native
scales) and FP8 fp32 block-scale (K-panel B), split by N over the job's
ranks (strong scaling: the whole problem is fixed, each rank holds N/P
columns of the weights, pre-sharded).  The replicated activation A (and its
scales) is made on rank 0 and broadcast once with NCCL, outside the timed
regions.  Per family it reports:

  - GEMM only: max over ranks of the per-rank CUDA-event time, with the
    min / median / max over ranks (the spread explains any per-GPU drop);
  - GEMM + all-gather of the bf16 column shards, serial: the GEMM, then one
    ncclAllGather into a rank-major [P][M][N/P] buffer;
  - GEMM + all-gather, overlapped: the GEMM in M strips on the compute stream
    and each finished strip's ncclAllGather on NCCL's stream, into a
    strip-major [S][P][M/S][N/P] buffer;
  - TFLOPS and the roofline fraction of each, the gather's bytes per GPU;
  - parity: on rank 0, sampled rows x one 128-column block of every rank's
    shard of the gathered C against the CPU oracle (its weights regenerated
    from their seeds), the overlapped buffer equal bit for bit to the serial
    one, and the last rank's shard equal bit for bit to the same columns
    computed by rank 0 alone.

The weights are generated in 1024-column blocks, each seeded by its global
block index, so every rank count produces the same global B and C.
"""
from __future__ import annotations

import statistics

M, N, K = 16384, 57344, 8192
BLOCK = 1024                 # weight columns per seeded generation block
LINK_GBS = 770.0             # measured peer copy per direction per GPU (NVLink 5)
FAMILIES = ("mxfp4", "fp8block")


def _quant_fp8block_rows(w, block_rows):
    """fp32 block scales amax/448 per block_rows x 128 and E4M3 elements."""
    import torch
    rows, k = w.shape
    g = w.view(rows // block_rows, block_rows, k // 128, 128)
    s = g.abs().amax(dim=(1, 3)).clamp_min(1e-30) / 448.0
    q = (g / s[:, None, :, None]).view(rows, k).to(torch.float8_e4m3fn)
    return q, s.contiguous()


def _weights(bench, fam, n0, n1, dev):
    """Raw quantised weight columns [n0, n1) of the global B: (q [n1-n0, K or
    K/2] bytes, scales) with E8M0 [n, K/32] (mxfp4) or fp32 [n/128, K/128]."""
    import torch
    qs, ss = [], []
    for blk in range(n0 // BLOCK, (n1 + BLOCK - 1) // BLOCK):
        gen = torch.Generator(device=dev)
        gen.manual_seed(900001 + blk)
        w = torch.randn(BLOCK, K, device=dev, generator=gen)
        lo, hi = max(n0, blk * BLOCK) - blk * BLOCK, min(n1, (blk + 1) * BLOCK) - blk * BLOCK
        if fam == "mxfp4":
            q, s = bench.quant_mx_torch(w[lo:hi].contiguous(), 6.0, True)
        else:
            q, s = _quant_fp8block_rows(w[lo:hi].contiguous(), 128)
            q = q.view(torch.uint8)
        qs.append(q)
        ss.append(s)
        del w
    return torch.cat(qs), torch.cat(ss)


def _activations(bench, fam, dev, rank, dist):
    import torch
    if fam == "mxfp4":
        qa = torch.empty(M, K // 2, dtype=torch.uint8, device=dev)
        sa = torch.empty(M, K // 32, dtype=torch.uint8, device=dev)
    else:
        qa = torch.empty(M, K, dtype=torch.uint8, device=dev)
        sa = torch.empty(M, K // 128, dtype=torch.float32, device=dev)
    if rank == 0:
        gen = torch.Generator(device=dev)
        gen.manual_seed(424242)
        x = torch.randn(M, K, device=dev, generator=gen)
        if fam == "mxfp4":
            q, s = bench.quant_mx_torch(x, 6.0, True)
        else:
            q, s = _quant_fp8block_rows(x, 1)
            q = q.view(torch.uint8)
        qa.copy_(q)
        sa.copy_(s)
        del x, q, s
    if dist is not None:
        dist.broadcast(qa, 0)
        dist.broadcast(sa, 0)
    return qa, sa


class _Gemm:
    """The family's GEMM over rows [r0, r1) of A into the same rows of C."""

    def __init__(self, bs, fam, qa, sa, qb, sb, nl, grid_blocks=0):
        import torch
        self.bs, self.fam, self.nl, self.grid = bs, fam, nl, grid_blocks
        self.qa = qa
        if fam == "mxfp4":
            self.sa = bs.pack_scales(sa)
            self.qb = bs.pack_b(qb, "shuffle16", unpack=True)
            self.sb = bs.pack_scales(sb)
            self.sf_rows128 = ((K // 32 + 3) // 4) * 512       # native atom bytes per 128 rows
        else:
            self.sa = sa
            self.qb = qb.view(nl, K // 128, 128).permute(1, 0, 2).contiguous().view(torch.float8_e4m3fn)
            self.sb = sb

    def __call__(self, out, r0=0, r1=M, grid_blocks=None):
        import torch
        g = self.grid if grid_blocks is None else grid_blocks
        if self.fam == "mxfp4":
            sa = self.sa[r0 // 128 * self.sf_rows128:]
            self.bs.gemm_a4w4_mxfp4(self.qa[r0:r1], self.qb, sa, self.sb, out=out[r0:r1], scale_format="native",
                                    b_format="shuffle16", kernel="auto", grid_blocks=g)
        else:
            # split_k 1: every tile whole, so a row's result does not depend on
            # the rows called with it (the serial and the strip-wise GEMMs agree
            # bit for bit); K slices of the partial last wave would move < 1 %
            # of the work at this size
            self.bs.gemm_a8w8_bpreshuffle(self.qa[r0:r1].view(torch.float8_e4m3fn), self.qb, self.sa[r0:r1],
                                          self.sb, torch.bfloat16, preshuffled=True, out=out[r0:r1],
                                          grid_blocks=g, split_k=1)


def _time(fn, steps, warmup, stream):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _over_ranks(v, dist, world, dev):
    """[values of every rank] (rank order)."""
    import torch
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    if world == 1:
        return [v]
    out = torch.empty(world, dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(out, t)
    return [float(x) for x in out.cpu()]


def run(bench, bs, dev, world, rank, dist, peaks, steps=8, warmup=3, strips=4, overlap_grid=0):
    """Returns the configs4 record on rank 0 (None elsewhere).  Every rank
    takes the same collective steps in the same order.  overlap_grid > 0
    caps the CTAs of the overlapped strip GEMMs, leaving SMs to NCCL's
    kernels; the GEMM-only and serial timings always use every SM."""
    import numpy as np
    import torch
    P = world
    nl = N // P
    n0 = rank * nl
    stream = torch.cuda.current_stream(dev)
    dist_ = dist if world > 1 else None
    rec = {"workload": f"M={M} N={N} K={K}, N-sharded over {P} GPU(s) ({nl} columns each), bf16 out",
           "scaling": "strong", "strips": strips, "overlap_grid": overlap_grid or "all SMs",
           "gather_layout": {"serial": "[P][M][N/P] rank-major", "overlapped": "[S][P][M/S][N/P] strip-major"},
           "link_gbs": LINK_GBS, "families": {}}
    flops = 2.0 * M * N * K
    for fam in FAMILIES:
        qa, sa = _activations(bench, fam, dev, rank, dist_)
        qb, sb = _weights(bench, fam, n0, n0 + nl, dev)
        gemm = _Gemm(bs, fam, qa, sa, qb, sb, nl)
        del qb, sb
        out = torch.empty(M, nl, dtype=torch.bfloat16, device=dev)
        t_gemm = _time(lambda: gemm(out), steps, warmup, stream)
        per_rank = _over_ranks(t_gemm, dist_, world, dev)
        r = {"gemm_ms": max(per_rank),
             "gemm_ms_per_rank": {"min": min(per_rank), "median": statistics.median(per_rank), "max": max(per_rank)}}
        mult = 4.0 if fam == "mxfp4" else 2.0
        peak_gpu = mult * peaks.get("bf16_tflops")
        r["tflops"] = flops / (r["gemm_ms"] * 1e-3) / 1e12
        r["frac"] = r["tflops"] / (P * peak_gpu)
        r["peak_per_gpu_tflops"] = peak_gpu
        if P > 1:
            gath = torch.empty(P, M, nl, dtype=torch.bfloat16, device=dev)
            ms = M // strips
            gath_s = torch.empty(strips, P, ms, nl, dtype=torch.bfloat16, device=dev)

            def serial():
                gemm(out)
                dist.all_gather_into_tensor(gath, out)

            def overlapped():
                works = []
                for s in range(strips):
                    gemm(out, s * ms, (s + 1) * ms, grid_blocks=overlap_grid)
                    works.append(dist.all_gather_into_tensor(gath_s[s], out[s * ms:(s + 1) * ms], async_op=True))
                for w in works:
                    w.wait()

            t_ser = max(_over_ranks(_time(serial, steps, warmup, stream), dist_, world, dev))
            t_ovl = max(_over_ranks(_time(overlapped, steps, warmup, stream), dist_, world, dev))
            recv = (P - 1) * M * nl * 2
            target = max(flops / P / (peak_gpu * 1e12), recv / (LINK_GBS * 1e9)) * 1e3
            r.update({"gemm_allgather_ms_serial": t_ser, "gemm_allgather_ms_overlapped": t_ovl,
                      "tflops_with_allgather": flops / (min(t_ser, t_ovl) * 1e-3) / 1e12,
                      "allgather_bytes_received_per_gpu": recv,
                      "gemm_allgather_target_ms": target,
                      "gemm_allgather_frac": target / min(t_ser, t_ovl)})
            # parity of the gathered C (rank 0), after one more of each
            serial()
            overlapped()
            torch.cuda.synchronize()
            same = all(torch.equal(gath_s[s], gath[:, s * ms:(s + 1) * ms]) for s in range(strips))
        else:
            gemm(out)
            torch.cuda.synchronize()
            gath = out.view(1, M, nl)
            same = True
        if rank == 0:
            r["parity"] = _parity(bench, bs, fam, gemm, gath, qa, sa, nl, P, dev)
            r["parity"]["overlapped_equals_serial"] = bool(same)
            if P > 1:
                # the last rank's shard, recomputed here alone
                qb2, sb2 = _weights(bench, fam, (P - 1) * nl, P * nl, dev)
                g2 = _Gemm(bs, fam, qa, sa, qb2, sb2, nl)
                out2 = torch.empty(M, nl, dtype=torch.bfloat16, device=dev)
                g2(out2)
                torch.cuda.synchronize()
                r["parity"]["last_shard_bitwise_equal_1gpu"] = bool(torch.equal(out2, gath[P - 1]))
                del g2, out2, qb2, sb2
            r["parity"]["ok"] = bool(r["parity"]["bad"] == 0 and same and
                                     r["parity"].get("last_shard_bitwise_equal_1gpu", True))
        rec["families"][fam] = r
        del gemm, out, gath, qa, sa
        if P > 1:
            del gath_s
        torch.cuda.empty_cache()
        if dist_ is not None:
            dist.barrier()
    return rec if rank == 0 else None


def _parity(bench, bs, fam, gemm, gath, qa, sa, nl, P, dev):
    """Sampled rows x one 128-column block per shard against the oracle."""
    import numpy as np
    import torch
    from oracle import oracle as orc
    orc.build()
    rng = np.random.default_rng(7)
    rows = np.sort(np.concatenate([[0, M - 1], rng.choice(np.arange(1, M - 1), 6, replace=False)]))
    ri = torch.from_numpy(rows).to(dev)
    qa_r, sa_r = qa[ri].cpu().numpy(), sa[ri].cpu().numpy()
    bad = checked = 0
    max_rel = 0.0
    for p in range(P):
        j0 = int(rng.integers(0, nl // 128)) * 128
        c0 = p * nl + j0
        qb, sb = _weights(bench, fam, c0, c0 + 128, dev)
        got = gath[p][ri, j0:j0 + 128].float().cpu().numpy()
        if fam == "mxfp4":
            ref, mag = orc.gemm_mxfp4(qa_r, qb.cpu().numpy(), sa_r, sb.cpu().numpy())
        else:
            ref, mag = orc.gemm_fp8_block(qa_r, qb.cpu().numpy(), sa_r, sb.cpu().numpy())
        b, mr, _ = orc.check_baseline_rule(ref, got, mag)
        bad += b
        checked += got.size
        max_rel = max(max_rel, mr)
    return {"checked": int(checked), "bad": int(bad), "max_rel": max_rel,
            "sample": f"{len(rows)} rows x one 128-column block of each of the {P} shard(s)"}

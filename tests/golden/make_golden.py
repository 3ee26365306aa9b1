"""Generate the golden fixtures under tests/golden/ (committed .npz files).

The reference ships no golden vectors and its host code cannot be compiled
here (it needs <hip/hip_fp8.h> and OPUS), so these fixtures come from an
implementation that is independent of oracle/oracle.c:
  - element codecs from torch (float8_e4m3fn) and ml_dtypes (float4_e2m1fn),
  - scale rules written with numpy (2^ceil(log2(amax/qmax)), amax/448),
  - GEMMs as float64 numpy matmuls of the dequantised operands,
  - layouts from the index formulas the reference states in its host drivers
    (source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:161-179,
     candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:194-227,
     block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_host.cc:96-111).
tests/test_oracle.py checks the C oracle against every fixture, which is how
the oracle is pinned.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import ml_dtypes
import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def e4m3(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def e4m3_dec(q: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(q)).view(torch.float8_e4m3fn).float().numpy()


def e2m1(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, np.float32).astype(ml_dtypes.float4_e2m1fn).view(np.uint8) & 15


def e2m1_dec(c: np.ndarray) -> np.ndarray:
    return (c & 15).astype(np.uint8).view(ml_dtypes.float4_e2m1fn).astype(np.float32)


def mx_quant(x: np.ndarray, qmax: float, fp4: bool):
    rows, k = x.shape
    g = x.reshape(rows, k // 32, 32).astype(np.float64)
    amax = np.abs(g).max(axis=2)
    with np.errstate(divide="ignore"):
        e = np.where(amax > 0, np.ceil(np.log2(amax / qmax)), 0.0)
    e = np.clip(e, -127, 127).astype(np.int32)
    sf = (e + 127).astype(np.uint8)
    scaled = (g * np.exp2(-e.astype(np.float64))[..., None]).astype(np.float32).reshape(rows, k)
    if fp4:
        codes = e2m1(scaled)
        q = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
        deq = e2m1_dec(codes).reshape(rows, k // 32, 32)
    else:
        q = e4m3(scaled)
        deq = e4m3_dec(q).reshape(rows, k // 32, 32)
    deq = (deq * np.exp2(e.astype(np.float64))[..., None]).reshape(rows, k)
    return q, sf, deq


def block_quant(x: np.ndarray, br: int):
    rows, k = x.shape
    nrb = (rows + br - 1) // br
    sf = np.zeros((nrb, k // 128), np.float32)
    q = np.zeros((rows, k), np.uint8)
    deq = np.zeros((rows, k), np.float64)
    for rb in range(nrb):
        r0, r1 = rb * br, min(rows, rb * br + br)
        for b in range(k // 128):
            blk = x[r0:r1, b * 128:(b + 1) * 128]
            amax = np.float32(np.abs(blk).max())
            s = np.float32(amax / np.float32(448.0)) if amax > 0 else np.float32(1.0)
            sf[rb, b] = s
            qq = e4m3(np.clip(blk / s, -448, 448))
            q[r0:r1, b * 128:(b + 1) * 128] = qq
            deq[r0:r1, b * 128:(b + 1) * 128] = e4m3_dec(qq).astype(np.float64)
    return q, sf, deq


def case_mxfp8(rng, m, n, k, name):
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    qa, sa, da = mx_quant(x, 448.0, False)
    qb, sb, db = mx_quant(w, 448.0, False)
    c = da @ db.T
    np.savez_compressed(HERE / f"{name}.npz", x=x, w=w, qa=qa, sa=sa, qb=qb, sb=sb, c=c)


def case_mxfp4(rng, m, n, k, name):
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    qa, sa, da = mx_quant(x, 6.0, True)
    qb, sb, db = mx_quant(w, 6.0, True)
    c = da @ db.T
    np.savez_compressed(HERE / f"{name}.npz", x=x, w=w, qa=qa, sa=sa, qb=qb, sb=sb, c=c)


def case_fp8_block(rng, m, n, k, name):
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    qa, sa, da = block_quant(x, 1)
    qb, sb, db = block_quant(w, 128)
    # C = sum_kb sa[m,kb] sb[n/128,kb] (A B^T)_kb
    c = np.zeros((m, n))
    for b in range(k // 128):
        part = da[:, b * 128:(b + 1) * 128] @ db[:, b * 128:(b + 1) * 128].T
        c += part * sa[:, b:b + 1].astype(np.float64) * np.repeat(sb[:, b].astype(np.float64), 128)[None, :n]
    np.savez_compressed(HERE / f"{name}.npz", x=x, w=w, qa=qa, sa=sa, qb=qb, sb=sb, c=c)


def case_layouts(rng, name):
    n, kb = 64, 256
    b = rng.integers(0, 256, size=(n, kb), dtype=np.uint8)
    # shuffle_weight(16,16): [n/16][kb/16][16][16]
    sh16 = b.reshape(n // 16, 16, kb // 16, 16).transpose(0, 2, 1, 3).reshape(n, kb).copy()
    # candidate_m10 formula for packed fp4 bytes (same permutation, stated differently)
    sh_m10 = np.zeros(n * kb, np.uint8)
    for r in range(n):
        for c in range(kb):
            o = (r // 16) * 16 * kb + (c // 32) * 512 + ((c // 16) % 2) * 256 + (r % 16) * 16 + c % 16
            sh_m10[o] = b[r, c]
    # K-panel B'[kt][n][128]
    kp = b.reshape(n, kb // 128, 128).transpose(1, 0, 2).copy()
    # e8m0_shuffle of a [rows, kg] scale matrix
    rows, kg = 40, 12
    sf = rng.integers(100, 140, size=(rows, kg), dtype=np.uint8)
    kg8 = (kg + 7) // 8 * 8
    rows32 = (rows + 31) // 32 * 32
    esh = np.full(rows32 * kg8, 0x7F, np.uint8)
    for r in range(rows):
        for g in range(kg):
            o = ((r // 32) * (kg8 // 8) + g // 8) * 256 + (g % 4) * 64 + (r % 16) * 4 + ((g % 8) // 4) * 2 + (r % 32) // 16
            esh[o] = sf[r, g]
    np.savez_compressed(HERE / f"{name}.npz", b=b, sh16=sh16, sh_m10=sh_m10.reshape(n, kb), kp=kp,
                        sf=sf, esh=esh)


def main():
    rng = np.random.default_rng(20261201)
    case_mxfp8(rng, 64, 64, 256, "mxfp8_64x64x256")
    case_mxfp8(rng, 40, 24, 128, "mxfp8_40x24x128")
    case_mxfp4(rng, 64, 64, 256, "mxfp4_64x64x256")
    case_fp8_block(rng, 48, 128, 256, "fp8block_48x128x256")
    case_layouts(rng, "layouts")
    # codec tables
    e4 = e4m3_dec(np.arange(256, dtype=np.uint8))
    e2 = e2m1_dec(np.arange(16, dtype=np.uint8))
    probe = np.concatenate([np.linspace(-470, 470, 4001, dtype=np.float32),
                            rng.standard_normal(4000).astype(np.float32) * 0.05,
                            np.float32([2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, -0.0])])
    probe4 = np.concatenate([np.linspace(-6.5, 6.5, 1301, dtype=np.float32),
                             np.float32([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25])])
    np.savez_compressed(HERE / "codecs.npz", e4m3_table=e4, e2m1_table=e2,
                        probe=probe, probe_e4m3=e4m3(np.clip(probe, -448, 448)),
                        probe4=probe4, probe_e2m1=e2m1(np.clip(probe4, -6, 6)))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()

"""E8M0 edge bytes and E4M3 NaN operands through every kernel family.

The scale byte 0 means 2^-127 in this library, as on the reference host
(mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:35-37) and in the OCP MX encoding that
tcgen05's block-scaled MMA implements; the reference's own device decode
(gemm_a8w8_mxfp8_kernel_template.hpp:23-25) would read it as 0.0.  The byte
255 means NaN (OCP MX), where the reference host's ldexp gives 2^128 (+inf
in fp32): every output of a row or column whose scales hold a 255 byte is NaN
(oracle.as_library_e8m0 states the mapping).  E4M3 0x7F / 0xFF operands are NaN and propagate to
their output rows.  Each case plants these values into seeded data; the
planted byte-0 group is scaled by 2^-127 x 2^127 = 1 against data scales near
2^-14, so reading byte 0 as zero would change that output by far more than the
tolerance.  Outputs in the rows and columns a 255 byte or a NaN operand
reaches must be NaN; all others must be finite and meet the usual rule.
"""
import numpy as np
import pytest
import torch

from helpers import assert_close, dev_u8, mxfp4_problem, mxfp8_problem

pytestmark = pytest.mark.gpu


def plant_mx(qa, sa, sb, fp8):
    """Edge bytes that cannot overflow: a planted 2^127 weight scale meets
    2^-127 (byte 0) activation scales in every row, so the products are 1,
    and only 255 bytes and NaN operands make outputs non-finite."""
    qa, sa, sb = qa.copy(), sa.copy(), sb.copy()
    sa[:, 0], sb[1, 0] = 0, 254        # group 0 of column 1: 2^-127 * 2^127 = 1 in every row
    sa[:, 2], sb[6, 2] = 1, 253        # group 2 of column 6: 2^-126 * 2^126
    sa[2, 1] = 255                     # row 2 NaN
    sa[3, 2], sb[3, 2] = 255, 0        # row 3 NaN (the host: inf * 2^-127)
    sb[5, 3] = 255                     # column 5 NaN
    if fp8:
        qa[4, 7] = 0x7F                # NaN operands: rows 4 and 7 NaN
        qa[7, 40] = 0xFF
    return qa, sa, sb


def check(orc, ref, got, mag, what, nan_rows, nan_cols):
    lib = orc.as_library_e8m0(ref, nan_rows, nan_cols)
    fin = ~np.isnan(lib)
    assert np.array_equal(np.isnan(got), ~fin), f"{what}: NaN pattern differs from the rows/columns a 255 byte or NaN reaches"
    assert np.isfinite(lib[fin]).all() and np.isfinite(got[fin]).all()
    assert_close(orc, lib[fin], got[fin], None if mag is None else mag[fin], what)
    return int((~fin).sum())


def mx_nan(orc, qa, sa, sb, fp8):
    rows = np.where((sa == 255).any(axis=1))[0]
    if fp8:
        rows = np.union1d(rows, orc.e4m3_nan_rows(qa))
    return rows, np.where((sb == 255).any(axis=1))[0]


@pytest.mark.parametrize("kernel,m,split_k,out_dtype", [
    ("1cta", 256, 0, torch.bfloat16), ("1cta", 256, 0, torch.float32), ("pair", 256, 0, torch.bfloat16),
    ("swap", 16, 0, torch.bfloat16), ("swap", 48, 3, torch.float32), ("1cta", 128, 2, torch.bfloat16)])
def test_mxfp8_edge_bytes_and_nan(bs, orc, cuda, kernel, m, split_k, out_dtype):
    n, k = 256, 512
    qa, qb, sa, sb = [x[0] for x in mxfp8_problem(orc, m, n, k, 61)]
    qa, sa, sb = plant_mx(qa, sa, sb, True)
    ref, mag = orc.gemm_mxfp8(qa, qb, sa, sb, f64=True)
    out = bs.gemm_a8w8_mxfp8(dev_u8(qa, cuda).view(torch.float8_e4m3fn), dev_u8(qb, cuda).view(torch.float8_e4m3fn),
                             dev_u8(sa, cuda), dev_u8(sb, cuda), kernel=kernel, split_k=split_k, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    got = out.float().cpu().numpy()
    assert check(orc, ref, got, mag, f"mxfp8 edges {kernel} m{m} s{split_k}", *mx_nan(orc, qa, sa, sb, True)) > 0
    # byte 0 read as 0.0 would drop group 0 of column 1, which dominates it
    zero_reading = ref[:, 1] - orc.gemm_mxfp8(qa[:, :32], qb[:, :32], sa[:, :1], sb[:, :1], f64=True)[0][:, 1]
    ok = np.isfinite(got[:, 1])
    assert (np.abs(got[ok, 1] - zero_reading[ok]) > 1.0).all()


@pytest.mark.parametrize("kernel,m", [("1cta", 256), ("pair", 256), ("swap", 32)])
def test_mxfp4_edge_bytes(bs, orc, cuda, kernel, m):
    n, k = 256, 512
    qa, qb, sa, sb = mxfp4_problem(orc, m, n, k, 62)
    qa, sa, sb = plant_mx(qa, sa, sb, False)
    ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
    out = bs.gemm_a4w4_mxfp4(dev_u8(qa, cuda), dev_u8(qb, cuda), dev_u8(sa, cuda), dev_u8(sb, cuda), kernel=kernel)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert check(orc, ref, out.float().cpu().numpy(), mag, f"mxfp4 edges {kernel} m{m}",
                 *mx_nan(orc, qa, sa, sb, False)) > 0


@pytest.mark.parametrize("tiles", [0, 1])
def test_e8m0_block_edge_bytes_and_nan(bs, orc, cuda, tiles):
    """launch_blockscale_bpreshuffle: E8M0 bytes 0 / 255 in both 1x128 and
    128x128 scales, NaN activations."""
    m, n, k = 256, 256, 512
    qa, _ = orc.quant_mxfp8(orc.normal((m, k), seed=63))
    qb, _ = orc.quant_mxfp8(orc.normal((n, k), seed=64))
    rng = np.random.default_rng(11)
    sfa_t = rng.integers(124, 131, (k // 128, m)).astype(np.uint8)
    sfb = rng.integers(124, 131, (n // 128, k // 128)).astype(np.uint8)
    sfa_t[0, :], sfb[0, 0] = 0, 254    # K block 0 of columns 0..127: 2^-127 * 2^127 = 1 in every row
    sfa_t[1, 2] = 255                  # row 2 NaN
    sfb[1, 3] = 255                    # columns 128..255 NaN
    qa[3, 5] = 0x7F                    # row 3 NaN
    ref, mag = orc.gemm_e8m0_block(qa, qb, sfa_t, sfb)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(orc.shuffle_weight16(qb), cuda).view(torch.float8_e4m3fn)
    out = bs.gemm_a8w8_blockscale_bpreshuffle(A, B, dev_u8(sfa_t, cuda).t(), dev_u8(sfb, cuda), tiles=tiles)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    nan_rows = np.union1d(np.where((sfa_t == 255).any(axis=0))[0], orc.e4m3_nan_rows(qa))
    nan_cols = np.concatenate([np.arange(cb * 128, cb * 128 + 128) for cb in np.where((sfb == 255).any(axis=1))[0]])
    assert check(orc, ref, out.float().cpu().numpy(), mag, f"e8m0 block edges tiles={tiles}", nan_rows, nan_cols) > 0


@pytest.mark.parametrize("kernel,m", [("auto", 256), ("swap", 16), ("1cta", 48)])
def test_fp8_block_nan_operands(bs, orc, cuda, kernel, m):
    n, k = 256, 512
    qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=65), 1)
    qb, sb = orc.quant_fp8_block(orc.normal((n, k), seed=66), 128)
    qa, qb = qa.copy(), qb.copy()
    qa[4, 7] = 0x7F
    qb[9, 300] = 0xFF                  # column 9 NaN
    ref, mag = orc.gemm_fp8_block(qa, qb, sa, sb)
    out = bs.gemm_a8w8_bpreshuffle(dev_u8(qa, cuda).view(torch.float8_e4m3fn),
                                   dev_u8(orc.shuffle_kpanel(qb), cuda).view(torch.float8_e4m3fn),
                                   torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda), kernel=kernel)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert check(orc, ref, out.float().cpu().numpy(), mag, f"fp8 block NaN operands {kernel} m{m}",
                 orc.e4m3_nan_rows(qa), orc.e4m3_nan_rows(qb)) > 0

"""Guard canaries around C: every kernel family writes exactly the M x N
output region and nothing else -- not the padding columns of a padded row
stride (ldc > N), not the rows before or after.  C lives inside a larger
buffer filled with a canary pattern; the call goes through the C ABI with
that ldc; afterwards every canary must be intact and every output finite.
Ragged M and N exercise the clipping of TMA stores and the masked stores of
the other epilogues."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import dev_u8

pytestmark = pytest.mark.gpu

CANARY = 0x7FBF   # a bf16 NaN pattern no kernel produces


def guarded_c(m, n, pad, out_dtype, device):
    """Buffer of (m + 2) rows x (n + 2 * pad) columns; C starts at row 1, column pad."""
    ldc = n + 2 * pad
    if out_dtype == torch.bfloat16:
        buf = torch.full((m + 2, ldc), CANARY, dtype=torch.int16, device=device)
    else:
        buf = torch.full((m + 2, ldc), float("nan"), dtype=torch.float32, device=device)
    return buf, ldc


def check_guard(buf, m, n, pad, out_dtype):
    host = buf.cpu()
    inside = torch.zeros_like(host, dtype=torch.bool)
    inside[1:m + 1, pad:pad + n] = True
    if out_dtype == torch.bfloat16:
        outside_ok = (host[~inside] == CANARY).all().item()
        c = host[1:m + 1, pad:pad + n].view(torch.bfloat16).float()
    else:
        outside_ok = torch.isnan(host[~inside]).all().item()
        c = host[1:m + 1, pad:pad + n]
    assert outside_ok, "a kernel wrote outside C"
    assert torch.isfinite(c).all().item(), "C has unwritten or non-finite elements"


def mx_args(bs, A, B, SA, SB, m, n, k, c_ptr, ldc, *, fp4, out_dtype, kernel, b_format=0, ws=None):
    a = bs.Args()
    bs.lib().bsgemm_args_init(ctypes.byref(a))
    a.ptr_a, a.ptr_b, a.ptr_c = A.data_ptr(), B.data_ptr(), c_ptr
    a.m, a.n, a.k, a.batch = m, n, k, 1
    a.stride_a, a.stride_b, a.stride_c = A.stride(0), B.stride(0), ldc
    a.ptr_sfa, a.ptr_sfb = SA.data_ptr(), SB.data_ptr()
    a.sfa_format = a.sfb_format = bs.SF_ROWMAJOR
    a.stride_sfa, a.stride_sfb = SA.stride(0), SB.stride(0)
    a.layout = bs.LAYOUTS["tn"]
    a.b_format = b_format
    a.out_dtype = bs.OUT_BF16 if out_dtype == torch.bfloat16 else bs.OUT_FP32
    a.kernel = bs.KERNELS[kernel]
    a.split_k = 1 if kernel == "pair" else 0
    need = int(bs.lib().bsgemm_workspace_size(bs.FAMILY_MXFP4 if fp4 else bs.FAMILY_MXFP8, ctypes.byref(a)))
    if need:
        ws = torch.empty(need, dtype=torch.uint8, device=A.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), need
    return a, ws


@pytest.mark.parametrize("fp4,kernel,m,n,out_dtype", [
    (False, "pair", 264, 520, torch.bfloat16),
    (False, "1cta", 136, 264, torch.bfloat16),
    (False, "1cta", 136, 264, torch.float32),
    (False, "swap", 30, 264, torch.bfloat16),
    (True, "pair", 264, 392, torch.bfloat16),
    (True, "swap", 16, 136, torch.float32),
])
def test_mx_writes_only_c(bs, orc, cuda, fp4, kernel, m, n, out_dtype):
    k = 512
    if fp4:
        qa, sa = orc.quant_mxfp4(orc.normal((m, k), seed=3))
        qb, sb = orc.quant_mxfp4(orc.normal((n, k), seed=4))
    else:
        qa, sa = orc.quant_mxfp8(orc.normal((m, k), seed=3))
        qb, sb = orc.quant_mxfp8(orc.normal((n, k), seed=4))
    A, B = dev_u8(qa, cuda), dev_u8(qb, cuda)
    SA, SB = dev_u8(sa, cuda), dev_u8(sb, cuda)
    pad = 8
    buf, ldc = guarded_c(m, n, pad, out_dtype, cuda)
    esz = 2 if out_dtype == torch.bfloat16 else 4
    c_ptr = buf.data_ptr() + (ldc + pad) * esz
    a, ws = mx_args(bs, A, B, SA, SB, m, n, k, c_ptr, ldc, fp4=fp4, out_dtype=out_dtype, kernel=kernel)
    fn = bs.lib().bsgemm_a4w4_mxfp4 if fp4 else bs.lib().bsgemm_a8w8_mxfp8
    status = fn(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert status == 0, bs.strerror(status)
    assert bs.check_device_error() == 0
    check_guard(buf, m, n, pad, out_dtype)


@pytest.mark.parametrize("kernel,m", [("swap", 20), ("1cta", 140)])
def test_fp8_block_writes_only_c(bs, orc, cuda, kernel, m):
    n, k = 392, 512
    qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=5), 1)
    qb, sb = orc.quant_fp8_block(orc.normal((n, k), seed=6), 128)
    A, B = dev_u8(qa, cuda), dev_u8(qb, cuda)
    SA, SB = torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda)
    pad = 8
    buf, ldc = guarded_c(m, n, pad, torch.bfloat16, cuda)
    a = bs.Args()
    bs.lib().bsgemm_args_init(ctypes.byref(a))
    a.ptr_a, a.ptr_b, a.ptr_c = A.data_ptr(), B.data_ptr(), buf.data_ptr() + (ldc + pad) * 2
    a.m, a.n, a.k, a.batch = m, n, k, 1
    a.stride_a, a.stride_b, a.stride_c = k, k, ldc
    a.ptr_sfa, a.ptr_sfb = SA.data_ptr(), SB.data_ptr()
    a.sfa_format = a.sfb_format = bs.SF_ROWMAJOR
    a.stride_sfa, a.stride_sfb = SA.stride(0), SB.stride(0)
    a.kernel = bs.KERNELS[kernel]
    need = int(bs.lib().bsgemm_workspace_size(bs.FAMILY_FP8_BLOCK, ctypes.byref(a)))
    ws = None
    if need:
        ws = torch.empty(need, dtype=torch.uint8, device=cuda)
        a.workspace, a.workspace_bytes = ws.data_ptr(), need
    status = bs.lib().bsgemm_a8w8_blockscale_bpreshuffle(ctypes.byref(a),
                                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert status == 0, bs.strerror(status)
    assert bs.check_device_error() == 0
    check_guard(buf, m, n, pad, torch.bfloat16)

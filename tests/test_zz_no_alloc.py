"""The allocation-free MXFP8 entry point (bsgemm_a8w8_mxfp8_noalloc).

Callers embedded in a runtime that owns all device memory (or that must not
take the synchronisation an allocation can cause) cannot hand the library a
workspace.  This entry point runs the same kernels with a fixed scratch array
inside the library instead.  The test calls it through the C ABI and checks
its output against the workspace-taking entry point, under the same tolerance
as every parity test, on two calls in a row (the scratch keeps the previous
call's contents, which must not matter).  It also checks that a problem too
large for the scratch is refused before anything runs.

The file name sorts last so that a run stopping at its first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import assert_close, dev_u8, mxfp8_problem

pytestmark = pytest.mark.gpu


def fill_args(bs, A, B, SA, SB, out, split_k=0):
    m, k = A.shape
    n = B.shape[0]
    a = bs.Args()
    bs.lib().bsgemm_args_init(ctypes.byref(a))
    a.ptr_a, a.ptr_b, a.ptr_c = A.data_ptr(), B.data_ptr(), out.data_ptr()
    a.m, a.n, a.k, a.batch = m, n, k, 1
    a.stride_a, a.stride_b, a.stride_c = k, k, n
    a.ptr_sfa, a.ptr_sfb = SA.data_ptr(), SB.data_ptr()
    a.sfa_format = a.sfb_format = bs.SF_ROWMAJOR
    a.stride_sfa, a.stride_sfb = k // 32, k // 32
    a.layout = bs.LAYOUTS["tn"]
    a.out_dtype = bs.OUT_BF16
    a.split_k = split_k
    return a


def noalloc_fn(bs):
    fn = bs.lib().bsgemm_a8w8_mxfp8_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(bs.Args), ctypes.c_void_p]
    return fn


def test_noalloc_matches_workspace_entry_twice(bs, orc, cuda):
    fn = noalloc_fn(bs)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    # two problems in a row: a skinny one (auto split-K -> partials in the
    # scratch) and a square one (row-major scales repacked into the scratch)
    for (m, n, k, seed) in ((32, 512, 4096, 21), (256, 384, 512, 22)):
        qa, qb, sa, sb = [x[0] for x in mxfp8_problem(orc, m, n, k, seed, "kpattern")]
        ref, mag = orc.gemm_mxfp8(qa, qb, sa, sb, f64=True)
        A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
        B = dev_u8(qb, cuda).view(torch.float8_e4m3fn)
        SA, SB = dev_u8(sa, cuda), dev_u8(sb, cuda)
        expected = bs.gemm_a8w8_mxfp8(A, B, SA, SB)      # workspace-taking entry point
        torch.cuda.synchronize()
        for call in range(2):
            out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
            args = fill_args(bs, A, B, SA, SB, out)
            assert fn(ctypes.byref(args), stream) == bs.OK
            torch.cuda.synchronize()
            assert bs.check_device_error() == 0
            got = out.float().cpu().numpy()
            assert_close(orc, expected.float().cpu().numpy().astype(np.float64), got, mag,
                         f"noalloc vs workspace entry {m}x{n}x{k} call {call}")
            assert_close(orc, ref, got, mag, f"noalloc vs oracle {m}x{n}x{k} call {call}")


def test_noalloc_drops_auto_split_that_exceeds_its_scratch(bs, orc, cuda):
    """A skinny problem whose automatic split-K partials would not fit in the
    fixed scratch runs unsplit instead of failing, with the same results."""
    fn = noalloc_fn(bs)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    m, n, k = 128, 8192, 16384   # the library splits this K in two (12 MB of partials and scales)
    qa, qb, sa, sb = [x[0] for x in mxfp8_problem(orc, m, n, k, 23, "rowpattern")]
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(qb, cuda).view(torch.float8_e4m3fn)
    SA, SB = dev_u8(sa, cuda), dev_u8(sb, cuda)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    args = fill_args(bs, A, B, SA, SB, out)
    size = bs.lib().bsgemm_workspace_size
    limit = bs.lib().bsgemm_noalloc_scratch_bytes
    limit.restype = ctypes.c_size_t
    assert size(bs.FAMILY_MXFP8, ctypes.byref(args)) > limit()      # the automatic plan splits K
    expected = bs.gemm_a8w8_mxfp8(A, B, SA, SB)
    assert fn(ctypes.byref(args), stream) == bs.OK
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert torch.isfinite(out).all()
    rows = np.arange(0, m, 9)
    got = out.float().cpu().numpy()[rows]
    ref, mag = orc.gemm_mxfp8(qa[rows], qb, sa[rows], sb, f64=True)
    # the workspace entry splits K and this one does not: they agree within
    # the fp32-accumulation tolerance, not bit for bit
    assert_close(orc, expected.float().cpu().numpy()[rows].astype(np.float64), got, mag, "noalloc unsplit vs entry")
    assert_close(orc, ref, got, mag, "noalloc unsplit vs oracle")


def test_noalloc_rejects_problems_beyond_its_scratch(bs, cuda):
    fn = noalloc_fn(bs)
    limit = bs.lib().bsgemm_noalloc_scratch_bytes
    limit.restype = ctypes.c_size_t
    assert limit() == 8 << 20
    m = n = 1024
    k = 4096
    A = torch.zeros(m, k, dtype=torch.uint8, device=cuda).view(torch.float8_e4m3fn)
    B = torch.zeros(n, k, dtype=torch.uint8, device=cuda).view(torch.float8_e4m3fn)
    SA = torch.full((m, k // 32), 127, dtype=torch.uint8, device=cuda)
    SB = torch.full((n, k // 32), 127, dtype=torch.uint8, device=cuda)
    out = torch.zeros(m, n, dtype=torch.bfloat16, device=cuda)
    # forced split of 4: 4 * 1024 * 1024 * 4 bytes of partials = 16 MiB > 8 MiB
    args = fill_args(bs, A, B, SA, SB, out, split_k=4)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    assert fn(ctypes.byref(args), stream) == bs.ERR_SCRATCH_LIMIT
    assert "scratch" in bs.strerror(bs.ERR_SCRATCH_LIMIT)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0                # nothing ran

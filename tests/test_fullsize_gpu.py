"""Full-size parity for every BASELINE configuration, through the C ABI.

Each GEMM runs at its full size on the GPU; the oracle (pinned bit-equal to
the reference's own CPU code by tests/test_ref_pin.py) checks a sample of
output rows against the target rule
    |err| <= 2^-7 |ref| + 1e-3 + 1e-6 * sum|term|,  max rel err <= 1e-2,
and every output element must be finite.  The configurations:
  - FP8 fp32 block-scale, K-panel B, bf16 out, M in {1, 16, 64,
    128, 1024, 8192} x (N, K) in {(7168, 2048), (4096, 7168), (24576, 1536),
    (7168, 18432)}, once with the library's own choice of kernel and split
    and once with the shipped tuned table's;
  - MXFP8 8192^3 in the nn and tt layouts (tn and nt are in
    test_gemm_gpu.py);
  - MXFP4 M in {16, 128, 1024} x N = K = 8192, B in
    shuffle_weight(16,16) read in place, native scales (the benchmark form);
  - DeepSeek-V4 traced a8w8 shapes with M not a multiple of 16
    (dsv4_a8w8_all_traced_shapes.csv: M = 6 and 27 at (N, K) = (1536, 7168),
    M = 27 at (7168, 21504)) through the shipped tuned table.
"""
import importlib

import numpy as np
import pytest
import torch

from helpers import assert_close, dev_u8, mxfp4_problem

pytestmark = pytest.mark.gpu

SWEEP_NK = [(7168, 2048), (4096, 7168), (24576, 1536), (7168, 18432)]
SWEEP_M = [1, 16, 64, 128, 1024, 8192]

_weights = {}


def block_weights(orc, cuda, n, k):
    """K-panel B and its 128x128 fp32 scales for one (N, K), made once."""
    if (n, k) not in _weights:
        qb, sb = orc.quant_fp8_block(orc.normal((n, k), seed=n * 7 + k), 128)
        B = dev_u8(orc.shuffle_kpanel(qb), cuda).view(torch.float8_e4m3fn)
        _weights[(n, k)] = (qb, sb, B, torch.from_numpy(sb).to(cuda))
    return _weights[(n, k)]


def sample_rows(m, count=16, seed=0):
    if m <= count:
        return np.arange(m)
    rows = np.random.default_rng(seed + m).choice(m - 2, count - 2, replace=False) + 1
    return np.sort(np.concatenate([[0, m - 1], rows]))      # first and last (ragged) rows always


def check_fp8_block(bs, orc, cuda, m, n, k, *, tuned, seed):
    tuning = importlib.import_module("355_1_trans_b200.tuning")
    qb, sb, B, SB = block_weights(orc, cuda, n, k)
    qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=seed), 1)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    prev = tuning.active()
    tuning.use_tuned(tuning.DEFAULT_TABLE if tuned else None)
    try:
        bs.gemm_a8w8_bpreshuffle(A, B, torch.from_numpy(sa).to(cuda), SB, torch.bfloat16, out=out)
    finally:
        tuning.use_tuned(prev)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert torch.isfinite(out).all()
    rows = sample_rows(m)
    ref, mag = orc.gemm_fp8_block(qa[rows], qb, sa[rows], sb)
    got = out[torch.from_numpy(rows).to(cuda)].float().cpu().numpy()
    assert_close(orc, ref, got, mag, f"fp8 block {m}x{n}x{k} {'tuned' if tuned else 'auto'}")


@pytest.mark.parametrize("tuned", [False, True], ids=["auto", "tuned"])
@pytest.mark.parametrize("n,k", SWEEP_NK, ids=[f"n{n}k{k}" for n, k in SWEEP_NK])
@pytest.mark.parametrize("m", SWEEP_M)
def test_fp8_block_sweep_full_size(bs, orc, cuda, m, n, k, tuned):
    """all 24 sweep shapes at full size."""
    check_fp8_block(bs, orc, cuda, m, n, k, tuned=tuned, seed=1000 + m)


@pytest.mark.parametrize("m,n,k", [(6, 1536, 7168), (27, 1536, 7168), (27, 7168, 21504)])
def test_dsv4_traced_shapes_through_tuned_table(bs, orc, cuda, m, n, k):
    """Traced DeepSeek-V4 a8w8 shapes with odd M, through the shipped tuned
    table's kernel / split choice; every row checked."""
    check_fp8_block(bs, orc, cuda, m, n, k, tuned=True, seed=2000 + m)


@pytest.mark.parametrize("layout", ["nn", "tt"])
def test_mxfp8_8192_nn_tt_row_sample(bs, orc, cuda, layout):
    """MXFP8 8192^3 in the two layouts with one MN-major operand
    (nn: A stored [K, M]; tt: B stored [K, N])."""
    m = n = k = 8192
    qa, sa = orc.quant_mxfp8(orc.normal((m, k), seed=83))
    qb, sb = orc.quant_mxfp8(orc.normal((n, k), seed=84))
    A = dev_u8(qa if layout[0] == "t" else np.ascontiguousarray(qa.T), cuda).view(torch.float8_e4m3fn)
    B = dev_u8(qb if layout[1] == "n" else np.ascontiguousarray(qb.T), cuda).view(torch.float8_e4m3fn)
    out = bs.gemm_a8w8_mxfp8(A, B, dev_u8(sa, cuda), dev_u8(sb, cuda), layout=layout)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert torch.isfinite(out).all()
    rows = sample_rows(m, 48, seed=5)
    ref, mag = orc.gemm_mxfp8(qa[rows], qb, sa[rows], sb, f64=True)
    got = out[torch.from_numpy(rows).to(cuda)].float().cpu().numpy()
    assert_close(orc, ref, got, mag, f"mxfp8 8192^3 {layout} sample")


@pytest.mark.parametrize("m", [16, 128, 1024])
def test_mxfp4_skinny_full_size(bs, orc, cuda, m):
    """MXFP4 M x 8192 x 8192, shuffled B read in place, native
    scales, automatic kernel and split-K."""
    n = k = 8192
    qa, qb, sa, sb = mxfp4_problem(orc, m, n, k, 40 + m)
    SA = bs.pack_scales(dev_u8(sa, cuda))
    SB = bs.pack_scales(dev_u8(sb, cuda))
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    bs.gemm_a4w4_mxfp4(dev_u8(qa, cuda), dev_u8(orc.shuffle_weight16(qb), cuda), SA, SB, out=out,
                       scale_format="native", b_format="shuffle16")
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert torch.isfinite(out).all()
    rows = sample_rows(m, 32, seed=6)
    ref, mag = orc.gemm_mxfp4(qa[rows], qb, sa[rows], sb)
    got = out[torch.from_numpy(rows).to(cuda)].float().cpu().numpy()
    assert_close(orc, ref, got, mag, f"mxfp4 {m}x8192x8192 shuffled")


def test_mxfp8_256_against_fp32_sequential_checker(bs, orc, cuda):
    """configs[0] against the reference's own fp32 sequential-accumulation
    loop (oracle.gemm_mxfp8 without f64 is bit-equal to
    mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:98-122 compiled from source); the
    floor term uses the fp64 sum|term|."""
    from helpers import mxfp8_problem
    qa, qb, sa, sb = [x[0] for x in mxfp8_problem(orc, 256, 256, 256, 1)]
    ref32 = orc.gemm_mxfp8(qa, qb, sa, sb).astype(np.float64)
    _, mag = orc.gemm_mxfp8(qa, qb, sa, sb, f64=True)
    for kernel in ("auto", "1cta", "pair"):
        out = bs.gemm_a8w8_mxfp8(dev_u8(qa, cuda).view(torch.float8_e4m3fn), dev_u8(qb, cuda).view(torch.float8_e4m3fn),
                                 dev_u8(sa, cuda), dev_u8(sb, cuda), kernel=kernel)
        torch.cuda.synchronize()
        assert_close(orc, ref32, out.float().cpu().numpy(), mag, f"mxfp8 256^3 {kernel} vs fp32 sequential")

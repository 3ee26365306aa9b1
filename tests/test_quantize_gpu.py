"""Device quantise + pack (bsgemm_quantize) against the CPU oracle's
quantisers: elements and scales bit for bit, every scale layout, bf16 and
fp32 input, ragged rows and edge values; then quantise -> GEMM end to end."""
import numpy as np
import pytest
import torch

from helpers import assert_close

pytestmark = pytest.mark.gpu


def edge_rows(orc, rows, cols, seed):
    """N(0,1) data with planted edge cases: an all-zero group, huge values
    (saturation), tiny values (subnormal after scaling), exact powers of two
    times qmax, and negative zeros."""
    x = orc.normal((rows, cols), seed=seed).astype(np.float32)
    x[0, :32] = 0.0
    x[1, :32] *= 1e30
    x[2, 32:64] *= 1e-30
    x[3, 64:96] = 448.0 * 2.0 ** np.arange(-16, 16)[:32]
    x[4, 96:128] = -0.0
    x[5, :128] = 6.0 * 2.0 ** -3
    return x


def as_bf16(x):
    t = torch.from_numpy(x).to(torch.bfloat16)
    return t, t.float().numpy()


@pytest.mark.parametrize("in_dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("rows", [200, 256])
def test_quantize_mxfp8_bit_exact(bs, orc, cuda, in_dtype, rows):
    cols = 1024
    x = edge_rows(orc, rows, cols, 11 + rows)
    if in_dtype == "bf16":
        xt, xref = as_bf16(x)
    else:
        xt, xref = torch.from_numpy(x), x
    qa, sa = orc.quant_mxfp8(xref)
    q, sf = bs.quantize(xt.to(cuda), "mxfp8", scale_format="rowmajor")
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), qa)
    assert np.array_equal(sf.cpu().numpy(), sa)
    q2, sfn = bs.quantize(xt.to(cuda), "mxfp8", scale_format="native")
    assert np.array_equal(q2.view(torch.uint8).cpu().numpy(), qa)
    assert np.array_equal(sfn.cpu().numpy(), orc.sf_to_native(sa))


@pytest.mark.parametrize("in_dtype", ["bf16", "fp32"])
def test_quantize_mxfp4_bit_exact(bs, orc, cuda, in_dtype):
    rows, cols = 136, 512
    x = edge_rows(orc, rows, cols, 21)
    if in_dtype == "bf16":
        xt, xref = as_bf16(x)
    else:
        xt, xref = torch.from_numpy(x), x
    qa, sa = orc.quant_mxfp4(xref)
    q, sf = bs.quantize(xt.to(cuda), "mxfp4", scale_format="rowmajor")
    assert np.array_equal(q.cpu().numpy(), qa)
    assert np.array_equal(sf.cpu().numpy(), sa)
    _, sfn = bs.quantize(xt.to(cuda), "mxfp4")
    assert np.array_equal(sfn.cpu().numpy(), orc.sf_to_native(sa))


@pytest.mark.parametrize("in_dtype", ["bf16", "fp32"])
def test_quantize_fp8_block_bit_exact(bs, orc, cuda, in_dtype):
    rows, cols = 77, 896
    x = edge_rows(orc, rows, cols, 31)
    if in_dtype == "bf16":
        xt, xref = as_bf16(x)
    else:
        xt, xref = torch.from_numpy(x), x
    qa, sa = orc.quant_fp8_block(xref, 1)
    q, sf = bs.quantize(xt.to(cuda), "fp8_block")
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), qa)
    assert np.array_equal(sf.cpu().numpy().view(np.uint32), sa.astype(np.float32).view(np.uint32))
    _, sft = bs.quantize(xt.to(cuda), "fp8_block", scale_format="kmajor_t")
    assert np.array_equal(sft.cpu().numpy(), np.ascontiguousarray(sa.T))


def test_quantize_then_gemm(bs, orc, cuda):
    """Activations quantised on the device feed the MXFP8 GEMM directly
    (native scales); the result matches the oracle GEMM of the oracle's
    quantisation of the same data."""
    m, n, k = 96, 384, 512
    x = orc.normal((m, k), seed=41).astype(np.float32)
    w = orc.normal((n, k), seed=42).astype(np.float32)
    xt, xref = as_bf16(x)
    qa, sa = orc.quant_mxfp8(xref)
    qb, sb = orc.quant_mxfp8(w)
    ref, mag = orc.gemm_mxfp8(qa, qb, sa, sb, f64=True)
    q, sfn = bs.quantize(xt.to(cuda), "mxfp8")
    B = torch.from_numpy(qb).to(cuda).view(torch.float8_e4m3fn)
    SB = bs.pack_scales(torch.from_numpy(sb).to(cuda))
    out = bs.gemm_a8w8_mxfp8(q, B, sfn, SB, scale_format="native")
    torch.cuda.synchronize()
    assert_close(orc, ref, out.float().cpu().numpy(), mag, "quantize -> mxfp8 gemm")


def test_quantize_rejects_bad_shapes(bs, cuda):
    x = torch.zeros((4, 100), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(bs.BsgemmError):
        bs.quantize(x, "mxfp8", scale_format="rowmajor")      # cols % 32
    y = torch.zeros((4, 96), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(bs.BsgemmError):
        bs.quantize(y, "mxfp8", scale_format="native")        # native atoms need cols % 128
    with pytest.raises(bs.BsgemmError):
        bs.quantize(y, "fp8_block")                           # cols % 128

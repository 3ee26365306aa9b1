"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Each case follows the reference's self-checking host drivers: inputs are
seeded and quantised on the host, the raw operands go to the oracle and the
(possibly repacked) operands to the GPU, C is NaN-poisoned before the launch,
and the result must meet the target tolerance on bf16 outputs,
    |err| <= 2^-7 |ref| + 1e-3 + 1e-6 * sum|a*b*s|  per element,
    max relative error <= 1e-2 over non-cancelling elements,
where the last term is an fp32-accumulation floor for elements whose terms
cancel (see oracle.check_baseline_rule; measured GPU error is below
4e-7 * sum|term| and bit-identical from run to run).  Fixture patterns of the
reference (unit scales, K-pattern scales, persistent-grid overrides, ragged
shapes) are all exercised.
"""
import numpy as np
import pytest
import torch

from helpers import assert_close, dev_u8, mxfp4_problem, mxfp8_problem, scale_mode

pytestmark = pytest.mark.gpu


def poisoned(shape, dtype, device):
    return torch.full(shape, float("nan"), dtype=dtype, device=device)


def run_mxfp8(bs, orc, cuda, m, n, k, *, seed=1, layout="tn", sf_mode="data", out_dtype=torch.bfloat16,
              split_k=0, grid_blocks=0, batch=1, native=False, kernel="auto"):
    qa_l, qb_l, sa_l, sb_l = mxfp8_problem(orc, m, n, k, seed, sf_mode, batch)
    res = [orc.gemm_mxfp8(qa, qb, sa, sb, f64=True) for qa, qb, sa, sb in zip(qa_l, qb_l, sa_l, sb_l)]
    refs, mags = [r[0] for r in res], [r[1] for r in res]
    a_host = [qa if layout[0] == "t" else np.ascontiguousarray(qa.T) for qa in qa_l]
    b_host = [qb if layout[1] == "n" else np.ascontiguousarray(qb.T) for qb in qb_l]
    A = dev_u8(np.stack(a_host) if batch > 1 else a_host[0], cuda).view(torch.float8_e4m3fn)
    B = dev_u8(np.stack(b_host) if batch > 1 else b_host[0], cuda).view(torch.float8_e4m3fn)
    SA = dev_u8(np.stack(sa_l) if batch > 1 else sa_l[0], cuda)
    SB = dev_u8(np.stack(sb_l) if batch > 1 else sb_l[0], cuda)
    fmt = "rowmajor"
    if native:
        assert batch == 1
        SA, SB = bs.pack_scales(SA), bs.pack_scales(SB)
        fmt = "native"
    out = poisoned((m, n) if batch == 1 else (batch, m, n), out_dtype, cuda)
    bs.gemm_a8w8_mxfp8(A, B, SA, SB, layout=layout, out_dtype=out_dtype, out=out, scale_format=fmt,
                       split_k=split_k, grid_blocks=grid_blocks, kernel=kernel)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    got = out.float().cpu().numpy()
    if batch == 1:
        got = got[None]
    for b in range(batch):
        assert_close(orc, refs[b], got[b], mags[b], f"mxfp8 {m}x{n}x{k} {layout} b{b}")
    return refs, got


# ---- MXFP8 ---------------------------------------------------------------------------

def test_mxfp8_256_tn_bf16(bs, orc, cuda):
    """The CPU-runnable case: M=N=K=256, tn, bf16 out, data-derived scales."""
    refs, got = run_mxfp8(bs, orc, cuda, 256, 256, 256)
    # also the reference's own acceptance rule (valid_vector with bf16 bounds)
    mag = orc.gemm_mxfp8(*[x[0] for x in mxfp8_problem(orc, 256, 256, 256, 1)], f64=True)[1]
    errors, _ = orc.check_e8m0_rule(refs[0], got[0], mag, bf16=True)   # 1e-4 + 5e-5 * sum|term|
    assert errors == 0


@pytest.mark.parametrize("sf_mode", ["unit", "kpattern", "rowpattern"])
def test_mxfp8_scale_patterns(bs, orc, cuda, sf_mode):
    run_mxfp8(bs, orc, cuda, 256, 256, 512, seed=2, sf_mode=sf_mode)


def test_mxfp8_fp32_out(bs, orc, cuda):
    refs, got = run_mxfp8(bs, orc, cuda, 128, 256, 256, seed=3, out_dtype=torch.float32)
    # fp32 out: the reference's 1e-3-relative-to-magnitude rule holds tightly
    np.testing.assert_allclose(got[0], refs[0], rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize("layout", ["tn", "nn", "tt", "nt"])
def test_mxfp8_layouts(bs, orc, cuda, layout):
    run_mxfp8(bs, orc, cuda, 256, 384, 512, seed=4, layout=layout, sf_mode="kpattern")


def test_mxfp8_ragged(bs, orc, cuda):
    run_mxfp8(bs, orc, cuda, 200, 264, 384, seed=5)


def test_mxfp8_batched(bs, orc, cuda):
    run_mxfp8(bs, orc, cuda, 128, 256, 256, seed=6, batch=2)


@pytest.mark.parametrize("split_k", [2, 3])
def test_mxfp8_split_k(bs, orc, cuda, split_k):
    run_mxfp8(bs, orc, cuda, 128, 256, 1024, seed=7, split_k=split_k, sf_mode="kpattern")


def test_mxfp8_auto_split_skinny(bs, orc, cuda):
    run_mxfp8(bs, orc, cuda, 16, 512, 2048, seed=8)


def test_mxfp8_native_scales(bs, orc, cuda):
    run_mxfp8(bs, orc, cuda, 256, 256, 512, seed=9, native=True, sf_mode="rowpattern")


@pytest.mark.parametrize("grid_blocks", [1, 37])
def test_mxfp8_persistent_grid(bs, orc, cuda, grid_blocks):
    """The reference's PERSIST_GRID override: many tiles per CTA."""
    run_mxfp8(bs, orc, cuda, 512, 512, 256, seed=10, grid_blocks=grid_blocks)


# ---- CTA-pair (cta_group::2) kernel -----------------------------------------------------

@pytest.mark.parametrize("layout", ["tn", "nn", "tt", "nt"])
def test_mxfp8_pair_layouts(bs, orc, cuda, layout):
    run_mxfp8(bs, orc, cuda, 512, 512, 512, seed=31, layout=layout, sf_mode="kpattern", kernel="pair")


def test_mxfp8_pair_ragged_batched(bs, orc, cuda):
    run_mxfp8(bs, orc, cuda, 300, 392, 384, seed=32, sf_mode="rowpattern", kernel="pair")
    run_mxfp8(bs, orc, cuda, 256, 256, 256, seed=33, batch=2, kernel="pair")


def test_mxfp8_pair_native_and_grid(bs, orc, cuda):
    run_mxfp8(bs, orc, cuda, 768, 512, 256, seed=34, native=True, kernel="pair", grid_blocks=2)


def test_mxfp4_pair(bs, orc, cuda):
    run_mxfp4(bs, orc, cuda, 512, 512, 1024, seed=35, sf_mode="kpattern", kernel="pair")
    run_mxfp4(bs, orc, cuda, 260, 264, 512, seed=36, sf_mode="rowpattern", kernel="pair")


# ---- MXFP4 ---------------------------------------------------------------------------

def run_mxfp4(bs, orc, cuda, m, n, k, *, seed=1, sf_mode="data", split_k=0, out_dtype=torch.bfloat16,
              grid_blocks=0, kernel="auto"):
    qa, qb, sa, sb = mxfp4_problem(orc, m, n, k, seed, sf_mode)
    ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
    out = poisoned((m, n), out_dtype, cuda)
    bs.gemm_a4w4_mxfp4(dev_u8(qa, cuda), dev_u8(qb, cuda), dev_u8(sa, cuda), dev_u8(sb, cuda),
                       out=out, out_dtype=out_dtype, split_k=split_k, grid_blocks=grid_blocks,
                       kernel=kernel)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    got = out.float().cpu().numpy()
    calc_diff = assert_close(orc, ref, got, mag, f"mxfp4 {m}x{n}x{k}")
    assert calc_diff < 0.02      # the reference's cosine-style gate
    return ref, got, mag


def test_mxfp4_256(bs, orc, cuda):
    run_mxfp4(bs, orc, cuda, 256, 256, 512)


@pytest.mark.parametrize("sf_mode", ["unit", "kpattern", "rowpattern"])
def test_mxfp4_scale_patterns(bs, orc, cuda, sf_mode):
    run_mxfp4(bs, orc, cuda, 256, 512, 1024, seed=2, sf_mode=sf_mode)


def test_mxfp4_reference_rule(bs, orc, cuda):
    """mxfp4 host compare(): tol = 1e-4 + 5e-5 * sum|term| + |ref|/256."""
    ref, got, mag = run_mxfp4(bs, orc, cuda, 128, 256, 512, seed=3, out_dtype=torch.float32)
    tol = 1e-4 + 5e-5 * mag + np.abs(ref) / 256
    assert np.all(np.abs(got - ref) <= tol)


def test_mxfp4_ragged_and_split(bs, orc, cuda):
    run_mxfp4(bs, orc, cuda, 16, 384, 2048, seed=4, split_k=4)
    run_mxfp4(bs, orc, cuda, 130, 256, 512, seed=5)


def test_mxfp4_shuffled_b(bs, orc, cuda):
    """B given in aiter shuffle_weight(16,16) bytes: bsgemm_pack_b restores the
    raw layout bit-exactly on the device (candidate_m10 bs layout)."""
    qa, qb, sa, sb = mxfp4_problem(orc, 128, 256, 512, 6, "kpattern")
    sh = orc.shuffle_weight16(qb)
    raw = bs.pack_b(dev_u8(sh, cuda), "shuffle16")
    assert np.array_equal(raw.cpu().numpy(), qb)
    ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
    out = bs.gemm_a4w4_mxfp4(dev_u8(qa, cuda), raw, dev_u8(sa, cuda), dev_u8(sb, cuda))
    assert_close(orc, ref, out.float().cpu().numpy(), mag, "mxfp4 shuffled B")


@pytest.mark.parametrize("kernel", ["1cta", "pair"])
def test_mxfp4_shuffled_b_in_place(bs, orc, cuda, kernel):
    """shuffle_weight(16,16) B read in place (5-D tensor map into the
    no-swizzle K-major layout): bit-identical to the raw-B launch."""
    for m, n, k, seed in ((256, 512, 1024, 7), (200, 272, 512, 8)):
        qa, qb, sa, sb = mxfp4_problem(orc, m, n, k, seed, "rowpattern")
        ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
        A, SA, SB = dev_u8(qa, cuda), dev_u8(sa, cuda), dev_u8(sb, cuda)
        raw = bs.gemm_a4w4_mxfp4(A, dev_u8(qb, cuda), SA, SB, kernel=kernel, split_k=1)
        shuf = bs.gemm_a4w4_mxfp4(A, dev_u8(orc.shuffle_weight16(qb), cuda), SA, SB, kernel=kernel,
                                  split_k=1, b_format="shuffle16")
        torch.cuda.synchronize()
        assert bs.check_device_error() == 0
        assert torch.equal(raw, shuf)
        assert_close(orc, ref, shuf.float().cpu().numpy(), mag, f"mxfp4 shuffled {kernel} {m}x{n}x{k}")


@pytest.mark.parametrize("kernel,out_dtype", [("1cta", torch.bfloat16), ("1cta", torch.float32),
                                              ("pair", torch.bfloat16)])
def test_mxfp8_shuffled_b_in_place(bs, orc, cuda, kernel, out_dtype):
    for m, n, k, seed in ((256, 512, 512, 9), (72, 400, 384, 10)):
        qa_l, qb_l, sa_l, sb_l = mxfp8_problem(orc, m, n, k, seed, "rowpattern")
        qa, qb, sa, sb = qa_l[0], qb_l[0], sa_l[0], sb_l[0]
        ref, mag = orc.gemm_mxfp8(qa, qb, sa, sb, f64=True)
        A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
        SA, SB = dev_u8(sa, cuda), dev_u8(sb, cuda)
        raw = bs.gemm_a8w8_mxfp8(A, dev_u8(qb, cuda).view(torch.float8_e4m3fn), SA, SB, kernel=kernel,
                                 out_dtype=out_dtype, split_k=1)
        shuf = bs.gemm_a8w8_mxfp8(A, dev_u8(orc.shuffle_weight16(qb), cuda).view(torch.float8_e4m3fn), SA, SB,
                                  kernel=kernel, out_dtype=out_dtype, split_k=1, b_format="shuffle16")
        torch.cuda.synchronize()
        assert bs.check_device_error() == 0
        assert torch.equal(raw, shuf)
        assert_close(orc, ref, shuf.float().cpu().numpy(), mag, f"mxfp8 shuffled {kernel} {m}x{n}x{k}")


# ---- transposed (swap-AB) MX decode kernel -------------------------------------------

@pytest.mark.parametrize("m", [1, 16, 30, 64])
def test_mxfp8_swap_decode(bs, orc, cuda, m):
    run_mxfp8(bs, orc, cuda, m, 640, 1024, seed=80 + m, sf_mode="rowpattern", kernel="swap")


def test_mxfp8_swap_variants(bs, orc, cuda):
    """fp32 out, forced split-K, native scales, batch 2 through the swap kernel."""
    run_mxfp8(bs, orc, cuda, 24, 520, 2048, seed=90, out_dtype=torch.float32, split_k=3, kernel="swap")
    run_mxfp8(bs, orc, cuda, 40, 384, 512, seed=91, native=True, kernel="swap")
    run_mxfp8(bs, orc, cuda, 8, 256, 1024, seed=92, batch=2, kernel="swap")


@pytest.mark.parametrize("m,k,split_k", [(16, 128, 1), (5, 384, 1), (32, 640, 5), (64, 896, 2), (16, 1152, 9)])
def test_mxfp8_swap_short_units(bs, orc, cuda, m, k, split_k):
    """Units of 1, 3 and odd numbers of K blocks (including split-K slices of one K block): the
    transposed kernel accumulates alternate K blocks in two TMEM chains and sums only the chains a
    unit reached."""
    run_mxfp8(bs, orc, cuda, m, 384, k, seed=200 + k + split_k, sf_mode="rowpattern", split_k=split_k,
              kernel="swap")


@pytest.mark.parametrize("m,k,split_k", [(1, 256, 1), (16, 768, 1), (40, 1280, 5)])
def test_mxfp4_swap_short_units(bs, orc, cuda, m, k, split_k):
    qa, qb, sa, sb = mxfp4_problem(orc, m, 512, k, 300 + k, "kpattern")
    ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
    out = poisoned((m, 512), torch.bfloat16, cuda)
    bs.gemm_a4w4_mxfp4(dev_u8(qa, cuda), dev_u8(orc.shuffle_weight16(qb), cuda), dev_u8(sa, cuda), dev_u8(sb, cuda),
                       out=out, kernel="swap", b_format="shuffle16", split_k=split_k)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert_close(orc, ref, out.float().cpu().numpy(), mag, f"mxfp4 swap {m}x512x{k} split {split_k}")


@pytest.mark.parametrize("m", [1, 16, 64])
def test_mxfp4_swap_decode_shuffled(bs, orc, cuda, m):
    qa, qb, sa, sb = mxfp4_problem(orc, m, 768, 2048, 95 + m, "kpattern")
    ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
    A, SA, SB = dev_u8(qa, cuda), dev_u8(sa, cuda), dev_u8(sb, cuda)
    for b_format, Bh in (("raw", qb), ("shuffle16", orc.shuffle_weight16(qb))):
        out = poisoned((m, 768), torch.bfloat16, cuda)
        bs.gemm_a4w4_mxfp4(A, dev_u8(Bh, cuda), SA, SB, out=out, kernel="swap", b_format=b_format)
        torch.cuda.synchronize()
        assert bs.check_device_error() == 0
        assert_close(orc, ref, out.float().cpu().numpy(), mag, f"mxfp4 swap {m} {b_format}")


# ---- E8M0 1x128 / 128x128 block scale: the reference's launch_blockscale_bpreshuffle --

def e8m0_block_problem(orc, m, n, k, seed):
    """E4M3 values of N(0,1) data, E8M0 scale bytes 124 + r % 7 as the
    reference's fill_scales (source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:154-159)."""
    qa, _ = orc.quant_mxfp8(orc.normal((m, k), seed=seed * 31))
    qb, _ = orc.quant_mxfp8(orc.normal((n, k), seed=seed * 31 + 1))
    rng = np.random.default_rng(seed)
    sfa_t = (124 + rng.integers(0, 7, size=(k // 128, m))).astype(np.uint8)
    sfb = (124 + rng.integers(0, 7, size=(n // 128, k // 128))).astype(np.uint8)
    return qa, qb, sfa_t, sfb


def run_e8m0_block(bs, orc, cuda, m, n, k, *, seed=1, dtype=torch.bfloat16, colmajor=True):
    qa, qb, sfa_t, sfb = e8m0_block_problem(orc, m, n, k, seed)
    ref, mag = orc.gemm_e8m0_block(qa, qb, sfa_t, sfb)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(orc.shuffle_weight16(qb), cuda).view(torch.float8_e4m3fn)
    if colmajor:
        SA = dev_u8(sfa_t, cuda).t()                       # [M, K/128], strides (1, M)
    else:
        SA = dev_u8(sfa_t, cuda).reshape(m, k // 128)      # contiguous, transposed bytes
    SB = dev_u8(sfb, cuda)
    out = poisoned((m, n), dtype, cuda)
    bs.gemm_a8w8_blockscale_bpreshuffle(A, B, SA, SB, dtype, out)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    got = out.float().cpu().numpy()
    errors, ratio = orc.check_e8m0_rule(ref, got, mag, bf16=dtype == torch.bfloat16)
    assert errors == 0, f"e8m0 block {m}x{n}x{k}: {errors} errors, max ratio {ratio}"
    if dtype == torch.bfloat16:
        assert_close(orc, ref, got, mag, f"e8m0 block {m}x{n}x{k}")
    return ref, got


def test_e8m0_block_256(bs, orc, cuda):
    run_e8m0_block(bs, orc, cuda, 256, 256, 512)


def test_e8m0_block_fp32_and_ragged(bs, orc, cuda):
    run_e8m0_block(bs, orc, cuda, 256, 512, 1024, seed=2, dtype=torch.float32)
    run_e8m0_block(bs, orc, cuda, 200, 384, 256, seed=3, colmajor=False)
    run_e8m0_block(bs, orc, cuda, 16, 1024, 2048, seed=4)


def test_e8m0_block_pair_path(bs, orc, cuda):
    """Enough 256x256 tiles for the CTA-pair kernel (its scale builders arrive
    on the leader's barrier across the cluster)."""
    run_e8m0_block(bs, orc, cuda, 2048, 2560, 256, seed=5)


def test_e8m0_block_rejects_like_reference(bs, cuda):
    A = torch.zeros((256, 256), dtype=torch.float8_e4m3fn, device=cuda)
    B = torch.zeros((256, 256), dtype=torch.uint8, device=cuda)
    SA = torch.zeros((256, 2), dtype=torch.uint8, device=cuda)
    SB = torch.zeros((2, 2), dtype=torch.uint8, device=cuda)
    with pytest.raises(ValueError):
        bs.gemm_a8w8_blockscale_bpreshuffle(A, B, SA.float(), SB)      # fp32 scales
    with pytest.raises(ValueError):
        bs.gemm_a8w8_blockscale_bpreshuffle(A, B, SA, SB, tiles=2)
    with pytest.raises(ValueError):
        bs.gemm_a8w8_blockscale_bpreshuffle(A, B[:, :128].contiguous(), SA, SB)
    out = torch.empty((256, 256), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        bs.gemm_a8w8_blockscale_bpreshuffle(A, B, SA, SB, out=out[:, :128])


# ---- FP8 block-scale (fp32 scales) --------------------------------------------------

def run_fp8_block(bs, orc, cuda, m, n, k, *, seed=1, kpanel=True, transposed=False, split_k=0,
                  out_dtype=torch.bfloat16, kernel="auto", shuffle16=False, grid_blocks=0):
    x = orc.normal((m, k), seed=seed * 77)
    w = orc.normal((n, k), seed=seed * 77 + 1)
    qa, sa = orc.quant_fp8_block(x, 1)
    qb, sb = orc.quant_fp8_block(w, 128)
    ref, mag = orc.gemm_fp8_block(qa, qb, sa, sb)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    if shuffle16:
        B = dev_u8(orc.shuffle_weight16(qb), cuda).view(torch.float8_e4m3fn)
        b_layout = "shuffle16"
    elif kpanel:
        B = dev_u8(orc.shuffle_kpanel(qb), cuda).view(torch.float8_e4m3fn)
        b_layout = "kpanel"
    else:
        B = dev_u8(qb, cuda).view(torch.float8_e4m3fn)
        b_layout = "raw"
    SA = torch.from_numpy(np.ascontiguousarray(sa.T if transposed else sa)).to(cuda)
    SB = torch.from_numpy(sb).to(cuda)
    out = poisoned((m, n), out_dtype, cuda)
    bs.gemm_a8w8_bpreshuffle(A, B, SA, SB, out_dtype, b_layout=b_layout, x_scale_transposed=transposed,
                             out=out, split_k=split_k, kernel=kernel, grid_blocks=grid_blocks)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    got = out.float().cpu().numpy()
    assert_close(orc, ref, got, mag, f"fp8 block {m}x{n}x{k}")
    return ref, got


def test_fp8_block_kpanel(bs, orc, cuda):
    run_fp8_block(bs, orc, cuda, 256, 256, 512)


def test_fp8_block_raw_b_transposed_sfa(bs, orc, cuda):
    run_fp8_block(bs, orc, cuda, 256, 384, 384, seed=2, kpanel=False, transposed=True)


def test_fp8_block_fp32_out(bs, orc, cuda):
    ref, got = run_fp8_block(bs, orc, cuda, 128, 256, 512, seed=3, out_dtype=torch.float32)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("m", [1, 16, 64, 200])
def test_fp8_block_decode_shapes(bs, orc, cuda, m):
    run_fp8_block(bs, orc, cuda, m, 1024, 2048, seed=4 + m)


@pytest.mark.parametrize("m,kernel", [(1, "swap"), (7, "swap"), (16, "swap"), (30, "swap"), (64, "swap"),
                                      (16, "1cta"), (64, "1cta")])
def test_fp8_block_decode_kernels(bs, orc, cuda, m, kernel):
    """Decode shapes through the transposed kernel and the standard one."""
    run_fp8_block(bs, orc, cuda, m, 896, 2304, seed=40 + m, kernel=kernel, transposed=(m == 7))


def test_fp8_block_swap_raw_b_fp32_split(bs, orc, cuda):
    ref, got = run_fp8_block(bs, orc, cuda, 24, 640, 1536, seed=50, kpanel=False, kernel="swap",
                             split_k=3, out_dtype=torch.float32)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("m,k,split_k", [(16, 128, 1), (1, 384, 1), (30, 640, 5), (64, 384, 3), (8, 1152, 9)])
def test_fp8_block_swap_short_units(bs, orc, cuda, m, k, split_k):
    """Units of 1 and 3 K blocks and split-K slices of one K block: the two promotion sets take
    alternate K blocks, so a set may see none of a unit's K blocks and still hand over zeros."""
    run_fp8_block(bs, orc, cuda, m, 640, k, seed=70 + k + split_k, kernel="swap", split_k=split_k)


# ---- CTA-pair fp32 block-scale kernel (256 x 256 tiles) --------------------------------

@pytest.mark.parametrize("m,n,k,layout,out_dtype,transposed", [
    (256, 256, 512, "kpanel", torch.bfloat16, False),
    (512, 384, 1024, "raw", torch.bfloat16, True),
    (384, 768, 640, "shuffle16", torch.bfloat16, False),
    (300, 200, 384, "kpanel", torch.float32, False),
    (1, 128, 256, "raw", torch.bfloat16, False),
    (129, 1000, 1152, "kpanel", torch.bfloat16, True),
])
def test_fp8_block_pair(bs, orc, cuda, m, n, k, layout, out_dtype, transposed):
    """The pair kernel on every weight layout and both outputs.  M = 300 and 129
    leave the peer CTA's rows of the last pair tile wholly or partly past M; N =
    200 and 1000 end inside a tile's second column half (and the peer's B rows),
    N = 384 leaves that half wholly past N."""
    run_fp8_block(bs, orc, cuda, m, n, k, seed=90 + m, kpanel=layout == "kpanel", shuffle16=layout == "shuffle16",
                  transposed=transposed, out_dtype=out_dtype, kernel="pair")


@pytest.mark.parametrize("grid_blocks", [2, 6, 0])
def test_fp8_block_pair_persistent(bs, orc, cuda, grid_blocks):
    """More pair tiles (10 x 10) than clusters: 1, 3 and all co-resident pairs walk the tiles."""
    run_fp8_block(bs, orc, cuda, 2560, 2560, 384, seed=97, kernel="pair", grid_blocks=grid_blocks)


def test_fp8_block_pair_matches_1cta(bs, orc, cuda):
    """Each SM of a pair computes its 128 rows of the 128-K partial from the same
    bytes in the same K order as the 1-CTA kernel, and promotes them with the same
    fma.rn, so the two kernels agree bit for bit."""
    m, n, k = 1024, 1024, 2048
    qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=98), 1)
    qb, sb = orc.quant_fp8_block(orc.normal((n, k), seed=99), 128)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(orc.shuffle_kpanel(qb), cuda).view(torch.float8_e4m3fn)
    SA, SB = torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda)
    outs = [bs.gemm_a8w8_bpreshuffle(A, B, SA, SB, torch.float32, kernel=kern, split_k=1)
            for kern in ("1cta", "pair")]
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert torch.equal(outs[0], outs[1])


# ---- wide single-CTA kernel (128 x 256 tiles, K slices of every tile) -------------------
@pytest.mark.parametrize("m,n,k,split_k,layout,out_dtype,transposed", [
    (128, 768, 1024, 0, "kpanel", torch.bfloat16, False),
    (100, 520, 2048, 3, "raw", torch.float32, True),      # partial M and N tiles, slices of 5-6 K blocks
    (64, 512, 1536, 1, "shuffle16", torch.bfloat16, False),
    (200, 1032, 768, 2, "kpanel", torch.bfloat16, False),  # two M tiles, a last N tile of 8 columns
    (1, 256, 384, 3, "kpanel", torch.bfloat16, False),     # slices of one K block
    (300, 784, 3072, 0, "shuffle16", torch.float32, False),
])
def test_fp8_block_wide(bs, orc, cuda, m, n, k, split_k, layout, out_dtype, transposed):
    ref, got = run_fp8_block(bs, orc, cuda, m, n, k, seed=600 + m + n, kpanel=layout == "kpanel",
                             shuffle16=layout == "shuffle16", transposed=transposed, split_k=split_k,
                             out_dtype=out_dtype, kernel="wide")
    if out_dtype == torch.float32:
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("layout", ["kpanel", "raw", "shuffle16"])
def test_fp8_block_wide_matches_1cta(bs, orc, cuda, layout):
    """Whole tiles (split_k=1): the wide kernel promotes each element in the 1-CTA kernel's
    order with the same fma.rn, so the two agree bit for bit; with K slices the result is the
    same from run to run."""
    m, n, k = 200, 1040, 1536
    qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=620), 1)
    qb, sb = orc.quant_fp8_block(orc.normal((n, k), seed=621), 128)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    Bh = orc.shuffle_kpanel(qb) if layout == "kpanel" else orc.shuffle_weight16(qb) if layout == "shuffle16" else qb
    B = dev_u8(Bh, cuda).view(torch.float8_e4m3fn)
    SA, SB = torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda)
    run = lambda kern, sk: bs.gemm_a8w8_bpreshuffle(A, B, SA, SB, torch.float32, b_layout=layout, kernel=kern,
                                                    split_k=sk)
    one, wide, s1, s2 = run("1cta", 1), run("wide", 1), run("wide", 4), run("wide", 4)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert torch.equal(one, wide)
    assert torch.equal(s1, s2)
    ref, mag = orc.gemm_fp8_block(qa, qb, sa, sb)
    assert_close(orc, ref, s1.cpu().numpy(), mag, f"fp8 block wide split 4 {layout}")


@pytest.mark.parametrize("grid_blocks,split_k", [(7, 3), (1, 1), (5, 0)])
def test_fp8_block_wide_persistent_grid(bs, orc, cuda, grid_blocks, split_k):
    """A capped grid walks several units (and their K slices) per CTA: the TMEM buffers and the
    stage ring carry over between units."""
    run_fp8_block(bs, orc, cuda, 300, 1280, 1536, seed=660 + grid_blocks, split_k=split_k, kernel="wide",
                  grid_blocks=grid_blocks)


def test_fp8_block_wide_mx_rejects(bs, orc, cuda):
    """The wide kernel is for fp32 block scales only: the MX families refuse it."""
    qa, sa = orc.quant_mxfp8(orc.normal((128, 256), seed=650))
    qb, sb = orc.quant_mxfp8(orc.normal((256, 256), seed=651))
    with pytest.raises(bs.BsgemmError):
        bs.gemm_a8w8_mxfp8(dev_u8(qa, cuda).view(torch.float8_e4m3fn), dev_u8(qb, cuda).view(torch.float8_e4m3fn),
                           dev_u8(sa, cuda), dev_u8(sb, cuda), kernel="wide")


@pytest.mark.parametrize("m,n,k,grid_blocks,out_dtype", [
    (1024, 5120, 4096, 0, torch.bfloat16),   # 80 units on 74 clusters: 6 tail units x 4 slices
    (512, 2048, 4096, 0, torch.float32),     # 16 units, fewer than a wave: every unit in 4 slices
    (1024, 5120, 4096, 26, torch.bfloat16),  # 13 clusters: 80 = 6 x 13 + 2 tail units x 4 slices
])
def test_fp8_block_pair_tail_slices(bs, orc, cuda, m, n, k, grid_blocks, out_dtype):
    """The pair kernel's partial last wave as K slices (fp32 partials in the workspace, summed in
    slice order by the tail reduce): correct against the oracle, bit-identical from run to run,
    and within rounding of the unsplit run (split_k=1)."""
    qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=500 + m), 1)
    qb, sb = orc.quant_fp8_block(orc.normal((n, k), seed=501 + n), 128)
    ref, mag = orc.gemm_fp8_block(qa, qb, sa, sb)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(orc.shuffle_kpanel(qb), cuda).view(torch.float8_e4m3fn)
    SA, SB = torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda)
    outs = [bs.gemm_a8w8_bpreshuffle(A, B, SA, SB, out_dtype, kernel="pair", grid_blocks=grid_blocks, split_k=sk)
            for sk in (0, 0, 1)]
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    got = outs[0].float().cpu().numpy()
    assert_close(orc, ref, got, mag, f"fp8 block pair tail {m}x{n}x{k}")
    assert torch.equal(outs[0], outs[1])
    assert_close(orc, outs[2].float().cpu().numpy(), got, mag, "tail slices against unsplit")


@pytest.mark.parametrize("kernel,split_k", [("pair", 0), ("auto", 0), ("1cta", 0), ("wide", 0), ("wide", 3)])
def test_fp8_block_batched_c_abi(bs, orc, cuda, kernel, split_k):
    """Batched fp32 block-scale through the C ABI (the Python wrapper is batch 1): batch strides
    of A, K-panel B, both scales and C, with padding between A's and C's batch slices, checked
    per batch against the oracle.  At this size "auto" takes the pair kernel (2 waves of 120 pair
    units, counted 1.6 each, against 4 waves of 480 tiles)."""
    import ctypes
    batch, m, n, k = 2, 1536, 2560, 512
    kb = k // 128
    pads_a, pads_c = 64, 96   # extra rows between batch slices
    A = torch.zeros(batch, m + pads_a, k, dtype=torch.uint8, device=cuda)
    B = torch.empty(batch, kb, n, 128, dtype=torch.uint8, device=cuda)
    SA = torch.empty(batch, m, kb, dtype=torch.float32, device=cuda)
    SB = torch.empty(batch, n // 128, kb, dtype=torch.float32, device=cuda)
    C = torch.full((batch, m + pads_c, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    refs = []
    for e in range(batch):
        qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=300 + e), 1)
        qb, sb = orc.quant_fp8_block(orc.normal((n, k), seed=310 + e), 128)
        refs.append(orc.gemm_fp8_block(qa, qb, sa, sb))
        A[e, :m] = dev_u8(qa, cuda)
        B[e] = dev_u8(orc.shuffle_kpanel(qb), cuda).view(kb, n, 128)
        SA[e] = torch.from_numpy(sa).to(cuda)
        SB[e] = torch.from_numpy(sb).to(cuda)
    args = bs.Args()
    bs.lib().bsgemm_args_init(ctypes.byref(args))
    args.ptr_a, args.ptr_b, args.ptr_c = A.data_ptr(), B.data_ptr(), C.data_ptr()
    args.m, args.n, args.k, args.batch = m, n, k, batch
    args.stride_a, args.stride_b, args.stride_c = k, 128, n
    args.stride_a_batch, args.stride_b_batch, args.stride_c_batch = (m + pads_a) * k, n * k, (m + pads_c) * n
    args.ptr_sfa, args.ptr_sfb = SA.data_ptr(), SB.data_ptr()
    args.stride_sfa, args.stride_sfb = kb, kb
    args.stride_sfa_batch, args.stride_sfb_batch = m * kb, (n // 128) * kb
    args.layout, args.b_format = bs.LAYOUTS["tn"], bs.B_KPANEL128
    args.sfa_format, args.sfb_format, args.out_dtype = bs.SF_ROWMAJOR, bs.SF_ROWMAJOR, bs.OUT_BF16
    args.kernel = bs.KERNELS[kernel]
    args.split_k = split_k
    ws = bs._workspace(bs.FAMILY_FP8_BLOCK, args, None, cuda)
    status = bs.lib().bsgemm_a8w8_blockscale_bpreshuffle(ctypes.byref(args), bs._stream(cuda))
    torch.cuda.synchronize()
    del ws
    assert status == bs.OK, bs.strerror(status)
    assert bs.check_device_error() == 0
    for e in range(batch):
        ref, mag = refs[e]
        assert_close(orc, ref, C[e, :m].float().cpu().numpy(), mag, f"fp8 block batch {e} {kernel} split {split_k}")
        assert torch.isnan(C[e, m:].float()).all(), "padding rows after a batch slice were written"


# ---- grouped (MoE) fp32 block-scale GEMM ----------------------------------------------

def run_fp8_block_grouped(bs, orc, cuda, sizes, n, k, *, seed, b_layout="kpanel", tail=0, max_rows=None,
                          out_dtype=torch.bfloat16, kernel="auto"):
    """Groups of `sizes` rows concatenated (then `tail` rows in no group); each
    group against its own weights through the oracle.  Returns the output."""
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    t_rows = int(offs[-1]) + tail
    qa, sa = orc.quant_fp8_block(orc.normal((t_rows, k), seed=seed), 1)
    qbs, sbs = zip(*[orc.quant_fp8_block(orc.normal((n, k), seed=seed * 31 + e + 1), 128) for e in range(len(sizes))])
    if b_layout == "kpanel":
        bh = np.stack([orc.shuffle_kpanel(qb) for qb in qbs])
    elif b_layout == "shuffle16":
        bh = np.stack([orc.shuffle_weight16(qb) for qb in qbs])
    else:
        bh = np.stack(qbs)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(bh, cuda).view(torch.float8_e4m3fn)
    SA = torch.from_numpy(sa).to(cuda)
    SB = torch.from_numpy(np.stack(sbs)).to(cuda)
    G = torch.from_numpy(offs).to(cuda)
    max_rows = max_rows or max(max(sizes), 1)
    out = poisoned((t_rows, n), out_dtype, cuda)
    bs.gemm_a8w8_blockscale_grouped(A, B, SA, SB, G, max_rows, out_dtype, out=out, b_layout=b_layout, kernel=kernel)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    got = out.float().cpu().numpy()
    for e, sz in enumerate(sizes):
        o0, done = int(offs[e]), min(sz, max_rows)
        if done:
            ref, mag = orc.gemm_fp8_block(qa[o0:o0 + done], qbs[e], sa[o0:o0 + done], sbs[e])
            assert_close(orc, ref, got[o0:o0 + done], mag, f"grouped e{e} rows {sz} {b_layout}")
        # rows of the group beyond max_rows are not computed
        assert np.isnan(got[o0 + done:o0 + sz]).all(), f"group {e} wrote past max_rows"
    assert np.isnan(got[int(offs[-1]):]).all(), "rows outside every group were written"
    return got


@pytest.mark.parametrize("sizes,n,k,b_layout,out_dtype", [
    ((0, 5, 130, 17, 256, 1), 384, 512, "kpanel", torch.bfloat16),
    ((64, 64, 3), 256, 1024, "raw", torch.float32),
    ((200, 0, 40), 512, 384, "shuffle16", torch.bfloat16),
    ((1,), 128, 128, "kpanel", torch.bfloat16),
])
def test_fp8_block_grouped(bs, orc, cuda, sizes, n, k, b_layout, out_dtype):
    """Ragged groups (empty, single-row, several 128-row tiles), each against
    its own weights, with rows after the last group left untouched."""
    run_fp8_block_grouped(bs, orc, cuda, sizes, n, k, seed=400 + n + k, b_layout=b_layout, tail=9,
                          out_dtype=out_dtype)


@pytest.mark.parametrize("sizes,n,k,b_layout,out_dtype", [
    ((0, 5, 300, 17, 512, 1), 384, 512, "kpanel", torch.bfloat16),
    ((256, 257, 3), 512, 1024, "raw", torch.float32),
    ((600, 0, 40), 768, 384, "shuffle16", torch.bfloat16),
])
def test_fp8_block_grouped_pair(bs, orc, cuda, sizes, n, k, b_layout, out_dtype):
    """Grouped calls on CTA pairs (256-row tiles): groups that end inside a pair tile (the peer
    CTA's rows wholly or partly in the next group), empty and single-row groups, N ending
    inside a column half; rows after the last group left untouched."""
    run_fp8_block_grouped(bs, orc, cuda, sizes, n, k, seed=450 + n + k, b_layout=b_layout, tail=9,
                          out_dtype=out_dtype, kernel="pair")


def test_fp8_block_grouped_pair_many_experts(bs, orc, cuda):
    """More groups than the pair kernel's tile prefix holds (1024): the full tile grid is
    decoded and tiles past each group's rows are skipped by every role."""
    sizes = [0] * 1100
    for e, sz in ((3, 5), (500, 300), (1023, 1), (1024, 64), (1099, 200)):
        sizes[e] = sz
    run_fp8_block_grouped(bs, orc, cuda, tuple(sizes), 128, 256, seed=78, b_layout="raw", tail=3, kernel="pair")


def test_fp8_block_grouped_pair_matches_1cta(bs, orc, cuda):
    """Grouped pair and grouped 1-CTA results agree bit for bit (same per-row arithmetic)."""
    a = run_fp8_block_grouped(bs, orc, cuda, (512, 300, 129), 512, 768, seed=79, kernel="pair")
    b = run_fp8_block_grouped(bs, orc, cuda, (512, 300, 129), 512, 768, seed=79, kernel="1cta")
    assert np.array_equal(a, b, equal_nan=True)


def test_fp8_block_grouped_many_experts(bs, orc, cuda):
    """More experts than the kernel's shared-memory tile prefix holds (1024):
    the grouped kernel falls back to decoding the full tile grid and skipping
    tiles past each expert's rows."""
    sizes = [0] * 1100
    for e, sz in ((3, 5), (500, 130), (1023, 1), (1024, 64), (1099, 200)):
        sizes[e] = sz
    run_fp8_block_grouped(bs, orc, cuda, tuple(sizes), 128, 256, seed=77, b_layout="raw", tail=3)


def test_fp8_block_grouped_caps_rows_at_max_rows(bs, orc, cuda):
    """A group longer than max_rows is computed up to max_rows rows only: the
    kernel clamps groups, so routing offsets beyond the bound never reach
    past the tile grid."""
    run_fp8_block_grouped(bs, orc, cuda, (300, 20), 256, 512, seed=5, max_rows=256)


def run_mx_grouped(bs, orc, cuda, sizes, n, k, *, fp4, seed, b_format="raw", b_scale_format="rowmajor",
                   tail=0, max_rows=None, out_dtype=torch.bfloat16, sf_mode="data"):
    """Grouped MXFP8 / MXFP4: groups of `sizes` rows concatenated (then `tail`
    rows in no group), each checked against its own weights through the oracle."""
    quant = orc.quant_mxfp4 if fp4 else orc.quant_mxfp8
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    t_rows = int(offs[-1]) + tail
    qa, sa = quant(orc.normal((t_rows, k), seed=seed))
    sa = scale_mode(sa, sf_mode)
    qbs, sbs = zip(*[quant(orc.normal((n, k), seed=seed * 31 + e + 1)) for e in range(len(sizes))])
    sbs = [scale_mode(sb, sf_mode) for sb in sbs]
    bh = np.stack([orc.shuffle_weight16(qb) for qb in qbs]) if b_format == "shuffle16" else np.stack(qbs)
    A, B = dev_u8(qa, cuda), dev_u8(bh, cuda)
    if not fp4:
        A, B = A.view(torch.float8_e4m3fn), B.view(torch.float8_e4m3fn)
    SA = dev_u8(sa, cuda)
    SB = dev_u8(np.stack(sbs), cuda)
    if b_scale_format == "native":
        SB = torch.stack([bs.pack_scales(SB[e]) for e in range(len(sizes))])
    G = torch.from_numpy(offs).to(cuda)
    max_rows = max_rows or max(max(sizes), 1)
    out = poisoned((t_rows, n), out_dtype, cuda)
    fn = bs.gemm_a4w4_mxfp4_grouped if fp4 else bs.gemm_a8w8_mxfp8_grouped
    fn(A, B, SA, SB, G, max_rows, out_dtype, out=out, b_format=b_format, b_scale_format=b_scale_format)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    got = out.float().cpu().numpy()
    for e, sz in enumerate(sizes):
        o0, done = int(offs[e]), min(sz, max_rows)
        if done:
            rows = slice(o0, o0 + done)
            ref, mag = (orc.gemm_mxfp4(qa[rows], qbs[e], sa[rows], sbs[e]) if fp4
                        else orc.gemm_mxfp8(qa[rows], qbs[e], sa[rows], sbs[e], f64=True))
            assert_close(orc, ref, got[rows], mag, f"mx grouped fp4={fp4} e{e} rows {sz} {b_format}")
        assert np.isnan(got[o0 + done:o0 + sz]).all(), f"group {e} wrote past max_rows"
    assert np.isnan(got[int(offs[-1]):]).all(), "rows outside every group were written"
    return got


@pytest.mark.parametrize("fp4,sizes,n,k,b_format,b_sf,out_dtype", [
    (False, (0, 5, 130, 17, 256, 1), 384, 512, "raw", "rowmajor", torch.bfloat16),
    (False, (64, 64, 3), 256, 1024, "shuffle16", "native", torch.float32),
    (False, (200, 0, 40), 272, 384, "raw", "native", torch.bfloat16),
    (True, (0, 7, 129, 33), 256, 1024, "raw", "rowmajor", torch.bfloat16),
    (True, (96, 1, 250), 384, 512, "shuffle16", "native", torch.float32),
])
def test_mx_grouped(bs, orc, cuda, fp4, sizes, n, k, b_format, b_sf, out_dtype):
    """Ragged groups (empty, single-row, several 128-row tiles, N not a
    multiple of the tile), each against its own weights, with rows after the
    last group left untouched; B raw or shuffle_weight(16,16), B scales
    row-major or native atoms per expert."""
    run_mx_grouped(bs, orc, cuda, sizes, n, k, fp4=fp4, seed=700 + n + k + fp4, b_format=b_format,
                   b_scale_format=b_sf, tail=9, out_dtype=out_dtype)


@pytest.mark.parametrize("fp4", [False, True])
def test_mx_grouped_scale_patterns_and_cap(bs, orc, cuda, fp4):
    """The reference's row-pattern scales (a wrong row-to-group scale mapping
    shows at once) and a group longer than max_rows, computed up to max_rows."""
    run_mx_grouped(bs, orc, cuda, (300, 20, 77), 256, 512, fp4=fp4, seed=9, max_rows=256,
                   sf_mode="rowpattern")


def test_mx_grouped_matches_dense(bs, orc, cuda):
    """A single group covering all rows equals the dense MXFP8 GEMM bit for bit."""
    x = orc.normal((200, 1024), seed=77)
    w = orc.normal((384, 1024), seed=78)
    qa, sa = orc.quant_mxfp8(x)
    qb, sb = orc.quant_mxfp8(w)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(qb, cuda).view(torch.float8_e4m3fn)
    SA, SB = dev_u8(sa, cuda), dev_u8(sb, cuda)
    dense = bs.gemm_a8w8_mxfp8(A, B, SA, SB, kernel="1cta", split_k=1)
    G = torch.tensor([0, 200], dtype=torch.int32, device=cuda)
    grouped = bs.gemm_a8w8_mxfp8_grouped(A, B[None], SA, SB[None], G, 200)
    torch.cuda.synchronize()
    assert torch.equal(dense, grouped)


@pytest.mark.parametrize("fp4,m,n,k,chunks,b_format,out_dtype,pinned", [
    (False, 700, 640, 512, 3, "raw", torch.bfloat16, True),
    (False, 128, 256, 256, 1, "raw", torch.float32, False),
    (True, 300, 512, 1024, 2, "shuffle16", torch.bfloat16, True),
    (True, 1100, 1280, 512, 0, "raw", torch.bfloat16, True),
])
def test_mx_host_staged(bs, orc, cuda, fp4, m, n, k, chunks, b_format, out_dtype, pinned):
    """Host-resident operands through the pipelined copy-in / GEMM blocks /
    copy-out entry point: ragged last chunks in both dimensions, pinned and
    pageable host memory, against the oracle; a host C with a wider row pitch
    keeps its padding untouched."""
    if fp4:
        qa, qb, sa, sb = mxfp4_problem(orc, m, n, k, 40 + m, "rowpattern")
        ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
    else:
        qa_l, qb_l, sa_l, sb_l = mxfp8_problem(orc, m, n, k, 40 + m, "rowpattern")
        qa, qb, sa, sb = qa_l[0], qb_l[0], sa_l[0], sb_l[0]
        ref, mag = orc.gemm_mxfp8(qa, qb, sa, sb, f64=True)
    bh = orc.shuffle_weight16(qb) if b_format == "shuffle16" else qb

    def host(x):
        t = torch.from_numpy(np.ascontiguousarray(x))
        return t.pin_memory() if pinned else t

    A, B, SA, SB = host(qa), host(bh), host(sa), host(sb)
    if not fp4:
        A, B = A.view(torch.float8_e4m3fn), B.view(torch.float8_e4m3fn)
    wide = torch.full((m, n + 8), float("nan"), dtype=out_dtype)
    out = wide[:, :n]
    with torch.cuda.device(cuda):
        got = bs.gemm_mx_from_host(A, B, SA, SB, fp4=fp4, out_dtype=out_dtype, out=out, b_format=b_format,
                                   chunks=chunks)
    assert bs.check_device_error() == 0
    assert got.data_ptr() == out.data_ptr()
    assert_close(orc, ref, got.float().numpy(), mag, f"host-staged fp4={fp4} {m}x{n}x{k} chunks={chunks}")
    assert torch.isnan(wide[:, n:]).all(), "the row padding of C was written"


@pytest.mark.parametrize("m,kernel", [(16, "swap"), (48, "swap"), (200, "1cta")])
def test_fp8_block_shuffle16_b(bs, orc, cuda, m, kernel):
    """aiter shuffle_weight(16,16) weights read in place by both kernels."""
    run_fp8_block(bs, orc, cuda, m, 768, 1024, seed=60 + m, kernel=kernel, shuffle16=True)


@pytest.mark.parametrize("grid_blocks", [3, 7, 0])
def test_fp8_block_swap_grid_caps_deterministic(bs, orc, cuda, grid_blocks):
    """Decode kernel under persistent-grid caps with auto split-K: correct,
    bit-identical from launch to launch, and within tolerance unsplit."""
    m, n, k = 24, 640, 2304
    x = orc.normal((m, k), seed=70)
    w = orc.normal((n, k), seed=71)
    qa, sa = orc.quant_fp8_block(x, 1)
    qb, sb = orc.quant_fp8_block(w, 128)
    ref, mag = orc.gemm_fp8_block(qa, qb, sa, sb)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(orc.shuffle_kpanel(qb), cuda).view(torch.float8_e4m3fn)
    SA, SB = torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda)
    outs = []
    for _ in range(2):
        out = poisoned((m, n), torch.bfloat16, cuda)
        bs.gemm_a8w8_bpreshuffle(A, B, SA, SB, torch.bfloat16, out=out, kernel="swap", grid_blocks=grid_blocks)
        outs.append(out)
    whole = bs.gemm_a8w8_bpreshuffle(A, B, SA, SB, torch.bfloat16, kernel="swap", split_k=1)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert torch.equal(outs[0], outs[1])
    assert_close(orc, ref, outs[0].float().cpu().numpy(), mag, f"grid cap {grid_blocks}")
    assert_close(orc, ref, whole.float().cpu().numpy(), mag, "whole tiles")


def test_fp8_block_split_k(bs, orc, cuda):
    run_fp8_block(bs, orc, cuda, 64, 512, 2048, seed=9, split_k=5)


# ---- packers -------------------------------------------------------------------------

def test_pack_b_roundtrips(bs, orc, cuda):
    rng = np.random.default_rng(3)
    b = rng.integers(0, 256, size=(256, 512), dtype=np.uint8)
    for fmt, shuffled in (("shuffle16", orc.shuffle_weight16(b)), ("kpanel", orc.shuffle_kpanel(b))):
        raw = bs.pack_b(dev_u8(shuffled, cuda), fmt)
        assert np.array_equal(raw.cpu().numpy(), b), fmt
        back = bs.pack_b(raw, fmt, unpack=True)
        assert np.array_equal(back.cpu().numpy().reshape(-1), shuffled.reshape(-1)), fmt


def test_pack_scales_matches_oracle(bs, orc, cuda):
    rng = np.random.default_rng(4)
    for rows, kg in ((256, 16), (200, 12), (40, 8), (1, 4)):
        sf = rng.integers(0, 256, size=(rows, kg), dtype=np.uint8)
        nat = bs.pack_scales(dev_u8(sf, cuda))
        assert np.array_equal(nat.cpu().numpy(), orc.sf_to_native(sf)), (rows, kg)
        assert np.array_equal(bs.unpack_scales(nat, rows, kg).cpu().numpy(), sf)
        esh = orc.e8m0_shuffle(sf)
        nat2 = bs.pack_scales(dev_u8(esh, cuda), rows, kg, src_format="e8m0_shuffle")
        assert np.array_equal(nat2.cpu().numpy(), orc.sf_to_native(sf))
        assert np.array_equal(bs.unpack_scales(nat, rows, kg, dst_format="e8m0_shuffle").cpu().numpy(), esh)


# ---- failure detection ---------------------------------------------------------------

def test_bounded_wait_reports_timeout(bs, cuda):
    """A wait on an mbarrier that nothing arrives at returns an error status
    after its limit; the context stays usable."""
    assert bs.selftest_timeout(2000) == bs.ERR_TIMEOUT
    assert bs.check_device_error() == 0
    x = torch.ones(4, device=cuda)
    assert float(x.sum()) == 4.0


# ---- full size (row sample) ----------------------------------------------------------

@pytest.mark.parametrize("layout,kernel", [("tn", "auto"), ("nt", "auto"), ("tn", "1cta")])
def test_mxfp8_8192_row_sample(bs, orc, cuda, layout, kernel):
    """MXFP8 8192^3 at full size: every output row is produced by the GPU;
    64 sampled rows are checked against the oracle."""
    m = n = k = 8192
    x = orc.normal((m, k), seed=81)
    w = orc.normal((n, k), seed=82)
    qa, sa = orc.quant_mxfp8(x)
    qb, sb = orc.quant_mxfp8(w)
    A = dev_u8(qa if layout[0] == "t" else np.ascontiguousarray(qa.T), cuda).view(torch.float8_e4m3fn)
    B = dev_u8(qb if layout[1] == "n" else np.ascontiguousarray(qb.T), cuda).view(torch.float8_e4m3fn)
    out = bs.gemm_a8w8_mxfp8(A, B, dev_u8(sa, cuda), dev_u8(sb, cuda), layout=layout, kernel=kernel)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    rows = np.random.default_rng(0).choice(m, 64, replace=False)
    rows.sort()
    ref, mag = orc.gemm_mxfp8(qa[rows], qb, sa[rows], sb, f64=True)
    got = out[torch.from_numpy(rows).to(cuda)].float().cpu().numpy()
    assert_close(orc, ref, got, mag, f"mxfp8 8192^3 {layout} sample")
    assert not torch.isnan(out).any()


def test_mxfp4_8192_row_sample(bs, orc, cuda):
    m = n = k = 8192
    qa, qb, sa, sb = mxfp4_problem(orc, m, n, k, 11)
    out = bs.gemm_a4w4_mxfp4(dev_u8(qa, cuda), dev_u8(qb, cuda), dev_u8(sa, cuda), dev_u8(sb, cuda))
    torch.cuda.synchronize()
    rows = np.random.default_rng(1).choice(m, 64, replace=False)
    rows.sort()
    ref, mag = orc.gemm_mxfp4(qa[rows], qb, sa[rows], sb)
    got = out[torch.from_numpy(rows).to(cuda)].float().cpu().numpy()
    assert_close(orc, ref, got, mag, "mxfp4 8192^3 sample")
    assert not torch.isnan(out).any()


def test_mxfp4_8192_shuffled_b_row_sample(bs, orc, cuda):
    """The benchmark configuration: MXFP4 8192^3 with B in shuffle_weight(16,16)
    read in place, native scales, CTA pairs."""
    m = n = k = 8192
    qa, qb, sa, sb = mxfp4_problem(orc, m, n, k, 12)
    SA = bs.pack_scales(dev_u8(sa, cuda))
    SB = bs.pack_scales(dev_u8(sb, cuda))
    out = bs.gemm_a4w4_mxfp4(dev_u8(qa, cuda), dev_u8(orc.shuffle_weight16(qb), cuda), SA, SB,
                             scale_format="native", b_format="shuffle16")
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    rows = np.random.default_rng(2).choice(m, 64, replace=False)
    rows.sort()
    ref, mag = orc.gemm_mxfp4(qa[rows], qb, sa[rows], sb)
    got = out[torch.from_numpy(rows).to(cuda)].float().cpu().numpy()
    assert_close(orc, ref, got, mag, "mxfp4 8192^3 shuffled sample")
    assert not torch.isnan(out).any()


def test_e8m0_block_8192_row_sample(bs, orc, cuda):
    """launch_blockscale_bpreshuffle at 8192^3 (CTA pairs, scale builders):
    64 sampled rows against the oracle under the reference's valid_vector rule."""
    m = n = k = 8192
    qa, qb, sfa_t, sfb = e8m0_block_problem(orc, m, n, k, 13)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(orc.shuffle_weight16(qb), cuda).view(torch.float8_e4m3fn)
    out = bs.gemm_a8w8_blockscale_bpreshuffle(A, B, dev_u8(sfa_t, cuda).t(), dev_u8(sfb, cuda))
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    rows = np.random.default_rng(3).choice(m, 64, replace=False)
    rows.sort()
    ref, mag = orc.gemm_e8m0_block(qa[rows], qb, np.ascontiguousarray(sfa_t[:, rows]), sfb)
    got = out[torch.from_numpy(rows).to(cuda)].float().cpu().numpy()
    errors, ratio = orc.check_e8m0_rule(ref, got, mag, bf16=True)
    assert errors == 0, f"{errors} errors, max ratio {ratio}"
    assert_close(orc, ref, got, mag, "e8m0 block 8192^3 sample")


def test_fp8_block_largest_sweep_shape_row_sample(bs, orc, cuda):
    """The largest fp32 block-scale sweep shape, M=8192 N=7168 K=18432, K-panel B:
    32 sampled rows against the oracle."""
    m, n, k = 8192, 7168, 18432
    x = orc.normal((m, k), seed=14)
    w = orc.normal((n, k), seed=15)
    qa, sa = orc.quant_fp8_block(x, 1)
    qb, sb = orc.quant_fp8_block(w, 128)
    A = dev_u8(qa, cuda).view(torch.float8_e4m3fn)
    B = dev_u8(orc.shuffle_kpanel(qb), cuda).view(torch.float8_e4m3fn)
    out = bs.gemm_a8w8_bpreshuffle(A, B, torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda))
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    rows = np.random.default_rng(4).choice(m, 32, replace=False)
    rows.sort()
    ref, mag = orc.gemm_fp8_block(qa[rows], qb, sa[rows], sb)
    got = out[torch.from_numpy(rows).to(cuda)].float().cpu().numpy()
    assert_close(orc, ref, got, mag, "fp8 block 8192x7168x18432 sample")
    assert not torch.isnan(out).any()


def test_fp8_block_decode_full_shape(bs, orc, cuda):
    """Decode at full size, M=16 N=7168 K=18432 (transposed kernel, auto split-K),
    every element checked."""
    run_fp8_block(bs, orc, cuda, 16, 7168, 18432, seed=16)


# ---- split-K inside CTA clusters (decode calls without a workspace) ---------------------

@pytest.mark.parametrize("m,n,k,split_k,out_dtype", [
    (16, 7168, 2048, 0, torch.bfloat16), (1, 4096, 7168, 3, torch.bfloat16), (30, 896, 1536, 2, torch.float32),
    (48, 1000, 1152, 4, torch.bfloat16), (64, 640, 640, 3, torch.bfloat16), (7, 24576, 1536, 2, torch.bfloat16)])
def test_fp8_block_cluster_split_without_workspace(bs, orc, cuda, m, n, k, split_k, out_dtype):
    """No workspace: the K slices of each output tile are summed inside a
    cluster of CTAs (distributed shared memory), in slice order."""
    qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=300 + m), 1)
    qb, sb = orc.quant_fp8_block(orc.normal((n if n % 128 == 0 else (n + 127) // 128 * 128, k), seed=301 + m), 128)
    qb, sb = qb[:n], sb
    ref, mag = orc.gemm_fp8_block(qa, qb, sa, sb)
    out = poisoned((m, n), out_dtype, cuda)
    bs.gemm_a8w8_bpreshuffle(dev_u8(qa, cuda).view(torch.float8_e4m3fn),
                             dev_u8(np.ascontiguousarray(qb), cuda).view(torch.float8_e4m3fn),
                             torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda), out_dtype, b_layout="raw",
                             out=out, split_k=split_k, kernel="swap", workspace=False)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert_close(orc, ref, out.float().cpu().numpy(), mag, f"fp8 block cluster split {m}x{n}x{k} s{split_k}")


def test_fp8_block_cluster_split_more_tiles_than_clusters(bs, orc, cuda):
    """Persistent clusters: a grid cap of 6 CTAs (3 clusters of 2) walks 56 tiles."""
    m, n, k = 16, 7168, 1024
    qa, sa = orc.quant_fp8_block(orc.normal((m, k), seed=310), 1)
    qb, sb = orc.quant_fp8_block(orc.normal((n, k), seed=311), 128)
    ref, mag = orc.gemm_fp8_block(qa, qb, sa, sb)
    out = bs.gemm_a8w8_bpreshuffle(dev_u8(qa, cuda).view(torch.float8_e4m3fn),
                                   dev_u8(orc.shuffle_kpanel(qb), cuda).view(torch.float8_e4m3fn),
                                   torch.from_numpy(sa).to(cuda), torch.from_numpy(sb).to(cuda), split_k=2,
                                   kernel="swap", workspace=False, grid_blocks=6)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert_close(orc, ref, out.float().cpu().numpy(), mag, "fp8 block cluster split, 3 clusters")


@pytest.mark.parametrize("fp4,m,split_k", [(False, 16, 0), (False, 40, 3), (True, 1, 2), (True, 64, 4)])
def test_mx_cluster_split_without_workspace(bs, orc, cuda, fp4, m, split_k):
    n, k = 2048, 4096
    if fp4:
        qa, qb, sa, sb = mxfp4_problem(orc, m, n, k, 320 + m, "kpattern")
        ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
        A, B = dev_u8(qa, cuda), dev_u8(qb, cuda)
        fn = bs.gemm_a4w4_mxfp4
    else:
        qa, qb, sa, sb = [x[0] for x in mxfp8_problem(orc, m, n, k, 320 + m, "kpattern")]
        ref, mag = orc.gemm_mxfp8(qa, qb, sa, sb, f64=True)
        A, B = dev_u8(qa, cuda).view(torch.float8_e4m3fn), dev_u8(qb, cuda).view(torch.float8_e4m3fn)
        fn = bs.gemm_a8w8_mxfp8
    SA, SB = bs.pack_scales(dev_u8(sa, cuda)), bs.pack_scales(dev_u8(sb, cuda))
    out = poisoned((m, n), torch.bfloat16, cuda)
    fn(A, B, SA, SB, out=out, scale_format="native", split_k=split_k, kernel="swap", workspace=False)
    torch.cuda.synchronize()
    assert bs.check_device_error() == 0
    assert_close(orc, ref, out.float().cpu().numpy(), mag, f"{'mxfp4' if fp4 else 'mxfp8'} cluster split m{m} s{split_k}")

"""Pin the oracle to the reference's own code.

oracle/oracle.c restates the reference's CPU verification GEMMs, codecs,
acceptance rules and byte layouts; oracle/_ref/libref.so is those same
functions compiled from the reference's sources (oracle/ref_extract.py cuts
them out of its host drivers by checked line ranges; oracle/ref_shim.h stands
in for HIP's fp8 type).  Every test here runs both on the same seeded inputs
and the committed golden fixtures and requires:
  - bit-equal results for the codecs, the byte layouts and the fp32
    sequential-accumulation GEMMs (MXFP8, fp32 block-scale);
  - bit-equal results for the fp64-accumulating GEMMs (MXFP4, E8M0 block),
    whose sum orders match;
  - the same accept / reject decisions and statistics for the acceptance rules.
Skipped only where neither a reference checkout nor a built libref.so exists.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ref as rlib

GOLDEN = Path(__file__).resolve().parent / "golden"

pytestmark = pytest.mark.skipif(not rlib.available(),
                                reason="no reference checkout and no prebuilt oracle/_ref/libref.so")


@pytest.fixture(scope="module")
def rf():
    return rlib


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32 if a.dtype == np.float32 else np.uint64)


def assert_bit_equal(x, y, what):
    x, y = np.ascontiguousarray(x), np.ascontiguousarray(y)
    assert x.shape == y.shape and x.dtype == y.dtype, what
    diff = bits(x) != bits(y)
    assert not diff.any(), f"{what}: {int(diff.sum())} of {x.size} elements differ"


# ---- codecs --------------------------------------------------------------------------

def test_shim_e4m3_decode_matches_torch(rf):
    codes = np.arange(256, dtype=np.uint8)
    ours = np.array([rf.lib().ref_e4m3_to_f32(int(v)) for v in codes], np.float32)
    want = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(ours), np.isnan(want))
    ok = ~np.isnan(want)
    assert_bit_equal(ours[ok], want[ok], "E4M3 decode")


def test_codecs_match_reference(rf, orc):
    L, R = orc.lib(), rf.lib()
    for e in range(256):
        a = np.float32(L.or_e8m0_to_f32(e))
        assert bits(np.array([a])) == bits(np.array([np.float32(R.ref_mxfp8_e8m0_to_f32(e))])), e
        assert bits(np.array([a])) == bits(np.array([np.float32(R.ref_snap_e8m0_to_f32(e))])), e
        assert np.float64(a) == R.ref_mxfp4_e8m0_to_f64(e) or (e == 255 and np.isinf(a))
    # E8M0 byte 0 decodes to 2^-127 and byte 255 to +inf on the reference host
    assert R.ref_mxfp8_e8m0_to_f32(0) == 2.0 ** -127 and np.isinf(R.ref_mxfp8_e8m0_to_f32(255))
    rng = np.random.default_rng(5)
    probes = np.concatenate([rng.standard_normal(4000).astype(np.float32) * 10.0 ** rng.integers(-40, 40, 4000),
                             np.ldexp(np.float32(1), np.arange(-150, 128)).astype(np.float32),
                             np.float32([0.0, -1.0, 3.0e38, 1e-45])])
    for v in probes:
        assert L.or_f32_to_e8m0(float(v)) == R.ref_mxfp8_f32_to_e8m0(float(v)), v
    for c in range(16):
        assert L.or_e2m1_to_f32(c) == R.ref_e2m1_to_f32(c), c
    u = rng.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32)
    u = np.concatenate([u, np.uint32([0x7F800000, 0xFF800000, 0x7FC00000, 0x7F800001, 0x00000001, 0x3F808000,
                                      0x3F818000, 0x3F80FFFF])])
    for b in u:
        f = float(np.uint32(b).view(np.float32))
        assert L.or_f32_to_bf16(f) == R.ref_f32_to_bf16_rne(f), hex(b)
    for x in range(0, 2 ** 16, 97):
        y, z = L.or_bf16_to_f32(x), R.ref_bf16_to_f32(x)
        assert (np.isnan(y) and np.isnan(z)) or y == z


def test_generator_matches_reference(rf, orc):
    rng = np.random.default_rng(6)
    for x in rng.integers(0, 2 ** 63, 2000, dtype=np.uint64):
        assert orc.lib().or_mix64(int(x)) == rf.lib().ref_mix_bits(int(x))
    # the reference's scale filler, restated from mix_bits: 124 + mix(seed + i) % 7
    n, seed = 4099, 77
    got = np.empty(n, np.uint8)
    rf.lib().ref_fill_scales(got, n, seed)
    want = np.array([124 + orc.lib().or_mix64(seed + i) % 7 for i in range(n)], np.uint8)
    assert np.array_equal(got, want)


# ---- GEMMs ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", ["mxfp8_64x64x256", "mxfp8_40x24x128"])
def test_gemm_mxfp8_bit_equal_on_golden(rf, orc, name):
    g = np.load(GOLDEN / f"{name}.npz")
    ours = orc.gemm_mxfp8(g["qa"], g["qb"], g["sa"], g["sb"])
    theirs = rf.gemm_mxfp8(g["qa"], g["qb"], g["sa"], g["sb"])
    assert_bit_equal(ours, theirs, name)
    # and the fixture's float64 matmul agrees with the reference to fp32 rounding
    np.testing.assert_allclose(theirs, g["c"], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("sf_mode", ["data", "kpattern", "rowpattern", "edges"])
def test_gemm_mxfp8_bit_equal_random(rf, orc, sf_mode):
    from helpers import mxfp8_problem
    qa, qb, sa, sb = [x[0] for x in mxfp8_problem(orc, 72, 56, 384, 91, "data" if sf_mode == "edges" else sf_mode)]
    if sf_mode == "edges":      # E8M0 bytes 0 and 255 and E4M3 NaN operands
        sa, sb, qa = sa.copy(), sb.copy(), qa.copy()
        sa[1, 0], sb[1, 0] = 0, 254
        sa[2, 3] = 255
        sa[3, 1], sb[3, 1] = 255, 0
        qa[4, 5], qa[5, 7] = 0x7F, 0xFF
    ours, theirs = orc.gemm_mxfp8(qa, qb, sa, sb), rf.gemm_mxfp8(qa, qb, sa, sb)
    same_nan = np.array_equal(np.isnan(ours), np.isnan(theirs))
    assert same_nan
    ok = ~np.isnan(ours)
    assert_bit_equal(ours[ok], theirs[ok], f"mxfp8 {sf_mode}")


def test_gemm_fp8_block_bit_equal(rf, orc):
    g = np.load(GOLDEN / "fp8block_48x128x256.npz")
    ours, _ = orc.gemm_fp8_block(g["qa"], g["qb"], g["sa"], g["sb"])
    theirs = rf.gemm_fp8_block(g["qa"], g["qb"], g["sa"], g["sb"])
    assert_bit_equal(ours, theirs, "fp8 block golden")
    qa, sa = orc.quant_fp8_block(orc.normal((40, 640), seed=92), 1)
    qb, sb = orc.quant_fp8_block(orc.normal((384, 640), seed=93), 128)
    ours, _ = orc.gemm_fp8_block(qa, qb, sa, sb)
    assert_bit_equal(ours, rf.gemm_fp8_block(qa, qb, sa, sb), "fp8 block random")


def test_gemm_mxfp4_bit_equal(rf, orc):
    g = np.load(GOLDEN / "mxfp4_64x64x256.npz")
    ours, _ = orc.gemm_mxfp4(g["qa"], g["qb"], g["sa"], g["sb"])
    assert_bit_equal(ours, rf.gemm_mxfp4(g["qa"], g["qb"], g["sa"], g["sb"]), "mxfp4 golden")
    from helpers import mxfp4_problem
    for mode in ("data", "kpattern", "rowpattern"):
        qa, qb, sa, sb = mxfp4_problem(orc, 48, 80, 512, 94, mode)
        ours, _ = orc.gemm_mxfp4(qa, qb, sa, sb)
        assert_bit_equal(ours, rf.gemm_mxfp4(qa, qb, sa, sb), f"mxfp4 {mode}")


def test_gemm_e8m0_block_bit_equal(rf, orc):
    m, n, k = 40, 256, 512
    qa, _ = orc.quant_mxfp8(orc.normal((m, k), seed=95))
    qb, _ = orc.quant_mxfp8(orc.normal((n, k), seed=96))
    rng = np.random.default_rng(7)
    sfa_t = rng.integers(120, 135, (k // 128, m)).astype(np.uint8)
    sfb = rng.integers(120, 135, (n // 128, k // 128)).astype(np.uint8)
    c0, m0 = orc.gemm_e8m0_block(qa, qb, sfa_t, sfb)
    c1, m1 = rf.gemm_e8m0_block(qa, qb, sfa_t, sfb)
    assert_bit_equal(c0, c1, "e8m0 block C")
    assert_bit_equal(m0, m1, "e8m0 block sum|term|")


# ---- layouts -------------------------------------------------------------------------

def test_layouts_bit_equal(rf, orc):
    g = np.load(GOLDEN / "layouts.npz")
    b = g["b"]
    assert np.array_equal(rf.shuffle_kpanel(b), orc.shuffle_kpanel(b))
    assert np.array_equal(rf.shuffle_kpanel(b), g["kp"])
    assert np.array_equal(rf.pack_weight_16x16(b), orc.shuffle_weight16(b))
    assert np.array_equal(rf.pack_weight_16x16(b), g["sh16"])
    assert np.array_equal(rf.m10_shuffle_b(b), orc.shuffle_weight16(b))   # packed fp4 [N, K/2] bytes
    assert np.array_equal(rf.m10_shuffle_b(b), g["sh_m10"])
    assert np.array_equal(rf.m10_e8m0_shuffle(g["sf"]), orc.e8m0_shuffle(g["sf"]))
    assert np.array_equal(rf.m10_e8m0_shuffle(g["sf"]), g["esh"])
    rng = np.random.default_rng(8)
    for rows, kg in ((1, 1), (33, 9), (96, 24), (130, 40)):
        sf = rng.integers(0, 256, (rows, kg)).astype(np.uint8)
        assert np.array_equal(rf.m10_e8m0_shuffle(sf), orc.e8m0_shuffle(sf)), (rows, kg)
    bb = rng.integers(0, 256, (48, 384)).astype(np.uint8)
    assert np.array_equal(rf.pack_weight_16x16(bb), orc.shuffle_weight16(bb))
    assert np.array_equal(rf.shuffle_kpanel(bb), orc.shuffle_kpanel(bb))


# ---- acceptance rules ----------------------------------------------------------------

@pytest.mark.parametrize("bf16", [True, False])
def test_valid_vector_decisions_match(rf, orc, bf16):
    m, n, k = 24, 256, 384
    qa, _ = orc.quant_mxfp8(orc.normal((m, k), seed=97))
    qb, _ = orc.quant_mxfp8(orc.normal((n, k), seed=98))
    rng = np.random.default_rng(9)
    sfa_t = rng.integers(124, 131, (k // 128, m)).astype(np.uint8)
    sfb = rng.integers(124, 131, (n // 128, k // 128)).astype(np.uint8)
    ref, mag = rf.gemm_e8m0_block(qa, qb, sfa_t, sfb)
    good = orc.bf16_round(ref) if bf16 else ref.copy()
    for planted in (0, 1, 7):
        got = good.copy()
        idx = rng.choice(got.size, planted, replace=False)
        got.flat[idx] += np.float32(0.5) + np.abs(got.flat[idx]) * np.float32(0.1)
        errors, _ = orc.check_e8m0_rule(ref, got, mag, bf16=bf16)
        got_arg = (got.view(np.uint32) >> 16).astype(np.uint16) if bf16 else got
        assert rf.valid_vector(ref, got_arg, mag, bf16) == (errors == 0)
        assert errors == planted


def test_calc_diff_matches_mxfp4_compare(rf, orc):
    from helpers import mxfp4_problem
    qa, qb, sa, sb = mxfp4_problem(orc, 32, 64, 256, 99)
    ref, mag = orc.gemm_mxfp4(qa, qb, sa, sb)
    got = orc.bf16_round(ref)
    _, _, cd_ours = orc.check_baseline_rule(ref.astype(np.float64), got, mag)
    errors, _, _, cd_ref = rf.mxfp4_compare(ref, got, mag.astype(np.float32), 5e-5, 1e-4, 2.0 ** -8)
    assert errors == 0
    assert abs(cd_ours - cd_ref) <= 1e-12

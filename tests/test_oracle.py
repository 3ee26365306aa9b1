"""Pin the CPU oracle (oracle/oracle.c) against independent implementations.

The reference has no golden vectors and its host code needs HIP, so the
oracle is pinned against (a) torch / ml_dtypes codecs, (b) the golden
fixtures of tests/golden/make_golden.py (numpy float64 GEMMs on operands
quantised with torch / ml_dtypes casts) and (c) the layout formulas the
reference's host drivers state.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / f"{name}.npz")


# ---- codecs ------------------------------------------------------------------

def test_e4m3_decode_matches_torch(orc):
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    mine = orc.e4m3_table()
    assert np.array_equal(np.isnan(t), np.isnan(mine))
    assert np.array_equal(t[~np.isnan(t)], mine[~np.isnan(mine)])
    g = load("codecs")["e4m3_table"]
    assert np.array_equal(g[~np.isnan(g)], mine[~np.isnan(mine)])


def test_e4m3_encode_matches_torch_rne(orc):
    g = load("codecs")
    lib = orc.lib()
    got = np.array([lib.or_f32_to_e4m3(float(v)) for v in g["probe"]], np.uint8)
    assert np.array_equal(got, g["probe_e4m3"])
    # saturation (satfinite) and NaN
    assert lib.or_f32_to_e4m3(1e6) == 0x7E and lib.or_f32_to_e4m3(-1e6) == 0xFE
    assert lib.or_f32_to_e4m3(float("nan")) == 0x7F


def test_e2m1_codec_matches_ml_dtypes(orc):
    g = load("codecs")
    assert np.array_equal(orc.e2m1_table(), g["e2m1_table"])
    lib = orc.lib()
    got = np.array([lib.or_f32_to_e2m1(float(v)) for v in g["probe4"]], np.uint8)
    assert np.array_equal(got, g["probe_e2m1"])


def test_e8m0_decode_matches_torch(orc):
    codes = np.arange(1, 255, dtype=np.uint8)
    t = torch.from_numpy(codes).view(torch.float8_e8m0fnu).float().numpy()
    assert np.array_equal(orc.e8m0_decode(codes), t)
    lib = orc.lib()
    # reference host ldexp semantics at the ends (mxfp8_gemm/..._host.cc:35-37)
    assert lib.or_e8m0_to_f32(255) == float("inf")
    assert lib.or_e8m0_to_f32(0) == 2.0 ** -127
    # nearest-power-of-two-below encoder (:39-47)
    assert lib.or_f32_to_e8m0(1.0) == 127 and lib.or_f32_to_e8m0(3.0) == 128
    assert lib.or_f32_to_e8m0(0.0) == 0


def test_bf16_rne_matches_torch(orc):
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 1e3,
                        np.float32([1.00390625, 1.01171875, -2.00781250, 3.4e38])])
    t = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(orc.bf16_round(x), t)
    lib = orc.lib()
    assert all(lib.or_f32_to_bf16(float(v)) == (orc.bf16_round(np.float32([v])).view(np.uint32)[0] >> 16)
               for v in x[:200])


# ---- quantisers ------------------------------------------------------------------

@pytest.mark.parametrize("name", ["mxfp8_64x64x256", "mxfp8_40x24x128"])
def test_quant_mxfp8_matches_golden(orc, name):
    g = load(name)
    qa, sa = orc.quant_mxfp8(g["x"])
    qb, sb = orc.quant_mxfp8(g["w"])
    assert np.array_equal(sa, g["sa"]) and np.array_equal(sb, g["sb"])
    assert np.array_equal(qa, g["qa"]) and np.array_equal(qb, g["qb"])


def test_quant_mxfp4_matches_golden(orc):
    g = load("mxfp4_64x64x256")
    qa, sa = orc.quant_mxfp4(g["x"])
    qb, sb = orc.quant_mxfp4(g["w"])
    assert np.array_equal(sa, g["sa"]) and np.array_equal(sb, g["sb"])
    assert np.array_equal(qa, g["qa"]) and np.array_equal(qb, g["qb"])


def test_quant_fp8_block_matches_golden(orc):
    g = load("fp8block_48x128x256")
    qa, sa = orc.quant_fp8_block(g["x"], 1)
    qb, sb = orc.quant_fp8_block(g["w"], 128)
    assert np.array_equal(sa, g["sa"]) and np.array_equal(sb, g["sb"])
    assert np.array_equal(qa, g["qa"]) and np.array_equal(qb, g["qb"])


def test_mx_scale_rule_bounds(orc):
    """scale = 2^ceil(log2(amax/448)): every scaled block has amax in (224, 448]."""
    x = orc.normal((64, 512), seed=7)
    q, sf = orc.quant_mxfp8(x)
    amax = np.abs(x.reshape(64, 16, 32)).max(axis=2)
    s = np.ldexp(1.0, sf.astype(np.int32) - 127)
    r = amax / s
    assert np.all(r <= 448.0) and np.all(r > 224.0)


def test_fill_normal_is_thread_count_independent(orc):
    a = orc.normal((1000,), seed=3)
    b = orc.normal((1000,), seed=3)
    c = orc.normal((1000,), seed=4)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert abs(float(a.mean())) < 0.15 and 0.85 < float(a.std()) < 1.15


# ---- reference GEMMs ------------------------------------------------------------------

@pytest.mark.parametrize("name", ["mxfp8_64x64x256", "mxfp8_40x24x128"])
def test_gemm_mxfp8_matches_golden(orc, name):
    g = load(name)
    c64, mag = orc.gemm_mxfp8(g["qa"], g["qb"], g["sa"], g["sb"], f64=True)
    np.testing.assert_allclose(c64, g["c"], rtol=1e-6, atol=1e-6)
    c32 = orc.gemm_mxfp8(g["qa"], g["qb"], g["sa"], g["sb"])
    # fp32 sequential accumulation (the reference's) stays within its 1e-3 rule scaled by magnitude
    assert np.all(np.abs(c32 - g["c"]) <= 1e-4 + 1e-6 * mag)


def test_gemm_mxfp4_matches_golden(orc):
    g = load("mxfp4_64x64x256")
    c, mag = orc.gemm_mxfp4(g["qa"], g["qb"], g["sa"], g["sb"])
    np.testing.assert_allclose(c, g["c"], rtol=1e-6, atol=1e-6)
    assert np.all(mag >= np.abs(c) - 1e-3)


def test_gemm_fp8_block_matches_golden(orc):
    g = load("fp8block_48x128x256")
    c, mag = orc.gemm_fp8_block(g["qa"], g["qb"], g["sa"], g["sb"])
    assert np.all(np.abs(c - g["c"]) <= 1e-4 + 1e-5 * mag)


def test_gemm_e8m0_block_consistent_with_mxfp8(orc):
    """E8M0 1x128 block-scale == MXFP8 with each 128-K scale broadcast to its
    four 32-groups (source_snapshot/..._scale_host.cc:219-248)."""
    rng = np.random.default_rng(5)
    m, n, k = 16, 256, 256
    a = orc.quant_mxfp8(rng.standard_normal((m, k)).astype(np.float32))[0]
    b = orc.quant_mxfp8(rng.standard_normal((n, k)).astype(np.float32))[0]
    sa_t = rng.integers(124, 131, size=(k // 128, m), dtype=np.uint8)
    sb = rng.integers(124, 131, size=(n // 128, k // 128), dtype=np.uint8)
    c, _ = orc.gemm_e8m0_block(a, b, sa_t, sb)
    sa32 = np.repeat(sa_t.T, 4, axis=1)
    sb32 = np.repeat(np.repeat(sb, 128, axis=0), 4, axis=1)
    c2, _ = orc.gemm_mxfp8(a, b, sa32, sb32, f64=True)
    np.testing.assert_allclose(c, c2, rtol=1e-6, atol=1e-6)


def test_k_pattern_scales_change_result(orc):
    """The reference's MXFP4_SFA_K_PATTERN trick (scale = 120 + g % 13) must
    change the product versus unit scales -- guards group mix-ups."""
    rng = np.random.default_rng(9)
    m = n = 32
    k = 256
    a = orc.quant_mxfp8(rng.standard_normal((m, k)).astype(np.float32))[0]
    b = orc.quant_mxfp8(rng.standard_normal((n, k)).astype(np.float32))[0]
    unit = np.full((m, k // 32), 127, np.uint8)
    pat = np.tile((120 + np.arange(k // 32) % 13).astype(np.uint8), (m, 1))
    cu = orc.gemm_mxfp8(a, b, unit, np.full((n, k // 32), 127, np.uint8))
    cp = orc.gemm_mxfp8(a, b, pat, np.full((n, k // 32), 127, np.uint8))
    assert not np.allclose(cu, cp)


# ---- layouts ---------------------------------------------------------------------------

def test_layouts_match_reference_formulas(orc):
    g = load("layouts")
    b = g["b"]
    n, kb = b.shape
    sh = orc.shuffle_weight16(b)
    assert np.array_equal(sh, g["sh16"])
    assert np.array_equal(sh, g["sh_m10"])       # the fp4 formula is the same permutation
    assert np.array_equal(orc.unshuffle_weight16(sh, n, kb), b)
    kp = orc.shuffle_kpanel(b)
    assert np.array_equal(kp, g["kp"])
    assert np.array_equal(orc.unshuffle_kpanel(kp, n, kb), b)
    sf = g["sf"]
    esh = orc.e8m0_shuffle(sf)
    assert np.array_equal(esh, g["esh"])
    assert np.array_equal(orc.e8m0_unshuffle(esh, *sf.shape), sf)


def test_native_scale_layout_is_a_permutation(orc):
    rng = np.random.default_rng(2)
    rows, kg = 200, 12
    sf = rng.integers(0, 256, size=(rows, kg), dtype=np.uint8)
    nat = orc.sf_to_native(sf)
    assert nat.size == ((rows + 127) // 128) * ((kg + 3) // 4) * 512
    # every (r, g) lands at its documented offset
    for r in range(0, rows, 7):
        for gi in range(kg):
            off = ((r // 128) * ((kg + 3) // 4) + gi // 4) * 512 + ((r % 32) * 4 + (r % 128) // 32) * 4 + gi % 4
            assert nat[off] == sf[r, gi]

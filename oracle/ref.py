"""ctypes front end of oracle/_ref/libref.so: the reference's own CPU
verification functions, compiled from its sources (oracle/ref_extract.py,
oracle/ref_adapters.cc, `make -C oracle ref`).

TEST INFRASTRUCTURE ONLY.  tests/test_ref_pin.py uses it to pin the
restatement in oracle/oracle.c to the reference's code, and bench.py's CPU
legs time its MXFP8 / MXFP4 / block-scale GEMMs as the reference's CPU GEMM
("kind": "reference").  The product never imports it.

The library is built only where a reference checkout exists (the directory in
$BSGEMM_REFERENCE, default the reference's checkout path); elsewhere an
already-built libref.so is used if present, and `available()` is False
otherwise.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from functools import lru_cache
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB = _HERE / "_ref" / "libref.so"
_SOURCES = ("ref_extract.py", "ref_adapters.cc", "ref_shim.h")
REFERENCE_ROOT = Path(os.environ.get("BSGEMM_REFERENCE", "/root/reference"))

_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_I = ctypes.c_int


def build() -> Path | None:
    """Compile oracle/_ref/libref.so when a reference checkout is present and
    the library is missing or older than its recipe; returns the library path,
    or None when there is neither a checkout nor a built library."""
    stale = not _LIB.exists() or _LIB.stat().st_mtime < max((_HERE / s).stat().st_mtime for s in _SOURCES)
    if stale and (REFERENCE_ROOT / "mxfp8_gemm").is_dir():
        subprocess.run(["make", "-s", "-C", str(_HERE), "ref", f"REFERENCE={REFERENCE_ROOT}"], check=True)
    return _LIB if _LIB.exists() else None


def available() -> bool:
    return build() is not None


@lru_cache(None)
def lib() -> ctypes.CDLL:
    if build() is None:
        raise RuntimeError("oracle/_ref/libref.so is not built and no reference checkout is present")
    so = ctypes.CDLL(str(_LIB))
    S = ctypes.c_size_t
    sig = {
        "ref_e4m3_to_f32": (ctypes.c_float, [ctypes.c_uint8]),
        "ref_f32_to_e4m3": (ctypes.c_uint8, [ctypes.c_float]),
        "ref_mxfp8_e8m0_to_f32": (ctypes.c_float, [ctypes.c_uint8]),
        "ref_mxfp8_f32_to_e8m0": (ctypes.c_uint8, [ctypes.c_float]),
        "ref_mxfp8_gemm": (None, [_u8p, _u8p, _u8p, _u8p, _f32p, _I, _I, _I, _I, _I, _I, _I, _I]),
        "ref_fp8b_gemm": (None, [_u8p, _u8p, _f32p, _f32p, _f32p, _I, _I, _I, _I, _I, _I, _I, _I]),
        "ref_fp8b_shuffle_b": (None, [_u8p, _u8p, _I, _I, _I, _I]),
        "ref_e2m1_to_f32": (ctypes.c_float, [ctypes.c_uint]),
        "ref_mxfp4_e8m0_to_f64": (ctypes.c_double, [ctypes.c_uint8]),
        "ref_mxfp4_gemm": (None, [_u8p, _u8p, _u8p, _u8p, _f32p, _I, _I, _I]),
        "ref_mxfp4_compare": (None, [_f32p, _f32p, ctypes.c_void_p, S, ctypes.c_float, ctypes.c_float,
                                     ctypes.c_double, _f64p]),
        "ref_mix_bits": (ctypes.c_uint64, [ctypes.c_uint64]),
        "ref_fill_scales": (None, [_u8p, S, ctypes.c_uint64]),
        "ref_pack_weight_16x16": (None, [_u8p, _u8p, _I, _I, _I]),
        "ref_snap_e8m0_to_f32": (ctypes.c_float, [ctypes.c_uint8]),
        "ref_f32_to_bf16_rne": (ctypes.c_uint16, [ctypes.c_float]),
        "ref_bf16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "ref_e8m0_block_gemm": (None, [_u8p, _u8p, _u8p, _u8p, _f32p, _f64p, _I, _I, _I]),
        "ref_valid_vector": (_I, [_f32p, ctypes.c_void_p, _f64p, S, _I]),
        "ref_m10_e8m0_shuffle": (None, [_u8p, _u8p, _I, _I, _I]),
        "ref_m10_shuffle_b": (None, [_u8p, _u8p, _I, _I, _I]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(so, name)
        fn.restype = res
        fn.argtypes = args
    return so


def _c(a, dtype=np.uint8):
    return np.ascontiguousarray(a, dtype=dtype)


def gemm_mxfp8(qa, qb, sa, sb):
    """mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:98-122: fp32 C [M,N] of dense K-major
    A [M,K], B [N,K] with E8M0 scales [M,K/32], [N,K/32]."""
    qa, qb, sa, sb = _c(qa), _c(qb), _c(sa), _c(sb)
    m, k = qa.shape
    n = qb.shape[0]
    c = np.empty((m, n), np.float32)
    lib().ref_mxfp8_gemm(qa, qb, sa, sb, c, m, n, k, k, k, n, sa.shape[1], sb.shape[1])
    return c


def gemm_fp8_block(qa, qb, sa, sb):
    """block_scale_gemm_bpreshuffle/..._host.cc:66-90: fp32 C of A [M,K], raw B
    [N,K], SFA fp32 [M,K/128] (passed to the reference transposed, as its
    kernel layout [K/128,M]) and SFB fp32 [N/128,K/128]."""
    qa, qb = _c(qa), _c(qb)
    m, k = qa.shape
    n = qb.shape[0]
    sfa_t = _c(np.asarray(sa, np.float32).T, np.float32)
    sb = _c(sb, np.float32)
    c = np.empty((m, n), np.float32)
    lib().ref_fp8b_gemm(qa, qb, sfa_t, sb, c, m, n, k, k, k, n, m, sb.shape[1])
    return c


def gemm_mxfp4(qa, qb, sa, sb):
    """mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:97-115: exact
    fp64 sum rounded to fp32; dense A [M,K/2], B [N,K/2] bytes."""
    qa, qb, sa, sb = _c(qa), _c(qb), _c(sa), _c(sb)
    m, n, k = qa.shape[0], qb.shape[0], qa.shape[1] * 2
    c = np.empty((m, n), np.float32)
    lib().ref_mxfp4_gemm(qa, qb, sa, sb, c, m, n, k)
    return c


def gemm_e8m0_block(qa, qb, sfa_t, sfb):
    """source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:221-248: (C, sum|term|)."""
    qa, qb, sfa_t, sfb = _c(qa), _c(qb), _c(sfa_t), _c(sfb)
    m, k = qa.shape
    n = qb.shape[0]
    c = np.empty((m, n), np.float32)
    mag = np.empty((m, n), np.float64)
    lib().ref_e8m0_block_gemm(qa, qb, sfa_t, sfb, c, mag, m, n, k)
    return c, mag


def shuffle_kpanel(b, block_k=128):
    b = _c(b)
    n, k = b.shape
    out = np.empty(n * k, np.uint8)
    lib().ref_fp8b_shuffle_b(b, out, 1, n, k, block_k)
    return out.reshape(k // block_k, n, block_k)


def pack_weight_16x16(b):
    b = _c(b)
    n, k = b.shape
    out = np.empty(n * k, np.uint8)
    lib().ref_pack_weight_16x16(b, out, 1, n, k)
    return out.reshape(n, k)


def m10_shuffle_b(b_fp4):
    b = _c(b_fp4)
    n, kb = b.shape
    out = np.empty(n * kb, np.uint8)
    lib().ref_m10_shuffle_b(b, out, 1, n, kb * 2)
    return out.reshape(n, kb)


def m10_e8m0_shuffle(sf):
    sf = _c(sf)
    rows, kg = sf.shape
    out = np.empty(((rows + 31) // 32 * 32) * ((kg + 7) // 8 * 8), np.uint8)
    lib().ref_m10_e8m0_shuffle(sf, out, rows, 1, kg)
    return out


def valid_vector(ref, got, mag, bf16: bool) -> bool:
    """The reference's acceptance rule (source_snapshot/..._host.cc:250-291).
    got: bf16 bit patterns (uint16) when bf16, else float32."""
    ref, mag = _c(ref, np.float32).ravel(), _c(mag, np.float64).ravel()
    got = _c(got, np.uint16 if bf16 else np.float32).ravel()
    return bool(lib().ref_valid_vector(ref, got.ctypes.data, mag, ref.size, int(bf16)))


def mxfp4_compare(ref, got, mag=None, rel_mag=5e-5, abs_floor=1e-4, out_rel=0.0):
    """mxfp4 host's compare (gemm_a4w4_mxfp4_4wave_host.cc:117-144):
    (errors, max_diff, max_ratio, calc_diff)."""
    ref, got = _c(ref, np.float32).ravel(), _c(got, np.float32).ravel()
    mag_arr = None if mag is None else _c(mag, np.float32).ravel()
    out = np.empty(4, np.float64)
    lib().ref_mxfp4_compare(ref, got, None if mag_arr is None else mag_arr.ctypes.data, ref.size,
                            rel_mag, abs_floor, out_rel, out)
    return int(out[0]), float(out[1]), float(out[2]), float(out[3])


def num_threads() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))

"""ctypes/numpy front end of the CPU oracle (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() (as the
checker) and bench.py's cpu_baseline / ``--impl reference`` legs.  The product
package never imports this module and never falls back to it.

Each wrapper names the reference file:line its C function restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from functools import lru_cache
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB = _HERE / "_build" / "liboracle.so"

_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_L = ctypes.c_long
_I = ctypes.c_int


def build() -> Path:
    """Compile oracle/_build/liboracle.so with gcc -O3 -fopenmp (idempotent)."""
    src = _HERE / "oracle.c"
    if not _LIB.exists() or _LIB.stat().st_mtime < max(src.stat().st_mtime,
                                                      (_HERE / "oracle.h").stat().st_mtime):
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB


@lru_cache(None)
def lib() -> ctypes.CDLL:
    build()
    so = ctypes.CDLL(str(_LIB))
    sig = {
        "or_e4m3_to_f32": (ctypes.c_float, [ctypes.c_uint8]),
        "or_f32_to_e4m3": (ctypes.c_uint8, [ctypes.c_float]),
        "or_e2m1_to_f32": (ctypes.c_float, [ctypes.c_uint8]),
        "or_f32_to_e2m1": (ctypes.c_uint8, [ctypes.c_float]),
        "or_e8m0_to_f32": (ctypes.c_float, [ctypes.c_uint8]),
        "or_f32_to_e8m0": (ctypes.c_uint8, [ctypes.c_float]),
        "or_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
        "or_bf16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "or_mix64": (ctypes.c_uint64, [ctypes.c_uint64]),
        "or_fill_normal": (None, [_f32p, ctypes.c_size_t, ctypes.c_uint64]),
        "or_quant_mxfp8": (None, [_f32p, _I, _I, _L, _u8p, _u8p]),
        "or_quant_mxfp4": (None, [_f32p, _I, _I, _L, _u8p, _u8p]),
        "or_quant_fp8_block": (None, [_f32p, _I, _I, _L, _I, _u8p, _f32p]),
        "or_gemm_mxfp8": (None, [_u8p, _u8p, _u8p, _u8p, _f32p, _I, _I, _I, _L, _L, _L, _L, _L]),
        "or_gemm_mxfp8_f64": (None, [_u8p, _u8p, _u8p, _u8p, _f32p, _f64p, _I, _I, _I,
                                     _L, _L, _L, _L, _L]),
        "or_gemm_mxfp4": (None, [_u8p, _u8p, _u8p, _u8p, _f32p, _f64p, _I, _I, _I,
                                 _L, _L, _L, _L, _L]),
        "or_gemm_fp8_block": (None, [_u8p, _u8p, _f32p, _f32p, _f32p, _f64p, _I, _I, _I,
                                     _L, _L, _L, _L, _L, _L, _L]),
        "or_gemm_e8m0_block": (None, [_u8p, _u8p, _u8p, _u8p, _f32p, _f64p, _I, _I, _I]),
        "or_shuffle_kpanel": (None, [_u8p, _u8p, _I, _I, _I]),
        "or_unshuffle_kpanel": (None, [_u8p, _u8p, _I, _I, _I]),
        "or_shuffle_weight16": (None, [_u8p, _u8p, _I, _I]),
        "or_unshuffle_weight16": (None, [_u8p, _u8p, _I, _I]),
        "or_e8m0_shuffle_size": (ctypes.c_size_t, [_I, _I]),
        "or_e8m0_shuffle": (None, [_u8p, _u8p, _I, _I]),
        "or_e8m0_unshuffle": (None, [_u8p, _u8p, _I, _I]),
        "or_sf_native_size": (ctypes.c_size_t, [_I, _I]),
        "or_sf_to_native": (None, [_u8p, _L, _u8p, _I, _I]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(so, name)
        fn.restype = res
        fn.argtypes = args
    return so


# ---- codecs (vectorised through 256/16-entry tables) -----------------------

@lru_cache(None)
def e4m3_table() -> np.ndarray:
    return np.array([lib().or_e4m3_to_f32(v) for v in range(256)], dtype=np.float32)


@lru_cache(None)
def e2m1_table() -> np.ndarray:
    return np.array([lib().or_e2m1_to_f32(v) for v in range(16)], dtype=np.float32)


def e4m3_decode(q: np.ndarray) -> np.ndarray:
    return e4m3_table()[q]


def e8m0_decode(s: np.ndarray) -> np.ndarray:
    return np.ldexp(np.float32(1.0), s.astype(np.int32) - 127).astype(np.float32)


def e2m1_unpack(q: np.ndarray) -> np.ndarray:
    """[rows, k/2] packed bytes -> [rows, k] float32 (even k = low nibble)."""
    t = e2m1_table()
    out = np.empty(q.shape[:-1] + (q.shape[-1] * 2,), dtype=np.float32)
    out[..., 0::2] = t[q & 15]
    out[..., 1::2] = t[q >> 4]
    return out


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 RNE -> fp32 (source_snapshot/...scale_host.cc:185-204)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, (b >> 16) | 0x40, r).astype(np.uint32)
    return (r << 16).view(np.float32).reshape(np.shape(x))


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---- seeded inputs + quantisers ---------------------------------------------

def normal(shape, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    lib().or_fill_normal(out, n, seed)
    return out.reshape(shape)


def quant_mxfp8(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    q = np.zeros((rows, k), np.uint8)
    sf = np.zeros((rows, k // 32), np.uint8)
    lib().or_quant_mxfp8(x, rows, k, k, q, sf)
    return q, sf


def quant_mxfp4(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    q = np.zeros((rows, k // 2), np.uint8)
    sf = np.zeros((rows, k // 32), np.uint8)
    lib().or_quant_mxfp4(x, rows, k, k, q, sf)
    return q, sf


def quant_fp8_block(x: np.ndarray, block_rows: int):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    q = np.zeros((rows, k), np.uint8)
    sf = np.zeros(((rows + block_rows - 1) // block_rows, k // 128), np.float32)
    lib().or_quant_fp8_block(x, rows, k, k, block_rows, q, sf)
    return q, sf


# ---- reference GEMMs -----------------------------------------------------------

def gemm_mxfp8(a, b, sfa, sfb, f64: bool = False):
    """a [m,k] u8, b [n,k] u8, sfa [m,k/32], sfb [n,k/32] -> fp32 [m,n] (+mag)."""
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    sfa, sfb = np.ascontiguousarray(sfa), np.ascontiguousarray(sfb)
    m, k = a.shape
    n = b.shape[0]
    c = np.zeros((m, n), np.float32)
    if not f64:
        lib().or_gemm_mxfp8(a, b, sfa, sfb, c, m, n, k, k, k, n, sfa.shape[1], sfb.shape[1])
        return c
    mag = np.zeros((m, n), np.float64)
    lib().or_gemm_mxfp8_f64(a, b, sfa, sfb, c, mag, m, n, k, k, k, n, sfa.shape[1], sfb.shape[1])
    return c, mag


def gemm_mxfp4(a, b, sfa, sfb):
    """a [m,k/2], b [n,k/2] packed bytes -> (fp32 [m,n], mag)."""
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    sfa, sfb = np.ascontiguousarray(sfa), np.ascontiguousarray(sfb)
    m, kh = a.shape
    n = b.shape[0]
    c = np.zeros((m, n), np.float32)
    mag = np.zeros((m, n), np.float64)
    lib().or_gemm_mxfp4(a, b, sfa, sfb, c, mag, m, n, 2 * kh, kh, kh, n, sfa.shape[1], sfb.shape[1])
    return c, mag


def gemm_fp8_block(a, b, sfa, sfb):
    """a [m,k], b [n,k] E4M3 bytes; sfa fp32 [m,k/128]; sfb fp32 [n/128,k/128]."""
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    sfa = np.ascontiguousarray(sfa, dtype=np.float32)
    sfb = np.ascontiguousarray(sfb, dtype=np.float32)
    m, k = a.shape
    n = b.shape[0]
    c = np.zeros((m, n), np.float32)
    mag = np.zeros((m, n), np.float64)
    lib().or_gemm_fp8_block(a, b, sfa, sfb, c, mag, m, n, k, k, k, n,
                            sfa.shape[1], 1, sfb.shape[1], 1)
    return c, mag


def gemm_e8m0_block(a, b, sfa_t, sfb):
    """E8M0 1x128 / 128x128: sfa_t [k/128, m] bytes, sfb [n/128, k/128] bytes."""
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    m, k = a.shape
    n = b.shape[0]
    c = np.zeros((m, n), np.float32)
    mag = np.zeros((m, n), np.float64)
    lib().or_gemm_e8m0_block(a, b, np.ascontiguousarray(sfa_t), np.ascontiguousarray(sfb),
                             c, mag, m, n, k)
    return c, mag


# ---- layouts ---------------------------------------------------------------------

def shuffle_kpanel(b, block_k: int = 128):
    b = np.ascontiguousarray(b)
    n, k = b.shape
    out = np.empty(n * k, np.uint8)
    lib().or_shuffle_kpanel(b, out, n, k, block_k)
    return out.reshape(k // block_k, n, block_k)


def unshuffle_kpanel(bp, n: int, k: int, block_k: int = 128):
    out = np.empty((n, k), np.uint8)
    lib().or_unshuffle_kpanel(np.ascontiguousarray(bp).reshape(-1), out, n, k, block_k)
    return out


def shuffle_weight16(b):
    b = np.ascontiguousarray(b)
    n, kb = b.shape
    out = np.empty(n * kb, np.uint8)
    lib().or_shuffle_weight16(b, out, n, kb)
    return out.reshape(n, kb)


def unshuffle_weight16(bs, n: int, kbytes: int):
    out = np.empty((n, kbytes), np.uint8)
    lib().or_unshuffle_weight16(np.ascontiguousarray(bs).reshape(-1), out, n, kbytes)
    return out


def e8m0_shuffle(sf):
    sf = np.ascontiguousarray(sf)
    rows, kg = sf.shape
    out = np.empty(lib().or_e8m0_shuffle_size(rows, kg), np.uint8)
    lib().or_e8m0_shuffle(sf, out, rows, kg)
    return out


def e8m0_unshuffle(buf, rows: int, kg: int):
    out = np.empty((rows, kg), np.uint8)
    lib().or_e8m0_unshuffle(np.ascontiguousarray(buf), out, rows, kg)
    return out


def sf_to_native(sf):
    sf = np.ascontiguousarray(sf)
    rows, kg = sf.shape
    out = np.empty(lib().or_sf_native_size(rows, kg), np.uint8)
    lib().or_sf_to_native(sf, kg, out, rows, kg)
    return out


# ---- E8M0 edge bytes: the library's semantics ------------------------------------

def as_library_e8m0(ref: np.ndarray, nan_rows=(), nan_cols=()) -> np.ndarray:
    """Map a reference-host result onto what the block-scaled tensor cores
    produce for the two E8M0 edge bytes and for NaN operands.

    The reference host decodes a scale byte with ldexp(1, e - 127): byte 0 is
    2^-127, and byte 255 is 2^128 -- +inf in fp32
    (mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:35-37), a finite double in the MXFP4
    driver (mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:44).
    tcgen05's block-scaled MMA follows the OCP MX encoding: byte 0 is also
    2^-127, but byte 255 is NaN, so every output of a row whose activation
    scales hold a 255 byte, or of a column whose weight scales do, is NaN; an
    E4M3 NaN operand (0x7F / 0xFF) makes its output row or column NaN on both.
    (The reference's own device decode,
    mxfp8_gemm/gemm_a8w8_mxfp8_kernel_template.hpp:23-25, reads byte 0 as 0.0
    and 255 as +inf; neither is what this library does.)  All other outputs
    are the reference's values.  nan_rows / nan_cols: the rows and columns
    such a byte or operand reaches."""
    out = np.array(ref, dtype=np.float64, copy=True)
    out[np.asarray(nan_rows, dtype=np.int64), :] = np.nan
    out[:, np.asarray(nan_cols, dtype=np.int64)] = np.nan
    return out


def e4m3_nan_rows(q: np.ndarray) -> np.ndarray:
    """Rows of an E4M3 byte matrix holding a NaN code (0x7F or 0xFF)."""
    return np.where(((q & 0x7F) == 0x7F).any(axis=1))[0]


# ---- reference acceptance rules ---------------------------------------------------

def check_e8m0_rule(ref: np.ndarray, got: np.ndarray, mag: np.ndarray, bf16: bool,
                    rel_mag: float = 5e-5, abs_floor: float = 1e-4):
    """valid_vector of source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:250-291:
    |got - ref| within abs_floor + rel_mag*sum|term|, bounds RNE-rounded to bf16
    for bf16 output.  Returns (errors, max_ratio)."""
    ref = ref.astype(np.float32)
    tol = abs_floor + rel_mag * mag
    if bf16:
        expected = bf16_round(ref)
        lo = bf16_round((ref - tol).astype(np.float32)).astype(np.float64)
        hi = bf16_round((ref + tol).astype(np.float32)).astype(np.float64)
    else:
        expected = ref
        lo, hi = ref - tol, ref + tol
    got64 = got.astype(np.float64)
    bad = ~np.isfinite(got64) | (got64 < lo) | (got64 > hi)
    width = np.maximum(expected - lo, hi - expected)
    diff = np.abs(got64 - expected)
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = np.where(width > 0, diff / width, np.where(diff == 0, 0.0, np.inf))
    return int(bad.sum()), float(np.max(ratio)) if ratio.size else 0.0


def check_baseline_rule(ref: np.ndarray, got: np.ndarray, mag: np.ndarray | None = None,
                        mag_floor: float = 1e-6):
    """Target tolerance on bf16 outputs, per element
        |err| <= 2^-7*|ref| + 1e-3 + mag_floor * sum|term|.
    The last term is the fp32-accumulation floor: where the terms cancel
    (|ref| << sum|term|) no fp32 computation can meet a bound relative to |ref|;
    1e-6 * sum|term| is ~17 fp32 ulps of the term magnitude (the reference's own
    rule, source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:250-291, allows
    5e-5 * sum|term|).  max_rel is taken over the elements that are not
    cancellation-dominated (|ref| >= 1e-2 * sum|term|; |ref| > 1e-2 when mag is
    None).  Also returns the mxfp4 host's calc_diff = 1 - 2*sum(xy)/sum(x^2+y^2)
    (mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:119-144).
    Returns (bad_count, max_rel, calc_diff)."""
    r = ref.astype(np.float64)
    g = got.astype(np.float64)
    err = np.abs(g - r)
    floor = 0.0 if mag is None else mag_floor * mag
    bad = ~np.isfinite(g) | (err > (2.0 ** -7) * np.abs(r) + 1e-3 + floor)
    big = (np.abs(r) > 1e-2) if mag is None else (np.abs(r) >= 1e-2 * mag) & (np.abs(r) > 1e-2)
    max_rel = float(np.max(err[big] / np.abs(r[big]))) if big.any() else 0.0
    xx_yy = float(np.sum(r * r + g * g))
    calc_diff = 1.0 - 2.0 * float(np.sum(r * g)) / xx_yy if xx_yy > 0 else 0.0
    return int(bad.sum()), max_rel, calc_diff


def num_threads() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))

/*
 * oracle.h -- CPU restatement of the reference's host-side verification code
 * for the block-scaled GEMM path.  TEST INFRASTRUCTURE ONLY: nothing in the
 * product library links, loads or calls this code.  It is used by tests/,
 * __graft_entry__.smoke() and the cpu_baseline / --impl reference legs of
 * bench.py, always as the checker or the timed CPU baseline, never as the
 * measured GPU path.
 *
 * Every function names the reference file:line it restates (paths relative to
 * the reference project root).  The reference sources cannot be compiled here
 * (they include <hip/hip_fp8.h> and <opus/opus.hpp>), so this file is an
 * independent restatement, pinned by tests/test_oracle.py against torch's CPU
 * float8_e4m3fn / float4_e2m1fn_x2 / float8_e8m0fnu codecs and against the
 * golden fixtures under tests/golden/.
 */
#ifndef BSGEMM_ORACLE_H
#define BSGEMM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element codecs ---------------------------------------------------- */

/* OCP E4M3FN decode: bias 7, no infinities, 0x7F/0xFF are NaN, max 448.
 * Restates the __hip_fp8_e4m3 -> float conversion used by every reference
 * CPU GEMM (e.g. mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:115). */
float or_e4m3_to_f32(uint8_t v);
/* float -> E4M3FN, round-to-nearest-even, saturating to +-448 (satfinite);
 * NaN -> 0x7F.  Inputs produced by the quantisers never exceed 448. */
uint8_t or_f32_to_e4m3(float x);

/* E2M1 decode {0,.5,1,1.5,2,3,4,6} with sign bit 3.
 * mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:38-42 */
float or_e2m1_to_f32(uint8_t code);
/* float -> E2M1 code, round-to-nearest-even, saturating to +-6. */
uint8_t or_f32_to_e2m1(float x);

/* E8M0 decode as the reference host does it: ldexp(1, e - 127)
 * (mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:35-37; e = 255 gives +inf, e = 0 gives
 * 2^-127). */
float or_e8m0_to_f32(uint8_t e);
/* Nearest-power-of-two encoder of the reference
 * (mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:39-47). */
uint8_t or_f32_to_e8m0(float v);

/* fp32 -> bf16 round-to-nearest-even, NaN quieted.
 * trace_block_scale_latest_20260914_040021/source_snapshot/
 * gemm_a8w8_mxfp8_scale_host.cc:185-193 */
uint16_t or_f32_to_bf16(float x);
float or_bf16_to_f32(uint16_t b);

/* ---- seeded synthetic inputs --------------------------------------------
 * Counter-based splitmix64 (source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:
 * 139-159), so results do not depend on the OpenMP thread count; Box-Muller
 * turns two 24-bit uniforms into one N(0,1) sample. */
uint64_t or_mix64(uint64_t x);
void or_fill_normal(float *out, size_t n, uint64_t seed);

/* ---- quantisers (benchmark input recipes) --------------------------------
 * MX (1x32): per row, per 32-K group: scale = 2^ceil(log2(amax / qmax)),
 * elements = RNE(x / scale).  qmax = 448 (E4M3) or 6 (E2M1).  Zero groups get
 * scale byte 127.  x is [rows, k] with row stride ldx; q is [rows, k] bytes
 * (fp8) or [rows, k/2] bytes (fp4, even k in the low nibble); sf is
 * [rows, k/32] bytes. */
void or_quant_mxfp8(const float *x, int rows, int k, long ldx, uint8_t *q, uint8_t *sf);
void or_quant_mxfp4(const float *x, int rows, int k, long ldx, uint8_t *q, uint8_t *sf);
/* fp32 block scales, DeepSeek style: s = amax / 448 per block of br rows x 128
 * K (br = 1 for activations, 128 for weights); q = RNE(x / s).  sf is
 * [ceil(rows/br), k/128] fp32 row-major. */
void or_quant_fp8_block(const float *x, int rows, int k, long ldx, int br,
                        uint8_t *q, float *sf);

/* ---- reference CPU GEMMs ------------------------------------------------ */

/* MXFP8 C[m,n] fp32 = sum_g sa*sb * sum_{k in g} a*b, fp32 sequential
 * accumulation of a*b*scale, exactly as
 * mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:98-122.  A [m,k] K-major (lda), B [n,k]
 * K-major (ldb), SFA [m,k/32] (stride_sfa), SFB [n,k/32] (stride_sfb). */
void or_gemm_mxfp8(const uint8_t *a, const uint8_t *b, const uint8_t *sfa,
                   const uint8_t *sfb, float *c, int m, int n, int k, long lda,
                   long ldb, long ldc, long stride_sfa, long stride_sfb);

/* Same contraction with double accumulation; also returns sum|term| per
 * element (mag), the reference's tolerance basis
 * (source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:219-248, with 1x32 groups). */
void or_gemm_mxfp8_f64(const uint8_t *a, const uint8_t *b, const uint8_t *sfa,
                       const uint8_t *sfb, float *c, double *mag, int m, int n,
                       int k, long lda, long ldb, long ldc, long stride_sfa,
                       long stride_sfb);

/* MXFP4: exact double sum of e2m1(a)*e2m1(b)*2^(sa-127)*2^(sb-127).
 * mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:97-115; mag as in
 * :69-94.  A [m,k/2] bytes (lda bytes), B [n,k/2] bytes. */
void or_gemm_mxfp4(const uint8_t *a, const uint8_t *b, const uint8_t *sfa,
                   const uint8_t *sfb, float *c, double *mag, int m, int n,
                   int k, long lda, long ldb, long ldc, long stride_sfa,
                   long stride_sfb);

/* fp32 block-scale GEMM: sum += a*b*(sa*sb) in fp32, scale_a =
 * sfa[m*sfa_m + kb*sfa_k], scale_b = sfb[(n/128)*sfb_n + kb*sfb_k]
 * (block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_host.cc:
 * 66-90; its transposed SFA is sfa_m = 1, sfa_k = M).  Optionally mag. */
void or_gemm_fp8_block(const uint8_t *a, const uint8_t *b, const float *sfa,
                       const float *sfb, float *c, double *mag, int m, int n,
                       int k, long lda, long ldb, long ldc, long sfa_m,
                       long sfa_k, long sfb_n, long sfb_k);

/* E8M0 1x128 / 128x128 block-scale GEMM, double accumulation + mag.
 * source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:219-248: SFA bytes at
 * [kb*m_total + row], SFB bytes at [(n/128)*(k/128) + kb]. */
void or_gemm_e8m0_block(const uint8_t *a, const uint8_t *b, const uint8_t *sfa,
                        const uint8_t *sfb, float *c, double *mag, int m, int n,
                        int k);

/* ---- reference layouts (byte permutations) ------------------------------ */

/* K-panel preshuffle B'[kt][n][128] = B[n][kt*128 + ki].
 * block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_host.cc:96-111 */
void or_shuffle_kpanel(const uint8_t *src, uint8_t *dst, int n, int k, int block_k);
void or_unshuffle_kpanel(const uint8_t *src, uint8_t *dst, int n, int k, int block_k);

/* shuffle_weight(layout=(16,16)) over a byte matrix [n, kb] (kb = K bytes):
 * [n/16][kb/16][16][16] (source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:
 * 161-179).  For packed fp4 this equals the candidate_m10 formula
 * (n/16)*16*Kb + (kb/32)*512 + ((kb/16)%2)*256 + (n%16)*16 + kb%16
 * (mxfp4_gemm_4wave_20261112/candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:
 * 215-225) -- both are the same permutation. */
void or_shuffle_weight16(const uint8_t *src, uint8_t *dst, int n, int kbytes);
void or_unshuffle_weight16(const uint8_t *src, uint8_t *dst, int n, int kbytes);

/* aiter e8m0_shuffle of a [rows, kg] scale matrix: rows padded to 32, kg to 8
 * with 0x7F; offset (r/32*(kg8/8) + g/8)*256 + (g%4)*64 + (r%16)*4 +
 * ((g%8)/4)*2 + (r%32)/16.
 * candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:194-206 */
size_t or_e8m0_shuffle_size(int rows, int kg);
void or_e8m0_shuffle(const uint8_t *src, uint8_t *dst, int rows, int kg);
void or_e8m0_unshuffle(const uint8_t *src, uint8_t *dst, int rows, int kg);

/* This library's native (tcgen05 scale-factor) layout of a [rows, kg] E8M0
 * matrix, restated independently of the CUDA pack kernels so tests can check
 * them: atoms of 128 rows x 4 groups (512 bytes), atom (rb, kb) at
 * (rb*ceil(kg/4) + kb)*512, byte ((r%32)*4 + (r%128)/32)*4 + g%4; padding
 * 0x7F.  Not a reference layout. */
size_t or_sf_native_size(int rows, int kg);
void or_sf_to_native(const uint8_t *src, long stride, uint8_t *dst, int rows, int kg);

#ifdef __cplusplus
}
#endif
#endif

/*
 * ref_adapters.cc -- extern "C" entry points over the reference's own CPU
 * verification functions (TEST INFRASTRUCTURE ONLY).
 *
 * oracle/ref_extract.py copies those functions, by line range, out of the
 * reference's host drivers into oracle/_ref/ref_extracted.inc; this file
 * compiles them (with oracle/ref_shim.h standing in for HIP's fp8 type) into
 * oracle/_ref/libref.so, the "reference" build of the oracle.  The tests use
 * it to pin oracle/oracle.c (this project's restatement) to the reference's
 * code, and bench.py's CPU legs time it as the reference's CPU GEMM.  Nothing
 * in the product links or loads it.
 *
 * Each adapter passes its arguments straight through; where the reference
 * function takes extra constants the adapter supplies the values its driver
 * uses (group sizes 32 / 1 x 128 x 128).
 */
#include "ref_shim.h"

#include "ref_extracted.inc"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {
template <typename T>
const __hip_fp8_e4m3* fp8(const T* p) { return reinterpret_cast<const __hip_fp8_e4m3*>(p); }
}  // namespace

/* E4M3 decode of the shim type (the conversion every reference GEMM applies). */
REF_API float ref_e4m3_to_f32(uint8_t v) {
    __hip_fp8_e4m3 x;
    x.__x = v;
    return static_cast<float>(x);
}
REF_API uint8_t ref_f32_to_e4m3(float f) { return __hip_fp8_e4m3(f).__x; }

/* mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:35-47 */
REF_API float ref_mxfp8_e8m0_to_f32(uint8_t e) { return r_mxfp8::e8m0_to_f32(e); }
REF_API uint8_t ref_mxfp8_f32_to_e8m0(float v) { return r_mxfp8::f32_to_e8m0(v); }

/* mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:98-122, group_k = 32 as its driver. */
REF_API void ref_mxfp8_gemm(const uint8_t* a, const uint8_t* b, const uint8_t* sfa, const uint8_t* sfb, float* c,
                            int m, int n, int k, int lda, int ldb, int ldc, int stride_sfa, int stride_sfb) {
    r_mxfp8::gemm_ref(fp8(a), fp8(b), sfa, sfb, c, m, n, k, lda, ldb, ldc, stride_sfa, stride_sfb, 32);
}

/* block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_host.cc:66-90 with the driver's
 * group sizes (1 x 128 A, 128 x 128 B); sfa is [K/128][stride_sfa] (transposed, stride_sfa = M). */
REF_API void ref_fp8b_gemm(const uint8_t* a, const uint8_t* b, const float* sfa, const float* sfb, float* c,
                           int m, int n, int k, int lda, int ldb, int ldc, int stride_sfa, int stride_sfb) {
    r_fp8b::gemm_ref(fp8(a), fp8(b), sfa, sfb, c, m, n, k, lda, ldb, ldc, stride_sfa, stride_sfb, 1, 128, 128);
}

/* block_scale_gemm_bpreshuffle/..._host.cc:96-111 */
REF_API void ref_fp8b_shuffle_b(const uint8_t* src, uint8_t* dst, int batch, int n, int k, int block_k) {
    r_fp8b::shuffle_b(fp8(src), reinterpret_cast<__hip_fp8_e4m3*>(dst), batch, n, k, block_k);
}

/* mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:38-44 */
REF_API float ref_e2m1_to_f32(unsigned code) { return r_mxfp4::e2m1_to_f32(code); }
REF_API double ref_mxfp4_e8m0_to_f64(uint8_t e) { return r_mxfp4::e8m0_to_f64(e); }

/* mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:97-115 (dense [M,K/2] / [N,K/2]) */
REF_API void ref_mxfp4_gemm(const uint8_t* a, const uint8_t* b, const uint8_t* sfa, const uint8_t* sfb, float* c,
                            int m, int n, int k) {
    r_mxfp4::gemm_ref_cpu(a, b, sfa, sfb, c, m, n, k);
}

/* mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:117-144; out = errors, max_diff,
 * max_ratio, calc_diff.  mag may be null (|ref| is then the relative basis). */
REF_API void ref_mxfp4_compare(const float* ref, const float* got, const float* mag, size_t cnt, float rel_mag,
                               float abs_floor, double out_rel, double* out) {
    const r_mxfp4::cmp_stats s = r_mxfp4::compare(ref, got, mag, cnt, rel_mag, abs_floor, false, out_rel);
    out[0] = static_cast<double>(s.errors);
    out[1] = s.max_diff;
    out[2] = s.max_ratio;
    out[3] = s.calc_diff;
}

/* trace_block_scale_latest_20260914_040021/source_snapshot/gemm_a8w8_mxfp8_scale_host.cc */
REF_API uint64_t ref_mix_bits(uint64_t x) { return r_snap::mix_bits(x); }                       /* :139-144 */
REF_API void ref_fill_scales(uint8_t* p, size_t count, uint64_t seed) { r_snap::fill_scales(p, count, seed); }
REF_API void ref_pack_weight_16x16(const uint8_t* raw, uint8_t* packed, int batches, int n, int k) {  /* :163-179 */
    r_snap::pack_weight_16x16(fp8(raw), reinterpret_cast<__hip_fp8_e4m3*>(packed), batches, n, k);
}
REF_API float ref_snap_e8m0_to_f32(uint8_t e) { return r_snap::e8m0_to_f32(e); }              /* :181-183 */
REF_API uint16_t ref_f32_to_bf16_rne(float v) { return r_snap::f32_to_bf16_rne(v); }          /* :185-193 */
REF_API float ref_bf16_to_f32(uint16_t v) { return r_snap::bf16_to_f32(v); }                  /* :195-200 */
/* :221-248: E8M0 1x128 (A, SFA [K/128][M]) x 128x128 (B, SFB [N/128][K/128]), dense A [M,K], B [N,K]. */
REF_API void ref_e8m0_block_gemm(const uint8_t* a, const uint8_t* b, const uint8_t* sfa, const uint8_t* sfb,
                                 float* c, double* mag, int m, int n, int k) {
    r_snap::gemm_ref(fp8(a), fp8(b), sfa, sfb, c, mag, m, n, k);
}
/* :250-291 (prints its own statistics line, as in the reference). */
REF_API int ref_valid_vector(const float* ref, const void* out, const double* mag, size_t count, int bf16) {
    return r_snap::valid_vector(ref, out, mag, count, bf16 != 0) ? 1 : 0;
}

/* mxfp4_gemm_4wave_20261112/candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:196-206 (aiter e8m0_shuffle);
 * dst holds batch * rows32 * kg8 bytes. */
REF_API void ref_m10_e8m0_shuffle(const uint8_t* src, uint8_t* dst, int rows, int batch, int kg) {
    const std::vector<uint8_t> raw(src, src + static_cast<size_t>(batch) * rows * kg);
    const std::vector<uint8_t> out = r_m10::e8m0_shuffle(raw, rows, batch, kg);
    std::memcpy(dst, out.data(), out.size());
}
/* candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:219-225 (shuffle_weight(16,16) of packed fp4 B [N, K/2]). */
REF_API void ref_m10_shuffle_b(const uint8_t* src, uint8_t* dst, int batch, int n, int k) {
    const size_t bytes = static_cast<size_t>(batch) * n * (k / 2);
    const std::vector<uint8_t> h_b(src, src + bytes);
    std::vector<uint8_t> h_b_s(bytes);
    r_m10::shuffle_b(h_b, h_b_s, batch, n, k);
    std::memcpy(dst, h_b_s.data(), bytes);
}

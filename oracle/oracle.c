/*
 * oracle.c -- CPU restatement of the reference's verification GEMMs, codecs,
 * quantisers and byte layouts.  TEST INFRASTRUCTURE ONLY (see oracle.h): the
 * product library never links or calls it.  Built with gcc -O3 -fopenmp by
 * oracle/Makefile into oracle/_build/liboracle.so.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

/* ---- element codecs ---------------------------------------------------- */

float or_e4m3_to_f32(uint8_t v)
{
    const int s = v >> 7, e = (v >> 3) & 15, m = v & 7;
    float r;
    if (e == 15 && m == 7) return NAN;                 /* E4M3FN NaN */
    if (e == 0) r = ldexpf((float)m, -9);               /* m/8 * 2^-6 */
    else r = ldexpf((float)(8 + m), e - 10);            /* (1+m/8) * 2^(e-7) */
    return s ? -r : r;
}

/* Generic RNE minifloat encoder with saturation to the largest finite code.
 * ebits/mbits/bias describe the format; maxcode is the largest finite
 * magnitude code; sbit is the sign bit position. */
static uint8_t enc_minifloat(float x, int mbits, int bias, double maxv,
                             uint8_t maxcode, int sbit)
{
    const uint8_t sign = signbit(x) ? (uint8_t)(1u << sbit) : 0;
    const double a = fabs((double)x);
    int code;
    if (a >= maxv) {
        code = maxcode;
    } else if (a == 0.0) {
        code = 0;
    } else {
        int E;
        frexp(a, &E);
        const int e = E - 1;              /* a in [2^e, 2^(e+1)) */
        const int emin = 1 - bias;
        if (e < emin) {                   /* subnormal range: units of 2^(emin-mbits) */
            code = (int)rint(ldexp(a, mbits - emin));
        } else {
            int q = (int)rint(ldexp(a, mbits - e));   /* in [2^m, 2^(m+1)] */
            int ee = e;
            if (q == (2 << mbits)) { q = 1 << mbits; ++ee; }
            code = ((ee + bias) << mbits) | (q - (1 << mbits));
            if (code > maxcode) code = maxcode;
        }
    }
    return (uint8_t)(sign | code);
}

uint8_t or_f32_to_e4m3(float x)
{
    if (isnan(x)) return 0x7F;
    return enc_minifloat(x, 3, 7, 448.0, 0x7E, 7);
}

float or_e2m1_to_f32(uint8_t code)
{
    static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const float v = mag[code & 7];
    return (code & 8) ? -v : v;
}

uint8_t or_f32_to_e2m1(float x)
{
    if (isnan(x)) return 0x7;
    return enc_minifloat(x, 1, 1, 6.0, 0x7, 3);
}

float or_e8m0_to_f32(uint8_t e) { return ldexpf(1.0f, (int)e - 127); }

uint8_t or_f32_to_e8m0(float v)
{
    int exp, biased;
    if (v <= 0.0f) return 0;
    frexpf(v, &exp);
    biased = (exp - 1) + 127;
    if (biased < 0) biased = 0;
    if (biased > 255) biased = 255;
    return (uint8_t)biased;
}

uint16_t or_f32_to_bf16(float x)
{
    uint32_t bits;
    memcpy(&bits, &x, 4);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

float or_bf16_to_f32(uint16_t b)
{
    const uint32_t bits = (uint32_t)b << 16;
    float r;
    memcpy(&r, &bits, 4);
    return r;
}

/* ---- seeded inputs ------------------------------------------------------ */

uint64_t or_mix64(uint64_t x)
{
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

void or_fill_normal(float *out, size_t n, uint64_t seed)
{
    long i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < (long)n; ++i) {
        const uint64_t c = seed * 0x100000001b3ull + 2ull * (uint64_t)i;
        const double u1 = ((double)(or_mix64(c) >> 40) + 0.5) * 0x1p-24;
        const double u2 = (double)(or_mix64(c + 1) >> 40) * 0x1p-24;
        out[i] = (float)(sqrt(-2.0 * log(u1)) * cos(2.0 * M_PI * u2));
    }
}

/* ---- quantisers --------------------------------------------------------- */

/* exponent of 2^ceil(log2(r)) for r > 0, computed exactly */
static int ceil_log2(double r)
{
    int E;
    const double f = frexp(r, &E);   /* r = f * 2^E, f in [0.5, 1) */
    return (f == 0.5) ? E - 1 : E;
}

static void quant_mx(const float *x, int rows, int k, long ldx, uint8_t *q,
                     uint8_t *sf, int fp4)
{
    const int kg = k / 32;
    const double qmax = fp4 ? 6.0 : 448.0;
    int r;
#pragma omp parallel for schedule(static)
    for (r = 0; r < rows; ++r) {
        for (int g = 0; g < kg; ++g) {
            const float *xs = x + (long)r * ldx + g * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(xs[i]));
            int se = 0;
            if (amax > 0.0f) se = ceil_log2((double)amax / qmax);
            if (se < -127) se = -127;
            if (se > 127) se = 127;
            sf[(long)r * kg + g] = (uint8_t)(se + 127);
            for (int i = 0; i < 32; ++i) {
                const float v = (float)ldexp((double)xs[i], -se);
                if (fp4) {
                    const uint8_t c = or_f32_to_e2m1(v);
                    uint8_t *dst = q + (long)r * (k / 2) + (g * 32 + i) / 2;
                    if (((g * 32 + i) & 1) == 0) *dst = c;
                    else *dst = (uint8_t)(*dst | (c << 4));
                } else {
                    q[(long)r * k + g * 32 + i] = or_f32_to_e4m3(v);
                }
            }
        }
    }
}

void or_quant_mxfp8(const float *x, int rows, int k, long ldx, uint8_t *q, uint8_t *sf)
{
    quant_mx(x, rows, k, ldx, q, sf, 0);
}

void or_quant_mxfp4(const float *x, int rows, int k, long ldx, uint8_t *q, uint8_t *sf)
{
    quant_mx(x, rows, k, ldx, q, sf, 1);
}

void or_quant_fp8_block(const float *x, int rows, int k, long ldx, int br,
                        uint8_t *q, float *sf)
{
    const int kb = k / 128, nrb = (rows + br - 1) / br;
    int rb;
#pragma omp parallel for schedule(static)
    for (rb = 0; rb < nrb; ++rb) {
        const int r0 = rb * br, r1 = (r0 + br < rows) ? r0 + br : rows;
        for (int b = 0; b < kb; ++b) {
            float amax = 0.0f;
            for (int r = r0; r < r1; ++r)
                for (int i = 0; i < 128; ++i)
                    amax = fmaxf(amax, fabsf(x[(long)r * ldx + b * 128 + i]));
            const float s = amax > 0.0f ? amax / 448.0f : 1.0f;
            sf[(long)rb * kb + b] = s;
            for (int r = r0; r < r1; ++r)
                for (int i = 0; i < 128; ++i)
                    q[(long)r * k + b * 128 + i] =
                        or_f32_to_e4m3(x[(long)r * ldx + b * 128 + i] / s);
        }
    }
}

/* ---- reference GEMMs ---------------------------------------------------- */

void or_gemm_mxfp8(const uint8_t *a, const uint8_t *b, const uint8_t *sfa,
                   const uint8_t *sfb, float *c, int m, int n, int k, long lda,
                   long ldb, long ldc, long stride_sfa, long stride_sfb)
{
    /* decode tables keep the inner loop a plain fp32 multiply-add chain */
    float lut[256];
    for (int v = 0; v < 256; ++v) lut[v] = or_e4m3_to_f32((uint8_t)v);
    int i;
#pragma omp parallel for collapse(2) schedule(static)
    for (i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            const uint8_t *ar = a + (long)i * lda, *brw = b + (long)j * ldb;
            const uint8_t *sar = sfa + (long)i * stride_sfa, *sbr = sfb + (long)j * stride_sfb;
            float sum = 0.0f;
            for (int g = 0; g < k / 32; ++g) {
                const float scale = or_e8m0_to_f32(sar[g]) * or_e8m0_to_f32(sbr[g]);
                for (int p = g * 32; p < g * 32 + 32; ++p)
                    sum += lut[ar[p]] * lut[brw[p]] * scale;
            }
            c[(long)i * ldc + j] = sum;
        }
    }
}

void or_gemm_mxfp8_f64(const uint8_t *a, const uint8_t *b, const uint8_t *sfa,
                       const uint8_t *sfb, float *c, double *mag, int m, int n,
                       int k, long lda, long ldb, long ldc, long stride_sfa,
                       long stride_sfb)
{
    float lut[256];
    for (int v = 0; v < 256; ++v) lut[v] = or_e4m3_to_f32((uint8_t)v);
    int i;
#pragma omp parallel for collapse(2) schedule(static)
    for (i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            const uint8_t *ar = a + (long)i * lda, *brw = b + (long)j * ldb;
            double sum = 0.0, sabs = 0.0;
            for (int g = 0; g < k / 32; ++g) {
                const double scale = (double)or_e8m0_to_f32(sfa[(long)i * stride_sfa + g]) *
                                     (double)or_e8m0_to_f32(sfb[(long)j * stride_sfb + g]);
                double part = 0.0, pabs = 0.0;
                for (int p = g * 32; p < g * 32 + 32; ++p) {
                    const double t = (double)lut[ar[p]] * (double)lut[brw[p]];
                    part += t;
                    pabs += fabs(t);
                }
                sum += part * scale;
                sabs += pabs * scale;
            }
            c[(long)i * ldc + j] = (float)sum;
            if (mag) mag[(long)i * ldc + j] = sabs;
        }
    }
}

void or_gemm_mxfp4(const uint8_t *a, const uint8_t *b, const uint8_t *sfa,
                   const uint8_t *sfb, float *c, double *mag, int m, int n,
                   int k, long lda, long ldb, long ldc, long stride_sfa,
                   long stride_sfb)
{
    int i;
#pragma omp parallel for collapse(2) schedule(static)
    for (i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            const uint8_t *ar = a + (long)i * lda, *brw = b + (long)j * ldb;
            double sum = 0.0, sabs = 0.0;
            for (int g = 0; g < k / 32; ++g) {
                const double s = ldexp(1.0, (int)sfa[(long)i * stride_sfa + g] - 127) *
                                 ldexp(1.0, (int)sfb[(long)j * stride_sfb + g] - 127);
                double part = 0.0, pabs = 0.0;
                for (int p = g * 16; p < g * 16 + 16; ++p) {
                    const unsigned x = ar[p], y = brw[p];
                    const double t0 = (double)or_e2m1_to_f32(x & 15) * or_e2m1_to_f32(y & 15);
                    const double t1 = (double)or_e2m1_to_f32(x >> 4) * or_e2m1_to_f32(y >> 4);
                    part += t0 + t1;
                    pabs += fabs(t0) + fabs(t1);
                }
                sum += part * s;
                sabs += pabs * s;
            }
            c[(long)i * ldc + j] = (float)sum;
            if (mag) mag[(long)i * ldc + j] = sabs;
        }
    }
}

void or_gemm_fp8_block(const uint8_t *a, const uint8_t *b, const float *sfa,
                       const float *sfb, float *c, double *mag, int m, int n,
                       int k, long lda, long ldb, long ldc, long sfa_m,
                       long sfa_k, long sfb_n, long sfb_k)
{
    float lut[256];
    for (int v = 0; v < 256; ++v) lut[v] = or_e4m3_to_f32((uint8_t)v);
    int i;
#pragma omp parallel for collapse(2) schedule(static)
    for (i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            const uint8_t *ar = a + (long)i * lda, *brw = b + (long)j * ldb;
            float sum = 0.0f;
            double sabs = 0.0;
            for (int kb = 0; kb < k / 128; ++kb) {
                const float scale = sfa[(long)i * sfa_m + (long)kb * sfa_k] *
                                    sfb[(long)(j / 128) * sfb_n + (long)kb * sfb_k];
                for (int p = kb * 128; p < kb * 128 + 128; ++p) {
                    const float t = lut[ar[p]] * lut[brw[p]] * scale;
                    sum += t;
                    sabs += fabs((double)t);
                }
            }
            c[(long)i * ldc + j] = sum;
            if (mag) mag[(long)i * ldc + j] = sabs;
        }
    }
}

void or_gemm_e8m0_block(const uint8_t *a, const uint8_t *b, const uint8_t *sfa,
                        const uint8_t *sfb, float *c, double *mag, int m, int n,
                        int k)
{
    float lut[256];
    for (int v = 0; v < 256; ++v) lut[v] = or_e4m3_to_f32((uint8_t)v);
    const int groups_k = k / 128;
    int row;
#pragma omp parallel for collapse(2) schedule(static)
    for (row = 0; row < m; ++row) {
        for (int col = 0; col < n; ++col) {
            const uint8_t *ar = a + (long)row * k, *brw = b + (long)col * k;
            double sum = 0.0, sabs = 0.0;
            for (int kg = 0; kg < groups_k; ++kg) {
                const double scale = (double)or_e8m0_to_f32(sfa[(long)kg * m + row]) *
                                     (double)or_e8m0_to_f32(sfb[(long)(col / 128) * groups_k + kg]);
                for (int p = kg * 128; p < (kg + 1) * 128; ++p) {
                    const double t = (double)lut[ar[p]] * (double)lut[brw[p]] * scale;
                    sum += t;
                    sabs += fabs(t);
                }
            }
            c[(long)row * n + col] = (float)sum;
            if (mag) mag[(long)row * n + col] = sabs;
        }
    }
}

/* ---- layouts ------------------------------------------------------------ */

void or_shuffle_kpanel(const uint8_t *src, uint8_t *dst, int n, int k, int block_k)
{
    const int nkt = k / block_k;
    int r;
#pragma omp parallel for schedule(static)
    for (r = 0; r < n; ++r)
        for (int kt = 0; kt < nkt; ++kt)
            memcpy(dst + ((long)kt * n + r) * block_k, src + (long)r * k + (long)kt * block_k, block_k);
}

void or_unshuffle_kpanel(const uint8_t *src, uint8_t *dst, int n, int k, int block_k)
{
    const int nkt = k / block_k;
    int r;
#pragma omp parallel for schedule(static)
    for (r = 0; r < n; ++r)
        for (int kt = 0; kt < nkt; ++kt)
            memcpy(dst + (long)r * k + (long)kt * block_k, src + ((long)kt * n + r) * block_k, block_k);
}

void or_shuffle_weight16(const uint8_t *src, uint8_t *dst, int n, int kbytes)
{
    int nb;
#pragma omp parallel for schedule(static)
    for (nb = 0; nb < n / 16; ++nb)
        for (int kb = 0; kb < kbytes / 16; ++kb)
            for (int ni = 0; ni < 16; ++ni)
                memcpy(dst + ((long)nb * (kbytes / 16) + kb) * 256 + ni * 16,
                       src + (long)(nb * 16 + ni) * kbytes + kb * 16, 16);
}

void or_unshuffle_weight16(const uint8_t *src, uint8_t *dst, int n, int kbytes)
{
    int nb;
#pragma omp parallel for schedule(static)
    for (nb = 0; nb < n / 16; ++nb)
        for (int kb = 0; kb < kbytes / 16; ++kb)
            for (int ni = 0; ni < 16; ++ni)
                memcpy(dst + (long)(nb * 16 + ni) * kbytes + kb * 16,
                       src + ((long)nb * (kbytes / 16) + kb) * 256 + ni * 16, 16);
}

size_t or_e8m0_shuffle_size(int rows, int kg)
{
    return (size_t)((rows + 31) / 32 * 32) * (size_t)((kg + 7) / 8 * 8);
}

static size_t e8m0_shuffle_off(int r, int g, int kg8)
{
    return ((size_t)(r / 32) * (kg8 / 8) + g / 8) * 256 + (g % 4) * 64 + (r % 16) * 4 +
           ((g % 8) / 4) * 2 + (r % 32) / 16;
}

void or_e8m0_shuffle(const uint8_t *src, uint8_t *dst, int rows, int kg)
{
    const int kg8 = (kg + 7) / 8 * 8;
    memset(dst, 0x7F, or_e8m0_shuffle_size(rows, kg));
    for (int r = 0; r < rows; ++r)
        for (int g = 0; g < kg; ++g) dst[e8m0_shuffle_off(r, g, kg8)] = src[(long)r * kg + g];
}

void or_e8m0_unshuffle(const uint8_t *src, uint8_t *dst, int rows, int kg)
{
    const int kg8 = (kg + 7) / 8 * 8;
    for (int r = 0; r < rows; ++r)
        for (int g = 0; g < kg; ++g) dst[(long)r * kg + g] = src[e8m0_shuffle_off(r, g, kg8)];
}

size_t or_sf_native_size(int rows, int kg)
{
    return (size_t)((rows + 127) / 128) * (size_t)((kg + 3) / 4) * 512;
}

void or_sf_to_native(const uint8_t *src, long stride, uint8_t *dst, int rows, int kg)
{
    const int kb_total = (kg + 3) / 4;
    memset(dst, 0x7F, or_sf_native_size(rows, kg));
    for (int r = 0; r < rows; ++r)
        for (int g = 0; g < kg; ++g) {
            const size_t atom = ((size_t)(r / 128) * kb_total + g / 4) * 512;
            const size_t word = (size_t)((r % 32) * 4 + (r % 128) / 32);
            dst[atom + word * 4 + g % 4] = src[(long)r * stride + g];
        }
}

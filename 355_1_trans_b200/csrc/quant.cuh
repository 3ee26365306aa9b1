// quant.cuh -- activation quantise + pack: bf16 / fp32 rows -> the element
// and scale layouts the GEMM kernels read, in one pass over HBM.
//
// Quantisation rules (the input recipes of the reference's host drivers; the
// tests compare this kernel bit for bit with a CPU restatement of them):
//   MX (1 x 32), qmax = 448 (E4M3) or 6 (E2M1):
//     se = ceil(log2(amax / qmax)) over each 32-element group, exact, clamped
//     to [-127, 127], 0 for an all-zero group; scale byte = se + 127;
//     element = RNE-saturating cast of x * 2^-se (one rounding from fp32);
//     E2M1 codes packed two per byte, even k in the low nibble;
//     (E8M0 codec: mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:35-47)
//   FP8 1 x 128 block (activations of the fp32 block-scale GEMM):
//     s = amax / 448 in fp32 (1 for an all-zero group); element = RNE-
//     saturating E4M3 of x / s
//     (block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_host.cc
//      input generation).
// The casts use the sm_100a conversions cvt.rn.satfinite.{e4m3x2,e2m1x2}.f32
// (round to nearest even, saturate to the largest finite code, NaN -> NaN).
//
// Work split: a thread converts 8 consecutive elements (one 16-byte bf16 or
// two 16-byte fp32 loads) in each of eight (bf16) or four (fp32) 256-column
// segments, issuing all its loads first so that 128 bytes per thread are in
// flight to cover HBM latency (bf16 loads stay packed in 4 registers each
// until converted); 4 threads form an MX group, 16 a 128-block, and the
// group maximum is a butterfly of warp shuffles.  A warp covers 2048 (bf16)
// or 1024 (fp32) consecutive elements of one row, so loads and stores are
// contiguous.
#pragma once

#include "sm100.cuh"

namespace bsg {

constexpr int kQuantMxfp8 = 0, kQuantMxfp4 = 1, kQuantFp8Block = 2;

struct QuantParams {
  const void* x;
  int in_fp32;            // 0: bf16 input, 1: fp32
  int rows, cols;
  long long ldx;          // elements
  uint8_t* q;
  long long ldq;          // bytes
  void* sf;
  int sf_format;          // MX: 0 native atoms, 1 row-major bytes; fp8 block: 1 row-major, 2 [cols/128][rows]
  long long ld_sf;        // row-major: bytes (MX) / floats (fp8 block); [kb][rows]: floats between kb rows
  int rows_padded;        // native MX: rows rounded up to 128 (pad rows get scale 0x7F)
};

__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

// exponent of 2^ceil(log2(amax / qmax)) for amax > 0, exact, from the bits.
// With qmax = c 2^P (448 = 1.75 2^8, 6 = 1.5 2^2) and amax = m 2^e, m in
// [1, 2) (subnormals normalised first): amax / qmax = (m / c) 2^(e - P) with
// m / c in (1/2, 2), so the ceiling is e - P + 1 when m > c and e - P
// otherwise (m == c is an exact power of two).  Identical to ceil(log2())
// of the double quotient for every finite float (checked exhaustively over
// mantissas, subnormals and the clamp range); infinities keep that form.
template <int kP, uint32_t kCFrac>
__device__ __forceinline__ int mx_scale_exponent(float amax, double qmax) {
  if (!(amax > 0.0f)) return 0;
  const uint32_t bits = __float_as_uint(amax);
  uint32_t exp_field = bits >> 23, frac = bits & 0x7FFFFFu;
  int se;
  if (exp_field == 255u) {   // +inf
    int e;
    const double f = frexp(static_cast<double>(amax) / qmax, &e);
    se = f == 0.5 ? e - 1 : e;
  } else {
    int e;
    if (exp_field == 0u) {   // subnormal: normalise the fraction
      const int k = __clz(static_cast<int>(frac)) - 8;
      frac = (frac << k) & 0x7FFFFFu;
      e = -126 - k;
    } else {
      e = static_cast<int>(exp_field) - 127;
    }
    se = e - kP + (frac > kCFrac ? 1 : 0);
  }
  return se < -127 ? -127 : (se > 127 ? 127 : se);
}

// 2^-se for se in [-127, 127], exactly (2^-127 is subnormal)
__device__ __forceinline__ float pow2_neg(int se) {
  return __uint_as_float(se < 127 ? static_cast<uint32_t>(127 - se) << 23 : 0x00400000u);
}

// byte offset of (row, group) in the native scale layout
__device__ __forceinline__ long long native_sf_offset(int row, int g, int kg) {
  const int kb_atoms = (kg + 3) / 4;
  return (static_cast<long long>(row / 128) * kb_atoms + g / 4) * 512 +
         (((row % 32) * 4 + (row % 128) / 32) * 4 + (g % 4));
}

// Columns covered by one warp: quant_items segments of 256, every thread
// issuing its 16-byte loads (two per segment for fp32) before converting any.
constexpr int quant_items(bool f32_in) { return f32_in ? 4 : 8; }
constexpr int quant_warp_cols(bool f32_in) { return 256 * quant_items(f32_in); }

template <int kFormat, bool kF32In>
__global__ void __launch_bounds__(256, 4) quantize_kernel(const QuantParams p) {
  constexpr int kGroup = kFormat == kQuantFp8Block ? 128 : 32;
  constexpr int kLanes = kGroup / 8;   // threads per group
  constexpr int kQuantItems = quant_items(kF32In);
  constexpr int kQuantWarpCols = quant_warp_cols(kF32In);
  const int warps_per_row = (p.cols + kQuantWarpCols - 1) / kQuantWarpCols;
  const long long gw = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31u);
  const int row = static_cast<int>(gw / warps_per_row);
  const int col0 = static_cast<int>(gw % warps_per_row) * kQuantWarpCols + lane * 8;
  const int limit_rows = kFormat != kQuantFp8Block && p.sf_format == 0 ? p.rows_padded : p.rows;
  // A GEMM that consumes these activations may launch now (programmatic
  // dependent launch): its prologue and weight prefetch overlap this kernel,
  // and it waits for this grid's completion before it reads the outputs.
  griddep_launch_dependents();
  if (row >= limit_rows) return;
  // all loads first: raw 16-byte words (bf16 stays packed until converted)
  uint4 raw[kF32In ? 2 * kQuantItems : kQuantItems];
#pragma unroll
  for (int it = 0; it < kQuantItems; ++it) {
    const int col = col0 + it * 256;
    const bool live = row < p.rows && col < p.cols;   // cols % kGroup == 0: whole groups live or not
    if constexpr (kF32In) {
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const float*>(p.x) + row * p.ldx + col);
      raw[2 * it] = live ? __ldg(src) : make_uint4(0u, 0u, 0u, 0u);
      raw[2 * it + 1] = live ? __ldg(src + 1) : make_uint4(0u, 0u, 0u, 0u);
    } else {
      raw[it] = live ? __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) + row * p.ldx + col))
                     : make_uint4(0u, 0u, 0u, 0u);
    }
  }
#pragma unroll
  for (int it = 0; it < kQuantItems; ++it) {
    const int col = col0 + it * 256;
    if (col - lane * 8 >= p.cols) break;   // the whole warp is past the row end
    const bool live = row < p.rows && col < p.cols;
    float v[1][8];   // this segment's 8 elements (indexed [0][i] below)
    if constexpr (kF32In) {
      const uint4 a = raw[2 * it], b = raw[2 * it + 1];
      v[0][0] = __uint_as_float(a.x); v[0][1] = __uint_as_float(a.y);
      v[0][2] = __uint_as_float(a.z); v[0][3] = __uint_as_float(a.w);
      v[0][4] = __uint_as_float(b.x); v[0][5] = __uint_as_float(b.y);
      v[0][6] = __uint_as_float(b.z); v[0][7] = __uint_as_float(b.w);
    } else {
      const uint32_t u[4] = {raw[it].x, raw[it].y, raw[it].z, raw[it].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[0][2 * i] = __uint_as_float(u[i] << 16);
        v[0][2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
      }
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[0][i]));
#pragma unroll
    for (int d = 1; d < kLanes; d <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
    const int g = col / kGroup;
    const bool leader = (lane % kLanes) == 0;

    if constexpr (kFormat == kQuantFp8Block) {
      if (!live) continue;
      const float s = amax > 0.0f ? amax / 448.0f : 1.0f;
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int i = 0; i < 4; i += 2) {
        w0 |= cvt_e4m3x2(v[0][i] / s, v[0][i + 1] / s) << (8 * i);
        w1 |= cvt_e4m3x2(v[0][i + 4] / s, v[0][i + 5] / s) << (8 * i);
      }
      *reinterpret_cast<uint2*>(p.q + row * p.ldq + col) = make_uint2(w0, w1);
      if (leader) {
        float* sf = static_cast<float*>(p.sf);
        if (p.sf_format == 2)
          sf[static_cast<long long>(g) * p.ld_sf + row] = s;
        else
          sf[row * p.ld_sf + g] = s;
      }
    } else {
      constexpr double kQmax = kFormat == kQuantMxfp4 ? 6.0 : 448.0;
      const int se = kFormat == kQuantMxfp4 ? mx_scale_exponent<2, 0x400000u>(amax, kQmax)
                                            : mx_scale_exponent<8, 0x600000u>(amax, kQmax);
      if (live) {
        const float mul = pow2_neg(se);   // exact power of two (2^-127 .. 2^127)
        if constexpr (kFormat == kQuantMxfp8) {
          uint32_t w0 = 0, w1 = 0;
#pragma unroll
          for (int i = 0; i < 4; i += 2) {
            w0 |= cvt_e4m3x2(v[0][i] * mul, v[0][i + 1] * mul) << (8 * i);
            w1 |= cvt_e4m3x2(v[0][i + 4] * mul, v[0][i + 5] * mul) << (8 * i);
          }
          *reinterpret_cast<uint2*>(p.q + row * p.ldq + col) = make_uint2(w0, w1);
        } else {
          uint32_t w = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) w |= cvt_e2m1x2(v[0][2 * i] * mul, v[0][2 * i + 1] * mul) << (8 * i);
          *reinterpret_cast<uint32_t*>(p.q + row * p.ldq + col / 2) = w;
        }
      }
      if (leader && col < p.cols) {
        uint8_t* sf = static_cast<uint8_t*>(p.sf);
        const uint8_t byte = row < p.rows ? static_cast<uint8_t>(se + 127) : static_cast<uint8_t>(0x7F);
        if (p.sf_format == 0)
          sf[native_sf_offset(row, g, p.cols / 32)] = byte;
        else if (row < p.rows)
          sf[row * p.ld_sf + g] = byte;
      }
    }
  }
}

}  // namespace bsg

// pack.cuh -- device byte permutations between the reference's preshuffled
// formats and the layouts the sm_100a kernels read.  All are pure gathers
// (one thread per output 16-byte chunk or 4-byte word), HBM-bandwidth bound.
//
//   B operand:  aiter shuffle_weight(16,16)  [N/16][Kb/16][16][16]
//               (source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:161-179;
//                candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:215-225)
//               K-panel B'[K/128][N][128]
//               (block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_host.cc:96-111)
//           <-> raw [N][Kb] (Kb = K bytes), which TMA tiles directly.
//   E8M0 scales: row-major [rows][kg] or aiter e8m0_shuffle
//               (candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:194-206)
//           <-> native tcgen05 scale atoms: 512 bytes per (128 rows, 4 groups),
//               byte ((r%32)*4 + (r%128)/32)*4 + g%4, i.e. the 32x128-bit
//               image tcgen05.cp.32x128b.warpx4 copies into TMEM.
#pragma once

#include "sm100.cuh"

namespace bsg {

// ---- B operand ------------------------------------------------------------
// raw chunk (n, c16) <-> shuffle16 offset ((n/16)*(kb/16) + c16)*256 + (n%16)*16
__global__ void pack_b_shuffle16_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                        int rows, int kbytes, int unpack) {
  const long long chunks_per_row = kbytes / 16;
  const long long total = static_cast<long long>(rows) * chunks_per_row;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long n = i / chunks_per_row, c = i - n * chunks_per_row;
    const long long sh = ((n / 16) * chunks_per_row + c) * 16 + (n % 16);   // in 16B units
    if (unpack) dst[sh] = src[i];
    else dst[i] = src[sh];
  }
}

// raw chunk (n, kt, c) <-> kpanel offset (kt*rows + n)*8 + c  (16B units)
__global__ void pack_b_kpanel_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                     int rows, int kbytes, int unpack) {
  const long long chunks_per_row = kbytes / 16;
  const long long total = static_cast<long long>(rows) * chunks_per_row;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long n = i / chunks_per_row, c = i - n * chunks_per_row;
    const long long kt = c / 8, ci = c % 8;
    const long long kp = (kt * rows + n) * 8 + ci;
    if (unpack) dst[kp] = src[i];
    else dst[i] = src[kp];
  }
}

// ---- E8M0 scales -----------------------------------------------------------
__device__ __forceinline__ long long e8m0_shuffle_off(int r, int g, int kg8) {
  return (static_cast<long long>(r / 32) * (kg8 / 8) + g / 8) * 256 + (g % 4) * 64 + (r % 16) * 4 +
         ((g % 8) / 4) * 2 + (r % 32) / 16;
}

// One thread per native 32-bit word: word w of atom (rb, kb) holds row
// rb*128 + (w%4)*32 + w/4, groups kb*4 .. kb*4+3.
__global__ void pack_sf_native_kernel(const uint8_t* __restrict__ src, int src_stride,
                                      uint8_t* __restrict__ dst, int rows, int kg, int src_format,
                                      int unpack) {
  const int kb_total = (kg + 3) / 4;
  const long long words = static_cast<long long>((rows + 127) / 128) * kb_total * 128;
  const int kg8 = (kg + 7) / 8 * 8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < words;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long atom = i / 128;
    const int w = static_cast<int>(i % 128);
    const int rb = static_cast<int>(atom / kb_total), kb = static_cast<int>(atom % kb_total);
    const int r = rb * 128 + (w % 4) * 32 + w / 4;
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int g = kb * 4 + j;
      const bool valid = r < rows && g < kg;
      const long long so = !valid ? 0
                           : src_format == 3 ? e8m0_shuffle_off(r, g, kg8)
                                             : static_cast<long long>(r) * src_stride + g;
      if (!unpack) {
        const uint32_t v = valid ? src[so] : 0x7Fu;
        word |= v << (8 * j);
      } else if (valid) {
        dst[so] = src[i * 4 + j];
      }
    }
    if (!unpack) reinterpret_cast<uint32_t*>(dst)[i] = word;
  }
}

// Row-major E8M0 scales of a grouped (MoE) activation [total_rows][kg] into
// native atoms per group: group e (rows offsets[e] .. offsets[e+1], clamped to
// [0, total_rows] and to at most max_rows rows, as the grouped GEMM clamps
// them) gets its own ceil(max_rows/128) row blocks, so the GEMM finds group
// e's atoms at batch stride tiles * ceil(kg/4) * 512 bytes.  Rows past a
// group's end and groups past kg read 0x7F (2^0).
//
// The first warp of block 0 also writes tile_prefix[0 .. groups]: the
// exclusive prefix sum of the groups' 128-row tiles (ceil(rows / 128)), which
// the grouped GEMM uses to enumerate only the tiles that hold rows.
__global__ void pack_sf_grouped_kernel(const uint8_t* __restrict__ src, int src_stride,
                                       const int* __restrict__ offsets, int groups, int total_rows,
                                       int max_rows, int kg, uint8_t* __restrict__ dst,
                                       int* __restrict__ tile_prefix) {
  if (blockIdx.x == 0 && threadIdx.x < 32) {
    const int lane = static_cast<int>(threadIdx.x);
    int carry = 0;
    for (int base = 0; base < groups; base += 32) {
      const int e = base + lane;
      int t = 0;
      if (e < groups) {
        int a0 = __ldg(offsets + e), a1 = __ldg(offsets + e + 1);
        a0 = min(max(a0, 0), total_rows);
        a1 = min(max(a1, a0), total_rows);
        t = (min(a1 - a0, max_rows) + 127) / 128;
      }
      int v = t;   // inclusive warp scan
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += y;
      }
      if (e < groups) tile_prefix[e] = carry + v - t;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) tile_prefix[groups] = carry;
  }
  const int kb_total = (kg + 3) / 4;
  const int tiles = (max_rows + 127) / 128;
  const long long atoms_per_group = static_cast<long long>(tiles) * kb_total;
  const long long words = atoms_per_group * groups * 128;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < words;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long atom = i / 128;
    const int w = static_cast<int>(i % 128);
    const int e = static_cast<int>(atom / atoms_per_group);
    const long long rem = atom - e * atoms_per_group;
    const int rb = static_cast<int>(rem / kb_total), kb = static_cast<int>(rem % kb_total);
    int a0 = __ldg(offsets + e), a1 = __ldg(offsets + e + 1);
    a0 = min(max(a0, 0), total_rows);
    a1 = min(max(a1, a0), total_rows);
    const int rows = min(a1 - a0, max_rows);
    const int r = rb * 128 + (w % 4) * 32 + w / 4;
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int g = kb * 4 + j;
      const uint32_t v = r < rows && g < kg ? src[static_cast<long long>(a0 + r) * src_stride + g] : 0x7Fu;
      word |= v << (8 * j);
    }
    reinterpret_cast<uint32_t*>(dst)[i] = word;
  }
}

// Pads of an aiter e8m0_shuffle buffer are 0x7F; unpack writes them first.
__global__ void fill_u8_kernel(uint8_t* __restrict__ dst, long long n, uint8_t v) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    dst[i] = v;
}

// Bounded-wait self test: one thread waits on an mbarrier nothing arrives at;
// the expired wait records BSG_ERR_TIMEOUT in the device error word.
__global__ void selftest_timeout_kernel(unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // the phase with parity 0 never completes: no thread ever arrives
    (void)mbar_wait(&bar, 0, &abort_flag, timeout_ns);
  }
  __syncthreads();
}

}  // namespace bsg

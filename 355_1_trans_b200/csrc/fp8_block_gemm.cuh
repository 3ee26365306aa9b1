// fp8_block_gemm.cuh -- FP8 (E4M3) GEMM with fp32 block scales, DeepSeek
// style: one scale per (row, 128-K block) of A and per (128-N block, 128-K
// block) of B, for sm_100a.
//
// Semantics (reference, paths relative to its project root):
//   block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_kernel_template.hpp:
//   204-601 with scale_c_tile :24-39 and load_sfb :284-289: for each 128-K
//   block kb, the unscaled partial product (A B^T)_kb is multiplied by
//   sfa[m,kb] * sfb[n/128,kb] and added to an fp32 accumulator.
//
// Because the scales are arbitrary fp32 (not powers of two) they cannot be
// folded into a block-scaled MMA.  Instead:
//   - the single-thread issuer runs 4 x .kind::f8f6f4 MMAs (K = 32 each) per
//     128-K block into one of four TMEM buffers (128 x BN fp32 each), so the
//     tensor core fills the next buffers while buffer kb is being promoted;
//   - the epilogue warps (the "promotion" warps) tcgen05.ld each finished
//     partial and FMA it into a register accumulator with the per-row A scale
//     times the per-tile B scale, then release the buffer; after the last K
//     block they round to bf16 (RNE) and store.
// B is read either raw [N,K] or in the reference's K-panel preshuffle
// B'[K/128][N][128] (a 3D/4D tensor map makes both land identically in smem).
#pragma once

#include "mx_gemm.cuh"

namespace bsg {

struct Fp8BlockParams {
  int m, n, k;
  int batch;
  int num_kb;
  int tiles_m, tiles_n;
  int split_k, kb_per_split;
  int total_units;
  int group_m;
  const float* sfa;
  long long sfa_m, sfa_k, sfa_batch;   // float strides: row, k-block, batch
  const float* sfb;
  long long sfb_n, sfb_k, sfb_batch;   // float strides: 128-row block, k-block, batch
  void* c;
  long long ldc;
  long long c_batch_stride;
  float* ws;
  unsigned long long timeout_ns;
  // grouped (MoE) calls: group b owns rows [offsets[b], offsets[b + 1]) of the
  // concatenated A, its scales and C; total_rows bounds those arrays
  const int* group_offsets;
  int total_rows;
  // pair kernel only: the last tail_units units run as tail_split K slices
  // each (fp32 partials in ws, summed by fp8b_pair_tail_reduce_kernel);
  // total_items = total_units - tail_units + tail_units * tail_split
  int tail_units, tail_split, total_items;
};

// First row and row count of group b in a grouped call.  The offsets come
// from device memory written by the caller (the token routing); they are
// clamped to [0, total_rows] and a group to p.m rows, so an inconsistent
// offsets array cannot address outside A, its scales or C.
__device__ __forceinline__ void group_rows(const Fp8BlockParams& p, int b, int& row0, int& rows) {
  int a0 = __ldg(p.group_offsets + b);
  int a1 = __ldg(p.group_offsets + b + 1);
  a0 = min(max(a0, 0), p.total_rows);
  a1 = min(max(a1, a0), p.total_rows);
  row0 = a0;
  rows = min(a1 - a0, p.m);
}

// The unit a persistent CTA works on.  Plain calls decode the tile grid.  A
// grouped call with its groups' 128-row tile prefix in shared memory
// (`pre`, live = prefix[batch] M tiles) enumerates only the M tiles that hold
// rows, so ragged groups leave no CTA idle: gm belongs to the last group e
// with pre[e] <= gm (empty groups share their successor's prefix), as its M
// tile gm - pre[e].  Without the prefix (more groups than it holds), grouped
// calls decode the full grid and skip the tiles past a group's rows.
// Returns false for a unit to skip; every role skips the same units.
template <bool kGrouped>
__device__ __forceinline__ bool fp8b_unit(const Fp8BlockParams& p, const int* pre, int live, int u, int& b,
                                          int& mt, int& nt, int& s, int& row0, int& rows) {
  row0 = 0;
  rows = p.m;
  if constexpr (kGrouped) {
    if (pre != nullptr) {
      int gb, gm;
      decode_unit(u, live, p.tiles_n, 1, p.group_m, gb, gm, nt, s);
      int lo = 0, hi = p.batch - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= gm) lo = mid;
        else hi = mid - 1;
      }
      b = lo;
      mt = gm - pre[lo];
    } else {
      decode_unit(u, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
    }
    group_rows(p, b, row0, rows);
    return mt >= 0 && mt * 128 < rows;
  } else {
    decode_unit(u, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
    return true;
  }
}

// Weight (B) storage formats read in place:
//   kFmtRaw        [N, K] K-major rows (128B-swizzled stage tiles);
//   kFmtKPanel     the reference's shuffle_b K panels B'[K/128][N][128]
//                  (block_scale_gemm_bpreshuffle/..._host.cc:96-111);
//   kFmtShuffle16  aiter's shuffle_weight(16,16) [N/16][K/16][16][16]
//                  (source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:161-179),
//                  landed by a 5-D tensor map in the canonical no-swizzle
//                  K-major layout (see mx_gemm.cuh).
constexpr int kFmtRaw = 0, kFmtKPanel = 1, kFmtShuffle16 = 2;

// Shared-memory descriptor of K step t (32 bytes of K) of a 128-byte K stage
// of a weight tile stored in format kBFmt.
template <int kBFmt>
__device__ __forceinline__ uint64_t weight_sdesc(uint32_t tile_addr, int t) {
  if constexpr (kBFmt == kFmtShuffle16)
    return make_sdesc(tile_addr + 256u * static_cast<uint32_t>(t), 128u, 1024u, kLayoutNone);
  else
    return make_sdesc(tile_addr + 32u * static_cast<uint32_t>(t), 16u, 1024u, kLayoutSW128);
}

template <int BN>
struct Fp8BlockCfg {
  static_assert(BN == 128, "promotion accumulator holds 128 columns per thread");
  static constexpr uint32_t kABytes = 128u * 128u;
  static constexpr uint32_t kBBytes = static_cast<uint32_t>(BN) * 128u;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 6;
  static constexpr uint32_t kOffB = kABytes * kStages;
  static constexpr uint32_t kOffBar = kOffB + kBBytes * kStages;
  // grouped calls: the groups' M-tile prefix (up to kMaxPrefixGroups groups)
  static constexpr int kMaxPrefixGroups = 1024;
  static constexpr uint32_t kOffPrefix = kOffBar + 256u;
  static constexpr uint32_t kSmemBytes = kOffPrefix + 4u * (kMaxPrefixGroups + 1) + 1024u;
  // Four TMEM partial buffers (all 512 columns): the MMA runs up to four K
  // blocks ahead of the promotion (two buffers: 1666 against 1736 TFLOPS at
  // M=8192 N=7168 K=8192, together with the batched loads below).
  static constexpr int kAccBufs = 4;
  static constexpr uint32_t kTmemCols = kAccBufs * BN;
};

// kGrouped: the batch index is a group (expert) whose rows of A, sfa and C
// start at group_offsets[b] (A's tensor map spans all total_rows); tiles past
// a group's rows are skipped by every role alike, and B, sfb keep their
// per-group batch strides.  Grouped calls run without split-K.
template <int BN, int kBFmt, bool kOutF32, bool kGrouped = false>
__global__ void __launch_bounds__(256, 1)
    fp8_block_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmB, const Fp8BlockParams p) {
  using Cfg = Fp8BlockCfg<BN>;
  constexpr int S = Cfg::kStages;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::kOffB;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* empty_bar = full_bar + S;
  constexpr int NB = Cfg::kAccBufs;
  uint64_t* acc_full = empty_bar + S;    // [NB]
  uint64_t* acc_empty = acc_full + NB;   // [NB]
  uint64_t* drain_bar = acc_empty + NB;
  static_assert(8 * (2 * Cfg::kStages + 2 * Cfg::kAccBufs + 1) + 8 <= 256, "barrier area");
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;

  if (threadIdx.x == 32) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);   // one arrival per promotion warp
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (threadIdx.x == 0) griddep_launch_dependents();   // a split-K reduce may launch now
  // Launched with programmatic dependent launch, the prologue above overlaps
  // the previous kernel on the stream; nothing of global memory is touched
  // before that kernel has completed.
  griddep_wait();

  // Grouped calls: warp 0 writes the exclusive prefix of the groups' 128-row
  // tiles (clamped as group_rows clamps) for fp8b_unit.
  const int* pre = nullptr;
  int live = 0;
  int units = p.total_units;
  if constexpr (kGrouped) {
    if (p.batch <= Cfg::kMaxPrefixGroups) {
      int* pre_s = reinterpret_cast<int*>(smem + Cfg::kOffPrefix);
      if (warp == 0) {
        int carry = 0;
        for (int base = 0; base < p.batch; base += 32) {
          const int g = base + static_cast<int>(lane);
          int t = 0;
          if (g < p.batch) {
            int row0, rows;
            group_rows(p, g, row0, rows);
            t = (rows + 127) / 128;
          }
          int v = t;   // inclusive warp scan
#pragma unroll
          for (int d = 1; d < 32; d <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, v, d);
            if (static_cast<int>(lane) >= d) v += y;
          }
          if (g < p.batch) pre_s[g] = carry + v - t;
          carry += __shfl_sync(0xffffffffu, v, 31);
        }
        if (lane == 0) pre_s[p.batch] = carry;
      }
      __syncthreads();
      pre = pre_s;
      live = min(pre_s[p.batch], p.tiles_m * p.batch);
      units = live * p.tiles_n;
    }
  }

  if (warp == 0) {
    // producer warp: all lanes run the loop, the elected lane issues the copies
    const bool issuer = elect_one();
    // ------------------------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int last_stage = -1;
    uint32_t last_phase = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int b, mt, nt, s, row0, rows;
      if (!fp8b_unit<kGrouped>(p, pre, live, u, b, mt, nt, s, row0, rows)) continue;
      int a_row = mt * 128, a_batch = b;
      if constexpr (kGrouped) {
        a_row = row0 + mt * 128;
        a_batch = 0;
      }
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        uint64_t* fb = &full_bar[stage];
        if (issuer) {
          mbar_arrive_expect_tx(fb, Cfg::kStageBytes);
          tma_load_3d(sA + stage * Cfg::kABytes, &tmA, fb, kb * 128, a_row, a_batch);
          if constexpr (kBFmt == kFmtKPanel)
            tma_load_4d(sB + stage * Cfg::kBBytes, &tmB, fb, 0, nt * BN, kb, b);
          else if constexpr (kBFmt == kFmtShuffle16)
            tma_load_5d_hint(sB + stage * Cfg::kBBytes, &tmB, fb, 0, kb * 8, 0, nt * (BN / 16), b,
                             l2_policy_evict_first());
          else
            tma_load_3d(sB + stage * Cfg::kBBytes, &tmB, fb, kb * 128, nt * BN, b);
        }
        __syncwarp();
        last_stage = stage;
        last_phase = phase;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && last_stage >= 0) {
      int dummy = 0;
      mbar_wait(&full_bar[last_stage], last_phase, &dummy, p.timeout_ns);
    }
  } else if (warp == 1) {
    // MMA warp: all lanes run the loop, the elected lane issues
    const bool issuer = elect_one();
    // ------------------------------------------------------------------ MMA issuer
    // The descriptors of stage 0 are built once; a stage's are a constant
    // offset from them, so the issue path between two MMAs stays a few adds.
    const uint32_t idesc = idesc_f8f6f4(false, false, 128, BN);
    const uint64_t adesc0 = make_sdesc(smem_u32(sA), 16u, 1024u, kLayoutSW128);
    const uint64_t bdesc0 = weight_sdesc<kBFmt>(smem_u32(sB), 0);
    constexpr uint64_t kBStep = (kBFmt == kFmtShuffle16 ? 256u : 32u) >> 4;   // one K step, 16-byte units
    int stage = 0;
    uint32_t phase = 0;
    uint32_t kbi = 0;   // K blocks issued by this CTA, selects the TMEM buffer
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int b, mt, nt, s, row0, rows;
      if (!fp8b_unit<kGrouped>(p, pre, live, u, b, mt, nt, s, row0, rows)) continue;
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
      for (int kb = kb0; kb < kb1; ++kb, ++kbi) {
        const uint32_t buf = kbi % NB;
        const uint32_t use = kbi / NB;   // how many times this buffer was used before
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (issuer) {
          const uint32_t ust = static_cast<uint32_t>(stage);
          const uint64_t ad = adesc0 + static_cast<uint64_t>(ust * (Cfg::kABytes >> 4));
          const uint64_t bd = bdesc0 + static_cast<uint64_t>(ust * (Cfg::kBBytes >> 4));
          const uint32_t d = tmem_base + buf * BN;
          umma_f8f6f4(d, ad, bd, idesc, 0u);
          umma_f8f6f4(d, ad + 2u, bd + kBStep, idesc, 1u);
          umma_f8f6f4(d, ad + 4u, bd + 2u * kBStep, idesc, 1u);
          umma_f8f6f4(d, ad + 6u, bd + 3u * kBStep, idesc, 1u);
          tc_commit(&empty_bar[stage]);
          tc_commit(&acc_full[buf]);
        }
        __syncwarp();
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (issuer) tc_commit(drain_bar);
    int dummy = 0;
    mbar_wait(drain_bar, 0, &dummy, p.timeout_ns);
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ promotion + store
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    uint32_t kbi = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      // row0, rows: the group's first row and rows (the whole M when not grouped)
      int b, mt, nt, s, row0, rows;
      if (!fp8b_unit<kGrouped>(p, pre, live, u, b, mt, nt, s, row0, rows)) continue;
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
      const int row = mt * 128 + q * 32 + static_cast<int>(lane);
      const bool row_ok = row < rows;
      // a lane quarter whose 32 rows all lie beyond M (decode shapes) skips
      // the promotion work but still releases the buffers
      const bool quarter_live = mt * 128 + q * 32 < rows;
      const int n0 = nt * BN;
      const long long grow = static_cast<long long>(row0) + row;   // row in A, sfa and C
      const float* sfa_row = (kGrouped ? p.sfa : p.sfa + b * p.sfa_batch) + (row_ok ? grow : 0) * p.sfa_m;
      const float* sfb_blk = p.sfb + b * p.sfb_batch + static_cast<long long>(n0 / 128) * p.sfb_n;
      // column pairs as fp32 x 2 for fma.rn.f32x2: half the FMA instructions
      // in each warp's serial promotion round, and the same RN result per
      // element as two fmaf
      uint64_t accp[BN / 2];
#pragma unroll
      for (int i = 0; i < BN / 2; ++i) accp[i] = 0ull;
      float sa_next = row_ok ? __ldg(sfa_row + kb0 * p.sfa_k) : 0.0f;
      float sb_next = __ldg(sfb_blk + kb0 * p.sfb_k);
      for (int kb = kb0; kb < kb1; ++kb, ++kbi) {
        const uint64_t scale2 = pack_f32x2(sa_next * sb_next);
        if (kb + 1 < kb1) {
          sa_next = row_ok ? __ldg(sfa_row + (kb + 1) * p.sfa_k) : 0.0f;
          sb_next = __ldg(sfb_blk + (kb + 1) * p.sfb_k);
        }
        const uint32_t buf = kbi % NB;
        const uint32_t use = kbi / NB;
        if (!mbar_wait(&acc_full[buf], use & 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (quarter_live) {
          // two rounds of four 16-column loads in flight behind one wait
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) {
            uint32_t r[4][16];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tmem_ld16_async(tmem_base + lane_base + buf * BN + static_cast<uint32_t>(c * 64 + j * 16), r[j]);
            tmem_wait_ld16(r[0]);
#pragma unroll
            for (int j = 1; j < 4; ++j) tmem_reg_fence16(r[j]);
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int i = 0; i < 8; ++i) fma_f32x2(accp[(c * 64 + j * 16) / 2 + i], r[j][2 * i], r[j][2 * i + 1], scale2);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      if (!ok) break;
      if (!row_ok) continue;
      float acc[BN];
#pragma unroll
      for (int i = 0; i < BN / 2; ++i) unpack_f32x2(accp[i], acc[2 * i], acc[2 * i + 1]);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        const int col0 = n0 + c * 32;
        if (col0 >= p.n) continue;
        const bool full = col0 + 32 <= p.n;
        if (p.split_k > 1) {
          float* dst = p.ws + ((static_cast<long long>(s) * p.batch + b) * p.m + row) *
                                  static_cast<long long>(p.n) + col0;
          if (full) {
#pragma unroll
            for (int v = 0; v < 8; ++v)
              st_global_v4(dst + 4 * v, __float_as_uint(acc[c * 32 + 4 * v]),
                           __float_as_uint(acc[c * 32 + 4 * v + 1]),
                           __float_as_uint(acc[c * 32 + 4 * v + 2]),
                           __float_as_uint(acc[c * 32 + 4 * v + 3]));
          } else {
            #pragma unroll
            for (int v = 0; v < 32; ++v)
              if (col0 + v < p.n) dst[v] = acc[c * 32 + v];
          }
        } else if constexpr (kOutF32) {
          float* dst = reinterpret_cast<float*>(p.c) + (kGrouped ? 0 : b * p.c_batch_stride) + grow * p.ldc + col0;
          if (full) {
#pragma unroll
            for (int v = 0; v < 8; ++v)
              st_global_v4(dst + 4 * v, __float_as_uint(acc[c * 32 + 4 * v]),
                           __float_as_uint(acc[c * 32 + 4 * v + 1]),
                           __float_as_uint(acc[c * 32 + 4 * v + 2]),
                           __float_as_uint(acc[c * 32 + 4 * v + 3]));
          } else {
            #pragma unroll
            for (int v = 0; v < 32; ++v)
              if (col0 + v < p.n) dst[v] = acc[c * 32 + v];
          }
        } else {
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.c) + (kGrouped ? 0 : b * p.c_batch_stride) + grow * p.ldc + col0;
          if (full) {
            uint32_t w[16];
#pragma unroll
            for (int v = 0; v < 16; ++v) w[v] = pack_bf16x2(acc[c * 32 + 2 * v], acc[c * 32 + 2 * v + 1]);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              st_global_v4(dst + 8 * v, w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
          } else {
            #pragma unroll
              for (int v = 0; v < 32; ++v)
                if (col0 + v < p.n) dst[v] = static_cast<uint16_t>(pack_bf16x2(acc[c * 32 + v], 0.0f) & 0xFFFFu);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace bsg

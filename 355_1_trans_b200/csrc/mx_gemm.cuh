// mx_gemm.cuh -- MXFP8 (E4M3, .kind::mxf8f6f4) and MXFP4 (packed E2M1,
// .kind::mxf4 block32) block-scaled GEMM for sm_100a.
//
// Semantics (reference, paths relative to its project root):
//   mxfp8_gemm/gemm_a8w8_mxfp8_kernel_template.hpp:301-432 with
//   scale_and_accumulate :37-57, and
//   mxfp4_gemm_4wave_20261112/candidate_m10/gemm_a4w4_mxfp4_4wave_kernel_template.hpp:384-1169:
//   C[b,m,n] = sum_g 2^(sfa[m,g]-127) * 2^(sfb[n,g]-127) * sum_{k in g} A[m,k] B[n,k],
//   g = 32 consecutive K, fp32 accumulation, bf16 (RNE) or fp32 output.
//
// Design (one CTA per SM, persistent over output tiles of 128 x BN, grouped
// rasterisation so concurrently running CTAs share A/B panels in L2):
//   warp 0      TMA producer: A/B tiles (128-byte K slabs, 128B swizzle) by
//               tensor maps with L2 cache policies (A evict-last, B
//               evict-first), scale atoms by plain bulk copies; one mbarrier
//               per stage carries the transaction bytes;
//   warp 1      tcgen05 issuer (whole warp runs the loop, one elected lane
//               issues): scale atoms smem -> TMEM with tcgen05.cp into one of
//               two alternating TMEM regions, then 4 block-scaled MMAs per
//               stage into a 128 x BN fp32 TMEM accumulator; tcgen05.commit
//               frees stages;
//   warp 2      TMEM allocator;
//   warps 4-11  epilogue, two warps per TMEM lane quarter (warp w reads lanes
//               32*(w%4).., half of the columns each): the bf16 path drains
//               the whole accumulator into packed registers, releases TMEM at
//               once (the MMA warp starts the next tile) and then streams the
//               stores; fp32 / split-K partial outputs store chunk by chunk.
// The MMA instruction K is 32 (fp8) / 64 (fp4), i.e. 32 bytes of a 128-byte
// swizzled row; one stage holds 128 bytes of K per row (128 fp8 / 256 fp4
// elements) and 1 (fp8) or 2 (fp4) scale atoms per 128 rows.
//
// B operand modes (kBMode):
//   kBKMajor     [N, K] rows, 128B-swizzled K slabs;
//   kBMNMajor    [K, N] rows, 128B-swizzled N slabs (fp8 only);
//   kBShuffle16  the reference's shuffle_weight(16,16) byte layout
//                [N/16][Kbytes/16][16][16] read in place: every 16x16-byte
//                tile is two 8-row x 16-byte core matrices, so a 5-D tensor
//                map (core matrix, K chunk, half, N/16, batch) lands a stage
//                in the canonical no-swizzle K-major layout (K-adjacent core
//                matrices 128 B apart, 8-row groups 1024 B apart).
// Scale modes (kSfMode):
//   kSfNative        per-32-K E8M0 scales as native 512-byte atoms, copied
//                    with bulk copies;
//   kSfE8m0Block128  the reference's launch_blockscale_bpreshuffle scales:
//                    one E8M0 byte per row per 128 K, A's transposed
//                    [K/128][M], B's per 128 x 128 block [N/128][K/128]
//                    (source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:219-248).
//                    Warp 3 rewrites each stage's bytes into atoms with the
//                    byte replicated over the four 32-K groups, so the
//                    block-scaled MMA applies one scale per 128 K.
#pragma once

#include "sm100.cuh"

namespace bsg {

struct MxParams {
  int m, n, k;                   // k in elements
  int batch;
  int num_kb;                    // 128-byte K stages over the whole K
  int tiles_m, tiles_n;
  int split_k, kb_per_split;
  int total_units;               // batch * tiles_m * tiles_n * split_k
  int group_m;                   // rasterisation group (M tiles)
  const uint8_t* sfa;            // native scale atoms
  const uint8_t* sfb;
  long long sfa_batch_stride;    // bytes
  long long sfb_batch_stride;
  int sf_kb_total;               // scale atoms along K per 128-row block
  int sfb_row_blocks;            // 128-row blocks of the B scales, ceil(n / 128)
  long long sfa_ld, sfb_ld;      // kSfE8m0Block128: bytes between K blocks of A's
                                 // scales / between 128-column blocks of B's
  void* c;                       // output
  long long ldc;                 // elements
  long long c_batch_stride;      // elements
  float* ws;                     // split-K partials [split][batch][m][n]
  unsigned long long timeout_ns;
  const int* group_offsets;      // grouped mode: batch + 1 row offsets (device); else unused
  int total_rows;                // grouped mode: rows of A and C over all groups
  const int* tile_prefix;        // grouped mode: batch + 1 exclusive prefix of the groups' M tiles
};

// Grouped mode: group b owns rows group_offsets[b] .. group_offsets[b+1] of A
// and C, clamped to [0, total_rows] and to at most m rows (the tile grid's
// bound), so corrupt or oversized offsets never reach past the tensors.
__device__ __forceinline__ void mx_group_rows(const MxParams& p, int b, int& row0, int& rows) {
  int a0 = __ldg(p.group_offsets + b);
  int a1 = __ldg(p.group_offsets + b + 1);
  a0 = min(max(a0, 0), p.total_rows);
  a1 = min(max(a1, a0), p.total_rows);
  row0 = a0;
  rows = min(a1 - a0, p.m);
}

// Grouped mode enumerates only the M tiles that hold rows: unit u is (global
// M tile gm, N tile nt) over prefix[batch] M tiles (rasterised as a plain
// GEMM of that many M tiles), and gm belongs to the last group e with
// prefix[e] <= gm (empty groups share their successor's prefix), as its M
// tile gm - prefix[e].  Returns false for a tile past the group's rows, which
// the prefix never produces; every role skips such a unit alike.
__device__ __forceinline__ int mx_grouped_units(const MxParams& p) {
  const int live = min(__ldg(p.tile_prefix + p.batch), p.tiles_m * p.batch);
  return max(live, 0) * p.tiles_n;
}

__device__ __forceinline__ bool mx_grouped_unit(const MxParams& p, int u, int& e, int& mt, int& nt, int& row0,
                                                int& rows) {
  const int live = min(__ldg(p.tile_prefix + p.batch), p.tiles_m * p.batch);
  int b, gm, s;
  decode_unit(u, live, p.tiles_n, 1, p.group_m, b, gm, nt, s);
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.tile_prefix + mid) <= gm) lo = mid;
    else hi = mid - 1;
  }
  e = lo;
  mt = gm - __ldg(p.tile_prefix + lo);
  mx_group_rows(p, e, row0, rows);
  return mt >= 0 && mt * 128 < rows;
}

constexpr int kMxThreads = 384;     // 4 control warps + 8 epilogue warps
constexpr int kMxEpiThreads = 256;
constexpr int kMxEpiWarps = 8;      // one tmem_empty arrival per epilogue warp

constexpr int kBKMajor = 0, kBMNMajor = 1, kBShuffle16 = 2;
constexpr int kSfNative = 0, kSfE8m0Block128 = 1;

// Walks the (unit, K block) sequence a persistent CTA (or CTA pair) visits,
// across unit boundaries, so a warp can work several K blocks ahead.
struct KbCursor {
  int u, step, total;
  int tiles_m, tiles_n, split, group_m, kb_per, num_kb;
  int b, mt, nt, kb, kb1;
  __device__ __forceinline__ void settle() {
    while (u < total) {
      int s;
      decode_unit(u, tiles_m, tiles_n, split, group_m, b, mt, nt, s);
      kb = s * kb_per;
      kb1 = min(kb + kb_per, num_kb);
      if (kb < kb1) return;
      u += step;
    }
  }
  __device__ __forceinline__ bool valid() const { return u < total; }
  __device__ __forceinline__ void next() {
    if (++kb >= kb1) {
      u += step;
      settle();
    }
  }
};

__device__ __forceinline__ KbCursor make_cursor(int u0, int step, int total, int tiles_m, int tiles_n,
                                                int split, int group_m, int kb_per, int num_kb) {
  KbCursor c;
  c.u = u0;
  c.step = step;
  c.total = total;
  c.tiles_m = tiles_m;
  c.tiles_n = tiles_n;
  c.split = split;
  c.group_m = group_m;
  c.kb_per = kb_per;
  c.num_kb = num_kb;
  c.b = c.mt = c.nt = c.kb = c.kb1 = 0;
  c.settle();
  return c;
}

// Per-128-K E8M0 scale bytes of one K block: va[j] for A row
// lane + 32 j of the tile, vb[r] for B column block r of the tile.  Rows /
// blocks that do not exist read as 0x7F (2^0); their outputs are never
// stored.  The raw bytes are returned untouched: the first arithmetic use of
// a loaded register waits for the load, so the replication into atom words
// (e8m0_word) happens only when the stage is written, kSfPrefetch K blocks
// later.
template <int NBLK>
__device__ __forceinline__ void e8m0_block_bytes(const uint8_t* sa, int rows, const uint8_t* sb, int nblocks,
                                                 long long sfa_ld, long long sfb_ld, int kb, uint32_t lane,
                                                 uint32_t (&va)[4], uint32_t (&vb)[NBLK]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = static_cast<int>(lane) + 32 * j;
    va[j] = r < rows ? __ldg(sa + kb * sfa_ld + r) : 0x7Fu;
  }
#pragma unroll
  for (int r = 0; r < NBLK; ++r) vb[r] = r < nblocks ? __ldg(sb + r * sfb_ld + kb) : 0x7Fu;
}

// The byte repeated over the four 32-K groups of an atom word.
__device__ __forceinline__ uint32_t e8m0_word(uint32_t byte) { return byte * 0x01010101u; }

constexpr int kSfPrefetch = 4;   // K blocks of scale bytes in flight per builder

template <int BN, int kFp4>
struct MxCfg {
  static constexpr int kBlockM = 128;
  static constexpr int kSfAtomsK = kFp4 ? 2 : 1;           // scale atoms per stage along K
  static constexpr int kSfbRowBlocks = BN / 128;
  static constexpr uint32_t kABytes = 128u * 128u;
  static constexpr uint32_t kBBytes = static_cast<uint32_t>(BN) * 128u;
  static constexpr uint32_t kSfaBytes = 512u * kSfAtomsK;
  static constexpr uint32_t kSfbBytes = 512u * kSfAtomsK * kSfbRowBlocks;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  static constexpr uint32_t kSmemBudget = 225u * 1024u;
  static constexpr int kStages = static_cast<int>((kSmemBudget - 2048u) / kStageBytes) > 8
                                     ? 8
                                     : static_cast<int>((kSmemBudget - 2048u) / kStageBytes);
  // smem: [A x S][B x S][SFA x S][SFB x S][barriers]
  static constexpr uint32_t kOffB = kABytes * kStages;
  static constexpr uint32_t kOffSfa = kOffB + kBBytes * kStages;
  static constexpr uint32_t kOffSfb = kOffSfa + kSfaBytes * kStages;
  static constexpr uint32_t kOffBar = kOffSfb + kSfbBytes * kStages;
  static constexpr uint32_t kSmemBytes = kOffBar + 256u + 1024u;  // + alignment slack
  // TMEM columns: accumulator [0, BN), then two alternating scale-factor
  // regions (SFA: 4 columns per K atom, SFB: 4 per K atom and 128 rows), so
  // the scale copy of stage k+1 never overwrites columns the MMAs of stage k
  // are still reading.
  static constexpr uint32_t kSfRegionCols = 4u * kSfAtomsK * (1 + kSfbRowBlocks);
  static constexpr uint32_t kColSfa = BN;
  static constexpr uint32_t kColSfb = BN + 4u * kSfAtomsK;
  static constexpr uint32_t kColsUsed = BN + 2u * kSfRegionCols;
  static constexpr uint32_t kTmemCols = kColsUsed <= 32 ? 32 : kColsUsed <= 64 ? 64
                                        : kColsUsed <= 128 ? 128 : kColsUsed <= 256 ? 256 : 512;
  static constexpr int kHalfCols = BN / 2;   // columns per epilogue warp
  static_assert(kStages >= 2, "shared memory too small for two stages");
  static_assert(kColsUsed <= 512, "TMEM overflow");
};

// Store 32 fp32 accumulator columns of one row (fp32 output or split-K partial).
__device__ __forceinline__ void store_row32_f32(float* dst, const uint32_t (&r)[32], int valid) {
  if (valid >= 32) {
#pragma unroll
    for (int v = 0; v < 8; ++v) st_global_cs_v4(dst + 4 * v, r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
  } else {
#pragma unroll
    for (int v = 0; v < 32; ++v)
      if (v < valid) dst[v] = __uint_as_float(r[v]);
  }
}

// kGrouped: the batch index is a group (expert) whose rows of A and C start
// at group_offsets[b] (mx_group_rows); A is one [total_rows, K] matrix, the
// group's A scales are native atoms at batch stride sfa_batch_stride (packed
// per group), and the units are only the M tiles that hold rows
// (mx_grouped_unit), so the persistent grid stays balanced however ragged
// the groups are.
template <int BN, int kFp4, bool kAMN, int kBMode, bool kOutF32, int kSfMode, bool kGrouped = false>
__global__ void __launch_bounds__(kMxThreads, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const MxParams p) {
  using Cfg = MxCfg<BN, kFp4>;
  constexpr int S = Cfg::kStages;
  constexpr bool kBMN = kBMode == kBMNMajor;
  constexpr bool kBuildSf = kSfMode == kSfE8m0Block128;
  static_assert(!kBuildSf || !kFp4, "per-128 E8M0 scales are an fp8 format");
  static_assert(!kGrouped || (!kBuildSf && !kAMN), "grouped mode: K-major A, native scales");

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled operand tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::kOffB;
  uint8_t* sSfa = smem + Cfg::kOffSfa;
  uint8_t* sSfb = smem + Cfg::kOffSfb;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tmem_full = empty_bar + S;
  uint64_t* tmem_empty = tmem_full + 1;
  uint64_t* drain_bar = tmem_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;

  if (threadIdx.x == 32) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], kBuildSf ? 2 : 1);   // + the scale builder's arrival
      mbar_init(&empty_bar[i], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, kMxEpiWarps);
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

  if (warp == 0) {
    // producer warp: all lanes run the loop, the elected lane issues the copies
    const bool issuer = elect_one();
    // ------------------------------------------------------------------ TMA producer
    const uint64_t pol_a = l2_policy_evict_last();
    const uint64_t pol_b = l2_policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int last_stage = -1;
    uint32_t last_phase = 0;
    const int units = kGrouped ? mx_grouped_units(p) : p.total_units;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int b, mt, nt, s = 0;
      int a_row, a_batch;
      if constexpr (kGrouped) {
        int row0, rows;
        if (!mx_grouped_unit(p, u, b, mt, nt, row0, rows)) continue;
        a_row = row0 + mt * 128;
        a_batch = 0;
      } else {
        decode_unit(u, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
        a_row = mt * 128;
        a_batch = b;
      }
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
      const uint8_t* sfa_tile = p.sfa + b * p.sfa_batch_stride +
                                static_cast<long long>(mt) * p.sf_kb_total * 512;
      const uint8_t* sfb_tile = p.sfb + b * p.sfb_batch_stride +
                                static_cast<long long>(nt) * Cfg::kSfbRowBlocks * p.sf_kb_total * 512;
      // the last N tile may cover fewer 128-row scale blocks than BN / 128;
      // copy only the ones that exist (the columns beyond N are never stored)
      const int sfb_rows = min(Cfg::kSfbRowBlocks, p.sfb_row_blocks - nt * Cfg::kSfbRowBlocks);
      const uint32_t tx_bytes =
          kBuildSf ? Cfg::kABytes + Cfg::kBBytes
                   : Cfg::kStageBytes - static_cast<uint32_t>(Cfg::kSfbRowBlocks - sfb_rows) * 512u * Cfg::kSfAtomsK;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        uint64_t* fb = &full_bar[stage];
        if (issuer) mbar_arrive_expect_tx(fb, tx_bytes);
        uint8_t* a_dst = sA + stage * Cfg::kABytes;
        uint8_t* b_dst = sB + stage * Cfg::kBBytes;
        const int kbyte = kb * 128;
        if (issuer) {
          if constexpr (!kAMN) {
            tma_load_3d_hint(a_dst, &tmA, fb, kbyte, a_row, a_batch, pol_a);
          } else {
            tma_load_3d_hint(a_dst, &tmA, fb, a_row, kbyte, a_batch, pol_a);
          }
          if constexpr (kBMode == kBKMajor) {
            tma_load_3d_hint(b_dst, &tmB, fb, kbyte, nt * BN, b, pol_b);
          } else if constexpr (kBMode == kBShuffle16) {
            // (core-matrix byte, 16-byte K chunk, half, 16-row group, batch)
            tma_load_5d_hint(b_dst, &tmB, fb, 0, kb * 8, 0, nt * (BN / 16), b, pol_b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tma_load_3d_hint(b_dst + j * 16384, &tmB, fb, nt * BN + j * 128, kbyte, b, pol_b);
          }
          if constexpr (!kBuildSf) {
            const long long atom_k = static_cast<long long>(kb) * Cfg::kSfAtomsK;
            bulk_load(sSfa + stage * Cfg::kSfaBytes, sfa_tile + atom_k * 512, Cfg::kSfaBytes, fb);
#pragma unroll
            for (int r = 0; r < Cfg::kSfbRowBlocks; ++r)
              if (r < sfb_rows)
                bulk_load(sSfb + stage * Cfg::kSfbBytes + r * 512 * Cfg::kSfAtomsK,
                          sfb_tile + (static_cast<long long>(r) * p.sf_kb_total + atom_k) * 512,
                          512u * Cfg::kSfAtomsK, fb);
          }
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
      // give the copies already in flight a bounded chance to land before exit
      int dummy = 0;
      mbar_wait(&full_bar[last_stage], last_phase, &dummy, p.timeout_ns);
    }
  } else if (warp == 1) {
    // MMA warp: all lanes run the loop, the elected lane issues
    const bool issuer = elect_one();
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t kFmt = kFp4 ? 1u : 0u;
    constexpr uint32_t idesc0 = idesc_block_scaled(kFmt, kFmt, kAMN, kBMN, 128, BN);
    // K-major: SBO = 8 rows x 128 B; MN-major: LBO = next 128-element MN slab,
    // SBO = next 8 K rows.
    // Shuffled B (no swizzle): LBO = next 16-byte K chunk (128 B), SBO = next
    // 8-row group (1024 B), one MMA step = two K chunks.
    constexpr bool kBShuf = kBMode == kBShuffle16;
    constexpr uint32_t kALbo = kAMN ? 128u * 128u : 16u;
    constexpr uint32_t kBLbo = kBMN ? 128u * 128u : kBShuf ? 128u : 16u;
    constexpr uint32_t kSbo = 1024u;
    constexpr uint32_t kKStep = kAMN ? 32u * 128u : 32u;   // bytes per MMA along K (A)
    constexpr uint32_t kKStepB = kBMN ? 32u * 128u : kBShuf ? 256u : 32u;
    constexpr uint32_t kBLayout = kBShuf ? kLayoutNone : kLayoutSW128;
    // The descriptors of stage 0 are built once; a stage's are a constant
    // offset from them, so the issue path between two MMAs stays a few adds
    // (at N <= 128 the tensor pipe outruns a longer issue path).
    const uint64_t adesc0 = make_sdesc(smem_u32(sA), kALbo, kSbo, kLayoutSW128);
    const uint64_t bdesc0 = make_sdesc(smem_u32(sB), kBLbo, kSbo, kBLayout);
    const uint32_t sSfa0 = smem_u32(sSfa), sSfb0 = smem_u32(sSfb);
    int stage = 0;
    uint32_t phase = 0;
    int iter = 0;
    uint32_t sf_region = 0;   // alternates every stage
    bool ok = true;
    const int units = kGrouped ? mx_grouped_units(p) : p.total_units;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int b, mt, nt, s = 0;
      if constexpr (kGrouped) {
        int row0, rows;
        if (!mx_grouped_unit(p, u, b, mt, nt, row0, rows)) continue;   // uses no accumulator phase
      } else {
        decode_unit(u, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
      }
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
      if (!mbar_wait(tmem_empty, (static_cast<uint32_t>(iter) & 1u) ^ 1u, abort_flag,
                     p.timeout_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tsf = tmem_base + sf_region * Cfg::kSfRegionCols;
        sf_region ^= 1u;
        if (issuer) {
          const uint32_t ust = static_cast<uint32_t>(stage);
#pragma unroll
          for (int j = 0; j < Cfg::kSfAtomsK; ++j) {
            tmem_cp_sf_atom(tsf + Cfg::kColSfa + 4u * j, sSfa0 + ust * Cfg::kSfaBytes + 512u * j);
#pragma unroll
            for (int r = 0; r < Cfg::kSfbRowBlocks; ++r)
              tmem_cp_sf_atom(tsf + Cfg::kColSfb + 4u * (j * Cfg::kSfbRowBlocks + r),
                              sSfb0 + ust * Cfg::kSfbBytes + 512u * (r * Cfg::kSfAtomsK + j));
          }
          const uint64_t ad = adesc0 + static_cast<uint64_t>(ust * (Cfg::kABytes >> 4));
          const uint64_t bd = bdesc0 + static_cast<uint64_t>(ust * (Cfg::kBBytes >> 4));
          const uint32_t acc0 = kb > kb0 ? 1u : 0u;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t j = kFp4 ? static_cast<uint32_t>(t >> 1) : 0u;
            const uint32_t sf_id = kFp4 ? static_cast<uint32_t>((t & 1) * 2) : static_cast<uint32_t>(t);
            const uint64_t adesc = ad + static_cast<uint64_t>((t * kKStep) >> 4);
            const uint64_t bdesc = bd + static_cast<uint64_t>((t * kKStepB) >> 4);
            const uint32_t idesc = idesc_with_sf_id(idesc0, sf_id, sf_id);
            const uint32_t tsfa = tsf + Cfg::kColSfa + 4u * j;
            const uint32_t tsfb = tsf + Cfg::kColSfb + 4u * j * Cfg::kSfbRowBlocks;
            const uint32_t acc = t > 0 ? 1u : acc0;
            if constexpr (kFp4)
              umma_mxf4(tmem_base, adesc, bdesc, idesc, tsfa, tsfb, acc);
            else
              umma_mxf8f6f4(tmem_base, adesc, bdesc, idesc, tsfa, tsfb, acc);
          }
        }
        if (issuer) tc_commit(&empty_bar[stage]);
        __syncwarp();
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (issuer) tc_commit(tmem_full);
      ++iter;
    }
    // drain: wait until every tcgen05 op issued above has completed
    if (issuer) tc_commit(drain_bar);
    int dummy = 0;
    mbar_wait(drain_bar, 0, &dummy, p.timeout_ns);
  } else if (warp == 3) {
    if constexpr (kBuildSf) {
      // -------------------------------------------------------------- scale builder
      // Lane l owns 16 bytes of each atom: the words of rows l, l+32, l+64,
      // l+96.  The bytes of the next kSfPrefetch K blocks are in flight in a
      // register ring (statically indexed by unrolling), so global-load
      // latency never stalls the pipeline.
      constexpr int D = kSfPrefetch;
      constexpr int NBLK = Cfg::kSfbRowBlocks;
      KbCursor issue = make_cursor(blockIdx.x, gridDim.x, p.total_units, p.tiles_m, p.tiles_n, p.split_k,
                                   p.group_m, p.kb_per_split, p.num_kb);
      KbCursor cons = issue;
      uint32_t ra[D][4], rb[D][NBLK];
      auto load = [&](const KbCursor& c, uint32_t (&va)[4], uint32_t (&vb)[NBLK]) {
        const uint8_t* sa = p.sfa + c.b * p.sfa_batch_stride + c.mt * 128;
        const uint8_t* sb = p.sfb + c.b * p.sfb_batch_stride + static_cast<long long>(c.nt) * NBLK * p.sfb_ld;
        e8m0_block_bytes<NBLK>(sa, p.m - c.mt * 128, sb, min(NBLK, p.sfb_row_blocks - c.nt * NBLK), p.sfa_ld,
                               p.sfb_ld, c.kb, lane, va, vb);
      };
#pragma unroll
      for (int i = 0; i < D; ++i)
        if (issue.valid()) {
          load(issue, ra[i], rb[i]);
          issue.next();
        }
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      while (ok && cons.valid()) {
#pragma unroll
        for (int i = 0; i < D; ++i) {
          if (!cons.valid()) break;
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.timeout_ns)) {
            ok = false;
            break;
          }
          st_shared_v4(sSfa + stage * Cfg::kSfaBytes + lane * 16u, e8m0_word(ra[i][0]), e8m0_word(ra[i][1]),
                       e8m0_word(ra[i][2]), e8m0_word(ra[i][3]));
#pragma unroll
          for (int r = 0; r < NBLK; ++r) {
            const uint32_t w = e8m0_word(rb[i][r]);
            st_shared_v4(sSfb + stage * Cfg::kSfbBytes + r * 512 + lane * 16u, w, w, w, w);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full_bar[stage]);
          if (issue.valid()) {
            load(issue, ra[i], rb[i]);
            issue.next();
          }
          cons.next();
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    constexpr int HC = Cfg::kHalfCols;
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const uint32_t t_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(half * HC);
    int iter = 0;
    const int units = kGrouped ? mx_grouped_units(p) : p.total_units;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int b, mt, nt, s = 0;
      int row0 = 0, rows = p.m;   // the group's first row and rows (all of M when not grouped)
      if constexpr (kGrouped) {
        if (!mx_grouped_unit(p, u, b, mt, nt, row0, rows)) continue;
      } else {
        decode_unit(u, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
      }
      if (!mbar_wait(tmem_full, static_cast<uint32_t>(iter) & 1u, abort_flag, p.timeout_ns)) break;
      ++iter;
      tc_fence_after();
      const int row = mt * 128 + q * 32 + static_cast<int>(lane);
      const bool row_ok = row < rows;
      // C row of this lane and the batch's C origin (a group's rows live in one C)
      const long long crow = static_cast<long long>(row0) + row;
      const long long cbatch = kGrouped ? 0 : b * p.c_batch_stride;
      const int col_base = nt * BN + half * HC;
      const int valid_cols = p.n - col_base;   // may be <= 0 or > HC
      if (p.split_k > 1 || kOutF32) {
        float* dst = p.split_k > 1
                         ? p.ws + ((static_cast<long long>(s) * p.batch + b) * p.m + row) *
                                      static_cast<long long>(p.n) + col_base
                         : reinterpret_cast<float*>(p.c) + cbatch + crow * p.ldc + col_base;
#pragma unroll 1
        for (int c = 0; c < HC / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(t_base + static_cast<uint32_t>(c * 32), r);
          if (row_ok && valid_cols > c * 32) store_row32_f32(dst + c * 32, r, valid_cols - c * 32);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tmem_empty);
      } else {
        // drain the whole half-row into packed bf16 registers, release the
        // accumulator, then store
        uint32_t w[HC / 2];
#pragma unroll
        for (int c = 0; c < HC / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(t_base + static_cast<uint32_t>(c * 32), r);
#pragma unroll
          for (int v = 0; v < 16; ++v)
            w[c * 16 + v] = pack_bf16x2(__uint_as_float(r[2 * v]), __uint_as_float(r[2 * v + 1]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tmem_empty);
        if (row_ok && valid_cols > 0) {
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.c) + cbatch + crow * p.ldc + col_base;
          if (valid_cols >= HC) {
#pragma unroll
            for (int v = 0; v < HC / 8; ++v)
              st_global_cs_v4(dst + 8 * v, w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
          } else {
#pragma unroll
            for (int v = 0; v < HC / 2; ++v) {
              if (2 * v < valid_cols) dst[2 * v] = static_cast<uint16_t>(w[v] & 0xFFFFu);
              if (2 * v + 1 < valid_cols) dst[2 * v + 1] = static_cast<uint16_t>(w[v] >> 16);
            }
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

// Deterministic split-K reduction: C = sum_{s=0..S-1} ws[s] in fixed order.
template <bool kOutF32>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, void* __restrict__ c, int m,
                                     int n, int batch, int split, long long ldc,
                                     long long c_batch_stride) {
  griddep_wait();   // launched programmatically behind the GEMM: wait for its partials
  const long long per_batch = static_cast<long long>(m) * n;
  const long long total4 = per_batch * batch / 4;   // n % 4 == 0
  const long long slice = per_batch * batch;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = i * 4;
    // up to 8 slices' loads in flight at once, summed in slice order
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int s0 = 0; s0 < split; s0 += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < split) v[j] = __ldcg(reinterpret_cast<const float4*>(ws + (s0 + j) * slice) + i);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (s0 + j >= split) break;
        if (s0 + j == 0) {
          acc = v[0];
        } else {
          acc.x += v[j].x;
          acc.y += v[j].y;
          acc.z += v[j].z;
          acc.w += v[j].w;
        }
      }
    }
    const long long bb = e / per_batch;
    const long long rem = e - bb * per_batch;
    const long long row = rem / n, col = rem - row * n;
    if constexpr (kOutF32) {
      float* dst = reinterpret_cast<float*>(c) + bb * c_batch_stride + row * ldc + col;
      *reinterpret_cast<float4*>(dst) = acc;
    } else {
      uint16_t* dst = reinterpret_cast<uint16_t*>(c) + bb * c_batch_stride + row * ldc + col;
      uint2 w;
      w.x = pack_bf16x2(acc.x, acc.y);
      w.y = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(dst) = w;
    }
  }
}

}  // namespace bsg

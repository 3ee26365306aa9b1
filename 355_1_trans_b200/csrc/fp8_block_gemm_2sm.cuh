// fp8_block_gemm_2sm.cuh -- CTA-pair (tcgen05 cta_group::2) variant of the
// FP8 GEMM with fp32 block scales: a cluster of two CTAs on two SMs computes
// one 256 x 256 output tile.
//
// Semantics are those of fp8_block_gemm.cuh (reference, paths relative to its
// project root: block_scale_gemm_bpreshuffle/
// gemm_a8w8_blockscale_bpreshuffle_kernel_template.hpp:204-601): per 128-K
// block kb the unscaled partial (A B^T)_kb is multiplied by
// sfa[m,kb] * sfb[n/128,kb] and added to an fp32 accumulator, in the same
// order and with the same fma.rn as the 1-CTA kernel, so the two agree bit for
// bit.
//
// Why pairs of 256 x 256: the 1-CTA kernel's operand pipeline alone (its
// promotion switched off) reaches 0.57 of the FP8 peak with 128 x 128 tiles,
// and a pair of 256 x 128 tiles 0.64.  Here each SM loads 128 rows of A and
// 128 of the tile's 256 B rows per 128-K stage (32 KB) and owns a 128 x 256
// fp32 partial per K block -- twice the MMA work per stage and per hand-off --
// which is the MX pair kernel's shape (0.86 of the peak).  TMEM holds two such
// partials (2 x 256 columns), so the MMA runs one K block ahead of the
// promotion.
//
// Protocol (rank 0 = leader, rank 1 = peer; identical shared-memory layout;
// 384 threads: warpgroup 0 at 56 registers, warpgroups 1-2 at 224):
//   producer (warp 0, both CTAs)  waits its own empty[s]; loads its A rows and
//       its B rows with the pair form of the TMA load, whose transaction bytes
//       go to the LEADER's full[s]; the leader arms full[s] with both CTAs'
//       bytes;
//   MMA (warp 1 of the leader)     per K block waits acc_empty[buf] (sixteen
//       arrivals: eight promotion warps in each CTA) and full[s], issues four
//       pair MMAs (M = 256, N = 256, K = 32 each) into TMEM buffer buf of both
//       CTAs, and commits to empty[s] and acc_full[buf] of both CTAs;
//   promotion (warps 4-11, both)   warp w promotes lane quarter w % 4 and
//       column half (w - 4) / 4 (128 columns, one B-scale block) of the CTA's
//       own 128 rows, as the 1-CTA kernel does, then releases the buffer by a
//       relaxed arrive on the leader's acc_empty[buf].  The hand-off publishes
//       no memory: the warp's tcgen05.ld of the buffer have completed
//       (tcgen05.wait::ld) before it arrives.  With a cluster-scope release
//       (which waits for the warp's loads and stores in flight) and a
//       cluster-scope acquire on the MMA side, the 256 x 128 pair kernel ran at
//       576 and 1182 TFLOPS against 1612 relaxed.  The MMA waits for the
//       slowest of the sixteen warps, so each warp polls for its buffer
//       (mbar_wait_spin) and has its scales loaded four K blocks ahead.
//       After a unit's last K block: bf16 C through per-warp staging boxes
//       and TMA stores (fp32 C, and grouped calls, store each lane's row).
// The producer prefetches the next unit's first K blocks into L2 before the
// current unit ends.  The partial last wave of units can run as K slices
// (pair_item); their fp32 partials are summed by
// fp8b_pair_tail_reduce_kernel.  Grouped (MoE) calls enumerate live 256-row
// tiles per group (pair_work).  Every wait is bounded (sm100.cuh mbar_wait).
//
// The same body, with kPair false, is the wide single-CTA kernel
// (fp8_block_gemm_wide_kernel, on request): one CTA per 128 x 256 unit, the
// unit's 256 B rows loaded as two 128-row boxes per stage, single-CTA MMAs
// (M = 128, N = 256) and commits, and K split by cutting every unit into the
// same number of slices (the tail-slice mechanism with all units as tail).
// Whole units give the 1-CTA kernel's bits.  Per K block it costs what its
// area predicts (about 1.1 µs at 112 CTAs on 18432-deep K against 0.52 for a
// 128 x 128 tile), so it pays only where it needs fewer rounds of units
// (M=128 N=24576 K=1536: 14.1 against 17.5 µs).  Tiles of 72 rows or fewer
// run much slower for a reason not found (M=72 N=65536 K=1536: 44.9 against
// 28.6 µs), so neither the automatic choice nor the tuner uses it.
#pragma once

#include "fp8_block_gemm.cuh"

namespace bsg {

// kPair: the CTA-pair kernel (256 x 256 units over two SMs).  Otherwise the
// wide single-CTA kernel: one CTA computes a 128 x 256 unit with the same
// warp roles, promotion and epilogue; per 128-K stage it loads 128 rows of A
// and all 256 B rows (48 KB, 4 stages).
template <bool kPair = true>
struct Fp8Block2Cfg {
  static constexpr int kThreads = 384;
  static constexpr int kLaunchRegs = 168;      // 384 x 168 = 128 x 56 + 256 x 224
  static constexpr uint32_t kLowRegs = 56u;    // warpgroup 0: producer, MMA, TMEM allocation
  static constexpr uint32_t kHighRegs = 224u;  // warpgroups 1-2: promotion
  static_assert(128u * kLowRegs + 256u * kHighRegs <= static_cast<uint32_t>(kThreads * kLaunchRegs),
                "register split exceeds the launch");
  static constexpr uint32_t kABytes = 128u * 128u;   // this CTA's 128 rows of A, one 128-K block
  // the pair: this CTA's 128 of the tile's 256 B rows; wide: all 256
  static constexpr uint32_t kBBytes = (kPair ? 128u : 256u) * 128u;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kPair ? 6 : 4;
  static constexpr int kTileRows = kPair ? 256 : 128;   // output rows of one unit
  // a K slice's partial: one unit of fp32, row-major with 256 columns
  static constexpr long long kSlotFloats = static_cast<long long>(kTileRows) * 256LL;
  static constexpr uint32_t kOffB = kABytes * kStages;
  // bf16 epilogue staging: two 32-row x 32-column boxes (64-byte rows) per promotion warp
  static constexpr uint32_t kOutBytes = 32u * 64u;
  static constexpr uint32_t kOffOut = kOffB + kBBytes * kStages;
  static constexpr uint32_t kOffBar = kOffOut + 8u * 2u * kOutBytes;
  // grouped calls: the groups' pair-tile prefix lives in the staging area
  // (grouped calls store C with row masks, not through it)
  static constexpr int kMaxPrefixGroups = 1024;
  static_assert(4u * (kMaxPrefixGroups + 1) <= 8u * 2u * kOutBytes, "prefix does not fit the staging area");
  // next unit's first K blocks prefetched into L2, this many K blocks before the unit ends
  static constexpr int kPrefetchKb = 8;
  static constexpr int kPrefetchLead = 16;
  static constexpr uint32_t kSmemBytes = kOffBar + 256u + 1024u;
  static constexpr int kAccBufs = 2;
  static constexpr uint32_t kBN = 256u;
  static constexpr uint32_t kTmemCols = kAccBufs * kBN;
  static_assert(kSmemBytes <= 227u * 1024u, "shared memory");
  static_assert(kOffB % 1024u == 0 && kOffOut % 1024u == 0, "swizzled tiles need 1024-byte alignment");
  static_assert(kTmemCols <= 512u, "TMEM overflow");
};

// Stores one lane's row of a 128-column tile: acc[0..127] to columns
// [n0, n0 + 128) of `dst_row` (bf16 RNE or fp32), clipped at n.
template <bool kOutF32>
__device__ __forceinline__ void store_row128(const float (&acc)[128], void* dst_row, int n0, int n) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int col0 = n0 + c * 32;
    if (col0 >= n) continue;
    const bool full = col0 + 32 <= n;
    if constexpr (kOutF32) {
      float* dst = reinterpret_cast<float*>(dst_row) + col0;
      if (full) {
#pragma unroll
        for (int v = 0; v < 8; ++v)
          st_global_v4(dst + 4 * v, __float_as_uint(acc[c * 32 + 4 * v]), __float_as_uint(acc[c * 32 + 4 * v + 1]),
                       __float_as_uint(acc[c * 32 + 4 * v + 2]), __float_as_uint(acc[c * 32 + 4 * v + 3]));
      } else {
#pragma unroll
        for (int v = 0; v < 32; ++v)
          if (col0 + v < n) dst[v] = acc[c * 32 + v];
      }
    } else {
      uint16_t* dst = reinterpret_cast<uint16_t*>(dst_row) + col0;
      if (full) {
        uint32_t w[16];
#pragma unroll
        for (int v = 0; v < 16; ++v) w[v] = pack_bf16x2(acc[c * 32 + 2 * v], acc[c * 32 + 2 * v + 1]);
#pragma unroll
        for (int v = 0; v < 4; ++v) st_global_v4(dst + 8 * v, w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
      } else {
#pragma unroll
        for (int v = 0; v < 32; ++v)
          if (col0 + v < n) dst[v] = static_cast<uint16_t>(pack_bf16x2(acc[c * 32 + v], 0.0f) & 0xFFFFu);
      }
    }
  }
}

// Work item w of a pair launch: the whole units first (unit w, every K
// block), then the K slices of the last p.tail_units units, p.tail_split per
// unit (slice j covers K blocks [j*nkb/s, (j+1)*nkb/s)).  A persistent grid
// of C clusters thus runs its full waves of whole units and then spreads the
// tail over every cluster instead of leaving most of them idle for a whole
// unit's time.  slot: -1 for a whole unit, else the slice's fp32 partial slot.
struct PairItem {
  int unit, kb0, kb1, slot;
};
__device__ __forceinline__ PairItem pair_item(const Fp8BlockParams& p, int w) {
  const int whole = p.total_units - p.tail_units;
  PairItem it;
  if (w < whole) {
    it.unit = w;
    it.kb0 = 0;
    it.kb1 = p.num_kb;
    it.slot = -1;
    return it;
  }
  const int t = w - whole;
  const int j = t % p.tail_split;
  it.unit = whole + t / p.tail_split;
  it.kb0 = j * p.num_kb / p.tail_split;
  it.kb1 = (j + 1) * p.num_kb / p.tail_split;
  it.slot = t;
  return it;
}

// The work of item w, the same for every role: batch (group) b, pair M tile
// mt, N tile nt, K blocks [kb0, kb1), tail slot (-1: none) and the rows it
// covers, [row0, row0 + rows) of A, sfa and C (row0 = 0, rows = M unless
// grouped).  Grouped calls (no tail slices) enumerate, with the groups'
// 256-row tile prefix `pre` in shared memory (live_tiles of them), only the
// tiles that hold rows: tile gm belongs to the last group e with pre[e] <= gm.
// Without the prefix they decode the full grid; false marks a tile past its
// group's rows, which every role skips.
struct PairWork {
  int b, mt, nt, kb0, kb1, slot, row0, rows;
};
template <bool kGrouped>
__device__ __forceinline__ bool pair_work(const Fp8BlockParams& p, const int* pre, int live_tiles, int w,
                                          PairWork& x) {
  int s;
  if constexpr (kGrouped) {
    x.kb0 = 0;
    x.kb1 = p.num_kb;
    x.slot = -1;
    if (pre != nullptr) {
      int gb, gm;
      decode_unit(w, live_tiles, p.tiles_n, 1, p.group_m, gb, gm, x.nt, s);
      int lo = 0, hi = p.batch - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= gm) lo = mid;
        else hi = mid - 1;
      }
      x.b = lo;
      x.mt = gm - pre[lo];
    } else {
      decode_unit(w, p.tiles_m, p.tiles_n, 1, p.group_m, x.b, x.mt, x.nt, s);
    }
    group_rows(p, x.b, x.row0, x.rows);
    return x.mt >= 0 && x.mt * 256 < x.rows;
  } else {
    const PairItem it = pair_item(p, w);
    decode_unit(it.unit, p.tiles_m, p.tiles_n, 1, p.group_m, x.b, x.mt, x.nt, s);
    x.kb0 = it.kb0;
    x.kb1 = it.kb1;
    x.slot = it.slot;
    x.row0 = 0;
    x.rows = p.m;
    return true;
  }
}

// p.tiles_m counts 256-row pair tiles, p.tiles_n 256-column tiles; split_k 1
// (the tail slices above are the only K split).  kGrouped: the batch index is
// a group (expert) whose rows of A, sfa and C start at group_offsets[b] (A's
// tensor map spans all total_rows); B and sfb keep their per-group strides.
//
// kPair false (the wide kernel, fp8_block_gemm_wide_kernel): p.tiles_m counts
// 128-row tiles; each CTA is its own "cluster" of one, so the pair-only steps
// (pair TMA loads and MMAs, multicast commits, the pair TMEM allocation and
// cluster barriers) become their single-CTA forms, and every CTA issues its
// own MMAs.  Not used for grouped calls.
template <int kBFmt, bool kOutF32, bool kGrouped, bool kPair>
__device__ __forceinline__ void fp8b2_body(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                                           const Fp8BlockParams& p) {
  static_assert(kPair || !kGrouped, "the wide kernel has no grouped mode");
  using Cfg = Fp8Block2Cfg<kPair>;
  constexpr int TR = Cfg::kTileRows;
  constexpr int S = Cfg::kStages;
  constexpr int NB = Cfg::kAccBufs;
  constexpr uint32_t BN = Cfg::kBN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::kOffB;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* acc_full = empty_bar + S;    // [NB]
  uint64_t* acc_empty = acc_full + NB;   // [NB], the leader's are used
  uint64_t* drain_bar = acc_empty + NB;
  static_assert(8 * (2 * S + 2 * NB + 1) + 8 <= 256, "barrier area");
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;

  if (threadIdx.x == 32) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kPair ? 16 : 8);   // eight promotion warps in each CTA
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_holder, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if constexpr (!kOutF32 && !kGrouped) prefetch_tmap(&tmC);
  }
  tc_fence_before();
  if constexpr (kPair)
    cluster_sync_all();   // barriers of both CTAs initialised, TMEM allocated
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (threadIdx.x == 0) griddep_launch_dependents();   // the next kernel's prologue may start
  // Launched with programmatic dependent launch, the prologue above overlaps
  // the previous kernel on the stream; nothing of global memory is touched
  // before that kernel has completed.
  griddep_wait();
  const int cluster_id = static_cast<int>(kPair ? blockIdx.x >> 1 : blockIdx.x);
  const int num_clusters = static_cast<int>(kPair ? gridDim.x >> 1 : gridDim.x);

  // Grouped calls: warp 0 writes the exclusive prefix of the groups' 256-row
  // tiles (clamped as group_rows clamps); both CTAs of a pair compute the same.
  const int* pre = nullptr;
  int live_tiles = 0;
  int n_items = p.total_items;
  if constexpr (kGrouped) {
    n_items = p.total_units;
    if (p.batch <= Cfg::kMaxPrefixGroups) {
      int* pre_s = reinterpret_cast<int*>(smem + Cfg::kOffOut);
      if (warp == 0) {
        int carry = 0;
        for (int base = 0; base < p.batch; base += 32) {
          const int g = base + static_cast<int>(lane);
          int t = 0;
          if (g < p.batch) {
            int row0, rows;
            group_rows(p, g, row0, rows);
            t = (rows + 255) / 256;
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
      live_tiles = min(pre_s[p.batch], p.tiles_m * p.batch);
      n_items = live_tiles * p.tiles_n;
    }
  }

  if (warp < 4) {
    setmaxnreg_dec<Cfg::kLowRegs>();
    if (warp == 0) {
      // producer warp: all lanes run the loop, the elected lane issues the copies
      const bool issuer = elect_one();
      // ---------------------------------------------------------------- TMA producer (both CTAs)
      const uint64_t pol = l2_policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      for (int w = cluster_id; w < n_items; w += num_clusters) {
        PairWork x;
        if (!pair_work<kGrouped>(p, pre, live_tiles, w, x)) continue;
        const PairWork& it = x;
        const int b = x.b;
        const int a_batch = kGrouped ? 0 : x.b;
        const int row_a = x.row0 + x.mt * TR + static_cast<int>(rank) * 128;
        const int row_b = x.nt * 256 + static_cast<int>(rank) * 128;   // wide: the first of two 128-row boxes
        // every cluster reaches its next unit at about the same time, and the
        // new unit's A or B panel is often not in L2 yet: this CTA's operands of
        // that unit's first K blocks go to L2 a while before they are needed
        const int wn = w + num_clusters;
        const int kb_pf = max(it.kb0, it.kb1 - Cfg::kPrefetchLead);
        bool ok = true;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
          PairWork nx;
          if (kb == kb_pf && wn < n_items && issuer && pair_work<kGrouped>(p, pre, live_tiles, wn, nx)) {
            const int b2 = nx.b;
            const int ra = nx.row0 + nx.mt * TR + static_cast<int>(rank) * 128;
            for (int k2 = nx.kb0; k2 < min(nx.kb0 + Cfg::kPrefetchKb, nx.kb1); ++k2) {
              if (ra < (kGrouped ? p.total_rows : p.m)) tma_prefetch_3d(&tmA, k2 * 128, ra, kGrouped ? 0 : b2);
#pragma unroll
              for (int h = 0; h < (kPair ? 1 : 2); ++h) {
                const int rb = nx.nt * 256 + static_cast<int>(rank) * 128 + h * 128;
                if (rb >= p.n) continue;
                if constexpr (kBFmt == kFmtKPanel)
                  tma_prefetch_4d(&tmB, 0, rb, k2, b2);
                else if constexpr (kBFmt == kFmtShuffle16)
                  tma_prefetch_5d(&tmB, 0, k2 * 8, 0, rb / 16, b2);
                else
                  tma_prefetch_3d(&tmB, k2 * 128, rb, b2);
              }
            }
          }
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.timeout_ns)) {
            ok = false;
            break;
          }
          if constexpr (kPair) {
            const uint32_t fb_leader = mapa_shared(smem_u32(&full_bar[stage]), 0);
            if (issuer) {
              if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2u * Cfg::kStageBytes);
              tma_load_3d_pair(sA + stage * Cfg::kABytes, &tmA, fb_leader, kb * 128, row_a, a_batch, pol);
              if constexpr (kBFmt == kFmtKPanel)
                tma_load_4d_pair(sB + stage * Cfg::kBBytes, &tmB, fb_leader, 0, row_b, kb, b, pol);
              else if constexpr (kBFmt == kFmtShuffle16)
                tma_load_5d_pair(sB + stage * Cfg::kBBytes, &tmB, fb_leader, 0, kb * 8, 0, row_b / 16, b, pol);
              else
                tma_load_3d_pair(sB + stage * Cfg::kBBytes, &tmB, fb_leader, kb * 128, row_b, b, pol);
            }
          } else if (issuer) {
            // the unit's 256 B rows as two 128-row boxes, one after the other
            // in shared memory (the 8-row groups keep their 1024-byte stride)
            mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
            tma_load_3d_hint(sA + stage * Cfg::kABytes, &tmA, &full_bar[stage], kb * 128, row_a, a_batch, pol);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint8_t* dst = sB + stage * Cfg::kBBytes + static_cast<uint32_t>(h) * 16384u;
              const int rb = row_b + h * 128;
              if constexpr (kBFmt == kFmtKPanel)
                tma_load_4d_hint(dst, &tmB, &full_bar[stage], 0, rb, kb, b, pol);
              else if constexpr (kBFmt == kFmtShuffle16)
                tma_load_5d_hint(dst, &tmB, &full_bar[stage], 0, kb * 8, 0, rb / 16, b, pol);
              else
                tma_load_3d_hint(dst, &tmB, &full_bar[stage], kb * 128, rb, b, pol);
            }
          }
          __syncwarp();
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    } else if (warp == 1 && leader) {
      // MMA warp: all lanes run the loop, the elected lane issues
      const bool issuer = elect_one();
      // ---------------------------------------------------------------- MMA issuer (leader)
      constexpr uint32_t idesc = idesc_f8f6f4(false, false, kPair ? 256 : 128, BN);
      const uint64_t adesc0 = make_sdesc(smem_u32(sA), 16u, 1024u, kLayoutSW128);
      const uint64_t bdesc0 = weight_sdesc<kBFmt>(smem_u32(sB), 0);
      constexpr uint64_t kBStep = (kBFmt == kFmtShuffle16 ? 256u : 32u) >> 4;   // one K step, 16-byte units
      int stage = 0;
      uint32_t phase = 0;
      uint32_t kbi = 0;   // K blocks issued by this pair, selects the TMEM buffer
      bool ok = true;
      for (int w = cluster_id; w < n_items && ok; w += num_clusters) {
        PairWork it;
        if (!pair_work<kGrouped>(p, pre, live_tiles, w, it)) continue;
        for (int kb = it.kb0; kb < it.kb1; ++kb, ++kbi) {
          const uint32_t buf = kbi % NB;
          const uint32_t use = kbi / NB;   // how many times this buffer was used before
          if (!mbar_wait_cluster_relaxed(&acc_empty[buf], (use & 1u) ^ 1u, abort_flag, p.timeout_ns)) {
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
            if constexpr (kPair) {
              umma_f8f6f4_pair(d, ad, bd, idesc, 0u);
              umma_f8f6f4_pair(d, ad + 2u, bd + kBStep, idesc, 1u);
              umma_f8f6f4_pair(d, ad + 4u, bd + 2u * kBStep, idesc, 1u);
              umma_f8f6f4_pair(d, ad + 6u, bd + 3u * kBStep, idesc, 1u);
              tc_commit_pair(&empty_bar[stage], 0x3);
              tc_commit_pair(&acc_full[buf], 0x3);
            } else {
              umma_f8f6f4(d, ad, bd, idesc, 0u);
              umma_f8f6f4(d, ad + 2u, bd + kBStep, idesc, 1u);
              umma_f8f6f4(d, ad + 4u, bd + 2u * kBStep, idesc, 1u);
              umma_f8f6f4(d, ad + 6u, bd + 3u * kBStep, idesc, 1u);
              tc_commit(&empty_bar[stage]);
              tc_commit(&acc_full[buf]);
            }
          }
          __syncwarp();
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (issuer) {
        if constexpr (kPair)
          tc_commit_pair(drain_bar, 0x1);
        else
          tc_commit(drain_bar);
      }
      int dummy = 0;
      mbar_wait(drain_bar, 0, &dummy, p.timeout_ns);
    }
  } else {
    setmaxnreg_inc<Cfg::kHighRegs>();
    // ---------------------------------------------------------------- promotion + store (both CTAs)
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const uint32_t t_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(half) * 128u;
    // the leader's acc_empty (wide: this CTA's own, its shared::cta address
    // being a valid shared::cluster address of itself)
    const uint32_t ae_leader = kPair ? mapa_shared(smem_u32(acc_empty), 0) : smem_u32(acc_empty);
    uint8_t* out_buf = smem + Cfg::kOffOut + static_cast<uint32_t>(warp - 4) * 2u * Cfg::kOutBytes;
    uint32_t kbi = 0;
    bool ok = true;
    for (int w = cluster_id; w < n_items && ok; w += num_clusters) {
      PairWork it;
      if (!pair_work<kGrouped>(p, pre, live_tiles, w, it)) continue;
      const int b = it.b;
      const int rbase = it.mt * TR + static_cast<int>(rank) * 128;   // within the group (or matrix)
      const int row = rbase + q * 32 + static_cast<int>(lane);
      const bool row_ok = row < it.rows;
      const long long grow = static_cast<long long>(it.row0) + row;    // row of A, sfa and C
      const int n0 = it.nt * 256 + half * 128;   // this warp's 128 columns: one B-scale block
      // a warp whose 32 rows or 128 columns all lie beyond M or N skips the
      // promotion work (and the scale loads) but still releases the buffers
      const bool live = rbase + q * 32 < it.rows && n0 < p.n;
      const float* sfa_row =
          (kGrouped ? p.sfa : p.sfa + b * p.sfa_batch) + (row_ok ? grow : 0LL) * p.sfa_m;
      const float* sfb_blk = p.sfb + b * p.sfb_batch + static_cast<long long>(live ? n0 / 128 : 0) * p.sfb_n;
      uint64_t accp[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) accp[i] = 0ull;
      // scales of K blocks kb .. kb + 3 in a shift chain (static register
      // indices): each load has three K blocks to arrive -- the row scales
      // of the row-major layout miss L1, and one K block of distance left the
      // promotion stalled on them
      float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (live) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (it.kb0 + i < it.kb1) {
            sa[i] = row_ok ? __ldg(sfa_row + (it.kb0 + i) * p.sfa_k) : 0.0f;
            sb[i] = __ldg(sfb_blk + (it.kb0 + i) * p.sfb_k);
          }
      }
      for (int kb = it.kb0; kb < it.kb1; ++kb, ++kbi) {
        const uint64_t scale2 = pack_f32x2(sa[0] * sb[0]);
        const uint32_t buf = kbi % NB;
        const uint32_t use = kbi / NB;
        if (!mbar_wait_spin(&acc_full[buf], use & 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (live) {
          // two rounds of four 16-column loads in flight behind one wait
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[4][16];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tmem_ld16_async(t_base + buf * BN + static_cast<uint32_t>(c * 64 + j * 16), r[j]);
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
        if (lane == 0) mbar_arrive_cluster_relaxed(ae_leader + buf * 8u);
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          sa[i] = sa[i + 1];
          sb[i] = sb[i + 1];
        }
        if (live && kb + 4 < it.kb1) {
          sa[3] = row_ok ? __ldg(sfa_row + (kb + 4) * p.sfa_k) : 0.0f;
          sb[3] = __ldg(sfb_blk + (kb + 4) * p.sfb_k);
        }
      }
      if (!ok || !live) continue;
      if (!kGrouped && it.slot >= 0) {
        // a tail slice: this warp's 32 rows x 128 columns of the fp32 partial
        // go to the slice's slot (rows past M too; the reduce clips)
        float* dst = p.ws + it.slot * Cfg::kSlotFloats +
                     static_cast<long long>(static_cast<int>(rank) * 128 + q * 32 + static_cast<int>(lane)) * 256 +
                     half * 128;
#pragma unroll
        for (int v = 0; v < 32; ++v)
          st_global_v4(dst + 4 * v, static_cast<uint32_t>(accp[2 * v]), static_cast<uint32_t>(accp[2 * v] >> 32),
                       static_cast<uint32_t>(accp[2 * v + 1]), static_cast<uint32_t>(accp[2 * v + 1] >> 32));
        continue;
      }
      if constexpr (kOutF32 || kGrouped) {
        // fp32 C, and grouped calls (a TMA box would cross into the next
        // group's rows): each lane stores its own row
        if (!row_ok) continue;
        float acc[128];
#pragma unroll
        for (int i = 0; i < 64; ++i) unpack_f32x2(accp[i], acc[2 * i], acc[2 * i + 1]);
        const long long cb = kGrouped ? 0LL : b * p.c_batch_stride;
        if constexpr (kOutF32)
          store_row128<true>(acc, reinterpret_cast<float*>(p.c) + cb + grow * p.ldc, n0, p.n);
        else
          store_row128<false>(acc, reinterpret_cast<uint16_t*>(p.c) + cb + grow * p.ldc, n0, p.n);
      } else {
        // bf16 through TMA stores: per 32-column box each lane writes its row
        // (64 bytes, 64-byte swizzle, so the 32 lanes' 16-byte writes spread
        // over all banks) into one of this warp's two staging buffers; TMA
        // clips the box at the M and N edges
        const uint32_t swz = (lane >> 1) & 3u;
        const int row0 = rbase + q * 32;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (n0 + c * 32 >= p.n) break;
          uint8_t* sbuf = out_buf + static_cast<uint32_t>(c & 1) * Cfg::kOutBytes;
          if (lane == 0) bulk_wait_group_read1();   // the box before the last has left sbuf
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float lo0, hi0;
              unpack_f32x2(accp[c * 16 + j * 4 + v], lo0, hi0);
              w[v] = pack_bf16x2(lo0, hi0);
            }
            st_shared_v4(sbuf + lane * 64u + ((static_cast<uint32_t>(j) ^ swz) * 16u), w[0], w[1], w[2], w[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmC, sbuf, n0 + c * 32, row0, b);
            bulk_commit_group();
          }
        }
      }
    }
    if constexpr (!kOutF32 && !kGrouped)
      if (lane == 0) bulk_wait_group0();   // every store of this warp has completed
  }

  __syncwarp();
  tc_fence_before();
  if constexpr (kPair)
    cluster_sync_all();   // both CTAs done with TMEM, barriers and remote arrives
  else
    __syncthreads();
  tc_fence_after();
  if (warp == 2) {
    if constexpr (kPair)
      tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else
      tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

template <int kBFmt, bool kOutF32, bool kGrouped = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Fp8Block2Cfg<true>::kThreads, 1)
    fp8_block_gemm_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                              const __grid_constant__ CUtensorMap tmC, const Fp8BlockParams p) {
  fp8b2_body<kBFmt, kOutF32, kGrouped, true>(tmA, tmB, tmC, p);
}

// The wide single-CTA kernel: 128 x 256 units, K slices through p.tail_*.
template <int kBFmt, bool kOutF32>
__global__ void __launch_bounds__(Fp8Block2Cfg<false>::kThreads, 1)
    fp8_block_gemm_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                               const __grid_constant__ CUtensorMap tmC, const Fp8BlockParams p) {
  fp8b2_body<kBFmt, kOutF32, false, false>(tmA, tmB, tmC, p);
}

// Sums the K slices of a pair or wide launch into C, in slice order (so the
// result does not depend on which slice finished first): p.tail_units units
// of kRows x 256 (256 for pairs, 128 for the wide kernel), clipped at M and N.
// Launched after the GEMM with programmatic stream serialization; waits for it
// before reading.
template <bool kOutF32, int kRows = 256>
__global__ void __launch_bounds__(256) fp8b_pair_tail_reduce_kernel(const Fp8BlockParams p) {
  constexpr long long kSlot = static_cast<long long>(kRows) * 256;
  griddep_wait();
  const int whole = p.total_units - p.tail_units;
  const long long groups = static_cast<long long>(p.tail_units) * kRows * 64;   // 4-float groups
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int tu = static_cast<int>(g / (kRows * 64));
    const int rem = static_cast<int>(g % (kRows * 64));
    const int r = rem >> 6;
    const int c4 = (rem & 63) * 4;
    int b, mt, nt, s;
    decode_unit(whole + tu, p.tiles_m, p.tiles_n, 1, p.group_m, b, mt, nt, s);
    const int row = mt * kRows + r;
    const int col = nt * 256 + c4;   // N is a multiple of 8, so col < N covers col + 3
    if (row >= p.m || col >= p.n) continue;
    const float* src = p.ws + static_cast<long long>(tu) * p.tail_split * kSlot + r * 256 + c4;
    float4 acc = __ldg(reinterpret_cast<const float4*>(src));
    for (int j = 1; j < p.tail_split; ++j) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + j * kSlot));
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    if constexpr (kOutF32) {
      float* dst = reinterpret_cast<float*>(p.c) + b * p.c_batch_stride + static_cast<long long>(row) * p.ldc + col;
      st_global_v4(dst, __float_as_uint(acc.x), __float_as_uint(acc.y), __float_as_uint(acc.z), __float_as_uint(acc.w));
    } else {
      uint16_t* dst =
          reinterpret_cast<uint16_t*>(p.c) + b * p.c_batch_stride + static_cast<long long>(row) * p.ldc + col;
      *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
    }
  }
}

}  // namespace bsg

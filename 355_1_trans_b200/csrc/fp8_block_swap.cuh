// fp8_block_swap.cuh -- decode-shaped (M <= 64) FP8 GEMM with fp32 block
// scales, computed transposed ("swap-AB") so that it streams B from HBM.
//
// Semantics are those of fp8_block_gemm.cuh (reference:
// block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_kernel_template.hpp:
// 204-601): C[m,n] = sum_kb sfa[m,kb] * sfb[n/128,kb] * (A B^T)_kb[m,n].
//
// For a handful of activation rows the 128-row MMA side is wasted on A, so
// the roles are swapped: the weight tile (128 rows of B = 128 output columns)
// is the MMA's M side and the MN (16, 32 or 64) activation rows its N side.  The
// per-128-K partial D^T[n, m] lands in TMEM lanes n, columns m; because all
// 128 lanes of a tile share one 128x128 weight scale sfb[n/128, kb], the
// promotion is acc[m] += D^T[n, m] * (sfb * sfa[m, kb]) per thread (lane n).
// With MN columns per partial, up to 8 partials are in flight in TMEM, so the
// MMA rarely waits for the promotion warps, and the small stages (16 KB of B
// + MN x 128 B of A) allow a deep TMA pipeline: the kernel is bound by the B
// stream from HBM.  The per-K-block scales (MN values of sfa and one sfb)
// are staged into shared memory by the producers with asynchronous 4-byte
// copies into a ring of 32 slots -- more K blocks than can sit between the
// producers and the promotion -- so neither ever waits on a global scale load.
//
// Roles: warps 0, 2 and 3 TMA producers (every third K block each, with its
// scales), warp 1 MMA (one elected thread runs the role), warp 2 also
// allocates TMEM, warps 4-11 promotion (two sets on alternate K blocks for
// MN <= 32, two column halves for MN = 64).
#pragma once

#include "fp8_block_gemm.cuh"

namespace bsg {

// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

constexpr uint32_t kSwapProducers = 3;   // TMA producer warps 0, 2 and 3

// L2 prefetch of the weight tile (N tile nt, K block kb, batch b) in each B layout.
template <int kBFmt>
__device__ __forceinline__ void prefetch_weight_tile(const CUtensorMap* tmB, int nt, int kb, int b) {
  if constexpr (kBFmt == kFmtKPanel)
    tma_prefetch_4d(tmB, 0, nt * 128, kb, b);
  else if constexpr (kBFmt == kFmtShuffle16)
    tma_prefetch_5d(tmB, 0, kb * 8, 0, nt * 8, b);
  else
    tma_prefetch_3d(tmB, kb * 128, nt * 128, b);
}

// Split-K inside the kernel (kCl): the split_k CTAs that share an output tile
// form one thread-block cluster, each computes one K slice, and the partial
// tiles are summed through distributed shared memory.  Output columns are
// dealt out in "channels" (the storing promotion warps: one per TMEM lane
// quarter for MN <= 32, two per quarter for MN = 64); channel ch is reduced
// and stored by cluster rank ch % split_k, which receives the other ranks'
// partials of that channel in slots of its shared memory and adds them in
// rank order, so the result does not depend on timing.
template <int MN, bool kCl = false>
struct SwapCfg {
  static_assert(MN == 16 || MN == 32 || MN == 64, "MN must be 16, 32 or 64");
  // Promotion: eight warps, two per TMEM lane quarter.  A warp's chain per
  // K block (barrier wait, TMEM load, scale reads, FMAs, arrivals) is ~600
  // cycles of latency, longer than the MMA and the weight stream need per
  // K block, so two warps share each lane quarter: for MN = 64 each takes
  // half of the columns of every K block; for MN <= 32 two sets of four
  // warps take alternate K blocks, and at the end of a unit the second set
  // hands its sums to the first through shared memory.
  static constexpr int kPromoWarps = 8;
  static constexpr int kPromoSets = MN >= 64 ? 1 : 2;
  static constexpr int kThreads = 128 + 32 * kPromoWarps;
  static constexpr int kCols = MN >= 64 ? MN / 2 : MN;        // accumulator columns per thread
  static constexpr int kArrivals = kPromoWarps / kPromoSets;  // promotion warps per K block
  static constexpr uint32_t kRedBytes = kPromoSets > 1 ? 128u * static_cast<uint32_t>(MN) * 4u : 0u;
  static constexpr uint32_t kWBytes = 128u * 128u;                 // weight tile
  static constexpr uint32_t kXBytes = static_cast<uint32_t>(MN) * 128u;
  static constexpr uint32_t kStageBytes = kWBytes + kXBytes;
  static constexpr int kChannels = MN >= 64 ? 8 : 4;
  static constexpr int kChanFloats = kCols * 32;                  // HC rows x 32 columns
  static constexpr uint32_t kClBytes =
      kCl ? static_cast<uint32_t>(swap_cl_slot_count(kChannels) * kChanFloats) * 4u : 0u;
  static constexpr uint32_t kStageBudget = 210u * 1024u - kRedBytes - kClBytes;
  static constexpr int kStages = static_cast<int>(kStageBudget / kStageBytes) > 12
                                     ? 12
                                     : static_cast<int>(kStageBudget / kStageBytes);
  static constexpr int kAccBufs = (512 / MN) > 8 ? 8 : 512 / MN;
  static constexpr uint32_t kTmemCols = static_cast<uint32_t>(kAccBufs * MN) < 32 ? 32u
                                        : static_cast<uint32_t>(kAccBufs * MN);
  static constexpr uint32_t kOffX = kWBytes * kStages;
  // scale ring: at least kStages + kAccBufs slots (the K blocks that can sit
  // between the producer and the promotion), a power of two so that the slot
  // and parity of a K block are a mask and a shift
  static constexpr int kScaleSlots = 32;
  static constexpr uint32_t kScaleSlot = static_cast<uint32_t>(MN + 4);   // floats: MN sfa, 1 sfb
  static constexpr uint32_t kOffScale = kOffX + kXBytes * kStages;
  static constexpr uint32_t kScaleBytes = static_cast<uint32_t>(kScaleSlots) * kScaleSlot * 4u;
  static constexpr uint32_t kOffRed = kOffScale + ((kScaleBytes + 15u) & ~15u);   // [MN][128] floats
  static constexpr uint32_t kOffCl = kOffRed + kRedBytes;          // cluster split-K slots
  static constexpr uint32_t kOffBar = kOffCl + kClBytes;
  static constexpr uint32_t kBarBytes = kCl ? 1536u : 1024u;
  static constexpr uint32_t kSmemBytes = kOffBar + kBarBytes + 1024u;
  static_assert(8u * (2u * kStages + 2u * kAccBufs + 2u * kScaleSlots + 1u + 8u + (kCl ? 2u * kChannels : 0u)) +
                        8u <= kBarBytes,
                "barrier area");
  static_assert(kSmemBytes <= 227u * 1024u, "shared memory");
  static_assert(kScaleSlots >= kStages + kAccBufs, "scale ring shorter than the pipeline");
};

template <int MN, int kBFmt, bool kOutF32, bool kCl = false>
__global__ void __launch_bounds__(SwapCfg<MN, kCl>::kThreads, 1)
    fp8_block_swap_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const Fp8BlockParams p) {
  using Cfg = SwapCfg<MN, kCl>;
  constexpr int S = Cfg::kStages;
  constexpr int NB = Cfg::kAccBufs;
  constexpr int R = Cfg::kScaleSlots;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  uint8_t* sW = smem;
  uint8_t* sX = smem + Cfg::kOffX;
  float* sScale = reinterpret_cast<float*>(smem + Cfg::kOffScale);   // slot: [MN] sfa, [MN] sfb
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* acc_full = empty_bar + S;   // [NB]
  uint64_t* acc_empty = acc_full + NB;  // [NB]
  uint64_t* scale_full = acc_empty + NB;  // [R]
  uint64_t* scale_empty = scale_full + R;  // [R]
  uint64_t* drain_bar = scale_empty + R;
  uint64_t* red_full = drain_bar + 1;   // [4] second promotion set -> first, per lane quarter
  uint64_t* red_empty = red_full + 4;   // [4]
  uint64_t* cl_full = red_empty + 4;                    // [kChannels] partials of the other ranks arrived
  uint64_t* cl_free = cl_full + (kCl ? Cfg::kChannels : 0);   // [kChannels] owner consumed this rank's partial
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(cl_free + (kCl ? Cfg::kChannels : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* cl_slots = reinterpret_cast<float*>(smem + Cfg::kOffCl);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;

  if (threadIdx.x == 32) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], Cfg::kArrivals);   // one arrival per promotion warp of the K block
    }
    for (int i = 0; i < R; ++i) {
      mbar_init(&scale_full[i], 32);  // one cp.async arrival per producer lane
      mbar_init(&scale_empty[i], Cfg::kArrivals);
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&red_full[i], 1);
      mbar_init(&red_empty[i], 1);
    }
    if constexpr (kCl) {
      for (int i = 0; i < Cfg::kChannels; ++i) {
        mbar_init(&cl_full[i], static_cast<uint32_t>(p.split_k - 1));   // one warp of each other rank
        mbar_init(&cl_free[i], 1u);                                      // the owner's warp
      }
    }
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
  // the peers' barriers must exist before any remote arrival: every thread
  // arrives here and waits just before its first remote access (or at the end)
  if constexpr (kCl) cluster_arrive();
  bool cl_waited = false;
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (threadIdx.x == 0) griddep_launch_dependents();   // a split-K reduce may launch now

  if (warp == 0 || warp == 2 || warp == 3) {
    // ------------------------------------------------------------------ TMA producers
    // Three warps take every third K block each.  One warp's issue chain per
    // K block (two barrier waits, the scale copies, two TMA issues) lasts
    // ~600 cycles, which alone would cap the weight stream at ~28 B/clk per
    // SM; three chains in flight keep a CTA near the TMA rate.
    const uint32_t pidx = warp == 0 ? 0u : static_cast<uint32_t>(warp - 1);
    const bool issuer = elect_one();
    const uint64_t pol_w = l2_policy_evict_first();   // weights stream through once
    const uint64_t pol_x = l2_policy_evict_last();    // activations are reread by every tile
    int stage = 0;
    uint32_t phase = 0;
    uint32_t kbi = 0;
    bool ok = true;
    int last_stage = -1;
    uint32_t last_phase = 0;
    // The weights do not come from the previous kernel on the stream: pull
    // this warp's share of the first unit's first S K blocks into L2, then
    // wait for that kernel (programmatic dependent launch) before anything is
    // read into shared memory.
    if (issuer && static_cast<int>(blockIdx.x) < p.total_units) {
      int b, mt, nt, s;
      decode_unit(blockIdx.x, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + min(p.kb_per_split, S), p.num_kb);
      for (int kb = kb0 + static_cast<int>(pidx); kb < kb1; kb += static_cast<int>(kSwapProducers))
        prefetch_weight_tile<kBFmt>(&tmB, nt, kb, b);
    }
    griddep_wait();
    for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
      int b, mt, nt, s;
      decode_unit(u, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
      const int m0 = mt * MN;
      const int rows = min(MN, p.m - m0);
      const float* sfa_t = p.sfa + b * p.sfa_batch + static_cast<long long>(m0) * p.sfa_m;
      const float* sfb_blk = p.sfb + b * p.sfb_batch + static_cast<long long>(nt) * p.sfb_n;
      for (int kb = kb0; kb < kb1; ++kb, ++kbi) {
        if (kbi % kSwapProducers != pidx) {
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
          continue;
        }
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        // this K block's scales into scale slot kbi % R (free once the
        // promotion of K block kbi - R is done, which the stage and TMEM
        // rings already imply, so this wait does not add a stall)
        const uint32_t sl = kbi % R;
        if (!mbar_wait(&scale_empty[sl], ((kbi / R) & 1u) ^ 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        float* slot = sScale + sl * Cfg::kScaleSlot;
#pragma unroll
        for (int i = static_cast<int>(lane); i < MN; i += 32)
          if (i < rows) cp_async_4(slot + i, sfa_t + i * p.sfa_m + kb * p.sfa_k);
        if (lane == 0) cp_async_4(slot + MN, sfb_blk + kb * p.sfb_k);
        cp_async_mbar_arrive(&scale_full[sl]);
        if (issuer) {
          uint64_t* fb = &full_bar[stage];
          mbar_arrive_expect_tx(fb, Cfg::kStageBytes);
          if constexpr (kBFmt == kFmtKPanel)
            tma_load_4d_hint(sW + stage * Cfg::kWBytes, &tmB, fb, 0, nt * 128, kb, b, pol_w);
          else if constexpr (kBFmt == kFmtShuffle16)
            tma_load_5d_hint(sW + stage * Cfg::kWBytes, &tmB, fb, 0, kb * 8, 0, nt * 8, b, pol_w);
          else
            tma_load_3d_hint(sW + stage * Cfg::kWBytes, &tmB, fb, kb * 128, nt * 128, b, pol_w);
          tma_load_3d_hint(sX + stage * Cfg::kXBytes, &tmA, fb, kb * 128, mt * MN, b, pol_x);
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
    if (!ok && last_stage >= 0) {   // let this warp's last copies land before the CTA exits
      int dummy = 0;
      mbar_wait(&full_bar[last_stage], last_phase, &dummy, p.timeout_ns);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // An M=128 N<=64 MMA occupies the tensor pipe for well under 100 cycles,
    // so the issue loop sets the pace.  One elected thread runs the whole
    // role (its barrier waits cost a fraction of a 32-lane wait; the tcgen05
    // instructions are single-thread anyway), the descriptors of stage 0 are
    // built once and a stage's are a constant offset from them.
    if (elect_one()) {
      const uint32_t idesc = idesc_f8f6f4(false, false, 128, MN);
      const uint64_t wdesc0 = weight_sdesc<kBFmt>(smem_u32(sW), 0);
      const uint64_t xdesc0 = make_sdesc(smem_u32(sX), 16u, 1024u, kLayoutSW128);
      constexpr uint64_t kWStep = (kBFmt == kFmtShuffle16 ? 256u : 32u) >> 4;   // one K step, 16-byte units
      int stage = 0;
      uint32_t phase = 0;
      uint32_t kbi = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
        int b, mt, nt, s;
        decode_unit(u, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
        for (int kb = kb0; kb < kb1; ++kb, ++kbi) {
          const uint32_t buf = kbi % NB;
          if (!mbar_wait(&acc_empty[buf], ((kbi / NB) & 1u) ^ 1u, abort_flag, p.timeout_ns) ||
              !mbar_wait(&full_bar[stage], phase, abort_flag, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t wd = wdesc0 + static_cast<uint64_t>(static_cast<uint32_t>(stage) * (Cfg::kWBytes >> 4));
          const uint64_t xd = xdesc0 + static_cast<uint64_t>(static_cast<uint32_t>(stage) * (Cfg::kXBytes >> 4));
          const uint32_t d = tmem_base + buf * MN;
          umma_f8f6f4(d, wd, xd, idesc, 0u);
          umma_f8f6f4(d, wd + kWStep, xd + 2u, idesc, 1u);
          umma_f8f6f4(d, wd + 2u * kWStep, xd + 4u, idesc, 1u);
          umma_f8f6f4(d, wd + 3u * kWStep, xd + 6u, idesc, 1u);
          tc_commit(&empty_bar[stage]);
          tc_commit(&acc_full[buf]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      tc_commit(drain_bar);
      int dummy = 0;
      mbar_wait(drain_bar, 0, &dummy, p.timeout_ns);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ promotion + store
    // warp w: TMEM lane quarter w % 4 (= output columns); MN = 64: activation
    // rows [c0, c0 + HC) of every K block; MN <= 32: all rows of the K blocks
    // whose parity is the warp's set
    constexpr int HC = Cfg::kCols;
    constexpr int PS = Cfg::kPromoSets;
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const uint32_t set = PS > 1 ? static_cast<uint32_t>(half) : 0u;
    const int c0 = PS > 1 ? 0 : half * HC;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + Cfg::kOffRed);   // [HC][128]: conflict-free per column
    uint32_t kbi = 0;
    uint32_t ui = 0;   // units done, for the hand-off barriers' parity
    bool ok = true;
    griddep_wait();   // C and the split-K partials may still be read by the previous kernel
    for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x, ++ui) {
      int b, mt, nt, s;
      decode_unit(u, p.tiles_m, p.tiles_n, p.split_k, p.group_m, b, mt, nt, s);
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
      const int n = nt * 128 + q * 32 + static_cast<int>(lane);   // output column of this lane
      const int m0 = mt * MN;
      const int rows = min(MN, p.m - m0);
      float acc[HC];
#pragma unroll
      for (int i = 0; i < HC; ++i) acc[i] = 0.0f;
      constexpr int CH = HC / 16;   // 16-column TMEM loads per K block
      for (int kb = kb0; kb < kb1; ++kb, ++kbi) {
        if (PS > 1 && (kbi & 1u) != set) continue;
        const uint32_t buf = kbi % NB;
        const uint32_t sl = kbi % R;
        if (!mbar_wait(&acc_full[buf], (kbi / NB) & 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // the partial's TMEM loads are in flight while this K block's scales
        // are checked (they landed long before the MMA ran)
        uint32_t r[CH][16];
        const uint32_t taddr = tmem_base + lane_base + buf * MN + static_cast<uint32_t>(c0);
#pragma unroll
        for (int c = 0; c < CH; ++c) tmem_ld16_async(taddr + static_cast<uint32_t>(c * 16), r[c]);
        const bool sc_ok = mbar_wait(&scale_full[sl], (kbi / R) & 1u, abort_flag, p.timeout_ns);
        tmem_wait_ld16(r[0]);
#pragma unroll
        for (int c = 1; c < CH; ++c) tmem_reg_fence16(r[c]);
        if (!sc_ok) {
          ok = false;
          break;
        }
        const float* slot = sScale + sl * Cfg::kScaleSlot;
        const float sb = slot[MN];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int row = c0 + c * 16 + i;
            const float comb = row < rows ? sb * slot[row] : 0.0f;
            acc[c * 16 + i] = fmaf(__uint_as_float(r[c][i]), comb, acc[c * 16 + i]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&acc_empty[buf]);
          mbar_arrive(&scale_empty[sl]);
        }
      }
      if (!ok) break;
      if constexpr (PS > 1) {
        // the second set hands its sums to the first (per lane quarter,
        // through [HC][128] floats of shared memory)
        const int lrow = q * 32 + static_cast<int>(lane);
        if (set == 1) {
          if (!mbar_wait(&red_empty[q], (ui & 1u) ^ 1u, abort_flag, p.timeout_ns)) break;
#pragma unroll
          for (int i = 0; i < HC; ++i) red[i * 128 + lrow] = acc[i];
          __syncwarp();
          if (lane == 0) mbar_arrive(&red_full[q]);
          continue;
        }
        if (!mbar_wait(&red_full[q], ui & 1u, abort_flag, p.timeout_ns)) break;
#pragma unroll
        for (int i = 0; i < HC; ++i) acc[i] += red[i * 128 + lrow];
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_empty[q]);
      }
      if constexpr (kCl) {
        // split-K across the cluster: this warp's channel goes to its owner
        const int ch = PS > 1 ? q : warp - 4;
        const int S_ = p.split_k;
        const int rank = static_cast<int>(blockIdx.x) % S_;
        const int owner = ch % S_;
        const int owned = (Cfg::kChannels + S_ - 1) / S_;
        const int lch = ch / S_;
        if (!cl_waited) {   // the peers' barriers are initialised (see the arrival above)
          cluster_wait();
          cl_waited = true;
        }
        if (rank != owner) {
          // the owner has consumed this channel's previous partial from our slot
          if (ui > 0 && !mbar_wait_cluster(&cl_free[ch], (ui - 1u) & 1u, abort_flag, p.timeout_ns)) {
            ok = false;
            break;
          }
          const uint32_t dst =
              mapa_shared(smem_u32(cl_slots + (rank * owned + lch) * Cfg::kChanFloats + static_cast<int>(lane)),
                          static_cast<uint32_t>(owner));
#pragma unroll
          for (int i = 0; i < HC; ++i) st_cluster_f32(dst + static_cast<uint32_t>(i * 32 * 4), acc[i]);
          fence_acq_rel_cluster();   // this lane's remote stores before the warp's arrival
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&cl_full[ch]), static_cast<uint32_t>(owner)));
          continue;
        }
        if (!mbar_wait_cluster(&cl_full[ch], ui & 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        // rank order: partial 0 + partial 1 + ...
        float sum[HC];
        for (int r = 0; r < S_; ++r) {
          const float* src = cl_slots + (r * owned + lch) * Cfg::kChanFloats + static_cast<int>(lane);
#pragma unroll
          for (int i = 0; i < HC; ++i) {
            const float v = r == rank ? acc[i] : src[i * 32];
            sum[i] = r == 0 ? v : sum[i] + v;
          }
        }
#pragma unroll
        for (int i = 0; i < HC; ++i) acc[i] = sum[i];
        __syncwarp();   // every lane has read the slots before they are freed
        for (int r = 0; r < S_; ++r)
          if (r != rank && lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&cl_free[ch]), static_cast<uint32_t>(r)));
      }
      if (n >= p.n) continue;
      // store: lane n writes column n of every valid row (64 B per warp per row)
#pragma unroll
      for (int i = 0; i < HC; ++i) {
        if (c0 + i >= rows) break;
        const int m = m0 + c0 + i;
        if (!kCl && p.split_k > 1) {
          p.ws[((static_cast<long long>(s) * p.batch + b) * p.m + m) * static_cast<long long>(p.n) + n] = acc[i];
        } else if constexpr (kOutF32) {
          reinterpret_cast<float*>(p.c)[b * p.c_batch_stride + static_cast<long long>(m) * p.ldc + n] = acc[i];
        } else {
          reinterpret_cast<uint16_t*>(p.c)[b * p.c_batch_stride + static_cast<long long>(m) * p.ldc + n] =
              static_cast<uint16_t>(pack_bf16x2(acc[i], 0.0f) & 0xFFFFu);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (kCl) {
    if (!cl_waited) cluster_wait();
    cluster_sync_all();   // no peer touches this CTA's slots or barriers any more
  }
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace bsg

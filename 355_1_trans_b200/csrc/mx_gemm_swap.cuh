// mx_gemm_swap.cuh -- decode-shaped (M <= 64) MXFP8 / MXFP4 GEMM computed
// transposed ("swap-AB"), so that the MMA's 128-row side streams the weights.
//
// Semantics are those of mx_gemm.cuh (reference: mxfp8_gemm/
// gemm_a8w8_mxfp8_kernel_template.hpp:301-432, mxfp4_gemm_4wave_20261112/
// candidate_m10/gemm_a4w4_mxfp4_4wave_kernel_template.hpp:384-1169).
//
// With a handful of activation rows the normal orientation spends a 16 KB
// A tile per stage on (say) 16 useful rows.  Here the block-scaled MMA
// computes D^T[n, m] = sum_g sfb[n,g] sfa[m,g] (B A^T): the 128 weight rows of
// an N tile are the MMA's M side (with their scale atoms in the A-scale TMEM
// slot) and the MN = 16, 32 or 64 activation rows its N side (block-scaled
// shapes M = 128, N = 8..256 step 8).  A stage is 16 KB of weights plus
// MN x 128 bytes of activations, so 9-10 stages fit and the kernel streams
// the weights at HBM speed.  The activation rows of one batch all lie in the
// first 128-row scale atom (M <= 64), so the activation scales are that atom.
//
// Roles: warps 0, 2 and 3 TMA producers (every third K block each), warp 1
// MMA, warp 2 also allocates TMEM, warps 4-7 epilogue.  Two TMEM
// accumulators (MN columns each) alternate between units, so the MMA starts
// the next unit while the epilogue drains the last one: lane n of the
// accumulator is output column n, column m is output row m; a thread stores
// its column for every row (64 contiguous bytes per warp per row), or its
// split-K partial.
#pragma once

#include "mx_gemm.cuh"

namespace bsg {

// 32 lanes x 8 consecutive 32-bit TMEM columns -> 8 registers per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
}

constexpr uint32_t kMxSwapProducers = 3;   // TMA producer warps 0, 2 and 3
constexpr uint32_t kMxSwapChains = 2;      // accumulators per unit (alternate K blocks)

// Split-K inside the kernel (kCl), as in fp8_block_swap.cuh: the split_k CTAs
// of a tile form a cluster and sum their partial tiles through distributed
// shared memory.  The channels are the four epilogue warps (TMEM lane
// quarters); channel q is reduced and stored by cluster rank q % split_k in
// rank order.
template <int MN, int kFp4, bool kCl = false>
struct MxSwapCfg {
  static_assert(MN == 16 || MN == 32 || MN == 64, "MN must be 16, 32 or 64");
  static constexpr int kSfAtomsK = kFp4 ? 2 : 1;             // scale atoms per stage along K
  static constexpr uint32_t kWBytes = 128u * 128u;           // 128 weight rows x 128 bytes of K
  static constexpr uint32_t kXBytes = static_cast<uint32_t>(MN) * 128u;
  static constexpr uint32_t kSfwBytes = 512u * kSfAtomsK;
  static constexpr uint32_t kSfxBytes = 512u * kSfAtomsK;
  static constexpr uint32_t kStageBytes = kWBytes + kXBytes + kSfwBytes + kSfxBytes;
  static constexpr int kChannels = 4;
  static constexpr int kChanFloats = MN * 32;                // MN rows x 32 columns
  static constexpr uint32_t kClBytes =
      kCl ? static_cast<uint32_t>(swap_cl_slot_count(kChannels) * kChanFloats) * 4u : 0u;
  static constexpr uint32_t kStageBudget = 218u * 1024u - kClBytes;
  static constexpr int kStages = static_cast<int>(kStageBudget / kStageBytes) > 10
                                     ? 10
                                     : static_cast<int>(kStageBudget / kStageBytes);
  static constexpr uint32_t kOffX = kWBytes * kStages;
  static constexpr uint32_t kOffSfw = kOffX + kXBytes * kStages;
  static constexpr uint32_t kOffSfx = kOffSfw + kSfwBytes * kStages;
  static constexpr uint32_t kOffCl = kOffSfx + kSfxBytes * kStages;
  static constexpr uint32_t kOffBar = kOffCl + kClBytes;
  static constexpr uint32_t kBarBytes = kCl ? 512u : 256u;
  static constexpr uint32_t kSmemBytes = kOffBar + kBarBytes + 1024u;
  // TMEM: two accumulators [0, 2 MN), then two alternating scale regions
  // (weight atoms: 4 columns per K atom, activation atoms: 4 per K atom)
  // Each unit accumulates its K blocks alternately into kMxSwapChains TMEM
  // accumulators (summed in the epilogue): consecutive MMAs of one
  // accumulator wait for each other, so two chains keep the tensor pipe
  // busy at these small N.  Two units alternate, so the MMA starts the next
  // unit while the epilogue drains the last one.
  static constexpr uint32_t kChains = kMxSwapChains;
  static constexpr uint32_t kAccCols = kChains * static_cast<uint32_t>(MN);   // one unit's accumulators
  static constexpr uint32_t kColSf = 2u * kAccCols;
  static constexpr uint32_t kSfRegionCols = 8u * kSfAtomsK;
  static constexpr uint32_t kColsUsed = kColSf + 2u * kSfRegionCols;
  static constexpr uint32_t kTmemCols =
      kColsUsed <= 32 ? 32 : kColsUsed <= 64 ? 64 : kColsUsed <= 128 ? 128 : kColsUsed <= 256 ? 256 : 512;
  static_assert(kColsUsed <= 512, "TMEM columns");
  static_assert(kStages >= 4, "pipeline too shallow");
  static_assert(kSmemBytes <= 227u * 1024u, "shared memory");
  static_assert(8u * (2u * kStages + 5u + (kCl ? 2u * kChannels : 0u)) + 8u <= kBarBytes, "barrier area");
};

template <int MN, int kFp4, int kBMode, bool kOutF32, bool kCl = false>
__global__ void __launch_bounds__(256, 1)
    mx_gemm_swap_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const MxParams p) {
  using Cfg = MxSwapCfg<MN, kFp4, kCl>;
  constexpr int S = Cfg::kStages;
  static_assert(kBMode != kBMNMajor, "the weights are the K-major MMA A operand");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  uint8_t* sW = smem;
  uint8_t* sX = smem + Cfg::kOffX;
  uint8_t* sSfw = smem + Cfg::kOffSfw;
  uint8_t* sSfx = smem + Cfg::kOffSfx;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* acc_full = empty_bar + S;   // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* drain_bar = acc_empty + 2;
  uint64_t* cl_full = drain_bar + 1;                           // [4] partials of the other ranks arrived
  uint64_t* cl_free = cl_full + (kCl ? Cfg::kChannels : 0);    // [4] owner consumed this rank's partial
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);   // one arrival per epilogue warp
    }
    mbar_init(drain_bar, 1);
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

  // units: (batch, N tile, K slice); the activation tile is the batch's rows 0..MN-1
  if (warp == 0 || warp == 2 || warp == 3) {
    // ------------------------------------------------------------------ TMA producers
    // Three warps take every third K block each: one warp's issue chain per
    // K block (a barrier wait and four copies) would alone cap the weight
    // stream well below the TMA rate of an SM.
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
      decode_unit(blockIdx.x, 1, p.tiles_n, p.split_k, 1, b, mt, nt, s);
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + min(p.kb_per_split, S), p.num_kb);
      for (int kb = kb0 + static_cast<int>(pidx); kb < kb1; kb += static_cast<int>(kMxSwapProducers)) {
        if constexpr (kBMode == kBShuffle16)
          tma_prefetch_5d(&tmB, 0, kb * 8, 0, nt * 8, b);
        else
          tma_prefetch_3d(&tmB, kb * 128, nt * 128, b);
      }
    }
    griddep_wait();
    for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
      int b, mt, nt, s;
      decode_unit(u, 1, p.tiles_n, p.split_k, 1, b, mt, nt, s);
      const int kb0 = s * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
      const uint8_t* sfw_tile = p.sfb + b * p.sfb_batch_stride + static_cast<long long>(nt) * p.sf_kb_total * 512;
      const uint8_t* sfx_tile = p.sfa + b * p.sfa_batch_stride;
      for (int kb = kb0; kb < kb1; ++kb, ++kbi) {
        if (kbi % kMxSwapProducers != pidx) {
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
        if (issuer) {
          uint64_t* fb = &full_bar[stage];
          mbar_arrive_expect_tx(fb, Cfg::kStageBytes);
          const int kbyte = kb * 128;
          if constexpr (kBMode == kBShuffle16)
            tma_load_5d_hint(sW + stage * Cfg::kWBytes, &tmB, fb, 0, kb * 8, 0, nt * 8, b, pol_w);
          else
            tma_load_3d_hint(sW + stage * Cfg::kWBytes, &tmB, fb, kbyte, nt * 128, b, pol_w);
          tma_load_3d_hint(sX + stage * Cfg::kXBytes, &tmA, fb, kbyte, 0, b, pol_x);
          const long long atom_k = static_cast<long long>(kb) * Cfg::kSfAtomsK;
          bulk_load(sSfw + stage * Cfg::kSfwBytes, sfw_tile + atom_k * 512, Cfg::kSfwBytes, fb);
          bulk_load(sSfx + stage * Cfg::kSfxBytes, sfx_tile + atom_k * 512, Cfg::kSfxBytes, fb);
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
    // ------------------------------------------------------------------ MMA issuer
    // An M=128 N<=64 MMA occupies the tensor pipe for well under 100 cycles,
    // so the issue loop sets the pace.  One elected thread runs the whole
    // role (its barrier waits cost a fraction of a 32-lane wait; the tcgen05
    // instructions are single-thread anyway), the descriptors of stage 0 are
    // built once and a stage's are a constant offset from them.
    if (elect_one()) {
      constexpr uint32_t kFmt = kFp4 ? 1u : 0u;
      constexpr uint32_t idesc0 = idesc_block_scaled(kFmt, kFmt, false, false, 128, MN);
      constexpr bool kWShuf = kBMode == kBShuffle16;
      constexpr uint32_t kWLbo = kWShuf ? 128u : 16u;
      constexpr uint64_t kWStep = (kWShuf ? 256u : 32u) >> 4;   // one K step, 16-byte units
      constexpr uint32_t kWLayout = kWShuf ? kLayoutNone : kLayoutSW128;
      const uint64_t wdesc0 = make_sdesc(smem_u32(sW), kWLbo, 1024u, kWLayout);
      const uint64_t xdesc0 = make_sdesc(smem_u32(sX), 16u, 1024u, kLayoutSW128);
      const uint32_t sSfw0 = smem_u32(sSfw), sSfx0 = smem_u32(sSfx);
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      uint32_t sf_region = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x, ++iter) {
        int b, mt, nt, s;
        decode_unit(u, 1, p.tiles_n, p.split_k, 1, b, mt, nt, s);
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);
        const uint32_t ub = static_cast<uint32_t>(iter) & 1u;
        if (!mbar_wait(&acc_empty[ub], ((static_cast<uint32_t>(iter) >> 1) & 1u) ^ 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dunit = tmem_base + ub * Cfg::kAccCols;
        for (int kb = kb0; kb < kb1; ++kb) {
          const uint32_t chain = static_cast<uint32_t>(kb - kb0) % Cfg::kChains;
          const uint32_t d = dunit + chain * MN;
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tsf = tmem_base + Cfg::kColSf + sf_region * Cfg::kSfRegionCols;
          sf_region ^= 1u;
          const uint32_t ust = static_cast<uint32_t>(stage);
#pragma unroll
          for (int j = 0; j < Cfg::kSfAtomsK; ++j) {
            tmem_cp_sf_atom(tsf + 4u * j, sSfw0 + ust * Cfg::kSfwBytes + 512u * j);
            tmem_cp_sf_atom(tsf + 4u * (Cfg::kSfAtomsK + j), sSfx0 + ust * Cfg::kSfxBytes + 512u * j);
          }
          const uint64_t wd = wdesc0 + static_cast<uint64_t>(ust * (Cfg::kWBytes >> 4));
          const uint64_t xd = xdesc0 + static_cast<uint64_t>(ust * (Cfg::kXBytes >> 4));
          const uint32_t acc0 = kb - kb0 >= static_cast<int>(Cfg::kChains) ? 1u : 0u;   // first K block of its chain
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t j = kFp4 ? static_cast<uint32_t>(t >> 1) : 0u;
            const uint32_t sf_id = kFp4 ? static_cast<uint32_t>((t & 1) * 2) : static_cast<uint32_t>(t);
            const uint32_t idesc = idesc_with_sf_id(idesc0, sf_id, sf_id);
            const uint64_t adesc = wd + static_cast<uint64_t>(t) * kWStep;
            const uint64_t bdesc = xd + 2u * static_cast<uint64_t>(t);
            const uint32_t acc = t > 0 ? 1u : acc0;
            if constexpr (kFp4)
              umma_mxf4(d, adesc, bdesc, idesc, tsf + 4u * j, tsf + 4u * (Cfg::kSfAtomsK + j), acc);
            else
              umma_mxf8f6f4(d, adesc, bdesc, idesc, tsf + 4u * j, tsf + 4u * (Cfg::kSfAtomsK + j), acc);
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[ub]);
      }
      tc_commit(drain_bar);
      int dummy = 0;
      mbar_wait(drain_bar, 0, &dummy, p.timeout_ns);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int iter = 0;
    griddep_wait();   // C and the split-K partials may still be read by the previous kernel
    for (int u = blockIdx.x; u < p.total_units; u += gridDim.x, ++iter) {
      int b, mt, nt, s;
      decode_unit(u, 1, p.tiles_n, p.split_k, 1, b, mt, nt, s);
      const uint32_t ub = static_cast<uint32_t>(iter) & 1u;
      if (!mbar_wait(&acc_full[ub], (static_cast<uint32_t>(iter) >> 1) & 1u, abort_flag, p.timeout_ns)) break;
      tc_fence_after();
      float v[MN];
      const int kb0 = s * p.kb_per_split;
      const int nkb = min(kb0 + p.kb_per_split, p.num_kb) - kb0;
      // chain c holds the unit's K blocks c, c + kChains, ...; chains the
      // unit did not reach hold nothing of it
      const uint32_t chains = static_cast<uint32_t>(min(nkb, static_cast<int>(Cfg::kChains)));
      const uint32_t taddr = tmem_base + lane_base + ub * Cfg::kAccCols;
#pragma unroll
      for (uint32_t ch = 0; ch < Cfg::kChains; ++ch) {
        if (ch >= chains) break;
        if constexpr (MN >= 32) {
#pragma unroll
          for (int c = 0; c < MN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(taddr + ch * MN + static_cast<uint32_t>(c * 32), r);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              v[c * 32 + i] = ch == 0 ? __uint_as_float(r[i]) : v[c * 32 + i] + __uint_as_float(r[i]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < MN / 8; ++c) {
            uint32_t r[8];
            tmem_ld8(taddr + ch * MN + static_cast<uint32_t>(c * 8), r);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              v[c * 8 + i] = ch == 0 ? __uint_as_float(r[i]) : v[c * 8 + i] + __uint_as_float(r[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ub]);
      if constexpr (kCl) {
        // split-K across the cluster: channel q (this warp's 32 columns) goes to its owner
        const int S_ = p.split_k;
        const int rank = static_cast<int>(blockIdx.x) % S_;
        const int owner = q % S_;
        const int owned = (Cfg::kChannels + S_ - 1) / S_;
        const int lch = q / S_;
        const uint32_t ui = static_cast<uint32_t>(iter);
        if (!cl_waited) {   // the peers' barriers are initialised (see the arrival above)
          cluster_wait();
          cl_waited = true;
        }
        if (rank != owner) {
          if (ui > 0 && !mbar_wait_cluster(&cl_free[q], (ui - 1u) & 1u, abort_flag, p.timeout_ns)) break;
          const uint32_t dst =
              mapa_shared(smem_u32(cl_slots + (rank * owned + lch) * Cfg::kChanFloats + static_cast<int>(lane)),
                          static_cast<uint32_t>(owner));
#pragma unroll
          for (int i = 0; i < MN; ++i) st_cluster_f32(dst + static_cast<uint32_t>(i * 32 * 4), v[i]);
          fence_acq_rel_cluster();   // this lane's remote stores before the warp's arrival
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&cl_full[q]), static_cast<uint32_t>(owner)));
          continue;
        }
        if (!mbar_wait_cluster(&cl_full[q], ui & 1u, abort_flag, p.timeout_ns)) break;
        // rank order: partial 0 + partial 1 + ...
        float sum[MN];
        for (int r = 0; r < S_; ++r) {
          const float* src = cl_slots + (r * owned + lch) * Cfg::kChanFloats + static_cast<int>(lane);
#pragma unroll
          for (int i = 0; i < MN; ++i) {
            const float x = r == rank ? v[i] : src[i * 32];
            sum[i] = r == 0 ? x : sum[i] + x;
          }
        }
#pragma unroll
        for (int i = 0; i < MN; ++i) v[i] = sum[i];
        __syncwarp();   // every lane has read the slots before they are freed
        for (int r = 0; r < S_; ++r)
          if (r != rank && lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&cl_free[q]), static_cast<uint32_t>(r)));
      }
      const int n = nt * 128 + q * 32 + static_cast<int>(lane);   // output column of this lane
      if (n >= p.n) continue;
#pragma unroll
      for (int i = 0; i < MN; ++i) {
        if (i >= p.m) break;
        if (!kCl && p.split_k > 1) {
          p.ws[((static_cast<long long>(s) * p.batch + b) * p.m + i) * static_cast<long long>(p.n) + n] = v[i];
        } else if constexpr (kOutF32) {
          reinterpret_cast<float*>(p.c)[b * p.c_batch_stride + static_cast<long long>(i) * p.ldc + n] = v[i];
        } else {
          reinterpret_cast<uint16_t*>(p.c)[b * p.c_batch_stride + static_cast<long long>(i) * p.ldc + n] =
              static_cast<uint16_t>(pack_bf16x2(v[i], 0.0f) & 0xFFFFu);
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

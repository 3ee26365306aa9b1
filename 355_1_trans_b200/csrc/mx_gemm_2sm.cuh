// mx_gemm_2sm.cuh -- CTA-pair (tcgen05 cta_group::2) variant of the MXFP8 /
// MXFP4 block-scaled GEMM: a cluster of two CTAs on two SMs computes one
// 256 x 256 output tile.
//
// Semantics are those of mx_gemm.cuh (reference: mxfp8_gemm/
// gemm_a8w8_mxfp8_kernel_template.hpp:301-432, mxfp4_gemm_4wave_20261112/
// candidate_m10/gemm_a4w4_mxfp4_4wave_kernel_template.hpp:384-1169).
//
// Why pairs: a 1-CTA 128 x 256 tile has to pull 48 KB of A+B into one SM per
// 128-K stage.  In a pair each SM loads its own 128 rows of A and its own 128
// rows (half) of B -- 32 KB per stage -- while the leader's pair-mode MMA
// (M = 256, N = 256) reads A from each CTA's shared memory for that CTA's rows
// and B from both, so per-SM load traffic per flop drops by a third and six
// stages fit in shared memory.
//
// Protocol (rank 0 = leader, rank 1 = peer; identical shared-memory layout):
//   producer (warp 0, both CTAs)  waits its own empty[s]; loads its A half, its
//       B half, the A scale atoms of its own 128 rows and the B scale atoms of
//       all 256 columns with the pair form of the TMA load, whose transaction
//       bytes go to the LEADER's full[s]; the leader arms full[s] with the
//       bytes of both CTAs;
//   MMA (warp 1 of the leader)     waits full[s], copies the scale atoms to
//       TMEM with the pair form of tcgen05.cp (each CTA's shared memory to its
//       own TMEM, same columns), issues 4 pair MMAs, and commits to empty[s]
//       of both CTAs (commit with a CTA mask); after the tile it commits to
//       tmem_full of both CTAs;
//   epilogue (warps 4-11, both)    wait their own tmem_full, drain their own
//       TMEM rows (128 x 256 per CTA) into packed bf16 registers, arrive on the
//       leader's tmem_empty (count 2 x 8 warps), then store through TMA: each
//       warp stages 32 rows x 32 columns (2 KB, 64-byte swizzle, so the 32
//       lanes' 16-byte writes spread over all banks) and issues a tensor store
//       of that box; TMA clips the box at the M and N edges.
//   scale builder (warp 3, both CTAs; kSfE8m0Block128 only)  writes its own
//       CTA's scale atoms for the stage from the per-128 E8M0 bytes
//       (mx_gemm.cuh), fences them for the async proxy (CTA scope) and
//       arrives on its CTA's sf_ready[s]; that CTA's producer waits for
//       sf_ready[s] before issuing the stage's pair loads, so the leader's
//       full[s] -- which needs both CTAs' transaction bytes -- completes only
//       after both CTAs' atoms are in place.  Every synchronisation stays at
//       CTA scope: a cluster-scope proxy fence or release per stage (the
//       builder writing the peer's atoms, or arriving on the leader's
//       barrier) measured at about one memory latency each, a third to a
//       half of the MMA rate.
// B may be K-major, MN-major or the shuffle_weight(16,16) layout, as in
// mx_gemm.cuh.  Every wait is bounded (sm100.cuh mbar_wait).
#pragma once

#include "mx_gemm.cuh"

namespace bsg {

struct Mx2Params {
  int m, n, k;
  int batch;
  int num_kb;                    // 128-byte K stages
  int tiles_m, tiles_n;          // 256-row / 256-column pair tiles
  int total_units;               // batch * tiles_m * tiles_n
  int group_m;
  int sf_kb_total;               // scale atoms along K per 128-row block
  int sfa_row_blocks, sfb_row_blocks;
  // kSfE8m0Block128: raw scale bytes, A's [K/128][M], B's [N/128][K/128]
  const uint8_t* sfa;
  const uint8_t* sfb;
  long long sfa_ld, sfb_ld, sfa_batch_stride, sfb_batch_stride;
  void* c;
  long long ldc;
  long long c_batch_stride;
  unsigned long long timeout_ns;
};

template <int kFp4>
struct Mx2Cfg {
  static constexpr int kSfAtomsK = kFp4 ? 2 : 1;
  static constexpr uint32_t kABytes = 128u * 128u;       // this CTA's 128 rows
  static constexpr uint32_t kBBytes = 128u * 128u;       // this CTA's half of B
  static constexpr uint32_t kSfaBytes = 512u * kSfAtomsK;        // this CTA's 128 rows
  static constexpr uint32_t kSfbBytes = 2u * 512u * kSfAtomsK;   // 256 columns
  static constexpr uint32_t kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  // shared memory left for stages after the epilogue staging (8 x 2 KB)
  static constexpr uint32_t kStageBudget = 225u * 1024u - 2048u - 8u * 2048u;
  static constexpr int kStages = static_cast<int>(kStageBudget / kStageBytes) > 8
                                     ? 8
                                     : static_cast<int>(kStageBudget / kStageBytes);
  static constexpr uint32_t kOffB = kABytes * kStages;
  static constexpr uint32_t kOffSfa = kOffB + kBBytes * kStages;
  static constexpr uint32_t kOffSfb = kOffSfa + kSfaBytes * kStages;
  static constexpr uint32_t kOffOut = kOffSfb + kSfbBytes * kStages;   // 8 epilogue warps x 2 KB
  static constexpr uint32_t kOutBytes = 32u * 64u;
  static constexpr uint32_t kOffBar = kOffOut + 8u * kOutBytes;
  static constexpr uint32_t kSmemBytes = kOffBar + 256u + 1024u;
  static_assert(kSmemBytes <= 227u * 1024u, "shared memory");
  static_assert(kOffOut % 1024u == 0, "swizzled staging buffers need 1024-byte alignment");
  // barriers: full, empty, sf_ready [S each], tmem_full, tmem_empty, drain; holder + abort flag
  static_assert(8u * (3u * kStages + 3u) + 8u <= 256u, "barrier area");
  // two alternating scale-factor regions after the 256 accumulator columns
  static constexpr uint32_t kSfRegionCols = 12u * kSfAtomsK;
  static constexpr uint32_t kColSfa = 256u;
  static constexpr uint32_t kColSfb = 256u + 4u * kSfAtomsK;
  static constexpr uint32_t kTmemCols = 512u;
  static_assert(256u + 2u * kSfRegionCols <= 512u, "TMEM overflow");
  static_assert(kStages >= 3, "pipeline too shallow");
};

template <int kFp4, bool kAMN, int kBMode, int kSfMode>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kMxThreads, 1)
    mx_gemm_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmSfa,
                       const __grid_constant__ CUtensorMap tmSfb, const __grid_constant__ CUtensorMap tmC,
                       const Mx2Params p) {
  using Cfg = Mx2Cfg<kFp4>;
  constexpr int S = Cfg::kStages;
  constexpr bool kBMN = kBMode == kBMNMajor;
  constexpr bool kBuildSf = kSfMode == kSfE8m0Block128;
  static_assert(!kBuildSf || !kFp4, "per-128 E8M0 scales are an fp8 format");

  extern __shared__ uint8_t smem_raw[];
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
  uint64_t* sf_ready = drain_bar + 1;   // [S], kSfE8m0Block128 only
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sf_ready + S);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 32) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
      mbar_init(&sf_ready[i], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, 2 * kMxEpiWarps);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmSfa);
    prefetch_tmap(&tmSfb);
    prefetch_tmap(&tmC);
  }
  tc_fence_before();
  cluster_sync_all();   // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (threadIdx.x == 0) griddep_launch_dependents();   // the next kernel's prologue may start
  // Launched with programmatic dependent launch, the prologue above overlaps
  // the previous kernel on the stream; nothing of global memory is touched
  // before that kernel has completed.
  griddep_wait();
  const int cluster_id = static_cast<int>(blockIdx.x >> 1);
  const int num_clusters = static_cast<int>(gridDim.x >> 1);

  if (warp == 0) {
    // producer warp: all lanes run the loop, the elected lane issues the copies
    const bool issuer = elect_one();
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    const uint64_t pol_a = l2_policy_evict_last();
    const uint64_t pol_b = l2_policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = cluster_id; u < p.total_units && ok; u += num_clusters) {
      int b, mt, nt, s;
      decode_unit(u, p.tiles_m, p.tiles_n, 1, p.group_m, b, mt, nt, s);
      // scale atoms that exist at ragged edges: A rows of the leader always,
      // of the peer only when its 128-row block is inside M; B columns of the
      // whole 256-column tile, loaded by both CTAs
      const bool peer_sfa = 2 * mt + 1 < p.sfa_row_blocks;
      const bool my_sfa = rank == 0 || peer_sfa;
      const int sfb_rows = min(2, p.sfb_row_blocks - 2 * nt);
      const uint32_t sf_bytes =
          (1u + (peer_sfa ? 1u : 0u) + 2u * static_cast<uint32_t>(sfb_rows)) * 512u * Cfg::kSfAtomsK;
      const uint32_t tx_bytes = 2u * (Cfg::kABytes + Cfg::kBBytes) + (kBuildSf ? 0u : sf_bytes);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        if constexpr (kBuildSf) {
          // this CTA's scale atoms for the stage are written before its loads go out
          if (!mbar_wait(&sf_ready[stage], phase, abort_flag, p.timeout_ns)) {
            ok = false;
            break;
          }
        }
        const uint32_t fb_leader = mapa_shared(smem_u32(&full_bar[stage]), 0);
        if (leader && issuer) mbar_arrive_expect_tx(&full_bar[stage], tx_bytes);
        uint8_t* a_dst = sA + stage * Cfg::kABytes;
        uint8_t* b_dst = sB + stage * Cfg::kBBytes;
        const int kbyte = kb * 128;
        const int row_a = mt * 256 + static_cast<int>(rank) * 128;
        const int row_b = nt * 256 + static_cast<int>(rank) * 128;
        if (issuer) {
          if constexpr (!kAMN)
            tma_load_3d_pair(a_dst, &tmA, fb_leader, kbyte, row_a, b, pol_a);
          else
            tma_load_3d_pair(a_dst, &tmA, fb_leader, row_a, kbyte, b, pol_a);
          if constexpr (kBMode == kBKMajor)
            tma_load_3d_pair(b_dst, &tmB, fb_leader, kbyte, row_b, b, pol_b);
          else if constexpr (kBMode == kBShuffle16)
            tma_load_5d_pair(b_dst, &tmB, fb_leader, 0, kb * 8, 0, row_b / 16, b, pol_b);
          else
            tma_load_3d_pair(b_dst, &tmB, fb_leader, row_b, kbyte, b, pol_b);
          if constexpr (!kBuildSf) {
            const int atom_k = kb * Cfg::kSfAtomsK;
            if (my_sfa)
              tma_load_3d_pair(sSfa + stage * Cfg::kSfaBytes, &tmSfa, fb_leader, 0,
                               (2 * mt + static_cast<int>(rank)) * p.sf_kb_total + atom_k, b, pol_a);
            for (int r = 0; r < sfb_rows; ++r)
              tma_load_3d_pair(sSfb + stage * Cfg::kSfbBytes + r * 512 * Cfg::kSfAtomsK, &tmSfb, fb_leader,
                               0, (2 * nt + r) * p.sf_kb_total + atom_k, b, pol_b);
          }
        }
        __syncwarp();
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1 && leader) {
    // MMA warp: all lanes run the loop, the elected lane issues
    const bool issuer = elect_one();
    // ------------------------------------------------------------------ MMA issuer (leader)
    constexpr uint32_t kFmt = kFp4 ? 1u : 0u;
    constexpr uint32_t idesc0 = idesc_block_scaled(kFmt, kFmt, kAMN, kBMN, 256, 256);
    constexpr bool kBShuf = kBMode == kBShuffle16;
    constexpr uint32_t kALbo = kAMN ? 128u * 128u : 16u;
    constexpr uint32_t kBLbo = kBMN ? 128u * 128u : kBShuf ? 128u : 16u;
    constexpr uint32_t kSbo = 1024u;
    constexpr uint32_t kKStep = kAMN ? 32u * 128u : 32u;
    constexpr uint32_t kKStepB = kBMN ? 32u * 128u : kBShuf ? 256u : 32u;
    constexpr uint32_t kBLayout = kBShuf ? kLayoutNone : kLayoutSW128;
    // The descriptors of stage 0 are built once; a stage's are a constant
    // offset from them, and a stage's scale copies and MMAs are one branch,
    // so the issue path per stage stays short of the MMAs' own time.
    const uint64_t adesc0 = make_sdesc(smem_u32(sA), kALbo, kSbo, kLayoutSW128);
    const uint64_t bdesc0 = make_sdesc(smem_u32(sB), kBLbo, kSbo, kBLayout);
    const uint32_t sSfa0 = smem_u32(sSfa), sSfb0 = smem_u32(sSfb);
    int stage = 0;
    uint32_t phase = 0;
    int iter = 0;
    uint32_t sf_region = 0;   // alternates every stage
    bool ok = true;
    for (int u = cluster_id; u < p.total_units && ok; u += num_clusters, ++iter) {
      if (!mbar_wait_cluster(tmem_empty, (static_cast<uint32_t>(iter) & 1u) ^ 1u, abort_flag,
                             p.timeout_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kb = 0; kb < p.num_kb; ++kb) {
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
            // A scales: 4 columns per K atom (each CTA's own rows)
            tmem_cp_sf_atom_pair(tsf + Cfg::kColSfa + 4u * j, sSfa0 + ust * Cfg::kSfaBytes + 512u * j);
            // B scales: 8 columns per K atom (all 256 columns, in both CTAs)
#pragma unroll
            for (int r = 0; r < 2; ++r)
              tmem_cp_sf_atom_pair(tsf + Cfg::kColSfb + 4u * (j * 2 + r),
                                   sSfb0 + ust * Cfg::kSfbBytes + 512u * (r * Cfg::kSfAtomsK + j));
          }
          const uint64_t ad = adesc0 + static_cast<uint64_t>(ust * (Cfg::kABytes >> 4));
          const uint64_t bd = bdesc0 + static_cast<uint64_t>(ust * (Cfg::kBBytes >> 4));
          const uint32_t acc0 = kb > 0 ? 1u : 0u;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t j = kFp4 ? static_cast<uint32_t>(t >> 1) : 0u;
            const uint32_t sf_id = kFp4 ? static_cast<uint32_t>((t & 1) * 2) : static_cast<uint32_t>(t);
            const uint64_t adesc = ad + static_cast<uint64_t>((t * kKStep) >> 4);
            const uint64_t bdesc = bd + static_cast<uint64_t>((t * kKStepB) >> 4);
            const uint32_t idesc = idesc_with_sf_id(idesc0, sf_id, sf_id);
            const uint32_t tsfa = tsf + Cfg::kColSfa + 4u * j;
            const uint32_t tsfb = tsf + Cfg::kColSfb + 8u * j;
            const uint32_t acc = t > 0 ? 1u : acc0;
            if constexpr (kFp4)
              umma_mxf4_pair(tmem_base, adesc, bdesc, idesc, tsfa, tsfb, acc);
            else
              umma_mxf8f6f4_pair(tmem_base, adesc, bdesc, idesc, tsfa, tsfb, acc);
          }
        }
        if (issuer) tc_commit_pair(&empty_bar[stage], 0x3);
        __syncwarp();
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (issuer) tc_commit_pair(tmem_full, 0x3);
    }
    if (issuer) tc_commit_pair(drain_bar, 0x1);
    int dummy = 0;
    mbar_wait(drain_bar, 0, &dummy, p.timeout_ns);
  } else if (warp == 3) {
    if constexpr (kBuildSf) {
      // -------------------------------------------------------------- scale builder (both CTAs)
      // this CTA's 128 A rows and all 256 B columns, kSfPrefetch K blocks
      // ahead, as in mx_gemm.cuh
      constexpr int D = kSfPrefetch;
      KbCursor issue = make_cursor(cluster_id, num_clusters, p.total_units, p.tiles_m, p.tiles_n, 1, p.group_m,
                                   p.num_kb, p.num_kb);
      KbCursor cons = issue;
      uint32_t ra[D][4], rb[D][2];
      auto load = [&](const KbCursor& c, uint32_t (&va)[4], uint32_t (&vb)[2]) {
        const int row_a = c.mt * 256 + static_cast<int>(rank) * 128;
        const uint8_t* sa = p.sfa + c.b * p.sfa_batch_stride + row_a;
        const uint8_t* sb = p.sfb + c.b * p.sfb_batch_stride + static_cast<long long>(2 * c.nt) * p.sfb_ld;
        e8m0_block_bytes<2>(sa, p.m - row_a, sb, min(2, p.sfb_row_blocks - 2 * c.nt), p.sfa_ld, p.sfb_ld, c.kb,
                            lane, va, vb);
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
          for (int r = 0; r < 2; ++r) {
            const uint32_t w = e8m0_word(rb[i][r]);
            st_shared_v4(sSfb + stage * Cfg::kSfbBytes + r * 512 + lane * 16u, w, w, w, w);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sf_ready[stage]);
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
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const uint32_t t_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(half * 128);
    const uint32_t te_leader = mapa_shared(smem_u32(tmem_empty), 0);
    uint8_t* out_buf = smem + Cfg::kOffOut + static_cast<uint32_t>(warp - 4) * Cfg::kOutBytes;
    int iter = 0;
    for (int u = cluster_id; u < p.total_units; u += num_clusters, ++iter) {
      int b, mt, nt, s;
      decode_unit(u, p.tiles_m, p.tiles_n, 1, p.group_m, b, mt, nt, s);
      if (!mbar_wait(tmem_full, static_cast<uint32_t>(iter) & 1u, abort_flag, p.timeout_ns)) break;
      tc_fence_after();
      const int col_base = nt * 256 + half * 128;
      const int valid_cols = p.n - col_base;
      uint32_t w[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(t_base + static_cast<uint32_t>(c * 32), r);
#pragma unroll
        for (int v = 0; v < 16; ++v)
          w[c * 16 + v] = pack_bf16x2(__uint_as_float(r[2 * v]), __uint_as_float(r[2 * v + 1]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(te_leader);
      // 4 boxes of 32 rows x 32 columns through this warp's staging buffer
      const int row0 = mt * 256 + static_cast<int>(rank) * 128 + q * 32;
      if (row0 < p.m && valid_cols > 0) {
        const uint32_t swz = (lane >> 1) & 3u;   // 64-byte swizzle of row `lane`
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (c * 32 >= valid_cols) break;
          if (lane == 0) bulk_wait_group_read0();   // the previous box has left the buffer
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            st_shared_v4(out_buf + lane * 64u + ((static_cast<uint32_t>(j) ^ swz) * 16u), w[c * 16 + 4 * j],
                         w[c * 16 + 4 * j + 1], w[c * 16 + 4 * j + 2], w[c * 16 + 4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmC, out_buf, col_base + c * 32, row0, b);
            bulk_commit_group();
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group0();   // every store of this warp has completed
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();   // both CTAs done with TMEM, barriers and remote arrives
  tc_fence_after();
  if (warp == 2) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
}

}  // namespace bsg

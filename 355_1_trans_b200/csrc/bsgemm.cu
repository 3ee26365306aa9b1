// bsgemm.cu -- host side of the C ABI declared in include/bsgemm_b200.h:
// argument validation, TMA tensor-map encoding, tile / split-K planning and
// kernel dispatch.  The whole library is this one translation unit, so the
// per-device error word (sm100.cuh) is shared by every kernel.
//
// Validation mirrors the reference launcher
// (source_snapshot/gemm_a8w8_blockscale_bpreshuffle_launch.cc:31-65): null
// pointers, flags, shapes, strides, 16-byte rules of TMA, and C overlapping an
// input are rejected before anything is enqueued.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/bsgemm_b200.h"
#include "fp8_block_gemm.cuh"
#include "fp8_block_gemm_2sm.cuh"
#include "fp8_block_swap.cuh"
#include "mx_gemm.cuh"
#include "mx_gemm_2sm.cuh"
#include "mx_gemm_swap.cuh"
#include "pack.cuh"
#include "quant.cuh"

namespace {

using bsg::Fp8BlockCfg;
using bsg::Fp8BlockParams;
using bsg::MxCfg;
using bsg::MxParams;

constexpr unsigned long long kTimeoutNs = 10ull * 1000ull * 1000ull * 1000ull;  // 10 s per wait
// M tiles per rasterisation group: the CTAs in flight share a 16 x 128-row A
// panel group and walk its N tiles together (L2 reuse of A and B).
constexpr int kGroupM = 16;

// ---------------------------------------------------------------------------
// driver entry point for tensor-map encoding (no link-time libcuda dependency)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map of rank 2 to 5; dims/strides innermost first; strides[i] is the
// byte stride of dim i+1.
bool make_tmap_swz(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, int rank,
                   const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                   CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i < rank - 1) s[i] = strides[i];
  }
  const CUresult r = fn(m, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, int rank,
               const uint64_t* dims, const uint64_t* strides, const uint32_t* box, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i < rank - 1) s[i] = strides[i];
  }
  const CUresult r =
      fn(m, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
         CU_TENSOR_MAP_INTERLEAVE_NONE,
         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Byte tensor map (uint8 elements), 128B swizzle for operand tiles.
bool make_tmap_u8(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, bool swizzle128) {
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, rank, dims, strides, box, swizzle128);
}

// ---------------------------------------------------------------------------
// device facts (cached per device)
// ---------------------------------------------------------------------------
struct DevInfo {
  int sms = 0;
  bool sm100 = false;
  bool valid = false;
};

int device_info(DevInfo* out) {
  static DevInfo cache[64];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BSG_ERR_CUDA;
  if (dev < 0 || dev >= 64) return BSG_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev].valid) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return BSG_ERR_CUDA;
    cache[dev].sms = prop.multiProcessorCount;
    cache[dev].sm100 = prop.major == 10 && prop.minor == 0;
    cache[dev].valid = true;
  }
  *out = cache[dev];
  return BSG_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool overlaps(const void* a, uint64_t a_bytes, const void* b, uint64_t b_bytes) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + b_bytes && y < x + a_bytes;
}

// The CUDA error behind the calling thread's last BSG_ERR_CUDA (the
// reference-compatible entry point returns CUDA error codes).
thread_local cudaError_t t_last_cuda_error = cudaSuccess;

// Dynamic shared memory opt-in of a kernel, set once per (kernel, device):
// the attribute persists, so a launch that needs no more than the largest
// value already set skips the driver call.  Keyed on the kernel's address,
// since kernels of one signature share a template instantiation here.
struct SmemOptIn {
  const void* fn;
  int dev;
  uint32_t bytes;
};

template <typename K>
int set_smem(K kernel, uint32_t bytes) {
  static std::mutex mu;
  static SmemOptIn done[256];
  static int count = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BSG_ERR_CUDA;
  const void* fn = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  int slot = -1;
  for (int i = 0; i < count; ++i)
    if (done[i].fn == fn && done[i].dev == dev) slot = i;
  if (slot >= 0 && done[slot].bytes >= bytes) return BSG_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) {
    t_last_cuda_error = e;
    return BSG_ERR_CUDA;
  }
  if (slot >= 0) {
    done[slot].bytes = bytes;
  } else if (count < 256) {
    done[count++] = SmemOptIn{fn, dev, bytes};
  }
  return BSG_OK;
}

// Launch with programmatic stream serialization: the grid may launch while
// the previous kernel on the stream drains, so its prologue (barriers, TMEM,
// tensor-map prefetch, L2 prefetch of weights) overlaps that kernel.  Every
// GEMM kernel of this library runs griddepcontrol.wait before it reads or
// writes global memory that an earlier kernel may still own.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), int grid, int block, uint32_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(block));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) {
    t_last_cuda_error = e;
    return BSG_ERR_CUDA;
  }
  return BSG_OK;
}

// Same, as 1-D clusters of `cluster` CTAs (the grid a multiple of it).
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kern)(KArgs...), int grid, int cluster, int block, uint32_t smem, cudaStream_t st,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(block));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) {
    t_last_cuda_error = e;
    return BSG_ERR_CUDA;
  }
  return BSG_OK;
}

// Clusters of `cluster` CTAs of `kern` that fit on the device at once (0 when
// none does or the query fails).  Cached per (kernel, device, cluster size).
template <typename K>
int cluster_capacity(K kern, int cluster, int block, uint32_t smem) {
  struct Entry {
    const void* fn;
    int dev, cluster, n;
  };
  static std::mutex mu;
  static Entry done[64];
  static int count = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const void* fn = reinterpret_cast<const void*>(kern);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < count; ++i)
    if (done[i].fn == fn && done[i].dev == dev && done[i].cluster == cluster) return done[i].n;
  if (set_smem(kern, smem) != BSG_OK) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster * 64));
  cfg.blockDim = dim3(static_cast<unsigned>(block));
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  if (count < 64) done[count++] = Entry{fn, dev, cluster, n};
  return n;
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return BSG_OK;
  t_last_cuda_error = e;
  return BSG_ERR_CUDA;
}

int grid_for(int units, const DevInfo& dev, int grid_blocks) {
  int g = std::min(units, dev.sms);
  if (grid_blocks > 0) g = std::min(g, grid_blocks);
  return std::max(g, 1);
}

// ---------------------------------------------------------------------------
// split-K planning
// ---------------------------------------------------------------------------
struct Plan {
  int bn = 256;
  int tiles_m = 1, tiles_n = 1;
  int split = 1, kb_per = 1;
  int num_kb = 1;
  size_t ws_partials = 0;       // bytes of fp32 partials
  bool cluster = false;         // split-K slices of a tile reduced inside a CTA cluster
  int clusters = 0;             // co-resident clusters used (grid = clusters * split)
};

// Split-K choice for a persistent grid of `sms` CTAs, by a time model of the
// call fitted to B200 measurements of the decode-shaped kernels (µs, L2
// flushed): a round of units streams ceil(num_kb / s) K stages, each taking
// the longer of one SM's streaming time (sm_bytes_per_kb at the kernel's
// per-SM rate: about 90 GB/s for the fp32 block-scale and transposed decode
// kernels, 130 GB/s for the single-CTA MX kernel) and the round's share of
// HBM (hbm_bytes_per_kb of every active CTA at about 6 TB/s); every further round adds about 1 µs; a split adds the reduce
// kernel (about 3 µs) and the fp32 partials, an M x N write and read per
// slice.  Slices keep at least 4 K stages.  (A count of rounds x K stages
// alone chose 5 to 18 slices where 1 or 2 were fastest: M=16, N=7168,
// K=18432 ran 28.3 µs at 5 slices against 26.3 at 2.)
constexpr double kSmStreamBytesPerUs = 90.0e3;
constexpr double kSmStreamMxBytesPerUs = 130.0e3;
constexpr double kHbmBytesPerUs = 6.0e6;
constexpr double kRoundUs = 1.0;
constexpr double kReduceUs = 3.0;
int timed_split(long long tiles, int num_kb, int sms, int max_split, double sm_bytes_per_kb,
                double hbm_bytes_per_kb, double partial_bytes_per_slice, double sm_bytes_per_us) {
  if (tiles >= sms || num_kb < 8) return 1;
  const int smax = std::max(1, std::min(std::min(max_split, 64), num_kb / 4));
  int best_s = 1;
  double best = 0.0;
  for (int s = 1; s <= smax; ++s) {
    const long long units = tiles * s;
    const long long rounds = (units + sms - 1) / sms;
    const double active = static_cast<double>(std::min<long long>(units, sms));
    const double t_kb = std::max(sm_bytes_per_kb / sm_bytes_per_us, active * hbm_bytes_per_kb / kHbmBytesPerUs);
    double t = static_cast<double>(rounds) * ((num_kb + s - 1) / s) * t_kb + static_cast<double>(rounds - 1) * kRoundUs;
    if (s > 1) t += kReduceUs + s * partial_bytes_per_slice / kHbmBytesPerUs;
    if (s == 1 || t < best) {
      best = t;
      best_s = s;
    }
  }
  return best_s;
}

// sm_bytes_per_kb: bytes one CTA streams per K stage (A and B tiles);
// hbm_bytes_per_kb: the part of them that comes from HBM at decode shapes
// (the weight tile; the activations are shared through L2).
void plan_split(Plan& pl, const bsgemm_args& a, int sms, bool allow_auto, double sm_bytes_per_kb,
                double hbm_bytes_per_kb, double sm_bytes_per_us = kSmStreamBytesPerUs) {
  const long long tiles = static_cast<long long>(pl.tiles_m) * pl.tiles_n * a.batch;
  int split = 1;
  if (a.split_k > 1) {
    split = a.split_k;
  } else if (a.split_k == 0 && allow_auto) {
    const double partial = 8.0 * a.m * a.n * a.batch;   // fp32 write + read of one slice
    split = timed_split(tiles, pl.num_kb, sms, 64, sm_bytes_per_kb, hbm_bytes_per_kb, partial, sm_bytes_per_us);
  }
  split = std::min(split, pl.num_kb);
  pl.kb_per = (pl.num_kb + split - 1) / split;
  pl.split = (pl.num_kb + pl.kb_per - 1) / pl.kb_per;   // no empty slice
  pl.ws_partials = pl.split > 1 ? static_cast<size_t>(pl.split) * a.batch * a.m * a.n * 4 : 0;
}

// ---------------------------------------------------------------------------
// MXFP8 / MXFP4
// ---------------------------------------------------------------------------
size_t native_sf_bytes(int rows, int kg) {
  return static_cast<size_t>((rows + 127) / 128) * static_cast<size_t>((kg + 3) / 4) * 512u;
}

size_t align256(size_t x) { return (x + 255u) & ~static_cast<size_t>(255u); }

struct MxPlan : Plan {
  size_t ws_sfa = 0, ws_sfb = 0;  // bytes of packed scales in the workspace
};

// Activation rows per transposed-kernel tile (the MMA's N side): 16, 32 or 64.
int swap_mn(int m) { return m <= 16 ? 16 : m <= 32 ? 32 : 64; }

// Transposed MX kernel: decode-shaped M (one activation tile), both operands
// K-major (B raw or shuffle_weight(16,16)).
bool mx_use_swap(const bsgemm_args& a) {
  const bool eligible = a.m <= 64 && a.layout == BSG_LAYOUT_TN &&
                        (a.b_format == BSG_B_RAW || a.b_format == BSG_B_SHUFFLE16);
  return eligible && (a.kernel == BSG_KERNEL_SWAP || a.kernel == BSG_KERNEL_AUTO);
}

// In-cluster split-K of the transposed decode kernels (for calls without the
// workspace a split needs) and the cluster capacities it consults; defined
// with the kernels' launchers below.
bool swap_split_in_cluster(Plan& pl, const bsgemm_args& a, int (*capacity)(int mn, int split));
int swap_cluster_capacity(int mn, int split);
int mxs_cluster_capacity_fp8(int mn, int split);
int mxs_cluster_capacity_fp4(int mn, int split);

int mx_plan(const bsgemm_args& a, bool fp4, const DevInfo& dev, MxPlan& pl, bool allow_auto) {
  const int kg = a.k / 32;
  pl.num_kb = fp4 ? a.k / 256 : a.k / 128;
  if (mx_use_swap(a)) {
    pl.bn = swap_mn(a.m);   // activation rows per tile
    pl.tiles_m = 1;
    pl.tiles_n = (a.n + 127) / 128;
    plan_split(pl, a, dev.sms, allow_auto, 128.0 * (128 + pl.bn), 128.0 * 128);
  } else {
    pl.tiles_m = (a.m + 127) / 128;
    pl.bn = 256;
    if (static_cast<long long>(pl.tiles_m) * ((a.n + 255) / 256) * a.batch < dev.sms / 2 || a.n <= 128)
      pl.bn = 128;
    pl.tiles_n = (a.n + pl.bn - 1) / pl.bn;
    plan_split(pl, a, dev.sms, allow_auto, 128.0 * (128 + pl.bn), 128.0 * pl.bn, kSmStreamMxBytesPerUs);
  }
  pl.ws_sfa = a.sfa_format == BSG_SF_ROWMAJOR ? align256(native_sf_bytes(a.m, kg) * a.batch) : 0;
  pl.ws_sfb = a.sfb_format == BSG_SF_ROWMAJOR ? align256(native_sf_bytes(a.n, kg) * a.batch) : 0;
  return BSG_OK;
}

int validate_common(const bsgemm_args* a) {
  if (!a || !a->ptr_a || !a->ptr_b || !a->ptr_c || !a->ptr_sfa || !a->ptr_sfb)
    return BSG_ERR_INVALID_VALUE;
  if (a->m <= 0 || a->n <= 0 || a->k <= 0 || a->batch <= 0) return BSG_ERR_INVALID_VALUE;
  if (a->out_dtype != BSG_OUT_BF16 && a->out_dtype != BSG_OUT_FP32) return BSG_ERR_INVALID_VALUE;
  if (a->split_k < 0 || a->grid_blocks < 0) return BSG_ERR_INVALID_VALUE;
  if (a->layout < 0 || a->layout > 3) return BSG_ERR_INVALID_VALUE;
  if (a->kernel < BSG_KERNEL_AUTO || a->kernel > BSG_KERNEL_WIDE) return BSG_ERR_INVALID_VALUE;
  const int vec = a->out_dtype == BSG_OUT_BF16 ? 8 : 4;
  if (a->n % vec || a->stride_c < a->n || a->stride_c % vec) return BSG_ERR_ALIGNMENT;
  if (!aligned16(a->ptr_c)) return BSG_ERR_ALIGNMENT;
  if (a->batch > 1 && (a->stride_c_batch < static_cast<long long>(a->m) * a->stride_c ||
                       a->stride_c_batch % vec))
    return BSG_ERR_INVALID_VALUE;
  return BSG_OK;
}

// Operand extents in bytes, for the overlap test and tensor maps.
uint64_t operand_bytes(long long rows_of_storage, long long ld, long long batch_stride, int batch) {
  return static_cast<uint64_t>(batch > 1 ? batch_stride * (batch - 1) : 0) +
         static_cast<uint64_t>(rows_of_storage) * ld;
}

template <int BN, int kFp4, bool kAMN, int kBMode, bool kOutF32, int kSfMode>
int mx_launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p, int grid,
                cudaStream_t st) {
  using Cfg = MxCfg<BN, kFp4>;
  auto* kern = bsg::mx_gemm_kernel<BN, kFp4, kAMN, kBMode, kOutF32, kSfMode>;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, bsg::kMxThreads, Cfg::kSmemBytes, st, ta, tb, p);
  return rc != BSG_OK ? rc : launch_status();
}

// Grouped (MoE) mode of the single-CTA kernel: K-major A, native scales.
template <int BN, int kFp4, int kBMode, bool kOutF32>
int mx_launch_t_grouped(const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p, int grid,
                        cudaStream_t st) {
  using Cfg = MxCfg<BN, kFp4>;
  auto* kern = bsg::mx_gemm_kernel<BN, kFp4, false, kBMode, kOutF32, bsg::kSfNative, true>;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, bsg::kMxThreads, Cfg::kSmemBytes, st, ta, tb, p);
  return rc != BSG_OK ? rc : launch_status();
}

template <int BN, int kFp4, bool kAMN, int kBMode>
int mx_launch_out(bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p, int grid,
                  cudaStream_t st) {
  return f32 ? mx_launch_t<BN, kFp4, kAMN, kBMode, true, bsg::kSfNative>(ta, tb, p, grid, st)
             : mx_launch_t<BN, kFp4, kAMN, kBMode, false, bsg::kSfNative>(ta, tb, p, grid, st);
}

// Native-scale instantiations: fp8 takes every A/B orientation and the
// shuffled B; fp4 (.kind::mxf4) is K-major only.
template <int BN, int kFp4>
int mx_launch_bn(bool amn, int bmode, bool f32, const CUtensorMap& ta, const CUtensorMap& tb,
                 const MxParams& p, int grid, cudaStream_t st) {
  if constexpr (kFp4) {
    if (amn || bmode == bsg::kBMNMajor) return BSG_ERR_UNSUPPORTED;
    return bmode == bsg::kBShuffle16 ? mx_launch_out<BN, 1, false, bsg::kBShuffle16>(f32, ta, tb, p, grid, st)
                                     : mx_launch_out<BN, 1, false, bsg::kBKMajor>(f32, ta, tb, p, grid, st);
  } else {
    if (amn) {
      switch (bmode) {
        case bsg::kBKMajor: return mx_launch_out<BN, 0, true, bsg::kBKMajor>(f32, ta, tb, p, grid, st);
        case bsg::kBMNMajor: return mx_launch_out<BN, 0, true, bsg::kBMNMajor>(f32, ta, tb, p, grid, st);
        default: return mx_launch_out<BN, 0, true, bsg::kBShuffle16>(f32, ta, tb, p, grid, st);
      }
    }
    switch (bmode) {
      case bsg::kBKMajor: return mx_launch_out<BN, 0, false, bsg::kBKMajor>(f32, ta, tb, p, grid, st);
      case bsg::kBMNMajor: return mx_launch_out<BN, 0, false, bsg::kBMNMajor>(f32, ta, tb, p, grid, st);
      default: return mx_launch_out<BN, 0, false, bsg::kBShuffle16>(f32, ta, tb, p, grid, st);
    }
  }
}

// Per-128 E8M0 scales (launch_blockscale_bpreshuffle): A K-major, B shuffled.
template <int BN>
int mx_launch_e8m0b(bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p, int grid,
                    cudaStream_t st) {
  return f32 ? mx_launch_t<BN, 0, false, bsg::kBShuffle16, true, bsg::kSfE8m0Block128>(ta, tb, p, grid, st)
             : mx_launch_t<BN, 0, false, bsg::kBShuffle16, false, bsg::kSfE8m0Block128>(ta, tb, p, grid, st);
}

// Operand list of a pair launch: A, B, the two scale maps, C.
struct Mx2Maps {
  CUtensorMap a, b, sfa, sfb, c;
};

template <int kFp4, bool kAMN, int kBMode, int kSfMode>
int mx2_launch_t(const Mx2Maps& t, const bsg::Mx2Params& p, int grid, cudaStream_t st) {
  using Cfg = bsg::Mx2Cfg<kFp4>;
  auto* kern = bsg::mx_gemm_2sm_kernel<kFp4, kAMN, kBMode, kSfMode>;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, bsg::kMxThreads, Cfg::kSmemBytes, st, t.a, t.b, t.sfa, t.sfb, t.c, p);
  return rc != BSG_OK ? rc : launch_status();
}

int mx2_launch(bool fp4, bool amn, int bmode, int sfmode, const Mx2Maps& t, const bsg::Mx2Params& p, int grid,
               cudaStream_t st) {
  using namespace bsg;
  if (sfmode == kSfE8m0Block128) {
    if (fp4 || amn || bmode != kBShuffle16) return BSG_ERR_UNSUPPORTED;
    return mx2_launch_t<0, false, kBShuffle16, kSfE8m0Block128>(t, p, grid, st);
  }
  if (fp4) {
    if (amn || bmode == kBMNMajor) return BSG_ERR_UNSUPPORTED;
    return bmode == kBShuffle16 ? mx2_launch_t<1, false, kBShuffle16, kSfNative>(t, p, grid, st)
                                : mx2_launch_t<1, false, kBKMajor, kSfNative>(t, p, grid, st);
  }
  if (amn) {
    switch (bmode) {
      case kBKMajor: return mx2_launch_t<0, true, kBKMajor, kSfNative>(t, p, grid, st);
      case kBMNMajor: return mx2_launch_t<0, true, kBMNMajor, kSfNative>(t, p, grid, st);
      default: return mx2_launch_t<0, true, kBShuffle16, kSfNative>(t, p, grid, st);
    }
  }
  switch (bmode) {
    case kBKMajor: return mx2_launch_t<0, false, kBKMajor, kSfNative>(t, p, grid, st);
    case kBMNMajor: return mx2_launch_t<0, false, kBMNMajor, kSfNative>(t, p, grid, st);
    default: return mx2_launch_t<0, false, kBShuffle16, kSfNative>(t, p, grid, st);
  }
}

// Scale-atom tensor map: a native scale buffer viewed as [batch][atoms][128 x u32].
bool make_sf_tmap(CUtensorMap* m, const void* base, long long atoms_per_batch, int batch,
                  long long batch_stride_bytes, int atoms_per_box) {
  const uint64_t dims[3] = {128u, static_cast<uint64_t>(atoms_per_batch), static_cast<uint64_t>(batch)};
  const uint64_t strides[2] = {512u, static_cast<uint64_t>(batch > 1 ? batch_stride_bytes
                                                                     : atoms_per_batch * 512)};
  const uint32_t box[3] = {128u, static_cast<uint32_t>(atoms_per_box), 1u};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, base, 3, dims, strides, box, false);
}

// Operand tensor map over a plain [rows][ld] byte matrix (K-major or MN-major
// tile of 128 bytes x box_rows, 128B swizzle).
bool make_operand_tmap(CUtensorMap* m, const void* base, long long cols, long long rows, long long ld,
                       long long batch_stride, int batch, uint32_t box_rows) {
  const uint64_t dims[3] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows),
                            static_cast<uint64_t>(batch)};
  const uint64_t strides[2] = {static_cast<uint64_t>(ld),
                               static_cast<uint64_t>(batch > 1 ? batch_stride : rows * ld)};
  const uint32_t box[3] = {128u, box_rows, 1u};
  return make_tmap_u8(m, base, 3, dims, strides, box, true);
}

// Tensor map over B in the shuffle_weight(16,16) layout [N/16][Kb/16][16][16]
// (Kb = K in bytes): dims (16-byte row x 8 rows = one 128-byte core matrix,
// 16-byte K chunk, 8-row half of the 16-row group, 16-row group, batch).  A
// box of (128, 8, 2, box_rows/16, 1) is one 128-byte K stage of box_rows rows
// in the canonical no-swizzle K-major layout.
bool make_shuffle16_tmap(CUtensorMap* m, const void* base, long long rows, long long kbytes,
                         long long batch_stride, int batch, uint32_t box_rows) {
  const uint64_t dims[5] = {128u, static_cast<uint64_t>(kbytes / 16), 2u, static_cast<uint64_t>(rows / 16),
                            static_cast<uint64_t>(batch)};
  const uint64_t strides[4] = {256u, 128u, static_cast<uint64_t>(kbytes) * 16u,
                               static_cast<uint64_t>(batch > 1 ? batch_stride : rows * kbytes)};
  const uint32_t box[5] = {128u, 8u, 2u, box_rows / 16u, 1u};
  return make_tmap_u8(m, base, 5, dims, strides, box, false);
}

// Deterministic split-K reduction, launched with programmatic stream
// serialization: its launch overlaps the GEMM (which signals
// launch_dependents at its start) and the kernel waits for the GEMM's
// completion with griddepcontrol.wait before reading the partials.
int splitk_reduce(const float* ws, const bsgemm_args& a, int split, int sms, cudaStream_t st) {
  const long long total4 = static_cast<long long>(a.m) * a.n * a.batch / 4;
  const int grid = static_cast<int>(std::min<long long>((total4 + 255) / 256, 8LL * sms));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float* w = ws;
  void* c = a.ptr_c;
  int m = a.m, n = a.n, batch = a.batch;
  long long ldc = a.stride_c, cbs = a.stride_c_batch;
  cudaError_t e;
  if (a.out_dtype == BSG_OUT_FP32)
    e = cudaLaunchKernelEx(&cfg, bsg::splitk_reduce_kernel<true>, w, c, m, n, batch, split, ldc, cbs);
  else
    e = cudaLaunchKernelEx(&cfg, bsg::splitk_reduce_kernel<false>, w, c, m, n, batch, split, ldc, cbs);
  if (e != cudaSuccess) {
    t_last_cuda_error = e;
    return BSG_ERR_CUDA;
  }
  return launch_status();
}

// Resolved operands of one MX launch.
struct MxOperands {
  bool fp4 = false, a_mn = false;
  int bmode = bsg::kBKMajor;
  int sfmode = bsg::kSfNative;
  long long a_rows = 0, a_cols = 0, b_rows = 0, b_cols = 0;   // storage extents (bytes)
  long long kbytes = 0;
  const uint8_t* sfa = nullptr;
  const uint8_t* sfb = nullptr;
  long long sfa_bs = 0, sfb_bs = 0;       // native: atom batch strides; e8m0: byte batch strides
  long long sfa_ld = 0, sfb_ld = 0;       // e8m0 block-128 only
  float* partials = nullptr;
};

bool make_b_tmap(CUtensorMap* m, const bsgemm_args& a, const MxOperands& o, uint32_t box_rows) {
  if (o.bmode == bsg::kBShuffle16)
    return make_shuffle16_tmap(m, a.ptr_b, a.n, o.kbytes, a.stride_b_batch, a.batch, box_rows);
  return make_operand_tmap(m, a.ptr_b, o.b_cols, o.b_rows, a.stride_b, a.stride_b_batch, a.batch,
                           o.bmode == bsg::kBMNMajor ? 128u : box_rows);
}

template <int MN, int kFp4, int kBMode, bool kOutF32>
int mxs_launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p, int grid, cudaStream_t st,
                 int cluster) {
  if (cluster > 1) {
    using Cfg = bsg::MxSwapCfg<MN, kFp4, true>;
    auto* kern = bsg::mx_gemm_swap_kernel<MN, kFp4, kBMode, kOutF32, true>;
    if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
    const int rc = launch_pdl_cluster(kern, grid, cluster, 256, Cfg::kSmemBytes, st, ta, tb, p);
    return rc != BSG_OK ? rc : launch_status();
  }
  using Cfg = bsg::MxSwapCfg<MN, kFp4>;
  auto* kern = bsg::mx_gemm_swap_kernel<MN, kFp4, kBMode, kOutF32>;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, 256, Cfg::kSmemBytes, st, ta, tb, p);
  return rc != BSG_OK ? rc : launch_status();
}

template <int MN, int kFp4>
int mxs_launch_mn(int bmode, bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p, int grid,
                  cudaStream_t st, int cluster) {
  if (bmode == bsg::kBShuffle16)
    return f32 ? mxs_launch_t<MN, kFp4, bsg::kBShuffle16, true>(ta, tb, p, grid, st, cluster)
               : mxs_launch_t<MN, kFp4, bsg::kBShuffle16, false>(ta, tb, p, grid, st, cluster);
  return f32 ? mxs_launch_t<MN, kFp4, bsg::kBKMajor, true>(ta, tb, p, grid, st, cluster)
             : mxs_launch_t<MN, kFp4, bsg::kBKMajor, false>(ta, tb, p, grid, st, cluster);
}

template <int kFp4>
int mxs_launch(int mn, int bmode, bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p,
               int grid, cudaStream_t st, int cluster) {
  switch (mn) {
    case 16: return mxs_launch_mn<16, kFp4>(bmode, f32, ta, tb, p, grid, st, cluster);
    case 32: return mxs_launch_mn<32, kFp4>(bmode, f32, ta, tb, p, grid, st, cluster);
    default: return mxs_launch_mn<64, kFp4>(bmode, f32, ta, tb, p, grid, st, cluster);
  }
}

// Co-resident clusters of the MX decode kernel; all variants of one (MN,
// element type) share the shared-memory size, so one instantiation answers.
template <int kFp4>
int mxs_cluster_capacity(int mn, int split) {
  switch (mn) {
    case 16:
      return cluster_capacity(bsg::mx_gemm_swap_kernel<16, kFp4, bsg::kBKMajor, false, true>, split, 256,
                              bsg::MxSwapCfg<16, kFp4, true>::kSmemBytes);
    case 32:
      return cluster_capacity(bsg::mx_gemm_swap_kernel<32, kFp4, bsg::kBKMajor, false, true>, split, 256,
                              bsg::MxSwapCfg<32, kFp4, true>::kSmemBytes);
    default:
      return cluster_capacity(bsg::mx_gemm_swap_kernel<64, kFp4, bsg::kBKMajor, false, true>, split, 256,
                              bsg::MxSwapCfg<64, kFp4, true>::kSmemBytes);
  }
}
int mxs_cluster_capacity_fp8(int mn, int split) { return mxs_cluster_capacity<0>(mn, split); }
int mxs_cluster_capacity_fp4(int mn, int split) { return mxs_cluster_capacity<1>(mn, split); }

bool mx_use_pair(const bsgemm_args& a, const MxPlan& pl, const DevInfo& dev) {
  const long long pair_tiles = static_cast<long long>((a.m + 255) / 256) * ((a.n + 255) / 256) * a.batch;
  return a.kernel == BSG_KERNEL_PAIR ||
         (a.kernel == BSG_KERNEL_AUTO && pl.split == 1 && a.out_dtype == BSG_OUT_BF16 &&
          pair_tiles * 2 >= dev.sms);
}

// Tensor maps, parameters and launch of the planned MX GEMM (+ split-K reduce).
int mx_launch_planned(const bsgemm_args& a, const MxOperands& o, const MxPlan& pl, const DevInfo& dev,
                      cudaStream_t st) {
  const bool e8m0b = o.sfmode == bsg::kSfE8m0Block128;
  const int kg = a.k / 32;
  if (!e8m0b && mx_use_swap(a)) {
    // transposed decode kernel: activations box MN rows, weights box 128 rows
    CUtensorMap ta, tb;
    if (!make_operand_tmap(&ta, a.ptr_a, o.a_cols, o.a_rows, a.stride_a, a.stride_a_batch, a.batch,
                           static_cast<uint32_t>(pl.bn)) ||
        !make_b_tmap(&tb, a, o, 128u))
      return BSG_ERR_CUDA;
    MxParams p{};
    p.m = a.m;
    p.n = a.n;
    p.k = a.k;
    p.batch = a.batch;
    p.num_kb = pl.num_kb;
    p.tiles_m = 1;
    p.tiles_n = pl.tiles_n;
    p.split_k = pl.split;
    p.kb_per_split = pl.kb_per;
    p.total_units = pl.tiles_n * a.batch * pl.split;
    p.group_m = 1;
    p.sfa = o.sfa;
    p.sfb = o.sfb;
    p.sfa_batch_stride = o.sfa_bs;
    p.sfb_batch_stride = o.sfb_bs;
    p.sf_kb_total = (kg + 3) / 4;
    p.sfb_row_blocks = (a.n + 127) / 128;
    p.c = a.ptr_c;
    p.ldc = a.stride_c;
    p.c_batch_stride = a.stride_c_batch;
    p.ws = pl.split > 1 && !pl.cluster ? o.partials : nullptr;
    p.timeout_ns = kTimeoutNs;
    const int grid = pl.cluster ? pl.clusters * pl.split : grid_for(p.total_units, dev, a.grid_blocks);
    const int cluster = pl.cluster ? pl.split : 1;
    const bool f32 = a.out_dtype == BSG_OUT_FP32;
    const int rc = o.fp4 ? mxs_launch<1>(pl.bn, o.bmode, f32, ta, tb, p, grid, st, cluster)
                         : mxs_launch<0>(pl.bn, o.bmode, f32, ta, tb, p, grid, st, cluster);
    if (rc != BSG_OK) return rc;
    if (pl.split > 1 && !pl.cluster) return splitk_reduce(p.ws, a, pl.split, dev.sms, st);
    return BSG_OK;
  }
  if (a.kernel == BSG_KERNEL_SWAP) return BSG_ERR_UNSUPPORTED;
  if (mx_use_pair(a, pl, dev)) {
    if (pl.split > 1 || a.out_dtype != BSG_OUT_BF16) return BSG_ERR_UNSUPPORTED;
    if (!e8m0b && (o.sfa_bs % 512 || o.sfb_bs % 512)) return BSG_ERR_UNSUPPORTED;
    Mx2Maps t;
    CUtensorMap &ta = t.a, &tb = t.b, &tsa = t.sfa, &tsb = t.sfb;
    if (!make_operand_tmap(&ta, a.ptr_a, o.a_cols, o.a_rows, a.stride_a, a.stride_a_batch, a.batch, 128u) ||
        !make_b_tmap(&tb, a, o, 128u))
      return BSG_ERR_CUDA;
    {
      // C (bf16) for the TMA-store epilogue: boxes of 32 columns x 32 rows, 64-byte swizzle
      const uint64_t dims[3] = {static_cast<uint64_t>(a.n), static_cast<uint64_t>(a.m),
                                static_cast<uint64_t>(a.batch)};
      const uint64_t strides[2] = {static_cast<uint64_t>(a.stride_c) * 2u,
                                   static_cast<uint64_t>(a.batch > 1 ? a.stride_c_batch
                                                                     : static_cast<long long>(a.m) * a.stride_c) *
                                       2u};
      const uint32_t box[3] = {32u, 32u, 1u};
      if (!make_tmap_swz(&t.c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.ptr_c, 3, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_64B))
        return BSG_ERR_CUDA;
    }
    const int sf_kb_total = (kg + 3) / 4;
    const int atoms_k = o.fp4 ? 2 : 1;
    if (e8m0b) {
      std::memset(&tsa, 0, sizeof(tsa));   // unused: the kernel builds its scale atoms
      std::memset(&tsb, 0, sizeof(tsb));
    } else if (!make_sf_tmap(&tsa, o.sfa, static_cast<long long>((a.m + 127) / 128) * sf_kb_total, a.batch,
                             o.sfa_bs, atoms_k) ||
               !make_sf_tmap(&tsb, o.sfb, static_cast<long long>((a.n + 127) / 128) * sf_kb_total, a.batch,
                             o.sfb_bs, atoms_k)) {
      return BSG_ERR_CUDA;
    }
    bsg::Mx2Params q{};
    q.m = a.m;
    q.n = a.n;
    q.k = a.k;
    q.batch = a.batch;
    q.num_kb = pl.num_kb;
    q.tiles_m = (a.m + 255) / 256;
    q.tiles_n = (a.n + 255) / 256;
    q.total_units = q.tiles_m * q.tiles_n * a.batch;
    // 16 pair M-tiles (4096 rows) per raster group: fewest DRAM re-reads of
    // the panels at 8192^3, which under the 1 kW power cap is clock (2544 vs
    // 2436 TFLOPS with 8, 2399 with 32; sustained 2000-launch runs)
    q.group_m = std::min(q.tiles_m, kGroupM);
    q.sf_kb_total = sf_kb_total;
    q.sfa_row_blocks = (a.m + 127) / 128;
    q.sfb_row_blocks = (a.n + 127) / 128;
    q.sfa = o.sfa;
    q.sfb = o.sfb;
    q.sfa_ld = o.sfa_ld;
    q.sfb_ld = o.sfb_ld;
    q.sfa_batch_stride = o.sfa_bs;
    q.sfb_batch_stride = o.sfb_bs;
    q.c = a.ptr_c;
    q.ldc = a.stride_c;
    q.c_batch_stride = a.stride_c_batch;
    q.timeout_ns = kTimeoutNs;
    int clusters = std::min(q.total_units, dev.sms / 2);
    if (a.grid_blocks > 0) clusters = std::min(clusters, std::max(1, a.grid_blocks / 2));
    return mx2_launch(o.fp4, o.a_mn, o.bmode, o.sfmode, t, q, 2 * clusters, st);
  }

  CUtensorMap ta, tb;
  if (!make_operand_tmap(&ta, a.ptr_a, o.a_cols, o.a_rows, a.stride_a, a.stride_a_batch, a.batch, 128u) ||
      !make_b_tmap(&tb, a, o, static_cast<uint32_t>(pl.bn)))
    return BSG_ERR_CUDA;
  MxParams p{};
  p.m = a.m;
  p.n = a.n;
  p.k = a.k;
  p.batch = a.batch;
  p.num_kb = pl.num_kb;
  p.tiles_m = pl.tiles_m;
  p.tiles_n = pl.tiles_n;
  p.split_k = pl.split;
  p.kb_per_split = pl.kb_per;
  p.total_units = pl.tiles_m * pl.tiles_n * a.batch * pl.split;
  p.group_m = std::min(pl.tiles_m, kGroupM);
  p.sfa = o.sfa;
  p.sfb = o.sfb;
  p.sfa_batch_stride = o.sfa_bs;
  p.sfb_batch_stride = o.sfb_bs;
  p.sf_kb_total = (kg + 3) / 4;
  p.sfb_row_blocks = (a.n + 127) / 128;
  p.sfa_ld = o.sfa_ld;
  p.sfb_ld = o.sfb_ld;
  p.c = a.ptr_c;
  p.ldc = a.stride_c;
  p.c_batch_stride = a.stride_c_batch;
  p.ws = pl.split > 1 ? o.partials : nullptr;
  p.timeout_ns = kTimeoutNs;
  const int grid = grid_for(p.total_units, dev, a.grid_blocks);
  const bool f32 = a.out_dtype == BSG_OUT_FP32;
  int rc;
  if (e8m0b)
    rc = pl.bn == 256 ? mx_launch_e8m0b<256>(f32, ta, tb, p, grid, st) : mx_launch_e8m0b<128>(f32, ta, tb, p, grid, st);
  else if (pl.bn == 256)
    rc = o.fp4 ? mx_launch_bn<256, 1>(o.a_mn, o.bmode, f32, ta, tb, p, grid, st)
               : mx_launch_bn<256, 0>(o.a_mn, o.bmode, f32, ta, tb, p, grid, st);
  else
    rc = o.fp4 ? mx_launch_bn<128, 1>(o.a_mn, o.bmode, f32, ta, tb, p, grid, st)
               : mx_launch_bn<128, 0>(o.a_mn, o.bmode, f32, ta, tb, p, grid, st);
  if (rc != BSG_OK) return rc;
  if (pl.split > 1) return splitk_reduce(p.ws, a, pl.split, dev.sms, st);
  return BSG_OK;
}


int pack_sf_launch(const void* src, int src_stride, void* dst, int rows, int kg, int fmt,
                   int unpack, cudaStream_t st) {
  const long long words = static_cast<long long>((rows + 127) / 128) * ((kg + 3) / 4) * 128;
  const int grid = static_cast<int>(std::min<long long>((words + 255) / 256, 4096));
  bsg::pack_sf_native_kernel<<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(src), src_stride,
                                                  static_cast<uint8_t*>(dst), rows, kg, fmt,
                                                  unpack);
  return launch_status();
}

int mx_run(const bsgemm_args* args, bool fp4, cudaStream_t st) {
  int rc = validate_common(args);
  if (rc != BSG_OK) return rc;
  const bsgemm_args& a = *args;
  if (a.kernel == BSG_KERNEL_WIDE) return BSG_ERR_UNSUPPORTED;   // fp32 block scales only
  DevInfo dev;
  if ((rc = device_info(&dev)) != BSG_OK) return rc;
  if (!dev.sm100) return BSG_ERR_ARCH;
  if (a.k % (fp4 ? 256 : 128)) return BSG_ERR_INVALID_VALUE;
  const bool a_km = (a.layout & 1) != 0, b_km = (a.layout & 2) != 0;
  if (fp4 && (!a_km || !b_km)) return BSG_ERR_UNSUPPORTED;   // .kind::mxf4 is K-major only
  if (a.b_format != BSG_B_RAW && a.b_format != BSG_B_SHUFFLE16) return BSG_ERR_UNSUPPORTED;
  const bool shuffled = a.b_format == BSG_B_SHUFFLE16;
  if (shuffled && !b_km) return BSG_ERR_UNSUPPORTED;   // shuffle_weight is a K-major format
  for (int f : {a.sfa_format, a.sfb_format})
    if (f != BSG_SF_NATIVE && f != BSG_SF_ROWMAJOR) return BSG_ERR_UNSUPPORTED;

  MxOperands o;
  o.fp4 = fp4;
  o.a_mn = !a_km;
  o.bmode = shuffled ? bsg::kBShuffle16 : (b_km ? bsg::kBKMajor : bsg::kBMNMajor);
  o.kbytes = fp4 ? a.k / 2 : a.k;
  // A: K-major [M, kbytes] with ld stride_a, or M-major [K, M] with ld stride_a
  o.a_rows = a_km ? a.m : a.k;
  o.a_cols = a_km ? o.kbytes : a.m;
  o.b_rows = b_km ? a.n : a.k;
  o.b_cols = b_km ? o.kbytes : a.n;
  if (a.stride_a < o.a_cols || a.stride_a % 16 || a.stride_b < o.b_cols || a.stride_b % 16)
    return BSG_ERR_ALIGNMENT;
  if (shuffled && (a.n % 16 || a.stride_b != o.kbytes)) return BSG_ERR_INVALID_VALUE;   // dense 16x16 tiles
  if (!aligned16(a.ptr_a) || !aligned16(a.ptr_b)) return BSG_ERR_ALIGNMENT;
  if (a.batch > 1 && (a.stride_a_batch < o.a_rows * a.stride_a || a.stride_a_batch % 16 ||
                      a.stride_b_batch < o.b_rows * a.stride_b || a.stride_b_batch % 16))
    return BSG_ERR_INVALID_VALUE;
  const int kg = a.k / 32;
  // scale operands
  const size_t sfa_nat = native_sf_bytes(a.m, kg), sfb_nat = native_sf_bytes(a.n, kg);
  if (a.sfa_format == BSG_SF_NATIVE) {
    if (!aligned16(a.ptr_sfa)) return BSG_ERR_ALIGNMENT;
    o.sfa_bs = a.batch > 1 ? (a.stride_sfa_batch ? a.stride_sfa_batch : static_cast<long long>(sfa_nat)) : 0;
    if (o.sfa_bs % 16 || (a.batch > 1 && o.sfa_bs < static_cast<long long>(sfa_nat))) return BSG_ERR_INVALID_VALUE;
  } else if (a.stride_sfa < kg ||
             (a.batch > 1 && a.stride_sfa_batch < static_cast<long long>(a.m) * a.stride_sfa)) {
    return BSG_ERR_INVALID_VALUE;
  }
  if (a.sfb_format == BSG_SF_NATIVE) {
    if (!aligned16(a.ptr_sfb)) return BSG_ERR_ALIGNMENT;
    o.sfb_bs = a.batch > 1 ? (a.stride_sfb_batch ? a.stride_sfb_batch : static_cast<long long>(sfb_nat)) : 0;
    if (o.sfb_bs % 16 || (a.batch > 1 && o.sfb_bs < static_cast<long long>(sfb_nat))) return BSG_ERR_INVALID_VALUE;
  } else if (a.stride_sfb < kg ||
             (a.batch > 1 && a.stride_sfb_batch < static_cast<long long>(a.n) * a.stride_sfb)) {
    return BSG_ERR_INVALID_VALUE;
  }
  // C must not overlap an input
  const uint64_t c_bytes =
      operand_bytes(a.m, a.stride_c, a.stride_c_batch, a.batch) * (a.out_dtype == BSG_OUT_BF16 ? 2 : 4);
  if (overlaps(a.ptr_c, c_bytes, a.ptr_a, operand_bytes(o.a_rows, a.stride_a, a.stride_a_batch, a.batch)) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_b, operand_bytes(o.b_rows, a.stride_b, a.stride_b_batch, a.batch)))
    return BSG_ERR_INVALID_VALUE;

  MxPlan pl;
  mx_plan(a, fp4, dev, pl, true);
  size_t need = pl.ws_sfa + pl.ws_sfb + pl.ws_partials;
  if (need > a.workspace_bytes || (need && !a.workspace)) {
    const size_t scales = pl.ws_sfa + pl.ws_sfb;
    if (mx_use_swap(a) && scales <= a.workspace_bytes && (scales == 0 || a.workspace) &&
        swap_split_in_cluster(pl, a, fp4 ? mxs_cluster_capacity_fp4 : mxs_cluster_capacity_fp8)) {
      need = scales;   // split inside clusters: no partials in the workspace
    } else if (a.split_k == 0 && pl.split > 1) {   // auto split-K: drop it rather than fail
      bsgemm_args b2 = a;
      b2.split_k = 1;
      mx_plan(b2, fp4, dev, pl, false);
      need = pl.ws_sfa + pl.ws_sfb + pl.ws_partials;
    }
    if (need > a.workspace_bytes || (need && !a.workspace)) return BSG_ERR_WORKSPACE;
  }
  if (need && !aligned16(a.workspace)) return BSG_ERR_ALIGNMENT;
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  if (need && overlaps(a.ptr_c, c_bytes, ws, need)) return BSG_ERR_INVALID_VALUE;
  if (a.kernel == BSG_KERNEL_PAIR && pl.split > 1) return BSG_ERR_UNSUPPORTED;

  // scales in row-major form are packed into the workspace first
  o.sfa = static_cast<const uint8_t*>(a.ptr_sfa);
  o.sfb = static_cast<const uint8_t*>(a.ptr_sfb);
  if (a.sfa_format == BSG_SF_ROWMAJOR) {
    for (int bb = 0; bb < a.batch; ++bb)
      if ((rc = pack_sf_launch(o.sfa + static_cast<long long>(bb) * a.stride_sfa_batch, a.stride_sfa,
                               ws + bb * sfa_nat, a.m, kg, BSG_SF_ROWMAJOR, 0, st)) != BSG_OK)
        return rc;
    o.sfa = ws;
    o.sfa_bs = static_cast<long long>(sfa_nat);
  }
  if (a.sfb_format == BSG_SF_ROWMAJOR) {
    for (int bb = 0; bb < a.batch; ++bb)
      if ((rc = pack_sf_launch(o.sfb + static_cast<long long>(bb) * a.stride_sfb_batch, a.stride_sfb,
                               ws + pl.ws_sfa + bb * sfb_nat, a.n, kg, BSG_SF_ROWMAJOR, 0, st)) != BSG_OK)
        return rc;
    o.sfb = ws + pl.ws_sfa;
    o.sfb_bs = static_cast<long long>(sfb_nat);
  }
  o.partials = pl.split > 1 ? reinterpret_cast<float*>(ws + pl.ws_sfa + pl.ws_sfb) : nullptr;
  return mx_launch_planned(a, o, pl, dev, st);
}

// ---------------------------------------------------------------------------
// E8M0 1x128 / 128x128 block scale (the reference's launch_blockscale_bpreshuffle)
// ---------------------------------------------------------------------------
// Element count rows * cols * batch * bytes below 2^31, as the reference's
// bounded_count (source_snapshot/gemm_a8w8_blockscale_bpreshuffle_launch.cc:10-15).
bool bounded_count(int rows, int cols, int batch, int bytes) {
  const uint64_t limit = static_cast<uint64_t>(INT32_MAX) / static_cast<uint64_t>(bytes);
  if (rows <= 0 || cols <= 0 || batch <= 0 || static_cast<uint64_t>(rows) > limit / static_cast<uint64_t>(cols))
    return false;
  return static_cast<uint64_t>(batch) <= limit / (static_cast<uint64_t>(rows) * static_cast<uint64_t>(cols));
}

// Returns a cudaError_t value.  Validation follows the reference launcher
// (…_launch.cc:33-54) except that M may be any positive size and N a
// multiple of 128 (the reference: M, N % 256).  `tiles` (0 or 1, the
// reference's output-tiles-per-workgroup switch) selects the tile shape:
// 0 = planned here (CTA pairs for large problems), 1 = single-CTA tiles.
int e8m0b_run(const bsgemm_args& in, bool bf16, int tiles, cudaStream_t st) {
  const bsgemm_args& a = in;
  if (!a.ptr_a || !a.ptr_b || !a.ptr_c || !a.ptr_sfa || !a.ptr_sfb) return cudaErrorInvalidValue;
  if (a.m <= 0 || a.n <= 0 || a.k <= 0 || a.batch <= 0 || a.n % 128 || a.k % 128)
    return cudaErrorInvalidValue;
  const int kb = a.k / 128, nb = a.n / 128;
  if (!bounded_count(a.m, a.k, a.batch, 1) || !bounded_count(a.n, a.k, a.batch, 1) ||
      !bounded_count(a.m, a.n, a.batch, bf16 ? 2 : 4) || !bounded_count(a.m, kb, a.batch, 1) ||
      !bounded_count(nb, kb, a.batch, 1))
    return cudaErrorInvalidValue;
  if (a.stride_a != a.k || a.stride_b != a.k || a.stride_c != a.n || a.stride_a_batch != a.m * a.k ||
      a.stride_b_batch != a.n * a.k || a.stride_c_batch != a.m * a.n || a.stride_sfa != a.m ||
      a.stride_sfb != kb || a.stride_sfa_batch != a.m * kb || a.stride_sfb_batch != nb * kb)
    return cudaErrorInvalidValue;
  const uint64_t c_bytes = static_cast<uint64_t>(a.m) * a.n * a.batch * (bf16 ? 2 : 4);
  if (overlaps(a.ptr_c, c_bytes, a.ptr_a, static_cast<uint64_t>(a.stride_a_batch) * a.batch) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_b, static_cast<uint64_t>(a.stride_b_batch) * a.batch) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_sfa, static_cast<uint64_t>(a.stride_sfa_batch) * a.batch) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_sfb, static_cast<uint64_t>(a.stride_sfb_batch) * a.batch))
    return cudaErrorInvalidValue;
  // TMA and the vector stores need 16-byte aligned A, B and C
  if (!aligned16(a.ptr_a) || !aligned16(a.ptr_b) || !aligned16(a.ptr_c)) return cudaErrorInvalidValue;
  DevInfo dev;
  if (device_info(&dev) != BSG_OK) {
    const cudaError_t e = cudaGetLastError();
    return e != cudaSuccess ? e : cudaErrorUnknown;
  }
  if (!dev.sm100) return cudaErrorInvalidDeviceFunction;

  bsgemm_args g = a;
  g.layout = BSG_LAYOUT_TN;
  g.b_format = BSG_B_SHUFFLE16;
  g.sfa_format = BSG_SF_NATIVE;   // no repack: the kernel builds its scale atoms
  g.sfb_format = BSG_SF_NATIVE;
  g.out_dtype = bf16 ? BSG_OUT_BF16 : BSG_OUT_FP32;
  g.split_k = 1;                  // no workspace in this ABI
  g.workspace = nullptr;
  g.workspace_bytes = 0;
  g.grid_blocks = 0;
  // decode-sized M also takes the single-CTA kernel (its scale builder is
  // the one that reads per-128 E8M0 bytes)
  g.kernel = tiles == 1 || a.m <= 64 ? BSG_KERNEL_1CTA : BSG_KERNEL_AUTO;
  MxOperands o;
  o.bmode = bsg::kBShuffle16;
  o.sfmode = bsg::kSfE8m0Block128;
  o.kbytes = a.k;
  o.a_rows = a.m;
  o.a_cols = a.k;
  o.b_rows = a.n;
  o.b_cols = a.k;
  o.sfa = static_cast<const uint8_t*>(a.ptr_sfa);
  o.sfb = static_cast<const uint8_t*>(a.ptr_sfb);
  o.sfa_bs = a.stride_sfa_batch;
  o.sfb_bs = a.stride_sfb_batch;
  o.sfa_ld = a.stride_sfa;
  o.sfb_ld = a.stride_sfb;
  MxPlan pl;
  mx_plan(g, false, dev, pl, false);
  t_last_cuda_error = cudaSuccess;
  const int rc = mx_launch_planned(g, o, pl, dev, st);
  if (rc == BSG_OK) return cudaSuccess;
  if (rc == BSG_ERR_CUDA) return t_last_cuda_error != cudaSuccess ? t_last_cuda_error : cudaErrorUnknown;
  return cudaErrorNotSupported;
}

// ---------------------------------------------------------------------------
// FP8 block-scale (fp32 scales)
// ---------------------------------------------------------------------------
template <int kBFmt, bool kOutF32>
int fp8b_launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8BlockParams& p, int grid,
                  cudaStream_t st) {
  using Cfg = Fp8BlockCfg<128>;
  auto* kern = bsg::fp8_block_gemm_kernel<128, kBFmt, kOutF32>;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, 256, Cfg::kSmemBytes, st, ta, tb, p);
  return rc != BSG_OK ? rc : launch_status();
}

template <int kBFmt, bool kOutF32, bool kGrouped>
int fp8b2_launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Fp8BlockParams& p,
                   int grid, cudaStream_t st) {
  using Cfg = bsg::Fp8Block2Cfg<true>;
  auto* kern = bsg::fp8_block_gemm_2sm_kernel<kBFmt, kOutF32, kGrouped>;
  // The kernel's warpgroups re-split their registers with setmaxnreg; the
  // split is sized for exactly Cfg::kLaunchRegs registers per thread at launch
  // (with fewer, the promotion warps' increase could never be granted).
  static const int regs = [kern] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, kern) == cudaSuccess ? fa.numRegs : -1;
  }();
  if (regs != Cfg::kLaunchRegs) return BSG_ERR_UNSUPPORTED;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, Cfg::kThreads, Cfg::kSmemBytes, st, ta, tb, tc, p);
  return rc != BSG_OK ? rc : launch_status();
}

template <bool kGrouped>
int fp8b2_launch(int fmt, bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                 const Fp8BlockParams& p, int grid, cudaStream_t st) {
  switch (fmt) {
    case bsg::kFmtKPanel:
      return f32 ? fp8b2_launch_t<bsg::kFmtKPanel, true, kGrouped>(ta, tb, tc, p, grid, st)
                 : fp8b2_launch_t<bsg::kFmtKPanel, false, kGrouped>(ta, tb, tc, p, grid, st);
    case bsg::kFmtShuffle16:
      return f32 ? fp8b2_launch_t<bsg::kFmtShuffle16, true, kGrouped>(ta, tb, tc, p, grid, st)
                 : fp8b2_launch_t<bsg::kFmtShuffle16, false, kGrouped>(ta, tb, tc, p, grid, st);
    default:
      return f32 ? fp8b2_launch_t<bsg::kFmtRaw, true, kGrouped>(ta, tb, tc, p, grid, st)
                 : fp8b2_launch_t<bsg::kFmtRaw, false, kGrouped>(ta, tb, tc, p, grid, st);
  }
}

// The wide single-CTA kernel (128 x 256 units); same register rule as the pair.
template <int kBFmt, bool kOutF32>
int fp8bw_launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Fp8BlockParams& p,
                   int grid, cudaStream_t st) {
  using Cfg = bsg::Fp8Block2Cfg<false>;
  auto* kern = bsg::fp8_block_gemm_wide_kernel<kBFmt, kOutF32>;
  static const int regs = [kern] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, kern) == cudaSuccess ? fa.numRegs : -1;
  }();
  if (regs != Cfg::kLaunchRegs) return BSG_ERR_UNSUPPORTED;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, Cfg::kThreads, Cfg::kSmemBytes, st, ta, tb, tc, p);
  return rc != BSG_OK ? rc : launch_status();
}

int fp8bw_launch(int fmt, bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                 const Fp8BlockParams& p, int grid, cudaStream_t st) {
  switch (fmt) {
    case bsg::kFmtKPanel:
      return f32 ? fp8bw_launch_t<bsg::kFmtKPanel, true>(ta, tb, tc, p, grid, st)
                 : fp8bw_launch_t<bsg::kFmtKPanel, false>(ta, tb, tc, p, grid, st);
    case bsg::kFmtShuffle16:
      return f32 ? fp8bw_launch_t<bsg::kFmtShuffle16, true>(ta, tb, tc, p, grid, st)
                 : fp8bw_launch_t<bsg::kFmtShuffle16, false>(ta, tb, tc, p, grid, st);
    default:
      return f32 ? fp8bw_launch_t<bsg::kFmtRaw, true>(ta, tb, tc, p, grid, st)
                 : fp8bw_launch_t<bsg::kFmtRaw, false>(ta, tb, tc, p, grid, st);
  }
}

// Clusters of a pair launch: one per two SMs, or per two CTAs of a grid cap.
int fp8b_pair_clusters(const bsgemm_args& a, int sms) {
  int c = std::max(1, sms / 2);
  if (a.grid_blocks > 0) c = std::min(c, std::max(1, a.grid_blocks / 2));
  return c;
}

// Tail split of a pair launch: the units past the last full wave of
// `clusters` (all units, when there are fewer than a wave) run as K slices,
// as many per unit as the clusters allow, each at least 8 K blocks (shorter
// slices cost more in pipeline fill and partials than they save: 1024 x 24576
// x 1536, 12 K blocks, ran slower in slices of 2 and of 4).  Returns the bytes
// of fp32 partials it needs, 0 for no split.
size_t fp8b_pair_tail(long long units, int clusters, int num_kb, int* tail_units, int* tail_split) {
  const long long t = units >= clusters ? units % clusters : units;
  const int s = t > 0 ? static_cast<int>(std::min<long long>(clusters / t, num_kb / 8)) : 1;
  // the slices' reduce costs about 6 µs: split only when the tail unit saves
  // at least 16 K blocks (~10 µs; 8192 x 7168 x 2048, 16 K blocks in two
  // slices, ran 3 % slower than whole)
  if (t == 0 || s < 2 || num_kb - (num_kb + s - 1) / s < 16) {
    *tail_units = 0;
    *tail_split = 1;
    return 0;
  }
  *tail_units = static_cast<int>(t);
  *tail_split = s;
  return static_cast<size_t>(t) * static_cast<size_t>(s) * 256u * 256u * 4u;
}

// CTA-pair kernel (256 x 256 tiles): on request, or for an automatic call
// that the 1-CTA kernel (128 x 128 tiles) would cover in more time, counted
// in waves: a pair unit's K block costs about 1.6 of a 1-CTA tile's (B200,
// 8192 x 7168 x 8192: 1100 against 680 cycles), and a wave is sms / 2 pair
// units or sms tiles.  With split_k 0 the pair's partial last wave runs as K
// slices (fp8b_pair_tail), counted as 1/s of a wave plus kPairTailCost for
// the partials and their reduction.
constexpr double kPairKbCost = 1.6;
constexpr double kPairTailCost = 0.1;
bool fp8b_use_pair(const bsgemm_args& a, int sms) {
  if (a.kernel == BSG_KERNEL_PAIR) return true;
  // at M <= 128 the peer CTA of every pair would hold no rows
  if (a.kernel != BSG_KERNEL_AUTO || a.m <= 128 || a.split_k > 1) return false;
  const long long units = static_cast<long long>((a.m + 255) / 256) * ((a.n + 255) / 256) * a.batch;
  const long long tiles = static_cast<long long>((a.m + 127) / 128) * ((a.n + 127) / 128) * a.batch;
  const int clusters = std::max(1, sms / 2);
  int tu = 0, ts = 1;
  fp8b_pair_tail(units, clusters, a.k / 128, &tu, &ts);
  double pair_waves = static_cast<double>(units / clusters);
  if (tu > 0)
    pair_waves += 1.0 / ts + kPairTailCost;
  else if (units % clusters)
    pair_waves += 1.0;
  const double one_waves = static_cast<double>((tiles + sms - 1) / sms);
  return pair_waves * kPairKbCost < one_waves;
}

// Sums the K slices of a pair launch (256-row units) or of a wide launch
// (128-row units, `wide`).
int fp8b2_tail_reduce(const Fp8BlockParams& p, bool f32, int sms, cudaStream_t st, bool wide = false) {
  const long long groups = static_cast<long long>(p.tail_units) * (wide ? 128 : 256) * 64;
  const int grid = static_cast<int>(std::min<long long>((groups + 255) / 256, 8LL * sms));
  int rc;
  if (wide)
    rc = f32 ? launch_pdl(bsg::fp8b_pair_tail_reduce_kernel<true, 128>, grid, 256, 0, st, p)
             : launch_pdl(bsg::fp8b_pair_tail_reduce_kernel<false, 128>, grid, 256, 0, st, p);
  else
    rc = f32 ? launch_pdl(bsg::fp8b_pair_tail_reduce_kernel<true>, grid, 256, 0, st, p)
             : launch_pdl(bsg::fp8b_pair_tail_reduce_kernel<false>, grid, 256, 0, st, p);
  return rc != BSG_OK ? rc : launch_status();
}

// Wide single-CTA kernel (128 x 256 units): on request.  K splits like the
// other kernels (split_k > 1 forced, 0 by the time model of a unit's 48 KB
// stage, 32 KB of it weights); every unit is then cut into that many K
// slices, summed by the reduce above.  Returns the split and, in *ws_bytes,
// the fp32 partials it needs.
bool fp8b_use_wide(const bsgemm_args& a) { return a.kernel == BSG_KERNEL_WIDE; }
int fp8b_wide_split(const bsgemm_args& a, int sms, size_t* ws_bytes) {
  const long long units = static_cast<long long>((a.m + 127) / 128) * ((a.n + 255) / 256) * a.batch;
  const int num_kb = a.k / 128;
  int s = 1;
  if (a.split_k > 1)
    s = std::min(a.split_k, num_kb);
  else if (a.split_k == 0)
    s = timed_split(units, num_kb, sms, 64, 49152.0, 32768.0, 8.0 * a.m * a.n * a.batch, kSmStreamBytesPerUs);
  *ws_bytes = s > 1 ? static_cast<size_t>(units) * static_cast<size_t>(s) * 128u * 256u * 4u : 0;
  return s;
}

// Transposed decode kernel: on request (M <= 64), and automatically for
// M <= 32.  From 33 to 64 rows the single-CTA kernel measured as fast or
// faster (M=64: 9.9 against 13.2 µs at N=7168 K=2048, 33.4 against 43.2 at
// K=18432; M=32 within 0.1 µs).
bool fp8b_use_swap(const bsgemm_args& a) {
  return a.kernel == BSG_KERNEL_SWAP || (a.kernel == BSG_KERNEL_AUTO && a.m <= 32);
}

// Split-K of the transposed decode kernels for a call without the workspace
// its split needs: the K slices of a tile run on the CTAs of one cluster and
// are summed through distributed shared memory, so no partials leave the
// chip.  (With a workspace the partials plus the reduce kernel measured as
// fast or faster, so that stays the first choice.)  An automatic split is
// capped at kSwapMaxClusterSplit; a forced one must not exceed it.  Returns
// false (plan unchanged) when no cluster of that size fits.
bool swap_split_in_cluster(Plan& pl, const bsgemm_args& a, int (*capacity)(int mn, int split)) {
  if (pl.split < 2 || (a.split_k > 1 && pl.split > bsg::kSwapMaxClusterSplit)) return false;
  const int want = std::min(pl.split, bsg::kSwapMaxClusterSplit);
  const int kb_per = (pl.num_kb + want - 1) / want;
  const int split = (pl.num_kb + kb_per - 1) / kb_per;   // no empty slice
  if (split < 2) return false;
  int cap = capacity(pl.bn, split);
  if (a.grid_blocks > 0) cap = std::min(cap, a.grid_blocks / split);
  if (cap <= 0) return false;
  const long long tiles = static_cast<long long>(pl.tiles_m) * pl.tiles_n * a.batch;
  pl.kb_per = kb_per;
  pl.split = split;
  pl.cluster = true;
  pl.clusters = static_cast<int>(std::min<long long>(tiles, cap));
  pl.ws_partials = 0;
  return true;
}

void fp8b_plan(const bsgemm_args& a, const DevInfo& dev, Plan& pl, bool allow_auto) {
  pl.num_kb = a.k / 128;
  pl.tiles_n = (a.n + 127) / 128;
  if (fp8b_use_swap(a)) {
    const int mn = swap_mn(a.m);
    pl.bn = mn;
    pl.tiles_m = (a.m + mn - 1) / mn;
    plan_split(pl, a, dev.sms, allow_auto, 16384.0 + 128.0 * mn, 16384.0);
  } else {
    pl.bn = 128;
    pl.tiles_m = (a.m + 127) / 128;
    plan_split(pl, a, dev.sms, allow_auto, 32768.0, 16384.0);
  }
}

template <int MN, int kBFmt, bool kOutF32>
int swap_launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8BlockParams& p, int grid,
                  cudaStream_t st, int cluster) {
  if (cluster > 1) {
    using Cfg = bsg::SwapCfg<MN, true>;
    auto* kern = bsg::fp8_block_swap_kernel<MN, kBFmt, kOutF32, true>;
    if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
    const int rc = launch_pdl_cluster(kern, grid, cluster, Cfg::kThreads, Cfg::kSmemBytes, st, ta, tb, p);
    return rc != BSG_OK ? rc : launch_status();
  }
  using Cfg = bsg::SwapCfg<MN>;
  auto* kern = bsg::fp8_block_swap_kernel<MN, kBFmt, kOutF32>;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, Cfg::kThreads, Cfg::kSmemBytes, st, ta, tb, p);
  return rc != BSG_OK ? rc : launch_status();
}

template <int MN>
int swap_cluster_capacity_mn(int split) {
  using Cfg = bsg::SwapCfg<MN, true>;
  return cluster_capacity(bsg::fp8_block_swap_kernel<MN, bsg::kFmtKPanel, false, true>, split, Cfg::kThreads,
                          Cfg::kSmemBytes);
}

// All variants of one MN share the shared-memory size, so one instantiation
// answers for all.
int swap_cluster_capacity(int mn, int split) {
  switch (mn) {
    case 16: return swap_cluster_capacity_mn<16>(split);
    case 32: return swap_cluster_capacity_mn<32>(split);
    default: return swap_cluster_capacity_mn<64>(split);
  }
}

template <int kBFmt>
int fp8b_launch_fmt(bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const Fp8BlockParams& p,
                    int grid, cudaStream_t st) {
  return f32 ? fp8b_launch_t<kBFmt, true>(ta, tb, p, grid, st) : fp8b_launch_t<kBFmt, false>(ta, tb, p, grid, st);
}

template <int MN, int kBFmt>
int swap_launch_fmt(bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const Fp8BlockParams& p,
                    int grid, cudaStream_t st, int cluster) {
  return f32 ? swap_launch_t<MN, kBFmt, true>(ta, tb, p, grid, st, cluster)
             : swap_launch_t<MN, kBFmt, false>(ta, tb, p, grid, st, cluster);
}

template <int MN>
int swap_launch_mn(int fmt, bool f32, const CUtensorMap& ta, const CUtensorMap& tb,
                   const Fp8BlockParams& p, int grid, cudaStream_t st, int cluster) {
  switch (fmt) {
    case bsg::kFmtKPanel: return swap_launch_fmt<MN, bsg::kFmtKPanel>(f32, ta, tb, p, grid, st, cluster);
    case bsg::kFmtShuffle16: return swap_launch_fmt<MN, bsg::kFmtShuffle16>(f32, ta, tb, p, grid, st, cluster);
    default: return swap_launch_fmt<MN, bsg::kFmtRaw>(f32, ta, tb, p, grid, st, cluster);
  }
}

// Tensor map of the fp8 block-scale weights (batch = experts for grouped
// calls): shuffle_weight(16,16), K panels B'[K/128][N][128], or raw [N, K].
bool make_fp8b_weight_tmap(CUtensorMap* tb, const bsgemm_args& a, bool kpanel, bool shuf, int kb,
                           long long b_elems) {
  if (shuf) return make_shuffle16_tmap(tb, a.ptr_b, a.n, a.k, a.stride_b_batch, a.batch, 128u);
  if (kpanel) {
    const uint64_t dims[4] = {128u, static_cast<uint64_t>(a.n), static_cast<uint64_t>(kb),
                              static_cast<uint64_t>(a.batch)};
    const uint64_t strides[3] = {128u, static_cast<uint64_t>(a.n) * 128u,
                                 static_cast<uint64_t>(a.batch > 1 ? a.stride_b_batch : b_elems)};
    const uint32_t box[4] = {128u, 128u, 1u, 1u};
    return make_tmap_u8(tb, a.ptr_b, 4, dims, strides, box, true);
  }
  const uint64_t dims[3] = {static_cast<uint64_t>(a.k), static_cast<uint64_t>(a.n),
                            static_cast<uint64_t>(a.batch)};
  const uint64_t strides[2] = {static_cast<uint64_t>(a.stride_b),
                               static_cast<uint64_t>(a.batch > 1 ? a.stride_b_batch : b_elems)};
  const uint32_t box[3] = {128u, 128u, 1u};
  return make_tmap_u8(tb, a.ptr_b, 3, dims, strides, box, true);
}

int fp8b_run(const bsgemm_args* args, cudaStream_t st) {
  int rc = validate_common(args);
  if (rc != BSG_OK) return rc;
  const bsgemm_args& a = *args;
  DevInfo dev;
  if ((rc = device_info(&dev)) != BSG_OK) return rc;
  if (!dev.sm100) return BSG_ERR_ARCH;
  if (a.k % 128) return BSG_ERR_INVALID_VALUE;
  if (a.layout != BSG_LAYOUT_TN) return BSG_ERR_UNSUPPORTED;
  if (a.b_format != BSG_B_RAW && a.b_format != BSG_B_KPANEL128 && a.b_format != BSG_B_SHUFFLE16)
    return BSG_ERR_UNSUPPORTED;
  if (a.kernel == BSG_KERNEL_SWAP && a.m > 64) return BSG_ERR_UNSUPPORTED;
  if (a.kernel == BSG_KERNEL_PAIR && a.split_k > 1) return BSG_ERR_UNSUPPORTED;
  if (a.sfa_format != BSG_SF_ROWMAJOR && a.sfa_format != BSG_SF_KMAJOR_T) return BSG_ERR_UNSUPPORTED;
  if (a.sfb_format != BSG_SF_ROWMAJOR) return BSG_ERR_UNSUPPORTED;
  const bool kpanel = a.b_format == BSG_B_KPANEL128;
  const bool shuf = a.b_format == BSG_B_SHUFFLE16;
  const int bfmt = kpanel ? bsg::kFmtKPanel : shuf ? bsg::kFmtShuffle16 : bsg::kFmtRaw;
  const int kb = a.k / 128, nb = (a.n + 127) / 128;
  if (a.stride_a < a.k || a.stride_a % 16 || !aligned16(a.ptr_a) || !aligned16(a.ptr_b))
    return BSG_ERR_ALIGNMENT;
  if (kpanel ? a.stride_b != 128 : (a.stride_b < a.k || a.stride_b % 16)) return BSG_ERR_ALIGNMENT;
  if (shuf && (a.stride_b != a.k || a.n % 16)) return BSG_ERR_INVALID_VALUE;   // dense 16x16 tiles
  const long long b_elems = kpanel ? static_cast<long long>(a.n) * a.k : static_cast<long long>(a.n) * a.stride_b;
  if (a.batch > 1 && (a.stride_a_batch < static_cast<long long>(a.m) * a.stride_a ||
                      a.stride_a_batch % 16 || a.stride_b_batch < b_elems || a.stride_b_batch % 16))
    return BSG_ERR_INVALID_VALUE;
  // fp32 scale strides (floats)
  long long sfa_m, sfa_k;
  if (a.sfa_format == BSG_SF_ROWMAJOR) {
    if (a.stride_sfa < kb) return BSG_ERR_INVALID_VALUE;
    sfa_m = a.stride_sfa;
    sfa_k = 1;
  } else {
    if (a.stride_sfa < a.m) return BSG_ERR_INVALID_VALUE;
    sfa_m = 1;
    sfa_k = a.stride_sfa;
  }
  if (a.stride_sfb < kb) return BSG_ERR_INVALID_VALUE;
  if (a.batch > 1 && (a.stride_sfa_batch < static_cast<long long>(a.m) * kb ||
                      a.stride_sfb_batch < static_cast<long long>(nb) * kb))
    return BSG_ERR_INVALID_VALUE;
  const uint64_t c_bytes =
      operand_bytes(a.m, a.stride_c, a.stride_c_batch, a.batch) * (a.out_dtype == BSG_OUT_BF16 ? 2 : 4);
  if (overlaps(a.ptr_c, c_bytes, a.ptr_a, operand_bytes(a.m, a.stride_a, a.stride_a_batch, a.batch)) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_b,
               static_cast<uint64_t>(a.batch > 1 ? a.stride_b_batch * (a.batch - 1) : 0) + b_elems) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_sfa,
               4ull * (a.batch > 1 ? a.stride_sfa_batch * a.batch : static_cast<long long>(a.m) * kb)) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_sfb,
               4ull * (a.batch > 1 ? a.stride_sfb_batch * a.batch : static_cast<long long>(nb) * kb)))
    return BSG_ERR_INVALID_VALUE;

  Plan pl;
  fp8b_plan(a, dev, pl, true);
  const bool pair = fp8b_use_pair(a, dev.sms);
  const bool wide = fp8b_use_wide(a);
  if (pair || wide) {   // these plan their K slices themselves (the tail / wide split)
    pl.tiles_m = pair ? (a.m + 255) / 256 : (a.m + 127) / 128;
    pl.tiles_n = (a.n + 255) / 256;
    pl.split = 1;
    pl.kb_per = pl.num_kb;
    pl.ws_partials = 0;
    pl.cluster = false;
  }
  if (pl.ws_partials > a.workspace_bytes || (pl.ws_partials && !a.workspace)) {
    if (fp8b_use_swap(a) && swap_split_in_cluster(pl, a, swap_cluster_capacity)) {
      // split inside clusters: no workspace
    } else if (a.split_k == 0) {
      bsgemm_args b2 = a;
      b2.split_k = 1;
      fp8b_plan(b2, dev, pl, false);
    } else {
      return BSG_ERR_WORKSPACE;
    }
  }
  if (pl.ws_partials && !aligned16(a.workspace)) return BSG_ERR_ALIGNMENT;
  if (pl.ws_partials && overlaps(a.ptr_c, c_bytes, a.workspace, pl.ws_partials))
    return BSG_ERR_INVALID_VALUE;

  CUtensorMap ta, tb;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(a.k), static_cast<uint64_t>(a.m),
                              static_cast<uint64_t>(a.batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(a.stride_a),
                                 static_cast<uint64_t>(a.batch > 1 ? a.stride_a_batch
                                                                   : static_cast<long long>(a.m) * a.stride_a)};
    const bool swap = fp8b_use_swap(a);
    const uint32_t box[3] = {128u, swap ? static_cast<uint32_t>(swap_mn(a.m)) : 128u, 1u};
    if (!make_tmap_u8(&ta, a.ptr_a, 3, dims, strides, box, true)) return BSG_ERR_CUDA;
  }
  if (!make_fp8b_weight_tmap(&tb, a, kpanel, shuf, kb, b_elems)) return BSG_ERR_CUDA;
  Fp8BlockParams p{};
  p.m = a.m;
  p.n = a.n;
  p.k = a.k;
  p.batch = a.batch;
  p.num_kb = pl.num_kb;
  p.tiles_m = pl.tiles_m;
  p.tiles_n = pl.tiles_n;
  p.split_k = pl.split;
  p.kb_per_split = pl.kb_per;
  p.total_units = pl.tiles_m * pl.tiles_n * a.batch * pl.split;
  p.group_m = std::min(pl.tiles_m, kGroupM);
  p.sfa = static_cast<const float*>(a.ptr_sfa);
  p.sfa_m = sfa_m;
  p.sfa_k = sfa_k;
  p.sfa_batch = a.stride_sfa_batch;
  p.sfb = static_cast<const float*>(a.ptr_sfb);
  p.sfb_n = a.stride_sfb;
  p.sfb_k = 1;
  p.sfb_batch = a.stride_sfb_batch;
  p.c = a.ptr_c;
  p.ldc = a.stride_c;
  p.c_batch_stride = a.stride_c_batch;
  p.ws = pl.split > 1 && !pl.cluster ? static_cast<float*>(a.workspace) : nullptr;
  p.timeout_ns = kTimeoutNs;
  const int grid = pl.cluster ? pl.clusters * pl.split : grid_for(p.total_units, dev, a.grid_blocks);
  const int cluster = pl.cluster ? pl.split : 1;
  const bool f32 = a.out_dtype == BSG_OUT_FP32;
  if (pair || wide) {
    // C (bf16) for the TMA-store epilogue: boxes of 32 columns x 32 rows,
    // 64-byte swizzle (fp32 C is stored directly)
    CUtensorMap tc;
    std::memset(&tc, 0, sizeof(tc));
    if (!f32) {
      const uint64_t dims[3] = {static_cast<uint64_t>(a.n), static_cast<uint64_t>(a.m),
                                static_cast<uint64_t>(a.batch)};
      const uint64_t strides[2] = {static_cast<uint64_t>(a.stride_c) * 2u,
                                   static_cast<uint64_t>(a.batch > 1 ? a.stride_c_batch
                                                                     : static_cast<long long>(a.m) * a.stride_c) *
                                       2u};
      const uint32_t box[3] = {32u, 32u, 1u};
      if (!make_tmap_swz(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.ptr_c, 3, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_64B))
        return BSG_ERR_CUDA;
    }
    if (wide) {
      // every unit in s K slices (s 1: whole units, stored directly)
      size_t ws_bytes = 0;
      int s = fp8b_wide_split(a, dev.sms, &ws_bytes);
      if (ws_bytes && (!a.workspace || a.workspace_bytes < ws_bytes)) {
        if (a.split_k > 1) return BSG_ERR_WORKSPACE;
        s = 1;
        ws_bytes = 0;
      }
      if (ws_bytes && !aligned16(a.workspace)) return BSG_ERR_ALIGNMENT;
      if (ws_bytes && overlaps(a.ptr_c, c_bytes, a.workspace, ws_bytes)) return BSG_ERR_INVALID_VALUE;
      p.tail_units = s > 1 ? p.total_units : 0;
      p.tail_split = s;
      p.total_items = p.total_units - p.tail_units + p.tail_units * s;
      p.ws = ws_bytes ? static_cast<float*>(a.workspace) : nullptr;
      rc = fp8bw_launch(bfmt, f32, ta, tb, tc, p, grid_for(p.total_items, dev, a.grid_blocks), st);
      if (rc != BSG_OK || p.tail_units == 0) return rc;
      return fp8b2_tail_reduce(p, f32, dev.sms, st, true);
    }
    // the partial last wave as K slices, when the caller's workspace holds
    // their fp32 partials (split_k 1 keeps every unit whole)
    const int cl = fp8b_pair_clusters(a, dev.sms);
    int tu = 0, ts = 1;
    size_t tail_bytes = a.split_k == 0 ? fp8b_pair_tail(p.total_units, cl, pl.num_kb, &tu, &ts) : 0;
    if (tail_bytes && (!a.workspace || a.workspace_bytes < tail_bytes || !aligned16(a.workspace) ||
                       overlaps(a.ptr_c, c_bytes, a.workspace, tail_bytes))) {
      tu = 0;
      ts = 1;
      tail_bytes = 0;
    }
    p.tail_units = tu;
    p.tail_split = ts;
    p.total_items = p.total_units - tu + tu * ts;
    p.ws = tail_bytes ? static_cast<float*>(a.workspace) : nullptr;
    const int clusters = std::min(p.total_items, cl);
    rc = fp8b2_launch<false>(bfmt, f32, ta, tb, tc, p, 2 * clusters, st);
    if (rc != BSG_OK || tu == 0) return rc;
    return fp8b2_tail_reduce(p, f32, dev.sms, st);
  }
  if (fp8b_use_swap(a)) {
    switch (swap_mn(a.m)) {
      case 16: rc = swap_launch_mn<16>(bfmt, f32, ta, tb, p, grid, st, cluster); break;
      case 32: rc = swap_launch_mn<32>(bfmt, f32, ta, tb, p, grid, st, cluster); break;
      default: rc = swap_launch_mn<64>(bfmt, f32, ta, tb, p, grid, st, cluster); break;
    }
  } else {
    switch (bfmt) {
      case bsg::kFmtKPanel: rc = fp8b_launch_fmt<bsg::kFmtKPanel>(f32, ta, tb, p, grid, st); break;
      case bsg::kFmtShuffle16: rc = fp8b_launch_fmt<bsg::kFmtShuffle16>(f32, ta, tb, p, grid, st); break;
      default: rc = fp8b_launch_fmt<bsg::kFmtRaw>(f32, ta, tb, p, grid, st); break;
    }
  }
  if (rc != BSG_OK) return rc;
  if (pl.split > 1 && !pl.cluster) return splitk_reduce(p.ws, a, pl.split, dev.sms, st);
  return BSG_OK;
}

template <int kBFmt, bool kOutF32>
int fp8b_grouped_launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8BlockParams& p, int grid,
                          cudaStream_t st) {
  using Cfg = Fp8BlockCfg<128>;
  auto* kern = bsg::fp8_block_gemm_kernel<128, kBFmt, kOutF32, true>;
  if (set_smem(kern, Cfg::kSmemBytes) != BSG_OK) return BSG_ERR_CUDA;
  const int rc = launch_pdl(kern, grid, 256, Cfg::kSmemBytes, st, ta, tb, p);
  return rc != BSG_OK ? rc : launch_status();
}

// Grouped (MoE) fp32 block-scale GEMM on the 1-CTA kernel.  a.batch groups
// (experts): group e multiplies rows [offsets[e], offsets[e + 1]) of the
// concatenated A [total_rows, K] (and the same rows of x_scale) by its own
// weights B_e and their scales, and writes the same rows of C [total_rows, N].
// a.m bounds the rows of one group (it sizes the tile grid); the offsets are
// read on the device, so the routing needs no host round trip.
int fp8b_grouped_run(const bsgemm_args* args, const int* group_offsets, int total_rows, cudaStream_t st) {
  if (!args || !group_offsets || total_rows <= 0) return BSG_ERR_INVALID_VALUE;
  const bsgemm_args& a = *args;
  if (!a.ptr_a || !a.ptr_b || !a.ptr_c || !a.ptr_sfa || !a.ptr_sfb) return BSG_ERR_INVALID_VALUE;
  if (a.m <= 0 || a.n <= 0 || a.k <= 0 || a.batch <= 0 || a.grid_blocks < 0 || a.split_k < 0)
    return BSG_ERR_INVALID_VALUE;
  if (a.out_dtype != BSG_OUT_BF16 && a.out_dtype != BSG_OUT_FP32) return BSG_ERR_INVALID_VALUE;
  if (a.split_k > 1) return BSG_ERR_UNSUPPORTED;
  if (a.kernel != BSG_KERNEL_AUTO && a.kernel != BSG_KERNEL_1CTA && a.kernel != BSG_KERNEL_PAIR)
    return BSG_ERR_UNSUPPORTED;
  if (a.layout != BSG_LAYOUT_TN) return BSG_ERR_UNSUPPORTED;
  if (a.sfa_format != BSG_SF_ROWMAJOR || a.sfb_format != BSG_SF_ROWMAJOR) return BSG_ERR_UNSUPPORTED;
  if (a.b_format != BSG_B_RAW && a.b_format != BSG_B_KPANEL128 && a.b_format != BSG_B_SHUFFLE16)
    return BSG_ERR_UNSUPPORTED;
  DevInfo dev;
  int rc;
  if ((rc = device_info(&dev)) != BSG_OK) return rc;
  if (!dev.sm100) return BSG_ERR_ARCH;
  if (a.k % 128) return BSG_ERR_INVALID_VALUE;
  const int vec = a.out_dtype == BSG_OUT_BF16 ? 8 : 4;
  if (a.n % vec || a.stride_c < a.n || a.stride_c % vec || !aligned16(a.ptr_c)) return BSG_ERR_ALIGNMENT;
  const bool kpanel = a.b_format == BSG_B_KPANEL128;
  const bool shuf = a.b_format == BSG_B_SHUFFLE16;
  const int bfmt = kpanel ? bsg::kFmtKPanel : shuf ? bsg::kFmtShuffle16 : bsg::kFmtRaw;
  const int kb = a.k / 128, nb = (a.n + 127) / 128;
  if (a.stride_a < a.k || a.stride_a % 16 || !aligned16(a.ptr_a) || !aligned16(a.ptr_b))
    return BSG_ERR_ALIGNMENT;
  if (kpanel ? a.stride_b != 128 : (a.stride_b < a.k || a.stride_b % 16)) return BSG_ERR_ALIGNMENT;
  if (shuf && (a.stride_b != a.k || a.n % 16)) return BSG_ERR_INVALID_VALUE;
  const long long b_elems = kpanel ? static_cast<long long>(a.n) * a.k : static_cast<long long>(a.n) * a.stride_b;
  if (a.batch > 1 && (a.stride_b_batch < b_elems || a.stride_b_batch % 16)) return BSG_ERR_INVALID_VALUE;
  if (a.stride_sfa < kb || a.stride_sfb < kb) return BSG_ERR_INVALID_VALUE;
  if (a.batch > 1 && a.stride_sfb_batch < static_cast<long long>(nb) * kb) return BSG_ERR_INVALID_VALUE;
  const uint64_t c_bytes =
      static_cast<uint64_t>(total_rows) * a.stride_c * (a.out_dtype == BSG_OUT_BF16 ? 2 : 4);
  const uint64_t b_bytes = static_cast<uint64_t>(a.batch > 1 ? a.stride_b_batch * (a.batch - 1) : 0) + b_elems;
  const uint64_t sfb_bytes = 4ull * (a.batch > 1 ? a.stride_sfb_batch * a.batch : static_cast<long long>(nb) * kb);
  if (overlaps(a.ptr_c, c_bytes, a.ptr_a, static_cast<uint64_t>(total_rows) * a.stride_a) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_b, b_bytes) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_sfa, 4ull * total_rows * a.stride_sfa) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_sfb, sfb_bytes) ||
      overlaps(a.ptr_c, c_bytes, group_offsets, 4ull * (a.batch + 1)))
    return BSG_ERR_INVALID_VALUE;

  CUtensorMap ta, tb;
  {
    // A over all rows of all groups; a tile that runs past its group's last
    // row reads the next group's rows (or zero fill past total_rows), and
    // those rows are not stored
    const uint64_t dims[3] = {static_cast<uint64_t>(a.k), static_cast<uint64_t>(total_rows), 1u};
    const uint64_t strides[2] = {static_cast<uint64_t>(a.stride_a),
                                 static_cast<uint64_t>(total_rows) * static_cast<uint64_t>(a.stride_a)};
    const uint32_t box[3] = {128u, 128u, 1u};
    if (!make_tmap_u8(&ta, a.ptr_a, 3, dims, strides, box, true)) return BSG_ERR_CUDA;
  }
  if (!make_fp8b_weight_tmap(&tb, a, kpanel, shuf, kb, b_elems)) return BSG_ERR_CUDA;
  Fp8BlockParams p{};
  p.m = a.m;
  p.n = a.n;
  p.k = a.k;
  p.batch = a.batch;
  p.num_kb = kb;
  p.tiles_m = (a.m + 127) / 128;
  p.tiles_n = nb;
  p.split_k = 1;
  p.kb_per_split = kb;
  p.total_units = p.tiles_m * p.tiles_n * a.batch;
  p.group_m = kGroupM;   // rasterises the live M tiles, whose count only the device knows
  p.sfa = static_cast<const float*>(a.ptr_sfa);
  p.sfa_m = a.stride_sfa;
  p.sfa_k = 1;
  p.sfa_batch = 0;
  p.sfb = static_cast<const float*>(a.ptr_sfb);
  p.sfb_n = a.stride_sfb;
  p.sfb_k = 1;
  p.sfb_batch = a.stride_sfb_batch;
  p.c = a.ptr_c;
  p.ldc = a.stride_c;
  p.c_batch_stride = 0;
  p.ws = nullptr;
  p.timeout_ns = kTimeoutNs;
  p.group_offsets = group_offsets;
  p.total_rows = total_rows;
  const bool f32 = a.out_dtype == BSG_OUT_FP32;
  if (a.kernel == BSG_KERNEL_PAIR) {
    // CTA pairs, 256-row tiles per group (on request: with groups of a few
    // hundred rows or more; the host does not see the group sizes); C is
    // stored with row masks, so no C tensor map
    p.tiles_m = (a.m + 255) / 256;
    p.tiles_n = (a.n + 255) / 256;
    p.total_units = p.tiles_m * p.tiles_n * a.batch;
    p.tail_units = 0;
    p.tail_split = 1;
    p.total_items = p.total_units;
    CUtensorMap tc;
    std::memset(&tc, 0, sizeof(tc));
    const int clusters = std::min(p.total_units, fp8b_pair_clusters(a, dev.sms));
    return fp8b2_launch<true>(bfmt, f32, ta, tb, tc, p, 2 * clusters, st);
  }
  const int grid = grid_for(p.total_units, dev, a.grid_blocks);
  switch (bfmt) {
    case bsg::kFmtKPanel:
      return f32 ? fp8b_grouped_launch_t<bsg::kFmtKPanel, true>(ta, tb, p, grid, st)
                 : fp8b_grouped_launch_t<bsg::kFmtKPanel, false>(ta, tb, p, grid, st);
    case bsg::kFmtShuffle16:
      return f32 ? fp8b_grouped_launch_t<bsg::kFmtShuffle16, true>(ta, tb, p, grid, st)
                 : fp8b_grouped_launch_t<bsg::kFmtShuffle16, false>(ta, tb, p, grid, st);
    default:
      return f32 ? fp8b_grouped_launch_t<bsg::kFmtRaw, true>(ta, tb, p, grid, st)
                 : fp8b_grouped_launch_t<bsg::kFmtRaw, false>(ta, tb, p, grid, st);
  }
}

// ---------------------------------------------------------------------------
// Grouped (MoE) MXFP8 / MXFP4: the grouped mode of the single-CTA MX kernel
// ---------------------------------------------------------------------------
template <int BN, int kFp4, int kBMode>
int mx_grouped_launch_t(bool f32, const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p, int grid,
                        cudaStream_t st) {
  return f32 ? mx_launch_t_grouped<BN, kFp4, kBMode, true>(ta, tb, p, grid, st)
             : mx_launch_t_grouped<BN, kFp4, kBMode, false>(ta, tb, p, grid, st);
}

template <int kFp4>
int mx_grouped_launch(int bn, int bmode, bool f32, const CUtensorMap& ta, const CUtensorMap& tb,
                      const MxParams& p, int grid, cudaStream_t st) {
  if (bn == 256)
    return bmode == bsg::kBShuffle16 ? mx_grouped_launch_t<256, kFp4, bsg::kBShuffle16>(f32, ta, tb, p, grid, st)
                                     : mx_grouped_launch_t<256, kFp4, bsg::kBKMajor>(f32, ta, tb, p, grid, st);
  return bmode == bsg::kBShuffle16 ? mx_grouped_launch_t<128, kFp4, bsg::kBShuffle16>(f32, ta, tb, p, grid, st)
                                   : mx_grouped_launch_t<128, kFp4, bsg::kBKMajor>(f32, ta, tb, p, grid, st);
}

// args: m = the most rows any group may have, batch = groups; A [total_rows,
// K] (packed bytes for fp4) with row-major E8M0 scales [total_rows, K/32]
// (stride_sfa), which are packed per group into the workspace; B [groups, N,
// K] raw or shuffle_weight(16,16) at stride_b_batch, its scales native or
// row-major per group.
int mx_grouped_run(const bsgemm_args* args, bool fp4, const int* group_offsets, int total_rows,
                   cudaStream_t st) {
  if (!args || !group_offsets || total_rows <= 0) return BSG_ERR_INVALID_VALUE;
  const bsgemm_args& a = *args;
  if (!a.ptr_a || !a.ptr_b || !a.ptr_c || !a.ptr_sfa || !a.ptr_sfb) return BSG_ERR_INVALID_VALUE;
  if (a.m <= 0 || a.n <= 0 || a.k <= 0 || a.batch <= 0 || a.grid_blocks < 0 || a.split_k < 0)
    return BSG_ERR_INVALID_VALUE;
  if (a.out_dtype != BSG_OUT_BF16 && a.out_dtype != BSG_OUT_FP32) return BSG_ERR_INVALID_VALUE;
  if (a.split_k > 1) return BSG_ERR_UNSUPPORTED;
  if (a.kernel != BSG_KERNEL_AUTO && a.kernel != BSG_KERNEL_1CTA) return BSG_ERR_UNSUPPORTED;
  if (a.layout != BSG_LAYOUT_TN) return BSG_ERR_UNSUPPORTED;
  if (a.b_format != BSG_B_RAW && a.b_format != BSG_B_SHUFFLE16) return BSG_ERR_UNSUPPORTED;
  if (a.sfa_format != BSG_SF_ROWMAJOR) return BSG_ERR_UNSUPPORTED;
  if (a.sfb_format != BSG_SF_NATIVE && a.sfb_format != BSG_SF_ROWMAJOR) return BSG_ERR_UNSUPPORTED;
  DevInfo dev;
  int rc;
  if ((rc = device_info(&dev)) != BSG_OK) return rc;
  if (!dev.sm100) return BSG_ERR_ARCH;
  if (a.k % (fp4 ? 256 : 128)) return BSG_ERR_INVALID_VALUE;
  const int vec = a.out_dtype == BSG_OUT_BF16 ? 8 : 4;
  if (a.n % vec || a.stride_c < a.n || a.stride_c % vec || !aligned16(a.ptr_c)) return BSG_ERR_ALIGNMENT;
  const bool shuffled = a.b_format == BSG_B_SHUFFLE16;
  const long long kbytes = fp4 ? a.k / 2 : a.k;
  const int kg = a.k / 32;
  if (a.stride_a < kbytes || a.stride_a % 16 || a.stride_b < kbytes || a.stride_b % 16 || !aligned16(a.ptr_a) ||
      !aligned16(a.ptr_b))
    return BSG_ERR_ALIGNMENT;
  if (shuffled && (a.n % 16 || a.stride_b != kbytes)) return BSG_ERR_INVALID_VALUE;
  const long long b_bytes1 = static_cast<long long>(a.n) * a.stride_b;
  if (a.batch > 1 && (a.stride_b_batch < b_bytes1 || a.stride_b_batch % 16)) return BSG_ERR_INVALID_VALUE;
  if (a.stride_sfa < kg) return BSG_ERR_INVALID_VALUE;
  const size_t sfa_nat = native_sf_bytes(a.m, kg), sfb_nat = native_sf_bytes(a.n, kg);
  long long sfb_bs = 0;
  uint64_t sfb_bytes;
  if (a.sfb_format == BSG_SF_NATIVE) {
    if (!aligned16(a.ptr_sfb)) return BSG_ERR_ALIGNMENT;
    sfb_bs = a.batch > 1 ? (a.stride_sfb_batch ? a.stride_sfb_batch : static_cast<long long>(sfb_nat)) : 0;
    if (sfb_bs % 16 || (a.batch > 1 && sfb_bs < static_cast<long long>(sfb_nat))) return BSG_ERR_INVALID_VALUE;
    sfb_bytes = static_cast<uint64_t>(sfb_bs) * (a.batch - 1) + sfb_nat;
  } else {
    if (a.stride_sfb < kg || (a.batch > 1 && a.stride_sfb_batch < static_cast<long long>(a.n) * a.stride_sfb))
      return BSG_ERR_INVALID_VALUE;
    sfb_bytes = static_cast<uint64_t>(a.batch > 1 ? a.stride_sfb_batch * (a.batch - 1) : 0) +
                static_cast<uint64_t>(a.n) * a.stride_sfb;
  }
  // workspace: the per-group A scale atoms, (row-major B scales) B's atoms,
  // then the prefix of the groups' M tiles
  const size_t ws_sfa = align256(sfa_nat * a.batch);
  const size_t ws_sfb = a.sfb_format == BSG_SF_ROWMAJOR ? align256(sfb_nat * a.batch) : 0;
  const size_t need = ws_sfa + ws_sfb + align256(4u * (static_cast<size_t>(a.batch) + 1));
  if (need > a.workspace_bytes || !a.workspace) return BSG_ERR_WORKSPACE;
  if (!aligned16(a.workspace)) return BSG_ERR_ALIGNMENT;
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  const uint64_t c_bytes =
      static_cast<uint64_t>(total_rows) * a.stride_c * (a.out_dtype == BSG_OUT_BF16 ? 2 : 4);
  const uint64_t b_bytes = static_cast<uint64_t>(a.batch > 1 ? a.stride_b_batch * (a.batch - 1) : 0) + b_bytes1;
  const uint64_t sfa_bytes = static_cast<uint64_t>(total_rows) * a.stride_sfa;
  const uint64_t off_bytes = 4ull * (a.batch + 1);
  if (overlaps(a.ptr_c, c_bytes, a.ptr_a, static_cast<uint64_t>(total_rows) * a.stride_a) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_b, b_bytes) || overlaps(a.ptr_c, c_bytes, a.ptr_sfa, sfa_bytes) ||
      overlaps(a.ptr_c, c_bytes, a.ptr_sfb, sfb_bytes) || overlaps(a.ptr_c, c_bytes, group_offsets, off_bytes) ||
      overlaps(a.ptr_c, c_bytes, ws, need) || overlaps(ws, need, a.ptr_a, static_cast<uint64_t>(total_rows) * a.stride_a) ||
      overlaps(ws, need, a.ptr_b, b_bytes) || overlaps(ws, need, a.ptr_sfa, sfa_bytes) ||
      overlaps(ws, need, a.ptr_sfb, sfb_bytes) || overlaps(ws, need, group_offsets, off_bytes))
    return BSG_ERR_INVALID_VALUE;

  CUtensorMap ta, tb;
  // A over all rows of all groups; a tile that runs past its group's last row
  // reads the next group's rows (or zero fill past total_rows), and those
  // rows are not stored
  if (!make_operand_tmap(&ta, a.ptr_a, kbytes, total_rows, a.stride_a, 0, 1, 128u)) return BSG_ERR_CUDA;
  const int tiles_m = (a.m + 127) / 128;
  int bn = 256;
  if (static_cast<long long>(tiles_m) * ((a.n + 255) / 256) * a.batch < dev.sms / 2 || a.n <= 128) bn = 128;
  MxOperands o;
  o.fp4 = fp4;
  o.bmode = shuffled ? bsg::kBShuffle16 : bsg::kBKMajor;
  o.kbytes = kbytes;
  o.b_rows = a.n;
  o.b_cols = kbytes;
  if (!make_b_tmap(&tb, a, o, static_cast<uint32_t>(bn))) return BSG_ERR_CUDA;

  // scale atoms: A per group (device offsets) with the M-tile prefix, B per
  // batch when row-major
  int* tile_prefix = reinterpret_cast<int*>(ws + ws_sfa + ws_sfb);
  {
    const long long words = static_cast<long long>(sfa_nat / 4) * a.batch;
    const int grid = static_cast<int>(std::min<long long>((words + 255) / 256, 4096));
    bsg::pack_sf_grouped_kernel<<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(a.ptr_sfa), a.stride_sfa,
                                                     group_offsets, a.batch, total_rows, a.m, kg, ws,
                                                     tile_prefix);
    if ((rc = launch_status()) != BSG_OK) return rc;
  }
  const uint8_t* sfb = static_cast<const uint8_t*>(a.ptr_sfb);
  if (a.sfb_format == BSG_SF_ROWMAJOR) {
    for (int bb = 0; bb < a.batch; ++bb)
      if ((rc = pack_sf_launch(sfb + static_cast<long long>(bb) * a.stride_sfb_batch, a.stride_sfb,
                               ws + ws_sfa + bb * sfb_nat, a.n, kg, BSG_SF_ROWMAJOR, 0, st)) != BSG_OK)
        return rc;
    sfb = ws + ws_sfa;
    sfb_bs = static_cast<long long>(sfb_nat);
  }

  MxParams p{};
  p.m = a.m;
  p.n = a.n;
  p.k = a.k;
  p.batch = a.batch;
  p.num_kb = fp4 ? a.k / 256 : a.k / 128;
  p.tiles_m = tiles_m;
  p.tiles_n = (a.n + bn - 1) / bn;
  p.split_k = 1;
  p.kb_per_split = p.num_kb;
  p.total_units = p.tiles_m * p.tiles_n * a.batch;
  p.group_m = std::min(p.tiles_m, kGroupM);
  p.sfa = ws;
  p.sfb = sfb;
  p.sfa_batch_stride = static_cast<long long>(sfa_nat);
  p.sfb_batch_stride = sfb_bs;
  p.sf_kb_total = (kg + 3) / 4;
  p.sfb_row_blocks = (a.n + 127) / 128;
  p.c = a.ptr_c;
  p.ldc = a.stride_c;
  p.c_batch_stride = 0;
  p.ws = nullptr;
  p.timeout_ns = kTimeoutNs;
  p.group_offsets = group_offsets;
  p.total_rows = total_rows;
  p.tile_prefix = tile_prefix;
  p.group_m = kGroupM;   // over the live M tiles, whose count only the device knows
  const int grid = grid_for(p.total_units, dev, a.grid_blocks);
  const bool f32 = a.out_dtype == BSG_OUT_FP32;
  return fp4 ? mx_grouped_launch<1>(bn, o.bmode, f32, ta, tb, p, grid, st)
             : mx_grouped_launch<0>(bn, o.bmode, f32, ta, tb, p, grid, st);
}

// ---------------------------------------------------------------------------
// Host-staged MX GEMM: operands and C in host memory, copies pipelined with
// the GEMM blocks (the reference drivers' copy-in / launch / copy-out flow)
// ---------------------------------------------------------------------------
constexpr int kHostMaxChunks = 8;

// Per-device streams and events of the pipeline, created once.  The whole
// enqueue sequence of a call holds the device's mutex, so two host threads
// never interleave their records and waits on the shared events.
struct HostPipe {
  bool ready = false;
  cudaStream_t comp = nullptr, d2h = nullptr;
  cudaEvent_t start = nullptr, end = nullptr;
  cudaEvent_t in_a[kHostMaxChunks] = {}, in_b[kHostMaxChunks] = {};
  cudaEvent_t blk[2 * kHostMaxChunks] = {};   // the two strips of each step
  std::mutex mu;
};

int host_pipe(HostPipe** out) {
  static HostPipe pipes[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BSG_ERR_CUDA;
  HostPipe& hp = pipes[dev];
  *out = &hp;
  std::lock_guard<std::mutex> lock(hp.mu);
  if (hp.ready) return BSG_OK;
  auto ev = [](cudaEvent_t* e) { return cudaEventCreateWithFlags(e, cudaEventDisableTiming) == cudaSuccess; };
  bool ok = cudaStreamCreateWithFlags(&hp.comp, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&hp.d2h, cudaStreamNonBlocking) == cudaSuccess && ev(&hp.start) &&
            ev(&hp.end);
  for (int i = 0; ok && i < kHostMaxChunks; ++i) ok = ev(&hp.in_a[i]) && ev(&hp.in_b[i]);
  for (int i = 0; ok && i < 2 * kHostMaxChunks; ++i) ok = ev(&hp.blk[i]);
  if (!ok) {
    t_last_cuda_error = cudaGetLastError();
    return BSG_ERR_CUDA;
  }
  hp.ready = true;
  return BSG_OK;
}

// Device workspace of the host-staged call: A, B, their row-major scales,
// their native scale atoms and C, each 256-byte aligned.
struct HostLayout {
  size_t a, b, sa, sb, na, nb, c, total;
};

HostLayout host_layout(const bsgemm_args& a, bool fp4) {
  const size_t kbytes = fp4 ? a.k / 2 : a.k, kg = a.k / 32;
  HostLayout l;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  l.a = take(static_cast<size_t>(a.m) * kbytes);
  l.b = take(static_cast<size_t>(a.n) * kbytes);
  l.sa = take(static_cast<size_t>(a.m) * kg);
  l.sb = take(static_cast<size_t>(a.n) * kg);
  l.na = take(native_sf_bytes(a.m, static_cast<int>(kg)));
  l.nb = take(native_sf_bytes(a.n, static_cast<int>(kg)));
  l.c = take(static_cast<size_t>(a.m) * a.n * (a.out_dtype == BSG_OUT_FP32 ? 4 : 2));
  l.total = off;
  return l;
}

// Chunk boundaries along one dimension: `chunks` pieces, multiples of 256
// rows except the last (native scale atoms and C columns stay aligned).
int chunk_bounds(int extent, int chunks, int* bounds) {
  const int step = std::max(256, (extent + chunks - 1) / chunks + 255) / 256 * 256;
  int c = 0;
  bounds[0] = 0;
  while (bounds[c] < extent && c < kHostMaxChunks) {
    bounds[c + 1] = std::min(extent, bounds[c] + step);
    ++c;
  }
  return c;
}

int host_gemm_run(int family, const bsgemm_args* args, void* dev_ws, size_t dev_ws_bytes, int chunks,
                  cudaStream_t st) {
  if (!args) return BSG_ERR_INVALID_VALUE;
  if (family != BSG_FAMILY_MXFP8 && family != BSG_FAMILY_MXFP4) return BSG_ERR_UNSUPPORTED;
  const bool fp4 = family == BSG_FAMILY_MXFP4;
  const bsgemm_args& a = *args;
  if (!a.ptr_a || !a.ptr_b || !a.ptr_c || !a.ptr_sfa || !a.ptr_sfb || !dev_ws) return BSG_ERR_INVALID_VALUE;
  if (a.m <= 0 || a.n <= 0 || a.k <= 0 || a.batch != 1 || chunks < 0 || chunks > kHostMaxChunks)
    return BSG_ERR_INVALID_VALUE;
  if (a.out_dtype != BSG_OUT_BF16 && a.out_dtype != BSG_OUT_FP32) return BSG_ERR_INVALID_VALUE;
  if (a.layout != BSG_LAYOUT_TN || a.sfa_format != BSG_SF_ROWMAJOR || a.sfb_format != BSG_SF_ROWMAJOR)
    return BSG_ERR_UNSUPPORTED;
  if (a.b_format != BSG_B_RAW && a.b_format != BSG_B_SHUFFLE16) return BSG_ERR_UNSUPPORTED;
  if (a.k % (fp4 ? 256 : 128)) return BSG_ERR_INVALID_VALUE;
  const int vec = a.out_dtype == BSG_OUT_BF16 ? 8 : 4;
  if (a.n % vec || a.stride_c < a.n) return BSG_ERR_ALIGNMENT;
  const size_t kbytes = fp4 ? a.k / 2 : a.k, kg = a.k / 32;
  const bool shuffled = a.b_format == BSG_B_SHUFFLE16;
  if (a.stride_a < static_cast<long long>(kbytes) || a.stride_b < static_cast<long long>(kbytes) ||
      a.stride_sfa < static_cast<long long>(kg) || a.stride_sfb < static_cast<long long>(kg))
    return BSG_ERR_INVALID_VALUE;
  if (shuffled && (a.n % 16 || a.stride_b != static_cast<long long>(kbytes))) return BSG_ERR_INVALID_VALUE;
  const HostLayout l = host_layout(a, fp4);
  if (dev_ws_bytes < l.total) return BSG_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(dev_ws) & 255u) return BSG_ERR_ALIGNMENT;
  DevInfo dev;
  int rc;
  if ((rc = device_info(&dev)) != BSG_OK) return rc;
  if (!dev.sm100) return BSG_ERR_ARCH;

  int mb[kHostMaxChunks + 1], nb[kHostMaxChunks + 1];
  const int auto_m = std::min(4, std::max(1, a.m / 1024)), auto_n = std::min(4, std::max(1, a.n / 1024));
  const int cm = chunk_bounds(a.m, chunks ? chunks : auto_m, mb);
  const int cn = chunk_bounds(a.n, chunks ? chunks : auto_n, nb);
  HostPipe* hp = nullptr;
  if ((rc = host_pipe(&hp)) != BSG_OK) return rc;
  std::lock_guard<std::mutex> lock(hp->mu);

  uint8_t* ws = static_cast<uint8_t*>(dev_ws);
  const uint8_t* ha = static_cast<const uint8_t*>(a.ptr_a);
  const uint8_t* hb = static_cast<const uint8_t*>(a.ptr_b);
  const uint8_t* hsa = static_cast<const uint8_t*>(a.ptr_sfa);
  const uint8_t* hsb = static_cast<const uint8_t*>(a.ptr_sfb);
  const size_t esz = a.out_dtype == BSG_OUT_FP32 ? 4 : 2;
  const int kb_atoms = static_cast<int>((kg + 3) / 4);
  cudaError_t e = cudaSuccess;
  auto chk = [&](cudaError_t r) {
    if (r != cudaSuccess && e == cudaSuccess) e = r;
    return r == cudaSuccess;
  };
  // rows [r0, r1) of a host matrix (pitch `ld` bytes) into dense device rows;
  // dense rows go as one linear copy (strided 2-D copies ran at half the
  // PCIe rate while copies in the other direction were running)
  auto h2d_rows = [&](uint8_t* dst, const uint8_t* src, long long ld, size_t width, int r0, int r1) {
    uint8_t* d = dst + static_cast<size_t>(r0) * width;
    const uint8_t* h = src + static_cast<size_t>(r0) * ld;
    const size_t rows = static_cast<size_t>(r1 - r0);
    if (static_cast<size_t>(ld) == width)
      return chk(cudaMemcpyAsync(d, h, rows * width, cudaMemcpyHostToDevice, st));
    return chk(cudaMemcpy2DAsync(d, width, h, static_cast<size_t>(ld), width, rows, cudaMemcpyHostToDevice, st));
  };

  chk(cudaEventRecord(hp->start, st));
  chk(cudaStreamWaitEvent(hp->comp, hp->start, 0));
  chk(cudaStreamWaitEvent(hp->d2h, hp->start, 0));
  const long long b_ld = shuffled ? static_cast<long long>(kbytes) : a.stride_b;
  int status = BSG_OK;   // a failed launch stops the enqueueing; the join below always runs
  // One GEMM over rows [r0, r1) x columns [c0, c1) of C from the device
  // copies, then its copy back to the host C (strided rows).
  auto strip = [&](int r0, int r1, int c0, int c1, cudaEvent_t done) {
    if (r1 <= r0 || c1 <= c0 || status != BSG_OK || e != cudaSuccess) return;
    bsgemm_args g = a;
    g.ptr_a = ws + l.a + static_cast<size_t>(r0) * kbytes;
    g.ptr_b = ws + l.b + static_cast<size_t>(c0) * kbytes;
    g.ptr_c = ws + l.c + (static_cast<size_t>(r0) * a.n + c0) * esz;
    g.ptr_sfa = ws + l.na + static_cast<size_t>(r0 / 128) * kb_atoms * 512;
    g.ptr_sfb = ws + l.nb + static_cast<size_t>(c0 / 128) * kb_atoms * 512;
    g.m = r1 - r0;
    g.n = c1 - c0;
    g.stride_a = static_cast<int>(kbytes);
    g.stride_b = static_cast<int>(kbytes);
    g.stride_c = a.n;
    g.sfa_format = g.sfb_format = BSG_SF_NATIVE;
    g.split_k = 1;
    g.workspace = nullptr;
    g.workspace_bytes = 0;
    const int r = mx_run(&g, fp4, hp->comp);
    if (r != BSG_OK) {
      status = r;
      return;
    }
    chk(cudaEventRecord(done, hp->comp));
    chk(cudaStreamWaitEvent(hp->d2h, done, 0));
    uint8_t* hc = static_cast<uint8_t*>(a.ptr_c) + (static_cast<size_t>(r0) * a.stride_c + c0) * esz;
    const uint8_t* dc = ws + l.c + (static_cast<size_t>(r0) * a.n + c0) * esz;
    if (c0 == 0 && c1 == a.n && a.stride_c == a.n)   // whole rows: one linear copy
      chk(cudaMemcpyAsync(hc, dc, static_cast<size_t>(r1 - r0) * a.n * esz, cudaMemcpyDeviceToHost, hp->d2h));
    else
      chk(cudaMemcpy2DAsync(hc, static_cast<size_t>(a.stride_c) * esz, dc, static_cast<size_t>(a.n) * esz,
                            static_cast<size_t>(c1 - c0) * esz, static_cast<size_t>(r1 - r0),
                            cudaMemcpyDeviceToHost, hp->d2h));
  };
  // Step t brings B chunk t, then A chunk t.  The C blocks that become
  // computable are the column strip (A chunks < t) x (B chunk t), which runs
  // while A chunk t is still in flight, and the row strip (A chunk t) x (B
  // chunks <= t): two GEMMs per step whatever the chunk count.
  // Every input copy is queued first, so the copy engine never waits for
  // the host to enqueue GEMMs.
  for (int t = 0; t < std::max(cm, cn) && e == cudaSuccess; ++t) {
    if (t < cn) {
      // shuffle_weight(16,16) bytes of rows [n0, n1) are contiguous (n0 % 16 == 0)
      h2d_rows(ws + l.b, hb, b_ld, kbytes, nb[t], nb[t + 1]);
      h2d_rows(ws + l.sb, hsb, a.stride_sfb, kg, nb[t], nb[t + 1]);
      chk(cudaEventRecord(hp->in_b[t], st));
    }
    if (t < cm) {
      h2d_rows(ws + l.a, ha, a.stride_a, kbytes, mb[t], mb[t + 1]);
      h2d_rows(ws + l.sa, hsa, a.stride_sfa, kg, mb[t], mb[t + 1]);
      chk(cudaEventRecord(hp->in_a[t], st));
    }
  }
  for (int t = 0; t < std::max(cm, cn) && e == cudaSuccess && status == BSG_OK; ++t) {
    if (t < cn) {
      chk(cudaStreamWaitEvent(hp->comp, hp->in_b[t], 0));
      const int rc2 = pack_sf_launch(ws + l.sb + static_cast<size_t>(nb[t]) * kg, static_cast<int>(kg),
                                     ws + l.nb + static_cast<size_t>(nb[t] / 128) * kb_atoms * 512, nb[t + 1] - nb[t],
                                     static_cast<int>(kg), BSG_SF_ROWMAJOR, 0, hp->comp);
      if (rc2 != BSG_OK) status = rc2;
      strip(0, mb[std::min(t, cm)], nb[t], nb[t + 1], hp->blk[2 * t]);
    }
    if (t < cm) {
      chk(cudaStreamWaitEvent(hp->comp, hp->in_a[t], 0));
      const int rc2 = pack_sf_launch(ws + l.sa + static_cast<size_t>(mb[t]) * kg, static_cast<int>(kg),
                                     ws + l.na + static_cast<size_t>(mb[t] / 128) * kb_atoms * 512, mb[t + 1] - mb[t],
                                     static_cast<int>(kg), BSG_SF_ROWMAJOR, 0, hp->comp);
      if (rc2 != BSG_OK && status == BSG_OK) status = rc2;
      strip(mb[t], mb[t + 1], 0, nb[std::min(t, cn - 1) + 1], hp->blk[2 * t + 1]);
    }
  }
  // the caller's stream resumes after every block is back in host memory
  // (and, after a failure, after whatever was enqueued on either stream)
  chk(cudaEventRecord(hp->end, hp->comp));
  chk(cudaStreamWaitEvent(hp->d2h, hp->end, 0));
  chk(cudaEventRecord(hp->end, hp->d2h));
  chk(cudaStreamWaitEvent(st, hp->end, 0));
  if (status != BSG_OK) return status;
  if (e != cudaSuccess) {
    t_last_cuda_error = e;
    return BSG_ERR_CUDA;
  }
  return BSG_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

void bsgemm_args_init(bsgemm_args* a) {
  if (!a) return;
  std::memset(a, 0, sizeof(*a));
  a->batch = 1;
  a->layout = BSG_LAYOUT_TN;
  a->b_format = BSG_B_RAW;
  a->sfa_format = BSG_SF_ROWMAJOR;
  a->sfb_format = BSG_SF_ROWMAJOR;
  a->out_dtype = BSG_OUT_BF16;
}

int bsgemm_a8w8_mxfp8(const bsgemm_args* args, bsg_stream_t stream) {
  return mx_run(args, false, reinterpret_cast<cudaStream_t>(stream));
}

int bsgemm_a4w4_mxfp4(const bsgemm_args* args, bsg_stream_t stream) {
  return mx_run(args, true, reinterpret_cast<cudaStream_t>(stream));
}

int bsgemm_a8w8_blockscale_bpreshuffle(const bsgemm_args* args, bsg_stream_t stream) {
  return fp8b_run(args, reinterpret_cast<cudaStream_t>(stream));
}

int bsgemm_a8w8_blockscale_grouped(const bsgemm_args* args, const int* group_offsets, int total_rows,
                                   bsg_stream_t stream) {
  return fp8b_grouped_run(args, group_offsets, total_rows, reinterpret_cast<cudaStream_t>(stream));
}

int bsgemm_a8w8_mxfp8_grouped(const bsgemm_args* args, const int* group_offsets, int total_rows,
                              bsg_stream_t stream) {
  return mx_grouped_run(args, false, group_offsets, total_rows, reinterpret_cast<cudaStream_t>(stream));
}

int bsgemm_a4w4_mxfp4_grouped(const bsgemm_args* args, const int* group_offsets, int total_rows,
                              bsg_stream_t stream) {
  return mx_grouped_run(args, true, group_offsets, total_rows, reinterpret_cast<cudaStream_t>(stream));
}

size_t bsgemm_mx_host_workspace_size(int family, const bsgemm_args* args) {
  if (!args || args->m <= 0 || args->n <= 0 || args->k <= 0) return 0;
  if (family != BSG_FAMILY_MXFP8 && family != BSG_FAMILY_MXFP4) return 0;
  return host_layout(*args, family == BSG_FAMILY_MXFP4).total;
}

int bsgemm_mx_host_gemm(int family, const bsgemm_args* args, void* dev_workspace, size_t dev_workspace_bytes,
                        int chunks, bsg_stream_t stream) {
  return host_gemm_run(family, args, dev_workspace, dev_workspace_bytes, chunks,
                       reinterpret_cast<cudaStream_t>(stream));
}

size_t bsgemm_mx_grouped_workspace_size(const bsgemm_args* args) {
  if (!args || args->m <= 0 || args->n <= 0 || args->k <= 0 || args->batch <= 0) return 0;
  const int kg = args->k / 32;
  return align256(native_sf_bytes(args->m, kg) * args->batch) +
         (args->sfb_format == BSG_SF_ROWMAJOR ? align256(native_sf_bytes(args->n, kg) * args->batch) : 0) +
         align256(4u * (static_cast<size_t>(args->batch) + 1));
}

size_t bsgemm_workspace_size(int family, const bsgemm_args* args) {
  if (!args || args->m <= 0 || args->n <= 0 || args->k <= 0 || args->batch <= 0) return 0;
  DevInfo dev;
  if (device_info(&dev) != BSG_OK) return 0;
  if (family == BSG_FAMILY_MXFP8 || family == BSG_FAMILY_MXFP4) {
    MxPlan pl;
    mx_plan(*args, family == BSG_FAMILY_MXFP4, dev, pl, true);
    return pl.ws_sfa + pl.ws_sfb + pl.ws_partials;
  }
  if (family == BSG_FAMILY_FP8_BLOCK) {
    if (fp8b_use_wide(*args)) {   // partials of the wide kernel's K slices
      size_t bytes = 0;
      fp8b_wide_split(*args, dev.sms, &bytes);
      return bytes;
    }
    if (fp8b_use_pair(*args, dev.sms)) {   // partials of the pair kernel's tail slices
      if (args->split_k != 0) return 0;
      int tu = 0, ts = 1;
      const long long units = static_cast<long long>((args->m + 255) / 256) * ((args->n + 255) / 256) * args->batch;
      return fp8b_pair_tail(units, fp8b_pair_clusters(*args, dev.sms), args->k / 128, &tu, &ts);
    }
    Plan pl;
    fp8b_plan(*args, dev, pl, true);
    return pl.ws_partials;
  }
  return 0;
}

int bsgemm_pack_b(const void* src, void* dst, int rows, int kbytes, int src_format, int unpack,
                  bsg_stream_t stream) {
  if (!src || !dst || rows <= 0 || kbytes <= 0 || (unpack != 0 && unpack != 1))
    return BSG_ERR_INVALID_VALUE;
  if (!aligned16(src) || !aligned16(dst) || kbytes % 16) return BSG_ERR_ALIGNMENT;
  const uint64_t bytes = static_cast<uint64_t>(rows) * kbytes;
  if (overlaps(src, bytes, dst, bytes)) return BSG_ERR_INVALID_VALUE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long chunks = static_cast<long long>(rows) * (kbytes / 16);
  const int grid = static_cast<int>(std::min<long long>((chunks + 255) / 256, 8192));
  if (src_format == BSG_B_SHUFFLE16) {
    if (rows % 16) return BSG_ERR_INVALID_VALUE;
    bsg::pack_b_shuffle16_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(src),
                                                       static_cast<uint4*>(dst), rows, kbytes, unpack);
  } else if (src_format == BSG_B_KPANEL128) {
    if (kbytes % 128) return BSG_ERR_INVALID_VALUE;
    bsg::pack_b_kpanel_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(src),
                                                    static_cast<uint4*>(dst), rows, kbytes, unpack);
  } else {
    return BSG_ERR_INVALID_VALUE;
  }
  return launch_status();
}

size_t bsgemm_native_scales_size(int rows, int kg) {
  if (rows <= 0 || kg <= 0) return 0;
  return native_sf_bytes(rows, kg);
}

int bsgemm_pack_scales(const void* src, int src_stride, void* dst, int rows, int kg,
                       int src_format, int unpack, bsg_stream_t stream) {
  if (!src || !dst || rows <= 0 || kg <= 0 || (unpack != 0 && unpack != 1))
    return BSG_ERR_INVALID_VALUE;
  if (src_format != BSG_SF_ROWMAJOR && src_format != BSG_SF_E8M0_SHUFFLE) return BSG_ERR_INVALID_VALUE;
  if (src_format == BSG_SF_ROWMAJOR && src_stride < kg) return BSG_ERR_INVALID_VALUE;
  const void* native = unpack ? src : dst;
  if (!aligned16(native)) return BSG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (unpack && src_format == BSG_SF_E8M0_SHUFFLE) {
    const long long n = static_cast<long long>((rows + 31) / 32 * 32) * ((kg + 7) / 8 * 8);
    bsg::fill_u8_kernel<<<static_cast<int>(std::min<long long>((n + 255) / 256, 4096)), 256, 0, st>>>(
        static_cast<uint8_t*>(dst), n, 0x7F);
  }
  return pack_sf_launch(src, src_stride, dst, rows, kg, src_format, unpack, st);
}

int launch_blockscale_bpreshuffle(const void* kargs, int output_bf16, int tiles,
                                  bsg_stream_t stream) {
  if (!kargs || (output_bf16 != 0 && output_bf16 != 1) || (tiles != 0 && tiles != 1))
    return static_cast<int>(cudaErrorInvalidValue);
  static_assert(offsetof(bsgemm_args, layout) == 96, "96-byte reference prefix");
  bsgemm_args a;
  bsgemm_args_init(&a);
  std::memcpy(&a, kargs, 96);
  return e8m0b_run(a, output_bf16 == 1, tiles, reinterpret_cast<cudaStream_t>(stream));
}

int bsgemm_quantize(const void* x, int in_dtype, int rows, int cols, long long ldx, int format, void* q,
                    long long ldq, void* sf, int sf_format, long long ld_sf, bsg_stream_t stream) {
  if (!x || !q || !sf || rows <= 0 || cols <= 0) return BSG_ERR_INVALID_VALUE;
  if (in_dtype != BSG_IN_BF16 && in_dtype != BSG_IN_FP32) return BSG_ERR_INVALID_VALUE;
  if (format != BSG_QUANT_MXFP8 && format != BSG_QUANT_MXFP4 && format != BSG_QUANT_FP8_BLOCK)
    return BSG_ERR_INVALID_VALUE;
  const bool mx = format != BSG_QUANT_FP8_BLOCK;
  const int group = mx ? 32 : 128;
  if (cols % group) return BSG_ERR_INVALID_VALUE;
  const int esz = in_dtype == BSG_IN_FP32 ? 4 : 2;
  if (ldx < cols || (ldx * esz) % 16 || !aligned16(x)) return BSG_ERR_ALIGNMENT;
  const long long qcols = format == BSG_QUANT_MXFP4 ? cols / 2 : cols;
  const int qalign = format == BSG_QUANT_MXFP4 ? 4 : 8;
  if (ldq < qcols || ldq % qalign || reinterpret_cast<uintptr_t>(q) % qalign) return BSG_ERR_ALIGNMENT;
  if (mx) {
    if (sf_format == BSG_SF_NATIVE) {
      if (cols % 128) return BSG_ERR_INVALID_VALUE;
    } else if (sf_format != BSG_SF_ROWMAJOR || ld_sf < cols / 32) {
      return BSG_ERR_INVALID_VALUE;
    }
  } else {
    if (sf_format == BSG_SF_ROWMAJOR) {
      if (ld_sf < cols / 128) return BSG_ERR_INVALID_VALUE;
    } else if (sf_format != BSG_SF_KMAJOR_T || ld_sf < rows) {
      return BSG_ERR_INVALID_VALUE;
    }
    if (reinterpret_cast<uintptr_t>(sf) % 4) return BSG_ERR_ALIGNMENT;
  }
  // q and the scales must not overlap x
  const uint64_t xbytes = static_cast<uint64_t>(rows - 1) * ldx * esz + static_cast<uint64_t>(cols) * esz;
  const uint64_t qbytes = static_cast<uint64_t>(rows - 1) * ldq + static_cast<uint64_t>(qcols);
  if (overlaps(x, xbytes, q, qbytes)) return BSG_ERR_INVALID_VALUE;
  bsg::QuantParams p{};
  p.x = x;
  p.in_fp32 = in_dtype == BSG_IN_FP32;
  p.rows = rows;
  p.cols = cols;
  p.ldx = ldx;
  p.q = static_cast<uint8_t*>(q);
  p.ldq = ldq;
  p.sf = sf;
  p.sf_format = sf_format == BSG_SF_NATIVE ? 0 : sf_format == BSG_SF_ROWMAJOR ? 1 : 2;
  p.ld_sf = ld_sf;
  p.rows_padded = (rows + 127) / 128 * 128;
  const int warp_cols = bsg::quant_warp_cols(in_dtype == BSG_IN_FP32);
  const int warps_per_row = (cols + warp_cols - 1) / warp_cols;
  const int launch_rows = mx && p.sf_format == 0 ? p.rows_padded : rows;
  const long long warps = static_cast<long long>(launch_rows) * warps_per_row;
  const long long blocks = (warps + 7) / 8;
  if (blocks > 0x7fffffffLL) return BSG_ERR_INVALID_VALUE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(blocks));
  const bool f32 = in_dtype == BSG_IN_FP32;
  switch (format) {
    case BSG_QUANT_MXFP8:
      if (f32) bsg::quantize_kernel<bsg::kQuantMxfp8, true><<<grid, 256, 0, st>>>(p);
      else bsg::quantize_kernel<bsg::kQuantMxfp8, false><<<grid, 256, 0, st>>>(p);
      break;
    case BSG_QUANT_MXFP4:
      if (f32) bsg::quantize_kernel<bsg::kQuantMxfp4, true><<<grid, 256, 0, st>>>(p);
      else bsg::quantize_kernel<bsg::kQuantMxfp4, false><<<grid, 256, 0, st>>>(p);
      break;
    default:
      if (f32) bsg::quantize_kernel<bsg::kQuantFp8Block, true><<<grid, 256, 0, st>>>(p);
      else bsg::quantize_kernel<bsg::kQuantFp8Block, false><<<grid, 256, 0, st>>>(p);
      break;
  }
  return launch_status();
}

const char* bsgemm_strerror(int status) {
  switch (status) {
    case BSG_OK: return "success";
    case BSG_ERR_INVALID_VALUE: return "invalid argument";
    case BSG_ERR_UNSUPPORTED: return "unsupported combination of formats or layouts";
    case BSG_ERR_ARCH: return "device is not sm_100 (B200)";
    case BSG_ERR_WORKSPACE: return "workspace missing or too small";
    case BSG_ERR_CUDA: return "CUDA call failed";
    case BSG_ERR_TIMEOUT: return "device-side bounded wait expired";
    case BSG_ERR_ALIGNMENT: return "pointer or stride violates the 16-byte rules";
    case BSG_ERR_SCRATCH_LIMIT:
      return "problem needs more than the fixed device scratch of the allocation-free entry point";
    default: return "unknown status";
  }
}

int bsgemm_check_device_error(void) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return BSG_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&v, bsg::g_bsg_device_error, sizeof(int)) != cudaSuccess)
    return BSG_ERR_CUDA;
  const int zero = 0;
  if (v != 0 && cudaMemcpyToSymbol(bsg::g_bsg_device_error, &zero, sizeof(int)) != cudaSuccess)
    return BSG_ERR_CUDA;
  return v == 0 ? BSG_OK : v;
}

int bsgemm_selftest_timeout(int timeout_us) {
  if (timeout_us <= 0 || timeout_us > 10 * 1000 * 1000) return BSG_ERR_INVALID_VALUE;
  int rc = bsgemm_check_device_error();   // start from a clean word
  if (rc == BSG_ERR_CUDA) return rc;
  bsg::selftest_timeout_kernel<<<1, 32>>>(static_cast<unsigned long long>(timeout_us) * 1000ull);
  if (cudaGetLastError() != cudaSuccess) return BSG_ERR_CUDA;
  return bsgemm_check_device_error();
}

const char* bsgemm_version(void) { return "bsgemm_b200 0.1 (sm_100a)"; }

}  // extern "C"

// ===========================================================================
// Allocation-free MXFP8 entry point
//
// Some callers cannot allocate device memory at all: a serving runtime that
// reserves the whole HBM budget up front and routes every byte through its
// own allocator, or a host application that must never take the implicit
// device synchronisation a cudaMalloc/cudaFree can cause in the middle of its
// stream work.  bsgemm_a8w8_mxfp8 asks such callers for a workspace whenever
// it repacks row-major scales or splits K; this variant instead uses a fixed
// scratch array that lives in the library's own device image.
//
// Limits and behaviour:
//   - the scratch is kNoAllocScratchBytes (8 MiB) on every GPU that loads the
//     library, held until the process exits;
//   - a problem whose repacked scales plus split-K partials exceed it is
//     rejected with BSG_ERR_SCRATCH_LIMIT before anything is enqueued (with
//     split_k == 0 the split is dropped first if that makes it fit);
//   - every call on a device shares the one array, and it keeps whatever the
//     last call left there.  The kernels overwrite every scratch byte they
//     read (scale atoms are written whole, each K slice writes its complete
//     partial tile), so nothing has to start at zero, but two calls whose
//     work overlaps on the GPU (different streams, or different host threads
//     without ordering) race on the scratch and corrupt each other;
//   - the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current); make
//     that first call before any stream capture on the device.
// ===========================================================================
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

// Device-side scratch.  In host code this name is only a host stand-in for
// the symbol: never pass it to a kernel, always the address looked up below.
static __device__ __align__(256) unsigned char g_bsg_noalloc_scratch[kNoAllocScratchBytes];

int noalloc_scratch_ptr(void** out) {
  static std::mutex mu;
  static void* ptrs[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BSG_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bsg_noalloc_scratch) != cudaSuccess || !p) return BSG_ERR_CUDA;
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return BSG_OK;
}

}  // namespace

extern "C" {

BSG_API int bsgemm_a8w8_mxfp8_noalloc(const bsgemm_args* args, bsg_stream_t stream) {
  int rc = validate_common(args);
  if (rc != BSG_OK) return rc;
  bsgemm_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  size_t need = bsgemm_workspace_size(BSG_FAMILY_MXFP8, &a);
  if (need > kNoAllocScratchBytes && a.split_k == 0) {
    a.split_k = 1;                     // auto split-K does not fit: run unsplit
    need = bsgemm_workspace_size(BSG_FAMILY_MXFP8, &a);
  }
  if (need > kNoAllocScratchBytes) return BSG_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch_ptr(&scratch)) != BSG_OK) return rc;
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  return mx_run(&a, false, reinterpret_cast<cudaStream_t>(stream));
}

BSG_API size_t bsgemm_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

}  // extern "C"

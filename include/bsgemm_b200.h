/*
 * bsgemm_b200.h -- C ABI of the B200 (sm_100a) block-scaled GEMM library.
 *
 * Drop-in boundary for the reference's host launchers of three GEMM families
 * (paths relative to the reference project root):
 *   MXFP8  a8w8  E4M3 x E4M3, one E8M0 scale per 32 K     mxfp8_gemm/
 *   MXFP4  a4w4  packed E2M1, one E8M0 scale per 32 K      mxfp4_gemm_4wave_20261112/
 *   FP8 block-scale, fp32 scales 1x128 (A) / 128x128 (B),
 *        K-panel preshuffled B                             block_scale_gemm_bpreshuffle/
 * plus the reference's one shipped extern "C" entry point,
 * launch_blockscale_bpreshuffle (E8M0 1x128/128x128 scales).
 *
 * Conventions kept from the reference launcher
 * (trace_block_scale_latest_20260914_040021/source_snapshot/
 *  gemm_a8w8_blockscale_bpreshuffle_launch.cc:29-65):
 *   - the caller owns every buffer; no entry point allocates device memory;
 *   - a GEMM entry point enqueues its kernels on the caller's stream and
 *     returns without synchronising;
 *   - arguments are validated first; errors are returned, never aborted on;
 *   - entry points keep no per-call state and may be called concurrently.
 *
 * Layout letters (CUTLASS convention; the reference's letters are
 * swapped, e.g. its "nt" is this "tn"):
 *   tn = A K-major [M,K], B K-major [N,K]      (BSG_LAYOUT_TN = 3)
 *   nn = A M-major [K,M], B K-major [N,K]      (BSG_LAYOUT_NN = 2)
 *   tt = A K-major [M,K], B N-major [K,N]      (BSG_LAYOUT_TT = 1)
 *   nt = A M-major [K,M], B N-major [K,N]      (BSG_LAYOUT_NT = 0)
 * i.e. bit0 = A is K-major, bit1 = B is K-major.
 */
#ifndef BSGEMM_B200_H
#define BSGEMM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BSG_API __attribute__((visibility("default")))
#else
#define BSG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *bsg_stream_t; /* == cudaStream_t */

/* ---- status codes ------------------------------------------------------- */
enum {
    BSG_OK = 0,
    BSG_ERR_INVALID_VALUE = 1,   /* null pointer, bad flag, bad shape/stride, overlap */
    BSG_ERR_UNSUPPORTED = 2,     /* valid but not implemented combination */
    BSG_ERR_ARCH = 3,            /* device is not sm_100 (B200) */
    BSG_ERR_WORKSPACE = 4,       /* split-K workspace missing or too small */
    BSG_ERR_CUDA = 5,            /* a CUDA runtime/driver call failed */
    BSG_ERR_TIMEOUT = 6,         /* a device-side bounded wait expired */
    BSG_ERR_ALIGNMENT = 7,       /* pointer/stride violates TMA 16-byte rules */
    BSG_ERR_SCRATCH_LIMIT = 8    /* bsgemm_a8w8_mxfp8_noalloc: problem exceeds its fixed scratch */
};

/* ---- enums of bsgemm_args ---------------------------------------------- */
enum { BSG_LAYOUT_NT = 0, BSG_LAYOUT_TT = 1, BSG_LAYOUT_NN = 2, BSG_LAYOUT_TN = 3 };

enum {
    BSG_B_RAW = 0,          /* plain [N,K] (K-major) or [K,N] (N-major) */
    BSG_B_KPANEL128 = 1,    /* B'[K/128][N][128] (reference shuffle_b) */
    BSG_B_SHUFFLE16 = 2     /* aiter shuffle_weight(16,16) [N/16][Kb/16][16][16], read in place */
};

enum {
    BSG_SF_NATIVE = 0,      /* E8M0 tcgen05 atoms, see bsgemm_pack_scales */
    BSG_SF_ROWMAJOR = 1,    /* E8M0 [rows, K/32] (reference raw) or fp32 [rows, K/128] */
    BSG_SF_KMAJOR_T = 2,    /* fp32 SFA stored transposed [K/128, M] (reference kernel) */
    BSG_SF_E8M0_SHUFFLE = 3 /* aiter e8m0_shuffle: needs bsgemm_pack_scales first */
};

enum { BSG_OUT_BF16 = 0, BSG_OUT_FP32 = 1 };

enum { BSG_FAMILY_MXFP8 = 0, BSG_FAMILY_MXFP4 = 1, BSG_FAMILY_FP8_BLOCK = 2 };

/*
 * Kernel arguments.  The first 96 bytes are field-for-field the reference's
 * opus_gemm_scale_kargs / opus_gemm_kargs / opus_gemm_mxfp4_scale_kargs
 * (source_snapshot/gemm_a8w8_mxfp8_scale_common.h:12-38,
 *  mxfp8_gemm/gemm_a8w8_mxfp8_common.h:4-25,
 *  mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_traits.hpp:7-27).
 * Units: strides of fp8 tensors and of C in ELEMENTS, of packed fp4 tensors in
 * BYTES (as the reference), E8M0 scale strides in bytes, fp32 scale strides
 * in floats.  For BSG_SF_NATIVE the scale strides are ignored except the batch
 * strides (bytes between batches; 0 = densely packed).
 */
typedef struct bsgemm_args {
    const void *ptr_a;
    const void *ptr_b;
    void *ptr_c;
    int m;
    int n;
    int k;
    int batch;
    int stride_a;
    int stride_b;
    int stride_c;
    int stride_a_batch;
    int stride_b_batch;
    int stride_c_batch;
    const void *ptr_sfa;
    const void *ptr_sfb;
    int stride_sfa;
    int stride_sfb;
    int stride_sfa_batch;
    int stride_sfb_batch;
    /* ---- extensions (not in the reference's 96-byte struct) ---- */
    int layout;             /* BSG_LAYOUT_* */
    int b_format;           /* BSG_B_* */
    int sfa_format;         /* BSG_SF_* */
    int sfb_format;         /* BSG_SF_* */
    int out_dtype;          /* BSG_OUT_* */
    int split_k;            /* 0 = auto, 1 = none, >1 = forced number of K slices */
    void *workspace;        /* caller-owned scratch for split-K partials (fp32) */
    size_t workspace_bytes;
    int grid_blocks;        /* 0 = one CTA per SM; >0 caps the persistent grid
                               (the reference's PERSIST_GRID / m10 grid_blocks) */
    int kernel;             /* BSG_KERNEL_*: 0 = auto, 1 = single-CTA tiles,
                               2 = CTA-pair (cta_group::2) 256x256 tiles,
                               3 = transposed decode kernel (M <= 64; MX: layout tn),
                               4 = wide single-CTA 128x256 tiles (fp32 block scales only) */
} bsgemm_args;

enum { BSG_KERNEL_AUTO = 0, BSG_KERNEL_1CTA = 1, BSG_KERNEL_PAIR = 2, BSG_KERNEL_SWAP = 3, BSG_KERNEL_WIDE = 4 };

/* Fill the 96-byte prefix's defaults and zero the extensions. */
BSG_API void bsgemm_args_init(bsgemm_args *args);

/*
 * MXFP8: C[b,m,n] = sum_g 2^(sfa[m,g]-127) 2^(sfb[n,g]-127) sum_{k in g} A*B,
 * g = 32 consecutive K.  A/B E4M3FN bytes in any of the four layouts
 * (args->layout); B also as BSG_B_SHUFFLE16 (K-major layouts, read in place);
 * SFA/SFB in BSG_SF_NATIVE or BSG_SF_ROWMAJOR ([rows,K/32] bytes, row stride
 * stride_sf*).  Requires K % 128 == 0, N % 8 == 0 (bf16) or N % 4 == 0 (fp32);
 * M arbitrary.  kernel: AUTO (M <= 64 tn -> transposed decode kernel; large
 * bf16 problems -> CTA pairs; else single-CTA tiles), 1CTA, PAIR or SWAP.
 * Replaces the launch of gemm_a8w8_mxfp8_kernel in
 * mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:287-295 (its kargs at :265-285), without
 * the reference's K == 256 and M/N % 256 limits.
 * E8M0 edge bytes (all MX and E8M0 block-scale entry points): byte 0 is
 * 2^-127, as on the reference host (gemm_a8w8_mxfp8_host.cc:35-37); byte 255
 * is NaN (OCP MX, what the block-scaled tensor cores implement), where the
 * reference host's ldexp gives 2^128 (+inf in fp32), so every output of a
 * row or column whose scales hold a 255 byte is NaN.  E4M3 0x7F / 0xFF
 * operands are NaN and propagate to their outputs.
 */
BSG_API int bsgemm_a8w8_mxfp8(const bsgemm_args *args, bsg_stream_t stream);

/*
 * MXFP4: same contraction with E2M1 elements packed two per byte, even k in
 * the low nibble; A [M,K/2] and B [N,K/2] bytes, K-major only (layout TN).
 * B may be BSG_B_RAW or BSG_B_SHUFFLE16 (aiter shuffle_weight(16,16) bytes,
 * stride_b = K/2, read in place).  Requires K % 256 == 0.  kernel: AUTO,
 * 1CTA, PAIR, or SWAP (transposed decode kernel, M <= 64).
 * Replaces gemm_a4w4_mxfp4_4wave_kernel's launch in
 * mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:211-213 and the
 * persistent launch of candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:242-250.
 */
BSG_API int bsgemm_a4w4_mxfp4(const bsgemm_args *args, bsg_stream_t stream);

/*
 * FP8 block-scale with fp32 scales: C = sum_kb sfa[m,kb] * sfb[n/128,kb] *
 * (A B^T)_kb over 128-K blocks.  A E4M3 [M,K] (K-major); B K-major as
 * BSG_B_RAW [N,K] or BSG_B_KPANEL128 B'[K/128][N][128] (stride_b = 128, as the
 * reference kargs); SFA fp32 BSG_SF_ROWMAJOR [M,K/128] (aiter x_scale) or
 * BSG_SF_KMAJOR_T [K/128,M] (reference kernel); SFB fp32 [N/128,K/128]
 * row-major.  Requires K % 128 == 0, N % 8 == 0.  kernel: AUTO (M <= 32 ->
 * transposed decode kernel; M > 128 -> CTA pairs when they cover the problem
 * in fewer waves than single-CTA tiles; else single-CTA tiles with automatic
 * split-K), 1CTA, PAIR, SWAP (M <= 64) or WIDE (one CTA per 128x256 tile,
 * every tile in split_k K slices; split_k 0 = the library's choice).  With
 * split_k 0 the pair kernel runs its partial last wave as K slices whose fp32
 * partials use the workspace (without one, the tail runs unsplit); split_k 1
 * keeps every tile whole, and then 1CTA, PAIR and WIDE give the same bits and
 * a row's result does not depend on the other rows.
 * Replaces gemm_a8w8_blockscale_bpreshuffle_kernel's launch in
 * block_scale_gemm_bpreshuffle/gemm_a8w8_blockscale_bpreshuffle_host.cc:
 * 275-281 and aiter's gemm_a8w8_bpreshuffle_opus.
 */
BSG_API int bsgemm_a8w8_blockscale_bpreshuffle(const bsgemm_args *args, bsg_stream_t stream);

/*
 * Grouped (MoE) FP8 block-scale GEMM: args->batch groups (experts), group e
 * multiplying rows [group_offsets[e], group_offsets[e+1]) of a concatenated
 * A E4M3 [total_rows, K] (and the same rows of SFA fp32 [total_rows, K/128],
 * BSG_SF_ROWMAJOR) by its own weights (args->ptr_b + e * stride_b_batch in any
 * B format above; SFB fp32 [N/128, K/128] at ptr_sfb + e * stride_sfb_batch)
 * and writing the same rows of C [total_rows, N].  group_offsets is a DEVICE
 * array of batch + 1 non-decreasing int32 row offsets (the token routing, so
 * no host round trip); args->m is the most rows any group can hold (it sizes
 * the tile grid; tiles past a group's rows are skipped).  Offsets are clamped
 * to [0, total_rows] and a group to args->m rows, so an inconsistent array
 * gives wrong rows, never an out-of-bounds access.  split_k must be 0 or 1;
 * kernel AUTO / 1CTA (128-row tiles) or PAIR (CTA pairs, 256-row tiles per
 * group; the same bits).
 * No launcher in the reference; its notes point at a batched mxscale GEMM
 * (opus_gemm_splitk_and_interface_refactor.md:10, aiter PR #4320).
 */
BSG_API int bsgemm_a8w8_blockscale_grouped(const bsgemm_args *args, const int *group_offsets, int total_rows,
                                           bsg_stream_t stream);

/*
 * Grouped (MoE) MXFP8 / MXFP4 GEMM, with the groups given as in
 * bsgemm_a8w8_blockscale_grouped: A [total_rows, K] E4M3 (MXFP4: packed E2M1
 * [total_rows, K/2] bytes), layout TN, with SFA E8M0 [total_rows, K/32]
 * (BSG_SF_ROWMAJOR, row stride stride_sfa bytes); group e's weights B
 * [N, K] (raw or BSG_B_SHUFFLE16) at ptr_b + e * stride_b_batch and their SFB
 * E8M0 in BSG_SF_ROWMAJOR or BSG_SF_NATIVE, per group at stride_sfb_batch.
 * The row-major scales are packed into tcgen05 atoms (A per group, from the
 * device offsets) in the caller's workspace, which must hold
 * bsgemm_mx_grouped_workspace_size(args) bytes.  Offsets are clamped as in
 * bsgemm_a8w8_blockscale_grouped.  split_k 0 or 1; kernel AUTO or 1CTA.
 * No launcher in the reference (same note as the FP8 block-scale form).
 */
BSG_API int bsgemm_a8w8_mxfp8_grouped(const bsgemm_args *args, const int *group_offsets, int total_rows,
                                      bsg_stream_t stream);
BSG_API int bsgemm_a4w4_mxfp4_grouped(const bsgemm_args *args, const int *group_offsets, int total_rows,
                                      bsg_stream_t stream);
BSG_API size_t bsgemm_mx_grouped_workspace_size(const bsgemm_args *args);

/*
 * Host-staged MXFP8 / MXFP4 GEMM (family BSG_FAMILY_MXFP8 or _MXFP4): A, B,
 * their E8M0 scales (BSG_SF_ROWMAJOR) and C are HOST pointers (pinned for
 * asynchronous copies), with the strides of bsgemm_a8w8_mxfp8; layout TN,
 * batch 1, B raw or BSG_B_SHUFFLE16.  The call copies the operands in
 * row chunks (chunks per dimension, 1..8; 0 = one per 1024 rows, at most 4)
 * on `stream`, runs each C block's GEMM on an internal stream as soon as its
 * A and B chunks have arrived, and copies each finished block back on a
 * second internal stream, so both copy directions and the GEMMs overlap.
 * dev_workspace (256-byte aligned) holds the device copies and C:
 * bsgemm_mx_host_workspace_size(family, args) bytes.  Asynchronous: C is
 * complete when `stream` reaches this point.  The block GEMMs run without
 * split-K (args->split_k and args->workspace are ignored).  The first call
 * on a device creates the two internal streams and their events (no device
 * memory); calls on one device are serialised while they enqueue.  C
 * should be pinned: with pageable host C each strip's copy-back is
 * synchronous, so the host waits for that strip's GEMM before it queues the
 * next one and the copies no longer overlap the GEMMs.  The internal streams
 * and events are cached per device ordinal for the life of the process: do
 * not use the library across cudaDeviceReset on that device.
 * Replaces the reference drivers' hipMemcpy-in / launch / hipMemcpy-out
 * sequence (mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:261-301,
 * mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:195-224).
 */
BSG_API size_t bsgemm_mx_host_workspace_size(int family, const bsgemm_args *args);
BSG_API int bsgemm_mx_host_gemm(int family, const bsgemm_args *args, void *dev_workspace,
                                size_t dev_workspace_bytes, int chunks, bsg_stream_t stream);

/*
 * Bytes of workspace the call would need (0 when it needs none): split-K
 * partials, the FP8 block-scale pair kernel's tail-slice partials and the
 * wide kernel's K-slice partials, row-major MX scales repacked into native
 * atoms.  family = BSG_FAMILY_*.
 */
BSG_API size_t bsgemm_workspace_size(int family, const bsgemm_args *args);

/*
 * Device repack of B between a reference preshuffle and the raw layout
 * (async on stream).  The GEMMs read BSG_B_SHUFFLE16 and BSG_B_KPANEL128 in
 * place; this converts weights for other consumers, or raw -> preshuffled.
 *   src_format BSG_B_KPANEL128 or BSG_B_SHUFFLE16; dst is [rows, kbytes] bytes
 *   (kbytes = K for fp8, K/2 for fp4).  rows % 16 == 0 and kbytes % 16 == 0
 *   for SHUFFLE16; kbytes % 128 == 0 for KPANEL128.  unpack = 1 runs the
 *   inverse permutation (raw -> src_format).
 * Replaces the host preshuffles of the reference (shuffle_b,
 * block_scale_gemm_bpreshuffle/..._host.cc:96-111; pack_weight_16x16,
 * source_snapshot/gemm_a8w8_mxfp8_scale_host.cc:161-179; candidate_m10 bs,
 * mxfp4_gemm_4wave_20261112/candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:215-225).
 */
BSG_API int bsgemm_pack_b(const void *src, void *dst, int rows, int kbytes, int src_format,
                  int unpack, bsg_stream_t stream);

/*
 * Device repack of an E8M0 scale matrix [rows, kg] (kg = K/32) into the
 * native tcgen05 layout: 512-byte atoms of 128 rows x 4 groups, atom (rb,kb)
 * at (rb*ceil(kg/4)+kb)*512, byte ((r%32)*4 + (r%128)/32)*4 + g%4; padding
 * 0x7F.  src_format BSG_SF_ROWMAJOR (row stride src_stride bytes) or
 * BSG_SF_E8M0_SHUFFLE (aiter layout, candidate_m10/..._host.cc:194-206).
 * unpack = 1 writes native -> src_format instead.
 */
BSG_API int bsgemm_pack_scales(const void *src, int src_stride, void *dst, int rows, int kg,
                       int src_format, int unpack, bsg_stream_t stream);
/* Bytes of a native scale buffer for [rows, kg]. */
BSG_API size_t bsgemm_native_scales_size(int rows, int kg);

/*
 * Exact drop-in for the reference's only extern "C" launcher
 * (source_snapshot/gemm_a8w8_blockscale_bpreshuffle_launch.cc:31-65):
 * E4M3 A [M,K], B in shuffle_weight(16,16) layout, E8M0 SFA [K/128,M],
 * E8M0 SFB [N/128,K/128]; bf16 (output_bf16 = 1) or fp32 C.  Same
 * validation rules (M,N % 256, K % 128, dense strides, no overlap).
 * Returns 0 (cudaSuccess) or a cudaError_t value, as the reference.
 * The kargs struct is the first 96 bytes of bsgemm_args.
 */
BSG_API int launch_blockscale_bpreshuffle(const void *opus_gemm_scale_kargs, int output_bf16,
                                  int tiles, bsg_stream_t stream);

/* ---- activation quantise + pack ----------------------------------------- */
enum { BSG_QUANT_MXFP8 = 0, BSG_QUANT_MXFP4 = 1, BSG_QUANT_FP8_BLOCK = 2 };
enum { BSG_IN_BF16 = 0, BSG_IN_FP32 = 1 };

/*
 * Quantise x [rows, cols] (bf16 or fp32, row stride ldx elements, 16-byte
 * aligned rows) in one pass, writing elements and scales in layouts the GEMM
 * entry points read:
 *   BSG_QUANT_MXFP8     q E4M3 [rows, cols] bytes (row stride ldq bytes, % 8),
 *                       one E8M0 scale per 32 columns = 2^ceil(log2(amax/448)),
 *                       elements RNE-saturated from x * 2^-scale; cols % 32;
 *   BSG_QUANT_MXFP4     q packed E2M1 [rows, cols/2] (even column in the low
 *                       nibble, ldq % 4), scale 2^ceil(log2(amax/6)); cols % 32;
 *   BSG_QUANT_FP8_BLOCK q E4M3 [rows, cols], one fp32 scale amax/448 per 128
 *                       columns (1 for an all-zero block); cols % 128.
 * MX scales: sf_format BSG_SF_NATIVE (tcgen05 atoms, bsgemm_native_scales_size(
 * rows, cols/32) bytes, padding rows 0x7F; cols % 128) or BSG_SF_ROWMAJOR
 * ([rows, cols/32] bytes, row stride ld_sf).  FP8 block scales:
 * BSG_SF_ROWMAJOR ([rows, cols/128], row stride ld_sf floats) or
 * BSG_SF_KMAJOR_T ([cols/128, rows], stride ld_sf floats).
 * Bit-identical to the reference drivers' host quantisation recipes (E8M0
 * codec: mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:35-47).  No reference entry
 * point: the reference quantises on the host only.
 */
BSG_API int bsgemm_quantize(const void *x, int in_dtype, int rows, int cols, long long ldx, int format,
                            void *q, long long ldq, void *sf, int sf_format, long long ld_sf,
                            bsg_stream_t stream);

/* Human-readable status. */
BSG_API const char *bsgemm_strerror(int status);

/*
 * Device-side error word of the current device (set by a kernel whose
 * bounded wait expired); reading it synchronises the device and clears it.
 * Returns BSG_OK or BSG_ERR_TIMEOUT (or BSG_ERR_CUDA if the read failed).
 */
BSG_API int bsgemm_check_device_error(void);

/*
 * Self-test of the bounded-wait path: launches one tiny kernel whose
 * mbarrier nothing ever arrives at, with a wait limit of timeout_us; returns
 * the status the kernel reported (BSG_ERR_TIMEOUT expected).  Synchronous.
 */
BSG_API int bsgemm_selftest_timeout(int timeout_us);

/*
 * Allocation-free variant of bsgemm_a8w8_mxfp8 (same arguments, same
 * results) for callers that cannot allocate device memory at all -- e.g. a
 * serving runtime that owns the whole HBM budget through its own allocator,
 * or code that must not take the device synchronisation an allocation can
 * cause.  args->workspace is ignored: the scale repacking and split-K
 * partials use a fixed 8 MiB scratch array in the library's device image
 * (held on every GPU that loads the library until exit; see
 * bsgemm_noalloc_scratch_bytes).  Problems that need more are rejected with
 * BSG_ERR_SCRATCH_LIMIT.  All calls on a device share that one array: calls
 * that overlap on the GPU race and corrupt each other.  The first call on a
 * device looks the array's address up (once per device); make it before any
 * stream capture.  That address is cached per device ordinal for the life of
 * the process: do not call this entry point across cudaDeviceReset on that
 * device (the reset unloads the module that holds the array).  No
 * counterpart in the reference, whose launchers need no scratch.
 */
BSG_API int bsgemm_a8w8_mxfp8_noalloc(const bsgemm_args *args, bsg_stream_t stream);
/* Size of that fixed scratch array in bytes. */
BSG_API size_t bsgemm_noalloc_scratch_bytes(void);

/* Library version string. */
BSG_API const char *bsgemm_version(void);

#ifdef __cplusplus
}
#endif
#endif

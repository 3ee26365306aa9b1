"""bsgemm_b200 -- B200 (sm_100a) block-scaled GEMM library, Python host side.

The package directory name starts with a digit, so import it with
``importlib.import_module("355_1_trans_b200")``.

Everything here is a thin host mirror of the reference's Python adapter
(trace_block_scale_latest_20260914_040021/source_snapshot/blockscale_bpreshuffle.py:15-97)
and of aiter's ``gemm_a8w8_bpreshuffle_opus`` API
(opus_a8w8_bpreshuffle_integration_and_benchmark.md:113-135): it validates
tensors, fills the C-ABI argument struct and calls the CUDA library
``_build/libbsgemm_b200.so`` through ctypes on the current torch stream.
There is no CPU or library fallback: if the shared library is missing or the
device is not an sm_100 GPU, calls raise.
"""
from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "_build" / "libbsgemm_b200.so"

# ---- C enums (include/bsgemm_b200.h) -----------------------------------------
(OK, ERR_INVALID_VALUE, ERR_UNSUPPORTED, ERR_ARCH, ERR_WORKSPACE, ERR_CUDA, ERR_TIMEOUT, ERR_ALIGNMENT,
 ERR_SCRATCH_LIMIT) = range(9)
LAYOUTS = {"nt": 0, "tt": 1, "nn": 2, "tn": 3}
B_RAW, B_KPANEL128, B_SHUFFLE16 = 0, 1, 2
SF_NATIVE, SF_ROWMAJOR, SF_KMAJOR_T, SF_E8M0_SHUFFLE = 0, 1, 2, 3
OUT_BF16, OUT_FP32 = 0, 1
KERNELS = {"auto": 0, "1cta": 1, "pair": 2, "swap": 3, "wide": 4}
FAMILY_MXFP8, FAMILY_MXFP4, FAMILY_FP8_BLOCK = 0, 1, 2


class BsgemmError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what} failed: {status} ({strerror(status)})")


class Args(ctypes.Structure):
    """bsgemm_args: the reference's 96-byte kargs prefix + extensions."""
    _fields_ = (
        [(name, ctypes.c_void_p) for name in ("ptr_a", "ptr_b", "ptr_c")]
        + [(name, ctypes.c_int) for name in (
            "m", "n", "k", "batch", "stride_a", "stride_b", "stride_c",
            "stride_a_batch", "stride_b_batch", "stride_c_batch")]
        + [(name, ctypes.c_void_p) for name in ("ptr_sfa", "ptr_sfb")]
        + [(name, ctypes.c_int) for name in (
            "stride_sfa", "stride_sfb", "stride_sfa_batch", "stride_sfb_batch",
            "layout", "b_format", "sfa_format", "sfb_format", "out_dtype", "split_k")]
        + [("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
           ("grid_blocks", ctypes.c_int), ("kernel", ctypes.c_int)]
    )


assert Args.ptr_sfa.offset == 64 and Args.stride_sfa.offset == 80
assert Args.layout.offset == 96


@lru_cache(None)
def lib() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python 355_1_trans_b200/build.py` "
            "(there is no fallback implementation)")
    so = ctypes.CDLL(str(LIB_PATH))
    P, I, S = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    sigs = {
        "bsgemm_args_init": (None, [ctypes.POINTER(Args)]),
        "bsgemm_a8w8_mxfp8": (I, [ctypes.POINTER(Args), P]),
        "bsgemm_a4w4_mxfp4": (I, [ctypes.POINTER(Args), P]),
        "bsgemm_a8w8_blockscale_bpreshuffle": (I, [ctypes.POINTER(Args), P]),
        "bsgemm_a8w8_blockscale_grouped": (I, [ctypes.POINTER(Args), P, I, P]),
        "bsgemm_a8w8_mxfp8_grouped": (I, [ctypes.POINTER(Args), P, I, P]),
        "bsgemm_a4w4_mxfp4_grouped": (I, [ctypes.POINTER(Args), P, I, P]),
        "bsgemm_mx_grouped_workspace_size": (S, [ctypes.POINTER(Args)]),
        "bsgemm_mx_host_workspace_size": (S, [I, ctypes.POINTER(Args)]),
        "bsgemm_mx_host_gemm": (I, [I, ctypes.POINTER(Args), P, S, I, P]),
        "bsgemm_workspace_size": (S, [I, ctypes.POINTER(Args)]),
        "bsgemm_pack_b": (I, [P, P, I, I, I, I, P]),
        "bsgemm_pack_scales": (I, [P, I, P, I, I, I, I, P]),
        "bsgemm_native_scales_size": (S, [I, I]),
        "launch_blockscale_bpreshuffle": (I, [P, I, I, P]),
        "bsgemm_strerror": (ctypes.c_char_p, [I]),
        "bsgemm_check_device_error": (I, []),
        "bsgemm_selftest_timeout": (I, [I]),
        "bsgemm_version": (ctypes.c_char_p, []),
        "bsgemm_quantize": (I, [P, I, I, I, ctypes.c_longlong, I, P, ctypes.c_longlong, P, I,
                                ctypes.c_longlong, P]),
    }
    for name, (res, argt) in sigs.items():
        fn = getattr(so, name)
        fn.restype = res
        fn.argtypes = argt
    return so


def strerror(status: int) -> str:
    return lib().bsgemm_strerror(int(status)).decode()


def version() -> str:
    return lib().bsgemm_version().decode()


def check_device_error() -> int:
    """Synchronise and read/clear the device error word (0 or ERR_TIMEOUT)."""
    return int(lib().bsgemm_check_device_error())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _check(status: int, what: str):
    if status != OK:
        raise BsgemmError(status, what)


_FP8 = (torch.float8_e4m3fn, torch.uint8)
_SCALE_U8 = (torch.uint8, getattr(torch, "float8_e8m0fnu", torch.uint8))
_FP4 = (torch.uint8, getattr(torch, "float4_e2m1fn_x2", torch.uint8))


def _out(out, m, n, dtype, device, batch):
    shape = (m, n) if batch == 1 else (batch, m, n)
    if out is None:
        return torch.empty(shape, device=device, dtype=dtype)
    if tuple(out.shape) != shape or out.dtype != dtype or out.device != device or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor of shape %s and dtype %s" % (shape, dtype))
    return out


def _workspace(family: int, args: Args, workspace, device):
    """workspace None: allocate what the call needs; a tensor: use it;
    False: pass none (a decode-shaped call then splits K inside CTA clusters,
    up to 4 slices, or runs unsplit; row-major MX scales still need one)."""
    if workspace is False:
        return None
    need = int(lib().bsgemm_workspace_size(family, ctypes.byref(args)))
    if need == 0:
        return None
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=device)
    elif workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"workspace needs {need} bytes")
    args.workspace = workspace.data_ptr()
    args.workspace_bytes = workspace.numel() * workspace.element_size()
    return workspace


def _record(tensors, device):
    stream = torch.cuda.current_stream(device)
    for t in tensors:
        if t is not None and t.is_cuda:
            t.record_stream(stream)


# ---------------------------------------------------------------------------
# MXFP8 / MXFP4
# ---------------------------------------------------------------------------

def gemm_a8w8_mxfp8(A, B, A_scale, B_scale, *, layout: str = "tn", out_dtype=torch.bfloat16,
                    out=None, scale_format: str = "rowmajor", split_k: int = 0,
                    workspace=None, grid_blocks: int = 0, kernel: str = "auto",
                    b_format: str = "raw"):
    """MXFP8 GEMM (mxfp8_gemm/gemm_a8w8_mxfp8_host.cc:98-122 semantics).

    A: E4M3 [M,K] (layout t*) or [K,M] (n*); B: E4M3 [N,K] (*n) or [K,N] (*t);
    optional leading batch dim.  A_scale/B_scale: E8M0 bytes, [rows, K/32]
    row-major (scale_format="rowmajor") or native atoms from pack_scales
    (scale_format="native").  Returns C [M,N] (or [batch,M,N]) of out_dtype.
    kernel: "auto", "1cta" (128 x BN tiles, one CTA each), "pair" (256 x 256
    tiles on CTA pairs, cta_group::2) or "swap" (transposed decode kernel,
    M <= 64, layout tn).  b_format "shuffle16": B holds aiter's
    shuffle_weight(16,16) bytes of a K-major [N,K] B (read in place).
    """
    return _mx(A, B, A_scale, B_scale, fp4=False, layout=layout, out_dtype=out_dtype, out=out,
               scale_format=scale_format, split_k=split_k, workspace=workspace,
               grid_blocks=grid_blocks, kernel=kernel, b_format=b_format)


def gemm_a4w4_mxfp4(A, B, A_scale, B_scale, *, out_dtype=torch.bfloat16, out=None,
                    scale_format: str = "rowmajor", split_k: int = 0, workspace=None,
                    grid_blocks: int = 0, kernel: str = "auto", b_format: str = "raw"):
    """MXFP4 GEMM (mxfp4_gemm_4wave_20261112/gemm_a4w4_mxfp4_4wave_host.cc:97-115
    semantics): A [M,K/2], B [N,K/2] packed E2M1 bytes (even k low nibble),
    K-major; scales E8M0 [rows, K/32] or native.  b_format "shuffle16": B is
    the shuffle_weight(16,16) form of the [N,K/2] bytes
    (candidate_m10/gemm_a4w4_mxfp4_4wave_host.cc:215-225), read in place."""
    return _mx(A, B, A_scale, B_scale, fp4=True, layout="tn", out_dtype=out_dtype, out=out,
               scale_format=scale_format, split_k=split_k, workspace=workspace,
               grid_blocks=grid_blocks, kernel=kernel, b_format=b_format)


_B_FORMATS = {"raw": B_RAW, "shuffle16": B_SHUFFLE16}


def _tuned(family: str, m: int, n: int, k: int, kernel: str, split_k: int):
    """(kernel, split_k) from the installed tuned table for "auto" calls."""
    if kernel != "auto" or split_k != 0:
        return kernel, split_k
    from . import tuning
    table = tuning.active()
    sel = table.lookup(family, m, n, k) if table is not None else None
    return sel if sel is not None else (kernel, split_k)


def _mx(A, B, A_scale, B_scale, *, fp4, layout, out_dtype, out, scale_format, split_k,
        workspace, grid_blocks, kernel="auto", b_format="raw"):
    if layout not in LAYOUTS:
        raise ValueError(f"layout must be one of {sorted(LAYOUTS)}")
    if b_format not in _B_FORMATS:
        raise ValueError(f"b_format must be one of {sorted(_B_FORMATS)}")
    if A.dim() != B.dim() or A.dim() not in (2, 3):
        raise ValueError("A and B must both be 2-D or both 3-D (batched)")
    tensors = (A, B, A_scale, B_scale)
    if not A.is_cuda or any(t.device != A.device for t in tensors):
        raise ValueError("all inputs must be on the same GPU")
    ok_types = _FP4 if fp4 else _FP8
    if A.dtype not in ok_types or B.dtype not in ok_types:
        raise ValueError("A/B must hold %s bytes" % ("packed E2M1" if fp4 else "E4M3FN"))
    if A_scale.dtype not in _SCALE_U8 or B_scale.dtype not in _SCALE_U8:
        raise ValueError("scales must be E8M0 bytes")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be bfloat16 or float32")
    batch = A.shape[0] if A.dim() == 3 else 1
    code = LAYOUTS[layout]
    a_km, b_km = bool(code & 1), bool(code & 2)
    a2 = A.shape[-2:]
    b2 = B.shape[-2:]
    if fp4:
        m, kh = a2
        n = b2[0]
        k = 2 * kh
        if b2[1] != kh:
            raise ValueError("A and B disagree on K")
    else:
        m, k = (a2[0], a2[1]) if a_km else (a2[1], a2[0])
        n, kb = (b2[0], b2[1]) if b_km else (b2[1], b2[0])
        if kb != k:
            raise ValueError("A and B disagree on K")
    for t in (A, B):
        if t.stride(-1) != 1:
            raise ValueError("A and B must have unit stride in the last dimension")
    out = _out(out, m, n, out_dtype, A.device, batch)
    kernel, split_k = _tuned("mxfp4" if fp4 else "mxfp8", m, n, k, kernel, split_k)
    args = Args()
    lib().bsgemm_args_init(ctypes.byref(args))
    args.ptr_a, args.ptr_b, args.ptr_c = A.data_ptr(), B.data_ptr(), out.data_ptr()
    args.m, args.n, args.k, args.batch = m, n, k, batch
    args.stride_a, args.stride_b, args.stride_c = A.stride(-2), B.stride(-2), n
    if batch > 1:
        args.stride_a_batch, args.stride_b_batch, args.stride_c_batch = A.stride(0), B.stride(0), m * n
    args.ptr_sfa, args.ptr_sfb = A_scale.data_ptr(), B_scale.data_ptr()
    if scale_format == "rowmajor":
        kg = k // 32
        for sc, rows in ((A_scale, m), (B_scale, n)):
            if tuple(sc.shape[-2:]) != (rows, kg) or sc.stride(-1) != 1:
                raise ValueError(f"scale must be [{rows}, {kg}] with unit inner stride")
        args.sfa_format = args.sfb_format = SF_ROWMAJOR
        args.stride_sfa, args.stride_sfb = A_scale.stride(-2), B_scale.stride(-2)
        if batch > 1:
            args.stride_sfa_batch, args.stride_sfb_batch = A_scale.stride(0), B_scale.stride(0)
    elif scale_format == "native":
        args.sfa_format = args.sfb_format = SF_NATIVE
        if batch > 1:
            args.stride_sfa_batch = A_scale.stride(0) if A_scale.dim() > 1 else 0
            args.stride_sfb_batch = B_scale.stride(0) if B_scale.dim() > 1 else 0
    else:
        raise ValueError("scale_format must be 'rowmajor' or 'native'")
    args.layout = code
    args.b_format = _B_FORMATS[b_format]
    args.out_dtype = OUT_BF16 if out_dtype == torch.bfloat16 else OUT_FP32
    args.split_k = split_k
    args.grid_blocks = grid_blocks
    args.kernel = KERNELS[kernel]
    ws = _workspace(FAMILY_MXFP4 if fp4 else FAMILY_MXFP8, args, workspace, A.device)
    fn = lib().bsgemm_a4w4_mxfp4 if fp4 else lib().bsgemm_a8w8_mxfp8
    with torch.cuda.device(A.device):
        status = fn(ctypes.byref(args), _stream(A.device))
        _record((*tensors, out, ws), A.device)
    _check(status, "bsgemm_a4w4_mxfp4" if fp4 else "bsgemm_a8w8_mxfp8")
    return out


# ---------------------------------------------------------------------------
# FP8 block-scale with fp32 scales (aiter gemm_a8w8_bpreshuffle_opus API)
# ---------------------------------------------------------------------------

def gemm_a8w8_bpreshuffle(A, B, x_scale, w_scale, out_dtype=torch.bfloat16, *,
                          preshuffled: bool = True, x_scale_transposed: bool = False,
                          out=None, split_k: int = 0, workspace=None, grid_blocks: int = 0,
                          kernel: str = "auto", b_layout: str | None = None):
    """a8w8 GEMM with fp32 1x128 (x_scale [M,K/128]) and 128x128
    (w_scale [N/128,K/128]) block scales, bf16/fp32 out.

    preshuffled=True: B is the K-panel layout B'[K/128][N][128] (given as a
    [K/128, N, 128] or flat [N, K] tensor), as aiter's wrapper produces
    (opus_a8w8_bpreshuffle_integration_and_benchmark.md:76-81);
    preshuffled=False: B is plain [N, K].  b_layout overrides both:
    "kpanel", "shuffle16" (aiter shuffle_weight(16,16) bytes of [N, K], read in
    place) or "raw".  x_scale_transposed=True takes the reference kernel's
    [K/128, M] SFA layout.  kernel: "auto", "1cta" (128x128 output tiles),
    "pair" (CTA pairs, 256x256 tiles), "swap" (transposed decode kernel,
    M <= 64) or "wide" (one CTA per 128x256 tile, every tile in the same
    number of K slices).  "auto" takes the decode kernel for M <= 32 and CTA pairs for
    M > 128 when they need fewer waves.  split_k 0 lets the library split K
    (and run the pair kernel's partial last wave as K slices); split_k 1 keeps
    every tile whole, so a row's result does not depend on the other rows.
    """
    if b_layout is None:
        b_layout = "kpanel" if preshuffled else "raw"
    if b_layout not in ("kpanel", "shuffle16", "raw"):
        raise ValueError("b_layout must be 'kpanel', 'shuffle16' or 'raw'")
    if A.dim() != 2:
        raise ValueError("A must be [M, K]")
    tensors = (A, B, x_scale, w_scale)
    if not A.is_cuda or any(t.device != A.device for t in tensors):
        raise ValueError("all inputs must be on the same GPU")
    if A.dtype not in _FP8 or B.dtype not in _FP8:
        raise ValueError("A/B must hold E4M3FN bytes")
    if x_scale.dtype != torch.float32 or w_scale.dtype != torch.float32:
        raise ValueError("scales must be fp32")
    m, k = A.shape
    if b_layout == "kpanel":
        if B.dim() == 3:
            kt, n, inner = B.shape
            if inner != 128 or kt * 128 != k:
                raise ValueError("K-panel B must be [K/128, N, 128]")
        else:
            n = B.numel() // k
        if not B.is_contiguous():
            raise ValueError("K-panel B must be contiguous")
    else:
        n, kb = B.shape
        if kb != k:
            raise ValueError("A and B disagree on K")
        if b_layout == "shuffle16" and not B.is_contiguous():
            raise ValueError("shuffled B must be contiguous")
    kblk = k // 128
    if x_scale_transposed:
        if tuple(x_scale.shape) != (kblk, m) or x_scale.stride(1) != 1:
            raise ValueError("transposed x_scale must be [K/128, M]")
    elif tuple(x_scale.shape) != (m, kblk) or x_scale.stride(1) != 1:
        raise ValueError("x_scale must be [M, K/128]")
    if tuple(w_scale.shape) != ((n + 127) // 128, kblk) or w_scale.stride(1) != 1:
        raise ValueError("w_scale must be [N/128, K/128]")
    out = _out(out, m, n, out_dtype, A.device, 1)
    kernel, split_k = _tuned("fp8_block", m, n, k, kernel, split_k)
    args = Args()
    lib().bsgemm_args_init(ctypes.byref(args))
    args.ptr_a, args.ptr_b, args.ptr_c = A.data_ptr(), B.data_ptr(), out.data_ptr()
    args.m, args.n, args.k, args.batch = m, n, k, 1
    args.stride_a, args.stride_c = A.stride(0), n
    args.stride_b = 128 if b_layout == "kpanel" else k if b_layout == "shuffle16" else B.stride(0)
    args.b_format = {"kpanel": B_KPANEL128, "shuffle16": B_SHUFFLE16, "raw": B_RAW}[b_layout]
    args.ptr_sfa, args.ptr_sfb = x_scale.data_ptr(), w_scale.data_ptr()
    args.sfa_format = SF_KMAJOR_T if x_scale_transposed else SF_ROWMAJOR
    args.stride_sfa = x_scale.stride(0)
    args.sfb_format = SF_ROWMAJOR
    args.stride_sfb = w_scale.stride(0)
    args.layout = LAYOUTS["tn"]
    args.out_dtype = OUT_BF16 if out_dtype == torch.bfloat16 else OUT_FP32
    args.split_k = split_k
    args.grid_blocks = grid_blocks
    args.kernel = KERNELS[kernel]
    ws = _workspace(FAMILY_FP8_BLOCK, args, workspace, A.device)
    with torch.cuda.device(A.device):
        status = lib().bsgemm_a8w8_blockscale_bpreshuffle(ctypes.byref(args), _stream(A.device))
        _record((*tensors, out, ws), A.device)
    _check(status, "bsgemm_a8w8_blockscale_bpreshuffle")
    return out


def gemm_a8w8_blockscale_grouped(A, B, x_scale, w_scale, group_offsets, max_rows: int,
                                 out_dtype=torch.bfloat16, *, out=None, b_layout: str = "kpanel",
                                 grid_blocks: int = 0, kernel: str = "auto"):
    """Grouped (MoE) a8w8 GEMM with fp32 1x128 / 128x128 block scales.

    The tokens of all groups (experts) are concatenated: A [T, K] E4M3 and
    x_scale [T, K/128]; group e owns rows group_offsets[e] .. group_offsets[e+1]
    (an int32 CUDA tensor of E + 1 offsets, as the routing writes it) and is
    multiplied by its own weights B[e] (layout b_layout, as in
    gemm_a8w8_bpreshuffle: B [E, K/128, N, 128] or [E, N, K]) with w_scale[e]
    [N/128, K/128].  max_rows bounds the rows of any group.  Returns C [T, N];
    rows outside every group are left unwritten.  kernel: "auto" / "1cta"
    (128-row tiles) or "pair" (CTA pairs, 256-row tiles: for groups of a few
    hundred rows or more)."""
    if kernel not in ("auto", "1cta", "pair"):
        raise ValueError("kernel must be 'auto', '1cta' or 'pair'")
    if b_layout not in ("kpanel", "shuffle16", "raw"):
        raise ValueError("b_layout must be 'kpanel', 'shuffle16' or 'raw'")
    tensors = (A, B, x_scale, w_scale, group_offsets)
    if A.dim() != 2 or not A.is_cuda or any(t.device != A.device for t in tensors):
        raise ValueError("A must be [T, K] and all inputs on the same GPU")
    if A.dtype not in _FP8 or B.dtype not in _FP8:
        raise ValueError("A/B must hold E4M3FN bytes")
    if x_scale.dtype != torch.float32 or w_scale.dtype != torch.float32:
        raise ValueError("scales must be fp32")
    if group_offsets.dtype != torch.int32 or group_offsets.dim() != 1 or not group_offsets.is_contiguous():
        raise ValueError("group_offsets must be a contiguous int32 tensor of E + 1 offsets")
    t_rows, k = A.shape
    groups = group_offsets.numel() - 1
    if groups < 1 or B.shape[0] != groups or w_scale.dim() != 3 or w_scale.shape[0] != groups:
        raise ValueError("B and w_scale need one entry per group")
    if not B.is_contiguous():
        raise ValueError("B must be contiguous")
    n = B.shape[2] if (b_layout == "kpanel" and B.dim() == 4) else B.shape[1]
    if B[0].numel() != n * k:
        raise ValueError("B and A disagree on K")
    kblk = k // 128
    if tuple(x_scale.shape) != (t_rows, kblk) or x_scale.stride(1) != 1:
        raise ValueError("x_scale must be [T, K/128]")
    if tuple(w_scale.shape[1:]) != ((n + 127) // 128, kblk) or w_scale.stride(2) != 1:
        raise ValueError("w_scale must be [E, N/128, K/128]")
    if max_rows < 1:
        raise ValueError("max_rows must be positive")
    out = _out(out, t_rows, n, out_dtype, A.device, 1)
    args = Args()
    lib().bsgemm_args_init(ctypes.byref(args))
    args.ptr_a, args.ptr_b, args.ptr_c = A.data_ptr(), B.data_ptr(), out.data_ptr()
    args.m, args.n, args.k, args.batch = int(max_rows), n, k, groups
    args.stride_a, args.stride_c = A.stride(0), n
    args.stride_b = 128 if b_layout == "kpanel" else k
    args.stride_b_batch = B.stride(0)
    args.b_format = {"kpanel": B_KPANEL128, "shuffle16": B_SHUFFLE16, "raw": B_RAW}[b_layout]
    args.ptr_sfa, args.ptr_sfb = x_scale.data_ptr(), w_scale.data_ptr()
    args.sfa_format = args.sfb_format = SF_ROWMAJOR
    args.stride_sfa = x_scale.stride(0)
    args.stride_sfb = w_scale.stride(1)
    args.stride_sfb_batch = w_scale.stride(0)
    args.layout = LAYOUTS["tn"]
    args.out_dtype = OUT_BF16 if out_dtype == torch.bfloat16 else OUT_FP32
    args.grid_blocks = grid_blocks
    args.kernel = KERNELS[kernel]
    with torch.cuda.device(A.device):
        status = lib().bsgemm_a8w8_blockscale_grouped(ctypes.byref(args), ctypes.c_void_p(group_offsets.data_ptr()),
                                                      t_rows, _stream(A.device))
        _record((*tensors, out), A.device)
    _check(status, "bsgemm_a8w8_blockscale_grouped")
    return out


def gemm_a8w8_mxfp8_grouped(A, B, A_scale, B_scale, group_offsets, max_rows: int,
                            out_dtype=torch.bfloat16, *, out=None, b_format: str = "raw",
                            b_scale_format: str = "rowmajor", workspace=None, grid_blocks: int = 0):
    """Grouped (MoE) MXFP8 GEMM.

    A [T, K] E4M3 with A_scale E8M0 [T, K/32]; group e owns rows
    group_offsets[e] .. group_offsets[e+1] (int32 CUDA tensor of E + 1
    offsets) and multiplies them by B[e] ([E, N, K], raw or shuffle_weight(16,16)
    bytes per b_format) with B_scale[e] (E8M0 [E, N, K/32] row-major, or native
    atoms per expert [E, bytes] with b_scale_format="native").  max_rows bounds
    the rows of any group.  Returns C [T, N]; rows outside every group are left
    unwritten."""
    return _mx_grouped(A, B, A_scale, B_scale, group_offsets, max_rows, fp4=False, out_dtype=out_dtype,
                       out=out, b_format=b_format, b_scale_format=b_scale_format, workspace=workspace,
                       grid_blocks=grid_blocks)


def gemm_a4w4_mxfp4_grouped(A, B, A_scale, B_scale, group_offsets, max_rows: int,
                            out_dtype=torch.bfloat16, *, out=None, b_format: str = "raw",
                            b_scale_format: str = "rowmajor", workspace=None, grid_blocks: int = 0):
    """Grouped (MoE) MXFP4 GEMM: as gemm_a8w8_mxfp8_grouped with A [T, K/2]
    and B [E, N, K/2] packed E2M1 bytes (even k in the low nibble)."""
    return _mx_grouped(A, B, A_scale, B_scale, group_offsets, max_rows, fp4=True, out_dtype=out_dtype,
                       out=out, b_format=b_format, b_scale_format=b_scale_format, workspace=workspace,
                       grid_blocks=grid_blocks)


def gemm_mx_from_host(A, B, A_scale, B_scale, *, fp4: bool, out_dtype=torch.bfloat16, out=None,
                      b_format: str = "raw", chunks: int = 0, workspace=None, device=None):
    """MXFP8 (fp4=False) or MXFP4 GEMM on host-resident operands, the
    reference drivers' copy-in / launch / copy-out sequence with the copies
    pipelined against the GEMM blocks (bsgemm_mx_host_gemm).

    A [M,K] E4M3 or [M,K/2] packed E2M1 bytes, B [N,K] (or its
    shuffle_weight(16,16) bytes with b_format="shuffle16") and row-major E8M0
    scales [rows, K/32], all CPU tensors (pinned for overlap).  Returns C
    [M,N] in host memory (pinned, unless `out` is given); the call returns once
    C is complete.  workspace: a CUDA uint8 tensor of at least
    bsgemm_mx_host_workspace_size bytes, allocated when omitted."""
    if b_format not in _B_FORMATS:
        raise ValueError(f"b_format must be one of {sorted(_B_FORMATS)}")
    tensors = (A, B, A_scale, B_scale)
    if any(t.is_cuda for t in tensors) or A.dim() != 2 or B.dim() != 2:
        raise ValueError("A, B and the scales must be 2-D host (CPU) tensors")
    ok_types = _FP4 if fp4 else _FP8
    if A.dtype not in ok_types or B.dtype not in ok_types:
        raise ValueError("A/B must hold %s bytes" % ("packed E2M1" if fp4 else "E4M3FN"))
    if A_scale.dtype not in _SCALE_U8 or B_scale.dtype not in _SCALE_U8:
        raise ValueError("scales must be E8M0 bytes")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be bfloat16 or float32")
    m, kb = A.shape
    n = B.shape[0]
    k = 2 * kb if fp4 else kb
    if B.shape[1] != kb or any(t.stride(-1) != 1 for t in tensors):
        raise ValueError("A and B must agree on K and have unit inner stride")
    if tuple(A_scale.shape) != (m, k // 32) or tuple(B_scale.shape) != (n, k // 32):
        raise ValueError("scales must be [rows, K/32]")
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, pin_memory=True)
    elif out.is_cuda or tuple(out.shape) != (m, n) or out.dtype != out_dtype or out.stride(1) != 1:
        raise ValueError("out must be a host tensor [M, N] of out_dtype with unit inner stride")
    args = Args()
    lib().bsgemm_args_init(ctypes.byref(args))
    args.ptr_a, args.ptr_b, args.ptr_c = A.data_ptr(), B.data_ptr(), out.data_ptr()
    args.m, args.n, args.k = m, n, k
    args.stride_a, args.stride_b, args.stride_c = A.stride(0), B.stride(0), out.stride(0)
    args.ptr_sfa, args.ptr_sfb = A_scale.data_ptr(), B_scale.data_ptr()
    args.stride_sfa, args.stride_sfb = A_scale.stride(0), B_scale.stride(0)
    args.b_format = _B_FORMATS[b_format]
    args.out_dtype = OUT_BF16 if out_dtype == torch.bfloat16 else OUT_FP32
    family = FAMILY_MXFP4 if fp4 else FAMILY_MXFP8
    need = int(lib().bsgemm_mx_host_workspace_size(family, ctypes.byref(args)))
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=device)
    elif not workspace.is_cuda or workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"workspace must be a CUDA tensor of at least {need} bytes")
    with torch.cuda.device(workspace.device):
        stream = torch.cuda.current_stream(workspace.device)
        status = lib().bsgemm_mx_host_gemm(family, ctypes.byref(args), ctypes.c_void_p(workspace.data_ptr()),
                                           workspace.numel() * workspace.element_size(), int(chunks),
                                           ctypes.c_void_p(stream.cuda_stream))
        _check(status, "bsgemm_mx_host_gemm")
        stream.synchronize()
    return out


def _mx_grouped(A, B, A_scale, B_scale, group_offsets, max_rows, *, fp4, out_dtype, out, b_format,
                b_scale_format, workspace, grid_blocks):
    if b_format not in _B_FORMATS:
        raise ValueError(f"b_format must be one of {sorted(_B_FORMATS)}")
    if b_scale_format not in ("rowmajor", "native"):
        raise ValueError("b_scale_format must be 'rowmajor' or 'native'")
    tensors = (A, B, A_scale, B_scale, group_offsets)
    if A.dim() != 2 or B.dim() != 3 or not A.is_cuda or any(t.device != A.device for t in tensors):
        raise ValueError("A must be [T, K], B [E, N, K], all on the same GPU")
    ok_types = _FP4 if fp4 else _FP8
    if A.dtype not in ok_types or B.dtype not in ok_types:
        raise ValueError("A/B must hold %s bytes" % ("packed E2M1" if fp4 else "E4M3FN"))
    if A_scale.dtype not in _SCALE_U8 or B_scale.dtype not in _SCALE_U8:
        raise ValueError("scales must be E8M0 bytes")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be bfloat16 or float32")
    if group_offsets.dtype != torch.int32 or group_offsets.dim() != 1 or not group_offsets.is_contiguous():
        raise ValueError("group_offsets must be a contiguous int32 tensor of E + 1 offsets")
    t_rows, kb = A.shape
    k = 2 * kb if fp4 else kb
    groups = group_offsets.numel() - 1
    if groups < 1 or B.shape[0] != groups:
        raise ValueError("B needs one entry per group")
    n = B.shape[1]
    if B.shape[2] != kb or not B.is_contiguous() or A.stride(1) != 1:
        raise ValueError("B must be a contiguous [E, N, K] and agree with A on K")
    kg = k // 32
    if tuple(A_scale.shape) != (t_rows, kg) or A_scale.stride(1) != 1:
        raise ValueError(f"A_scale must be [{t_rows}, {kg}]")
    if b_scale_format == "rowmajor" and (tuple(B_scale.shape) != (groups, n, kg) or B_scale.stride(2) != 1):
        raise ValueError(f"B_scale must be [{groups}, {n}, {kg}]")
    if b_scale_format == "native" and (B_scale.dim() != 2 or B_scale.shape[0] != groups):
        raise ValueError("native B_scale must be [E, bytes] (pack_scales per expert)")
    if max_rows < 1:
        raise ValueError("max_rows must be positive")
    out = _out(out, t_rows, n, out_dtype, A.device, 1)
    args = Args()
    lib().bsgemm_args_init(ctypes.byref(args))
    args.ptr_a, args.ptr_b, args.ptr_c = A.data_ptr(), B.data_ptr(), out.data_ptr()
    args.m, args.n, args.k, args.batch = int(max_rows), n, k, groups
    args.stride_a, args.stride_b, args.stride_c = A.stride(0), B.stride(1), n
    args.stride_b_batch = B.stride(0)
    args.b_format = _B_FORMATS[b_format]
    args.ptr_sfa, args.ptr_sfb = A_scale.data_ptr(), B_scale.data_ptr()
    args.sfa_format = SF_ROWMAJOR
    args.stride_sfa = A_scale.stride(0)
    if b_scale_format == "rowmajor":
        args.sfb_format = SF_ROWMAJOR
        args.stride_sfb, args.stride_sfb_batch = B_scale.stride(1), B_scale.stride(0)
    else:
        args.sfb_format = SF_NATIVE
        args.stride_sfb_batch = B_scale.stride(0)
    args.layout = LAYOUTS["tn"]
    args.out_dtype = OUT_BF16 if out_dtype == torch.bfloat16 else OUT_FP32
    args.grid_blocks = grid_blocks
    need = int(lib().bsgemm_mx_grouped_workspace_size(ctypes.byref(args)))
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=A.device)
    elif workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"workspace needs {need} bytes")
    args.workspace = workspace.data_ptr()
    args.workspace_bytes = workspace.numel() * workspace.element_size()
    fn = lib().bsgemm_a4w4_mxfp4_grouped if fp4 else lib().bsgemm_a8w8_mxfp8_grouped
    with torch.cuda.device(A.device):
        status = fn(ctypes.byref(args), ctypes.c_void_p(group_offsets.data_ptr()), t_rows, _stream(A.device))
        _record((*tensors, out, workspace), A.device)
    _check(status, "bsgemm_a4w4_mxfp4_grouped" if fp4 else "bsgemm_a8w8_mxfp8_grouped")
    return out


# ---------------------------------------------------------------------------
# E8M0 1x128 / 128x128 block scale: the reference's own ctypes adapter
# ---------------------------------------------------------------------------

class OpusGemmScaleKargs(ctypes.Structure):
    """opus_gemm_scale_kargs, the reference's 96-byte launcher argument
    (source_snapshot/gemm_a8w8_mxfp8_scale_common.h:12-38)."""
    _fields_ = Args._fields_[:19]


assert ctypes.sizeof(OpusGemmScaleKargs) == 96


def gemm_a8w8_blockscale_bpreshuffle(A, B, A_scale, B_scale, dtype=torch.bfloat16, out=None, *,
                                     tiles: int = 0):
    """One GEMM launch through launch_blockscale_bpreshuffle, as the reference
    adapter (source_snapshot/blockscale_bpreshuffle.py:37-97): A E4M3 [M,K];
    B the shuffle_weight(16,16) bytes of E4M3 [N,K]; A_scale E8M0 [M,K/128]
    stored column-major (strides (1, M)) or a contiguous tensor holding the
    transposed [K/128, M] bytes; B_scale E8M0 [N/128,K/128] contiguous; bf16 or
    fp32 out.  No input conversion and no workspace.  Differences from the
    reference: any M >= 1 and N % 128 == 0 are accepted (it: M, N % 256).
    Raises ValueError on bad inputs, RuntimeError on a nonzero CUDA status.
    """
    tensors = (A, B, A_scale, B_scale)
    if any(t.ndim != 2 for t in tensors):
        raise ValueError("A/B/A_scale/B_scale must be 2-D")
    if not A.is_cuda or any(t.device != A.device for t in tensors):
        raise ValueError("all inputs must be on the same GPU")
    if A.dtype != torch.float8_e4m3fn or B.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise ValueError("A/B must contain E4M3FN FP8 bytes")
    if A_scale.dtype not in _SCALE_U8 or B_scale.dtype not in _SCALE_U8:
        raise ValueError("scales must be E8M0 bytes, not FP32")
    m, k = A.shape
    n, bk = B.shape
    if min(m, n, k) <= 0 or k != bk or n % 128 or k % 128:
        raise ValueError("requires matching K, N % 128 == 0, K % 128 == 0")
    if dtype not in (torch.bfloat16, torch.float32) or tiles not in (0, 1):
        raise ValueError("dtype must be bf16/fp32; tiles must be 0 or 1")
    if not A.is_contiguous() or not B.is_contiguous() or not B_scale.is_contiguous():
        raise ValueError("A, packed B and B_scale must be contiguous")
    if tuple(A_scale.shape) != (m, k // 128) or tuple(B_scale.shape) != (n // 128, k // 128):
        raise ValueError("requires A_scale [M,K/128], B_scale [N/128,K/128]")
    if not A_scale.is_contiguous() and A_scale.stride() != (1, m):
        raise ValueError("A_scale must use dense column-major bytes")
    output_bytes = 2 if dtype == torch.bfloat16 else 4
    if max(m * k, n * k, m * n * output_bytes) > 2**31 - 1:
        raise ValueError("every tensor must stay below 2 GiB")
    if out is None:
        out = torch.empty((m, n), device=A.device, dtype=dtype)
    elif out.shape != (m, n) or out.dtype != dtype or out.device != A.device or not out.is_contiguous():
        raise ValueError("out must be contiguous [M,N] with the requested dtype/device")
    out_begin = out.data_ptr()
    out_end = out_begin + out.numel() * out.element_size()
    for tensor in tensors:
        begin = tensor.data_ptr()
        end = begin + tensor.numel() * tensor.element_size()
        if out_begin < end and begin < out_end:
            raise ValueError("out must not overlap any input tensor")
    args = OpusGemmScaleKargs(A.data_ptr(), B.data_ptr(), out.data_ptr(), m, n, k, 1,
                              k, k, n, m * k, n * k, m * n, A_scale.data_ptr(), B_scale.data_ptr(),
                              m, k // 128, m * (k // 128), (n // 128) * (k // 128))
    with torch.cuda.device(A.device):
        status = lib().launch_blockscale_bpreshuffle(
            ctypes.byref(args), int(dtype == torch.bfloat16), tiles, _stream(A.device))
        _record((*tensors, out), A.device)
    if status:
        raise RuntimeError(f"blockscale bpreshuffle launch failed: CUDA error {status}")
    return out


# ---------------------------------------------------------------------------
# activation quantise + pack (device)
# ---------------------------------------------------------------------------
QUANT_FORMATS = {"mxfp8": 0, "mxfp4": 1, "fp8_block": 2}


def quantize(x, fmt: str = "mxfp8", *, scale_format: str | None = None):
    """Quantise a bf16 or fp32 tensor [rows, cols] for the GEMMs in one device pass.

    fmt "mxfp8": (E4M3 [rows, cols], E8M0 per 32 columns), "mxfp4": (packed
    E2M1 [rows, cols/2] uint8, E8M0 per 32), "fp8_block": (E4M3, fp32 per 128).
    scale_format: MX "native" (tcgen05 atoms, default) or "rowmajor"
    [rows, cols/32]; fp8_block "rowmajor" [rows, cols/128] (default) or
    "kmajor_t" [cols/128, rows].  Returns (q, scales)."""
    if x.dim() != 2 or x.dtype not in (torch.bfloat16, torch.float32) or not x.is_cuda:
        raise ValueError("x must be a 2-D bf16 or fp32 CUDA tensor")
    if fmt not in QUANT_FORMATS:
        raise ValueError(f"fmt must be one of {sorted(QUANT_FORMATS)}")
    if x.stride(1) != 1:
        x = x.contiguous()
    rows, cols = x.shape
    dev = x.device
    if fmt == "fp8_block":
        scale_format = scale_format or "rowmajor"
        q = torch.empty((rows, cols), dtype=torch.float8_e4m3fn, device=dev)
        if scale_format == "rowmajor":
            sf = torch.empty((rows, cols // 128), dtype=torch.float32, device=dev)
            sff, ld = SF_ROWMAJOR, cols // 128
        elif scale_format == "kmajor_t":
            sf = torch.empty((cols // 128, rows), dtype=torch.float32, device=dev)
            sff, ld = SF_KMAJOR_T, rows
        else:
            raise ValueError("fp8_block scale_format must be 'rowmajor' or 'kmajor_t'")
        ldq = cols
    else:
        scale_format = scale_format or "native"
        q = torch.empty((rows, cols // 2 if fmt == "mxfp4" else cols),
                        dtype=torch.uint8 if fmt == "mxfp4" else torch.float8_e4m3fn, device=dev)
        ldq = q.shape[1]
        if scale_format == "native":
            sf = torch.empty(native_scales_size(rows, cols // 32), dtype=torch.uint8, device=dev)
            sff, ld = SF_NATIVE, 0
        elif scale_format == "rowmajor":
            sf = torch.empty((rows, cols // 32), dtype=torch.uint8, device=dev)
            sff, ld = SF_ROWMAJOR, cols // 32
        else:
            raise ValueError("MX scale_format must be 'native' or 'rowmajor'")
    with torch.cuda.device(dev):
        status = lib().bsgemm_quantize(x.data_ptr(), 1 if x.dtype == torch.float32 else 0, rows, cols,
                                       x.stride(0), QUANT_FORMATS[fmt], q.data_ptr(), ldq, sf.data_ptr(),
                                       sff, ld, _stream(dev))
        _record((x, q, sf), dev)
    _check(status, "bsgemm_quantize")
    return q, sf


# ---------------------------------------------------------------------------
# layout converters (device)
# ---------------------------------------------------------------------------

def pack_b(B, src_format: str, *, unpack: bool = False, out=None):
    """Byte permutation of a [rows, kbytes] operand between a reference
    preshuffle ('shuffle16' = aiter shuffle_weight(16,16), 'kpanel' =
    B'[K/128][N][128]) and the raw K-major layout (unpack=True: raw -> format).
    Returns a uint8 tensor of the same shape as the input's [rows, kbytes]."""
    fmt = {"shuffle16": B_SHUFFLE16, "kpanel": B_KPANEL128}[src_format]
    src = B.contiguous().view(torch.uint8)
    if src.dim() == 3:           # K-panel given as [K/128, N, 128]
        kt, rows, inner = src.shape
        kbytes = kt * inner
    else:
        rows, kbytes = src.shape
    if out is None:
        out = torch.empty((rows, kbytes), dtype=torch.uint8, device=B.device)
    with torch.cuda.device(B.device):
        status = lib().bsgemm_pack_b(src.data_ptr(), out.data_ptr(), rows, kbytes, fmt,
                                     int(unpack), _stream(B.device))
        _record((src, out), B.device)
    _check(status, "bsgemm_pack_b")
    return out


def native_scales_size(rows: int, kg: int) -> int:
    return int(lib().bsgemm_native_scales_size(rows, kg))


def pack_scales(sf, rows: int | None = None, kg: int | None = None, *, src_format: str = "rowmajor",
                out=None):
    """E8M0 [rows, kg] (row-major, or aiter e8m0_shuffle bytes with rows/kg given)
    -> native tcgen05 scale atoms (uint8, native_scales_size(rows, kg) bytes)."""
    src = sf.contiguous().view(torch.uint8)
    if src_format == "rowmajor":
        rows, kg = src.shape
        fmt, stride = SF_ROWMAJOR, kg
    elif src_format == "e8m0_shuffle":
        if rows is None or kg is None:
            raise ValueError("rows and kg are required for e8m0_shuffle input")
        fmt, stride = SF_E8M0_SHUFFLE, 0
    else:
        raise ValueError("src_format must be 'rowmajor' or 'e8m0_shuffle'")
    size = native_scales_size(rows, kg)
    if out is None:
        out = torch.empty(size, dtype=torch.uint8, device=sf.device)
    with torch.cuda.device(sf.device):
        status = lib().bsgemm_pack_scales(src.data_ptr(), stride, out.data_ptr(), rows, kg, fmt, 0,
                                          _stream(sf.device))
        _record((src, out), sf.device)
    _check(status, "bsgemm_pack_scales")
    return out


def unpack_scales(native, rows: int, kg: int, *, dst_format: str = "rowmajor"):
    """Inverse of pack_scales."""
    if dst_format == "rowmajor":
        out = torch.empty((rows, kg), dtype=torch.uint8, device=native.device)
        fmt, stride = SF_ROWMAJOR, kg
    elif dst_format == "e8m0_shuffle":
        size = ((rows + 31) // 32 * 32) * ((kg + 7) // 8 * 8)
        out = torch.empty(size, dtype=torch.uint8, device=native.device)
        fmt, stride = SF_E8M0_SHUFFLE, 0
    else:
        raise ValueError("dst_format must be 'rowmajor' or 'e8m0_shuffle'")
    with torch.cuda.device(native.device):
        status = lib().bsgemm_pack_scales(native.data_ptr(), stride, out.data_ptr(), rows, kg, fmt, 1,
                                          _stream(native.device))
        _record((native, out), native.device)
    _check(status, "bsgemm_pack_scales(unpack)")
    return out


def selftest_timeout(timeout_us: int = 2000) -> int:
    """Run the bounded-wait self test; returns the status (ERR_TIMEOUT expected)."""
    return int(lib().bsgemm_selftest_timeout(int(timeout_us)))


__all__ = [
    "Args", "BsgemmError", "lib", "strerror", "version", "check_device_error",
    "gemm_a8w8_mxfp8", "gemm_a4w4_mxfp4", "gemm_a8w8_bpreshuffle",
    "pack_b", "pack_scales", "unpack_scales", "native_scales_size", "selftest_timeout",
]

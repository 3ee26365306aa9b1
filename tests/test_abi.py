"""C-ABI checks that need no GPU: the shared library loads, exports every
symbol include/bsgemm_b200.h declares, the argument struct matches the
reference's 96-byte kargs, and invalid arguments are rejected before any
CUDA call."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "bsgemm_b200.h").read_text()
    return sorted(set(re.findall(r"BSG_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(bs):
    syms = declared_symbols()
    assert len(syms) >= 12
    lib = bs.lib()
    for s in syms:
        assert hasattr(lib, s), s


def test_args_struct_matches_reference_prefix(bs):
    A = bs.Args
    # opus_gemm_scale_kargs: 96 bytes, ptr_sfa at 64, stride_sfa at 80
    # (source_snapshot/gemm_a8w8_mxfp8_scale_common.h:35-37)
    assert A.ptr_sfa.offset == 64 and A.stride_sfa.offset == 80
    assert A.layout.offset == 96
    assert A.stride_c_batch.offset == 60 and A.ptr_sfb.offset == 72


def test_args_init_defaults(bs):
    a = bs.Args()
    bs.lib().bsgemm_args_init(ctypes.byref(a))
    assert a.batch == 1 and a.layout == bs.LAYOUTS["tn"] and a.out_dtype == bs.OUT_BF16


def test_strerror_and_version(bs):
    assert bs.strerror(0) == "success"
    assert "invalid" in bs.strerror(bs.ERR_INVALID_VALUE)
    assert "sm_100a" in bs.version()


def test_invalid_arguments_rejected_without_gpu(bs):
    lib = bs.lib()
    assert lib.bsgemm_a8w8_mxfp8(None, None) == bs.ERR_INVALID_VALUE
    a = bs.Args()
    lib.bsgemm_args_init(ctypes.byref(a))
    assert lib.bsgemm_a8w8_mxfp8(ctypes.byref(a), None) == bs.ERR_INVALID_VALUE  # null pointers
    a.ptr_a = a.ptr_b = a.ptr_c = a.ptr_sfa = a.ptr_sfb = 4096
    a.m, a.n, a.k = 256, 256, 256
    a.stride_a = a.stride_b = 256
    a.stride_c = 256
    a.out_dtype = 7
    assert lib.bsgemm_a8w8_mxfp8(ctypes.byref(a), None) == bs.ERR_INVALID_VALUE
    a.out_dtype = 0
    a.n = 260          # bf16 out needs N % 8
    a.stride_c = 260
    assert lib.bsgemm_a8w8_mxfp8(ctypes.byref(a), None) == bs.ERR_ALIGNMENT
    a.n = a.stride_c = 256
    for kernel in (-1, 5):   # kernel values outside BSG_KERNEL_*
        a.kernel = kernel
        assert lib.bsgemm_a8w8_mxfp8(ctypes.byref(a), None) == bs.ERR_INVALID_VALUE
    a.kernel = bs.KERNELS["wide"]   # the wide kernel is for fp32 block scales only
    assert lib.bsgemm_a8w8_mxfp8(ctypes.byref(a), None) == bs.ERR_UNSUPPORTED
    a.kernel = 0
    assert lib.bsgemm_pack_b(None, None, 16, 16, 2, 0, None) == bs.ERR_INVALID_VALUE
    assert lib.bsgemm_pack_scales(None, 0, None, 1, 1, 1, 0, None) == bs.ERR_INVALID_VALUE
    assert lib.bsgemm_native_scales_size(200, 12) == 2 * 3 * 512


def test_mx_grouped_workspace_and_rejections(bs):
    """Grouped MX: workspace = per-group A atoms (+ B atoms when row-major)
    + the groups' M-tile prefix, and missing arguments are rejected before any CUDA call."""
    lib = bs.lib()
    a = bs.Args()
    lib.bsgemm_args_init(ctypes.byref(a))
    a.m, a.n, a.k, a.batch = 200, 384, 1024, 8
    per_a = lib.bsgemm_native_scales_size(200, 32)
    per_b = lib.bsgemm_native_scales_size(384, 32)
    prefix = 256   # nine int32 M-tile prefix entries, 256-byte aligned
    assert lib.bsgemm_mx_grouped_workspace_size(ctypes.byref(a)) == 8 * per_a + 8 * per_b + prefix
    a.sfb_format = bs.SF_NATIVE
    assert lib.bsgemm_mx_grouped_workspace_size(ctypes.byref(a)) == 8 * per_a + prefix
    offs = (ctypes.c_int * 9)()
    for fn in (lib.bsgemm_a8w8_mxfp8_grouped, lib.bsgemm_a4w4_mxfp4_grouped):
        assert fn(None, offs, 100, None) == bs.ERR_INVALID_VALUE
        assert fn(ctypes.byref(a), None, 100, None) == bs.ERR_INVALID_VALUE
        assert fn(ctypes.byref(a), offs, 0, None) == bs.ERR_INVALID_VALUE
        assert fn(ctypes.byref(a), offs, 100, None) == bs.ERR_INVALID_VALUE   # null operands


def test_mx_host_workspace_and_rejections(bs):
    """Host-staged MX GEMM: the device workspace holds A, B, both scale forms
    and C (256-byte aligned pieces); bad arguments fail before any CUDA call."""
    lib = bs.lib()
    a = bs.Args()
    lib.bsgemm_args_init(ctypes.byref(a))
    a.m, a.n, a.k = 700, 640, 512

    def al(x):
        return (x + 255) // 256 * 256

    want = (al(700 * 512) + al(640 * 512) + al(700 * 16) + al(640 * 16) + al(lib.bsgemm_native_scales_size(700, 16))
            + al(lib.bsgemm_native_scales_size(640, 16)) + al(700 * 640 * 2))
    assert lib.bsgemm_mx_host_workspace_size(bs.FAMILY_MXFP8, ctypes.byref(a)) == want
    assert lib.bsgemm_mx_host_workspace_size(bs.FAMILY_FP8_BLOCK, ctypes.byref(a)) == 0
    fn = lib.bsgemm_mx_host_gemm
    assert fn(bs.FAMILY_MXFP8, None, None, 0, 0, None) == bs.ERR_INVALID_VALUE
    assert fn(bs.FAMILY_FP8_BLOCK, ctypes.byref(a), None, 0, 0, None) == bs.ERR_UNSUPPORTED
    assert fn(bs.FAMILY_MXFP8, ctypes.byref(a), None, 0, 0, None) == bs.ERR_INVALID_VALUE   # null pointers
    a.ptr_a = a.ptr_b = a.ptr_c = a.ptr_sfa = a.ptr_sfb = 4096
    a.stride_a = a.stride_b = 512
    a.stride_c = 640
    a.stride_sfa = a.stride_sfb = 16
    assert fn(bs.FAMILY_MXFP8, ctypes.byref(a), ctypes.c_void_p(1 << 20), 0, 9, None) == bs.ERR_INVALID_VALUE
    assert fn(bs.FAMILY_MXFP8, ctypes.byref(a), ctypes.c_void_p(1 << 20), 1024, 0, None) == bs.ERR_WORKSPACE
    a.layout = bs.LAYOUTS["nn"]
    assert fn(bs.FAMILY_MXFP8, ctypes.byref(a), ctypes.c_void_p(1 << 20), 1 << 30, 0, None) == bs.ERR_UNSUPPORTED


def test_python_api_rejects_cpu_tensors(bs):
    import torch
    a = torch.zeros(128, 128, dtype=torch.float8_e4m3fn)
    s = torch.zeros(128, 4, dtype=torch.uint8)
    with pytest.raises(ValueError):
        bs.gemm_a8w8_mxfp8(a, a, s, s)


def test_product_does_not_import_oracle():
    """The product package must never reach the CPU oracle."""
    for p in (ROOT / "355_1_trans_b200").rglob("*"):
        if p.suffix in (".py", ".cu", ".cuh", ".h", ".cpp"):
            assert "oracle" not in p.read_text(errors="ignore").replace("oracle-free", ""), p


def _opus_kargs(bs, m=256, n=256, k=256, base=1 << 20):
    """Dense kargs of the reference's launcher, fake (never dereferenced)
    16-byte aligned addresses in disjoint ranges."""
    kb = k // 128
    return bs.OpusGemmScaleKargs(base, base + (1 << 24), base + (2 << 24), m, n, k, 1, k, k, n,
                                 m * k, n * k, m * n, base + (3 << 24), base + (4 << 24),
                                 m, kb, m * kb, (n // 128) * kb)


def test_launch_blockscale_bpreshuffle_validation(bs):
    """Error behaviour of the reference launcher
    (source_snapshot/gemm_a8w8_blockscale_bpreshuffle_launch.cc:33-54): every
    rejected case returns cudaErrorInvalidValue (1) before any CUDA call."""
    lib = bs.lib()
    fn = lib.launch_blockscale_bpreshuffle
    INVALID = 1
    assert fn(None, 1, 0, None) == INVALID
    a = _opus_kargs(bs)
    assert fn(ctypes.byref(a), 2, 0, None) == INVALID          # output_bf16 not 0/1
    assert fn(ctypes.byref(a), 1, 2, None) == INVALID          # tiles not 0/1
    for field, value in (("ptr_a", None), ("ptr_sfb", None), ("k", 200), ("n", 200),
                         ("m", 0), ("batch", 0), ("stride_a", 512), ("stride_c", 512),
                         ("stride_sfa", 2), ("stride_sfb", 1), ("stride_sfa_batch", 1),
                         ("stride_b_batch", 1)):
        b = _opus_kargs(bs)
        setattr(b, field, value)
        assert fn(ctypes.byref(b), 1, 0, None) == INVALID, field
    c = _opus_kargs(bs)
    c.ptr_c = c.ptr_a + 64                                     # C overlaps A
    assert fn(ctypes.byref(c), 0, 0, None) == INVALID
    d = _opus_kargs(bs, m=1 << 16, n=1 << 16, k=1 << 16)       # int32 element-count overflow
    assert fn(ctypes.byref(d), 1, 0, None) == INVALID


def test_tuned_table_lookup(tmp_path):
    """aiter-schema tuned CSV: exact M, next bucket up, largest for big M,
    None for an untuned (N, K)."""
    import importlib
    tuning = importlib.import_module("355_1_trans_b200.tuning")
    path = tmp_path / "t.csv"
    rows = []
    for m, solidx, split in ((1, 3, 8), (16, 3, 4), (128, 1, 2), (1024, 1, 1)):
        r = {c: "" for c in tuning.TUNED_HEADER}
        r.update({"gfx": "sm_100a", "cu_num": 148, "M": m, "N": 7168, "K": 2048, "dtype": "fp8_block",
                  "solidx": solidx, "splitK": split})
        rows.append(r)
    import csv
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=tuning.TUNED_HEADER)
        w.writeheader()
        w.writerows(rows)
    t = tuning.TunedTable.load(path)
    assert t.lookup("fp8_block", 16, 7168, 2048) == ("swap", 4)
    assert t.lookup("fp8_block", 17, 7168, 2048) == ("1cta", 2)
    assert t.lookup("fp8_block", 5000, 7168, 2048) == ("1cta", 1)
    assert t.lookup("fp8_block", 16, 4096, 2048) is None
    assert t.lookup("mxfp8", 16, 7168, 2048) is None


def test_tuner_candidates():
    """The tuner times the kernels "auto" may use, never the wide kernel (slow on tiles of 72
    rows or fewer, which a tuned row's M bucket would route to it); split-K only while the
    output tiles leave SMs idle."""
    import importlib
    tuning = importlib.import_module("355_1_trans_b200.tuning")
    c = tuning.candidates("fp8_block", 128, 1536, 24576)
    assert ("auto", 0) in c and ("1cta", 1) in c
    assert not any(k == "wide" for k, _ in c)
    assert not any(s > 1 for _, s in c)            # 192 tiles fill the 148 SMs
    c = tuning.candidates("fp8_block", 16, 7168, 7168)
    assert ("swap", 4) in c and ("1cta", 2) in c
    c = tuning.candidates("fp8_block", 512, 7168, 7168)
    assert ("pair", 0) in c and ("pair", 1) in c and not any(k == "pair" and s > 1 for k, s in c)
    assert tuning.KERNEL_NAMES[4] == "wide"        # a table row may still name it explicitly


def test_shipped_tuned_table_loads():
    import importlib
    tuning = importlib.import_module("355_1_trans_b200.tuning")
    t = tuning.TunedTable.load(tuning.DEFAULT_TABLE)
    sel = t.lookup("fp8_block", 16, 7168, 18432)
    assert sel is not None and sel[0] in tuning.KERNEL_NAMES.values()
    # every (N, K) group of the traced DeepSeek-V4 shapes is tuned, with an M
    # bucket that covers the traced M range (6 .. 4096, or 16384)
    for n, k in ((1536, 7168), (2048, 7168), (6144, 7168), (7168, 3072), (7168, 7168), (7168, 16384),
                 (7168, 21504), (8192, 1536), (65536, 1536)):
        for m in (6, 66, 300, 4096):
            sel = t.lookup("fp8_block", m, n, k)
            assert sel is not None and sel[0] in tuning.KERNEL_NAMES.values(), (m, n, k)
        # a swap-kernel row is only ever chosen for M <= 64
        assert t.lookup("fp8_block", 4096, n, k)[0] != "swap"


def test_bench_l2_policy():
    """bench.py flushes L2 before every timed call when the inputs fit in it,
    and for skinny (weight-stream-bound) calls when they fit in twice the L2."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    mb = 1024 * 1024
    # MXFP8 8192^3: 138 MB of inputs, compute-bound -> no flush
    assert bench.l2_policy(8192, 138 * mb) == (False, False)
    # MXFP4 8192^3: 71 MB of inputs fit in L2 -> flush
    assert bench.l2_policy(8192, 71 * mb) == (True, False)
    # decode M=16 N=7168 K=18432: 132 MB < 2 x L2 -> flush, bandwidth roofline
    assert bench.l2_policy(16, 132 * mb) == (True, True)
    # skinny call streaming 300 MB of weights -> no flush needed
    assert bench.l2_policy(64, 300 * mb) == (False, True)

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
    assert lib.bsgemm_pack_b(None, None, 16, 16, 2, 0, None) == bs.ERR_INVALID_VALUE
    assert lib.bsgemm_pack_scales(None, 0, None, 1, 1, 1, 0, None) == bs.ERR_INVALID_VALUE
    assert lib.bsgemm_native_scales_size(200, 12) == 2 * 3 * 512


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

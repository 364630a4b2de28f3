"""The C ABI library: loads on a machine without a GPU, exports every entry point declared in
include/dm3.h, and rejects bad arguments before touching the device."""

import ctypes
import subprocess

import pytest
import torch


def test_library_exports_every_header_symbol(dm3):
    lib = dm3._lib.load()
    declared = dm3._lib.header_functions()
    assert len(declared) >= 9
    for name in declared:
        assert hasattr(lib, name), name
        assert name in dm3._lib.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", str(dm3._lib.LIB_PATH)], capture_output=True, text=True)
    if out.returncode == 0:
        for name in declared:
            assert f" T {name}" in out.stdout, name


def test_version_and_workspace_size(dm3):
    lib = dm3._lib.load()
    assert lib.dm3_version() == b"0.1.0"
    n = lib.dm3_moe_workspace_bytes(2, 2048, 512)
    assert n == lib.dm3_moe_workspace_bytes(4, 2048, 512)  # sized for the maximum row count
    assert 1 << 20 < n < 8 << 20


def test_invalid_arguments_are_rejected_without_a_device(dm3):
    lib = dm3._lib.load()
    p = ctypes.c_void_p(16)
    # M out of range
    rc = lib.dm3_fp8_gemv(p, 0, 2048, 16, p, 2048, p, 16, 1, None, 0, p, 16, 0, None)
    assert rc == dm3._lib.DM3_EINVAL and b"M must be" in lib.dm3_last_error()
    # K not a multiple of 128
    rc = lib.dm3_fp8_gemv(p, 2, 100, 16, p, 2048, p, 16, 1, None, 0, p, 16, 0, None)
    assert rc == dm3._lib.DM3_EINVAL
    # unsupported hidden size for the fused kernel
    rc = lib.dm3_moe_forward(p, 2, 4096, 512, p, p, 8, 32, p, 0, p, 0, p, 0, p, 0, 128, p, p, 1 << 30, None)
    assert rc == dm3._lib.DM3_EINVAL and b"H must be" in lib.dm3_last_error()
    # workspace too small
    rc = lib.dm3_moe_forward(p, 2, 2048, 512, p, p, 8, 32, p, 0, p, 0, p, 0, p, 0, 128, p, p, 16, None)
    assert rc == dm3._lib.DM3_ENOSPACE
    # misaligned weights
    q = ctypes.c_void_p(17)
    rc = lib.dm3_moe_forward(p, 2, 2048, 512, p, p, 8, 32, q, 0, p, 0, p, 0, p, 0, 128, p, p, 1 << 30, None)
    assert rc == dm3._lib.DM3_EINVAL


def test_ops_refuse_cpu_tensors(dm3):
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    q = torch.zeros(128, 256, dtype=torch.float8_e4m3fn)
    s = torch.ones(128, 2)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        dm3.ops.fp8_gemv(x, q, s)

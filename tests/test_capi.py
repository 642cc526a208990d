"""The C-ABI library loads without a GPU, exports every entry point declared in include/*.h and
rejects malformed arguments before touching the device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from mamba3_b200 import _ext

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> list[str]:
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = header.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*[A-Za-z_][\w \*]*?\b(m3_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = _ext.load()
    names = declared_functions()
    assert {"m3_scan_fwd", "m3_step_fwd", "m3_last_error", "m3_abi_version"} <= set(names)
    for name in names:
        assert hasattr(lib, name), name
    assert lib.m3_abi_version() == _ext.ABI_VERSION


def test_struct_layout_matches_header():
    # 12 ints + float + int, then 26 tensor descriptors of 64 bytes.
    assert ctypes.sizeof(_ext.M3Tensor) == 64
    assert ctypes.sizeof(_ext.ScanArgs) == 14 * 4 + 28 * 64
    assert ctypes.sizeof(_ext.StepArgs) == 8 * 4 + 26 * 64
    assert ctypes.sizeof(_ext.NormArgs) == 8 + 4 * 4 + 5 * 64


def test_residual_rmsnorm_rejects_bad_arguments_without_a_device():
    lib = _ext.load()
    assert lib.m3_residual_rmsnorm(None, None) == 4
    args = _ext.NormArgs()
    args.rows, args.dim, args.device = 4, 128, -1
    assert lib.m3_residual_rmsnorm(ctypes.byref(args), None) == 4  # x / w / out_n missing
    assert b"required" in lib.m3_last_error()
    args.dim = 0
    assert lib.m3_residual_rmsnorm(ctypes.byref(args), None) == 1


def test_null_and_invalid_arguments_are_rejected_without_a_device():
    lib = _ext.load()
    assert lib.m3_scan_fwd(None, None) == 4
    assert b"null" in lib.m3_last_error()
    args = _ext.ScanArgs()
    assert lib.m3_scan_fwd(ctypes.byref(args), None) == 1  # zero sizes
    args.batch, args.length, args.groups, args.heads, args.rank, args.d_state, args.head_dim = 1, 4, 1, 2, 3, 8, 4
    args.chunk_hint = 4
    assert lib.m3_scan_fwd(ctypes.byref(args), None) == 1
    assert b"rank" in lib.m3_last_error()
    args.rank = 1
    assert lib.m3_scan_fwd(ctypes.byref(args), None) == 4  # q missing
    assert b"missing required tensor q" in lib.m3_last_error()
    step = _ext.StepArgs()
    step.batch, step.heads, step.rank, step.d_state, step.head_dim, step.num_angles = 1, 2, 4, 16, 8, 2
    assert lib.m3_step_fwd(ctypes.byref(step), None) == 1
    assert b"4 * num_angles" in lib.m3_last_error()


def test_binding_refuses_host_tensors():
    """The binding never runs anything on the CPU: host tensors are an error, not a fallback."""
    with pytest.raises(ValueError, match="CUDA tensors"):
        _ext.scan_forward(sizes=dict(batch=1, length=2, groups=1, heads=1, rank=1, d_state=8, head_dim=4,
                                     num_angles=0), tensors=dict(value=torch.empty(1)))
    with pytest.raises(ValueError, match="CUDA tensors"):
        _ext.step_forward(sizes=dict(batch=1, heads=1, rank=1, d_state=8, head_dim=4, num_angles=2),
                          tensors=dict(value=torch.empty(1)))


def test_workspace_query_rejects_non_positive_sizes_without_a_device():
    """A negative size answers with minus an M3_ERR_* code and a message, and the allocation-free
    entry point passes that code on instead of a stray status."""
    lib = _ext.load()
    lib.m3_scan_fwd_noalloc.argtypes = [ctypes.POINTER(_ext.ScanArgs), ctypes.c_void_p]
    lib.m3_scan_fwd_noalloc.restype = ctypes.c_int
    args = _ext.ScanArgs()
    args.batch, args.length, args.groups, args.heads, args.rank = -3, 100, 1, 8, 1
    args.d_state, args.head_dim, args.num_angles, args.chunk_hint, args.device = 128, 64, 32, 256, -1
    assert lib.m3_scan_workspace_bytes(ctypes.byref(args)) == -1  # -M3_ERR_SHAPE
    assert b"positive" in lib.m3_last_error()
    args.device = 0
    rc = lib.m3_scan_fwd_noalloc(ctypes.byref(args), None)
    assert rc in (1, 5)  # M3_ERR_SHAPE, or M3_ERR_CUDA where no device can be selected


def test_gemv_rejects_bad_arguments_without_a_device():
    lib = _ext.load()
    assert lib.m3_gemv(None, None) == 4
    args = _ext.GemvArgs()
    args.out_dim, args.in_dim, args.rows, args.device = 16, 12, 1, -1
    assert lib.m3_gemv(ctypes.byref(args), None) == 1  # in_dim not a multiple of 8
    args.in_dim, args.rows = 16, 5
    assert lib.m3_gemv(ctypes.byref(args), None) == 1  # more than 4 rows
    args.rows = 1
    assert lib.m3_gemv(ctypes.byref(args), None) != 0  # tensors missing

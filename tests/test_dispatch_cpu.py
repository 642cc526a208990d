"""Host-side dispatch decisions of the decode projections and the training path, and the ctypes
mirrors of the argument structs added for them (no device needed)."""

from __future__ import annotations

import ctypes

import torch

from mamba3_b200 import _ext, ops


def test_gemv_is_never_chosen_off_the_gpu():
    x = torch.randn(1, 1, 2560, dtype=torch.bfloat16)
    w = torch.randn(10768, 2560, dtype=torch.bfloat16)
    assert not _ext.gemv_eligible(x, w)


def test_gemv_shape_and_dtype_limits(monkeypatch):
    # emulate device tensors: only is_cuda matters for the decision logic
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    w = torch.randn(64, 256, dtype=torch.bfloat16)
    ok = torch.randn(4, 1, 256, dtype=torch.bfloat16)
    assert _ext.gemv_eligible(ok, w)
    assert not _ext.gemv_eligible(torch.randn(5, 1, 256, dtype=torch.bfloat16), w)  # more than 4 rows
    assert not _ext.gemv_eligible(ok.float(), w.float())                             # fp32
    assert not _ext.gemv_eligible(ok, w.half())                                      # mixed dtypes
    w2 = torch.randn(64, 260, dtype=torch.bfloat16)
    assert not _ext.gemv_eligible(torch.randn(1, 260, dtype=torch.bfloat16), w2)     # 260 % 8 != 0
    wide = torch.randn(8, 8192, dtype=torch.bfloat16)
    assert _ext.gemv_eligible(torch.randn(1, 8192, dtype=torch.bfloat16), wide)
    big = torch.randn(8, 16392, dtype=torch.bfloat16)
    assert not _ext.gemv_eligible(torch.randn(1, 16392, dtype=torch.bfloat16), big)  # above 16384 columns


def test_training_kernel_eligibility(monkeypatch):
    q = torch.randn(1, 4, 1, 1, 128)
    v = torch.randn(1, 4, 2, 64)
    assert not ops._train_kernel_eligible(q, v)  # CPU tensors keep the PyTorch formulation
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    assert ops._train_kernel_eligible(q, v)
    assert not ops._train_kernel_eligible(torch.randn(1, 4, 1, 1, 256), v)  # d_state above 128
    assert not ops._train_kernel_eligible(q, torch.randn(1, 4, 2, 128))     # head_dim above 64
    phase4 = torch.randn(1, 4, 2, 32)
    assert ops._prelude_kernel_eligible(q, phase4, True)
    assert not ops._prelude_kernel_eligible(q, torch.randn(1, 4, 2, 30), True)  # MIMO angles % 4
    assert ops._prelude_kernel_eligible(q, torch.randn(1, 4, 2, 30), False)     # SISO: any count
    assert not ops._prelude_kernel_eligible(torch.randn(1, 4, 1, 1, 130), None, False)


def test_new_struct_layouts_match_the_header():
    # m3_gemv_args: two int64, two int32, three 64-byte tensor descriptors
    assert ctypes.sizeof(_ext.GemvArgs) == 2 * 8 + 2 * 4 + 3 * 64
    # m3_prelude_args: ten int32, fourteen descriptors
    assert ctypes.sizeof(_ext.PreludeArgs) == 10 * 4 + 14 * 64
    lib = _ext.load()
    assert lib.m3_ssd_prelude_fwd(None, None) == 4
    assert lib.m3_ssd_prelude_bwd(None, None) == 4
    args = _ext.PreludeArgs()
    args.batch, args.length, args.groups, args.heads, args.rank, args.d_state = 1, 4, 1, 2, 1, 130
    args.device = -1
    assert lib.m3_ssd_prelude_fwd(ctypes.byref(args), None) == 1  # d_state not a multiple of 4 / above 128

"""Host logic of the CUDA training path (``ops._scan_train``) on CPU: the prelude (group expansion,
bias, rotation, trapezoid scale, rank values, endpoint-cache term) and epilogue (D skip, SiLU
gate, rank sum) around the SSD core reproduce ``ops._scan_torch`` in value and gradient when the
core is evaluated by a plain token recurrence; and the C entry points of the training kernels
reject malformed arguments without a device."""

from __future__ import annotations

import ctypes

import pytest
import torch

from _train_cases import leaves, scan_case
from conftest import rel_err
from mamba3_b200 import _ext, ops


def core_recurrence(q, k, v, adt, diag, initial_state):
    """The SSD core token by token: S_t = e^{adt_t} S_{t-1} + sum_r v_{t,r} k_{t,r}^T,
    y_{t,r} = e^{adt_t} S_{t-1} q_{t,r} + diag_t sum_r' (q_{t,r} . k_{t,r'}) v_{t,r'}."""
    batch, length, heads, rank, n = q.shape
    p = v.shape[-1]
    state = torch.zeros(batch, heads, p, n, dtype=q.dtype) if initial_state is None else initial_state
    ys = []
    for t in range(length):
        decayed = torch.exp(adt[:, t])[..., None, None] * state
        inter = torch.einsum("bhpn,bhrn->bhrp", decayed, q[:, t])
        scores = torch.einsum("bhrn,bhsn->bhrs", q[:, t], k[:, t])
        intra = diag[:, t][..., None, None] * torch.einsum("bhrs,bhsp->bhrp", scores, v[:, t])
        ys.append(inter + intra)
        state = decayed + torch.einsum("bhrp,bhrn->bhpn", v[:, t], k[:, t])
    return torch.stack(ys, dim=1), state


class _RecurrenceCore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, *inputs):
        with torch.enable_grad():
            detached = [x.detach().requires_grad_(x.requires_grad) if x is not None else None for x in inputs]
            out = core_recurrence(*detached)
        ctx.detached, ctx.out = detached, out
        return out[0].detach(), out[1].detach()

    @staticmethod
    def backward(ctx, dy, dfinal):
        targets = [x for x in ctx.detached if x is not None and x.requires_grad]
        grads = torch.autograd.grad(ctx.out, targets, (dy, dfinal), allow_unused=True)
        it = iter(grads)
        return tuple(next(it) if (x is not None and x.requires_grad) else None for x in ctx.detached)


@pytest.mark.parametrize("rank", [1, 4])
@pytest.mark.parametrize("cache", [True, False])
def test_training_prelude_and_epilogue_match_the_pytorch_formulation(monkeypatch, rank, cache):
    args, kw = scan_case(rank, cache=cache, dtype=torch.float64)
    args = tuple(a.detach().double().requires_grad_(True) for a in args)
    kw = {key: (v.detach().double().requires_grad_(True) if isinstance(v, torch.Tensor) else v) for key, v in kw.items()}
    y0, s0 = ops._scan_torch(*args, **{key: kw.get(key) for key in (
        "mimo_x", "mimo_z", "mimo_out", "chunk_size", "initial_state", "initial_k", "initial_value", "phase",
        "mimo_rotation", "q_bias", "k_bias")})
    g = torch.Generator().manual_seed(5)
    wy, ws = torch.randn(y0.shape, generator=g, dtype=y0.dtype), torch.randn(s0.shape, generator=g, dtype=s0.dtype)
    ref = torch.autograd.grad((y0 * wy).sum() + (s0 * ws).sum(), leaves(args, kw))

    monkeypatch.setattr(ops._SSDCore, "apply", _RecurrenceCore.apply)
    full = dict(mimo_x=None, mimo_z=None, mimo_out=None, initial_state=None, initial_k=None, initial_value=None,
                phase=None, q_bias=None, k_bias=None)
    full.update(kw)
    y1, s1 = ops._scan_train(*args, **full)
    got = torch.autograd.grad((y1 * wy).sum() + (s1 * ws).sum(), leaves(args, kw))
    # _scan_torch computes in float32 whatever the input dtype: agreement to float32 rounding
    assert rel_err(y1.detach(), y0.detach()) < 1e-5 and rel_err(s1.detach(), s0.detach()) < 1e-5
    for a, b in zip(got, ref):
        assert rel_err(a, b) < 1e-4


def test_training_entry_points_reject_bad_arguments_without_a_device():
    lib = _ext.load()
    assert ctypes.sizeof(_ext.SSDArgs) == 8 * 4 + 18 * 64
    assert lib.m3_ssd_chunk_rows() == 32
    assert lib.m3_ssd_train_fwd(None, None) == 4
    assert lib.m3_ssd_train_bwd(None, None) == 4
    args = _ext.SSDArgs()
    assert lib.m3_ssd_train_fwd(ctypes.byref(args), None) == 1  # zero sizes
    args.batch, args.length, args.heads, args.rank, args.d_state, args.head_dim, args.device = 1, 8, 2, 3, 32, 16, -1
    assert lib.m3_ssd_train_fwd(ctypes.byref(args), None) == 1  # rank 3
    args.rank, args.d_state = 1, 256
    assert lib.m3_ssd_train_fwd(ctypes.byref(args), None) == 1  # d_state above 128
    assert b"d_state" in lib.m3_last_error()
    args.d_state = 32
    assert lib.m3_ssd_train_bwd(ctypes.byref(args), None) == 4  # tensors missing

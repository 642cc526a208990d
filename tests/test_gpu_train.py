"""Training kernels of the chunked SSD on the GPU (``m3_ssd_train_fwd`` / ``m3_ssd_train_bwd``):
``mamba3_scan`` under autograd on CUDA tensors runs them, and its outputs and every input gradient
match autograd through the plain PyTorch formulation (``ops._scan_torch``, float32 on the same
device), mirroring tests/test_scan.py:195-225 and 339-382 of jreoka/mamba3. Model level: one
training step of ``Mamba3`` on CUDA against the same model run on the PyTorch formulation."""

from __future__ import annotations

import pytest
import torch

from _train_cases import leaves, scan_case
from conftest import rel_err
from mamba3_b200 import Mamba3, ops

pytestmark = pytest.mark.gpu

_KW = ("mimo_x", "mimo_z", "mimo_out", "chunk_size", "initial_state", "initial_k", "initial_value", "phase",
       "mimo_rotation", "q_bias", "k_bias")


def _grads(fn, args, kw, targets, seed=11):
    y, s = fn(*args, **kw)
    g = torch.Generator(device=y.device).manual_seed(seed)
    wy = torch.randn(y.shape, generator=g, device=y.device).to(y.dtype)
    ws = torch.randn(s.shape, generator=g, device=y.device)
    loss = (y.float() * wy.float()).sum() + (s * ws).sum()
    return y.detach(), s.detach(), torch.autograd.grad(loss, targets)


@pytest.mark.parametrize("rank", [1, 2, 4, 8])
@pytest.mark.parametrize("cache", [True, False])
@pytest.mark.parametrize("length", [45, 200])
def test_training_kernels_match_autograd_fp32(rank, cache, length):
    args, kw = scan_case(rank, cache=cache, length=length, device="cuda", d_state=128, head_dim=64, angles=32 if rank > 1 else 16)
    y1, s1, g1 = _grads(ops.mamba3_scan, args, kw, leaves(args, kw))
    assert ops.LAST_SCAN_DISPATCH, "the training kernels did not run"
    full = {key: kw.get(key) for key in _KW}
    y0, s0, g0 = _grads(ops._scan_torch, args, full, leaves(args, kw))
    assert rel_err(y1, y0) < 1e-4
    assert rel_err(s1, s0) < 1e-4
    for i, (a, b) in enumerate(zip(g1, g0)):
        assert rel_err(a, b) < 1e-4, f"gradient {i} of {len(g0)}"


@pytest.mark.parametrize("rank", [1, 4])
def test_training_kernels_bf16_within_tolerance(rank):
    args, kw = scan_case(rank, length=130, device="cuda", d_state=128, head_dim=64, angles=32 if rank > 1 else 16,
                         dtype=torch.bfloat16, seed=3)
    y1, s1, g1 = _grads(ops.mamba3_scan, args, kw, leaves(args, kw))
    full = {key: kw.get(key) for key in _KW}
    y0, s0, g0 = _grads(ops._scan_torch, args, full, leaves(args, kw))
    assert rel_err(y1.float(), y0.float()) < 2e-2
    assert rel_err(s1, s0) < 1e-2
    for i, (a, b) in enumerate(zip(g1, g0)):
        assert rel_err(a.float(), b.float()) < 3e-2, f"gradient {i}"


def test_small_state_shapes_and_group_expansion():
    """d_state 16, head_dim 16, two Q/K groups over four heads, ragged length."""
    args, kw = scan_case(1, length=37, heads=4, groups=2, d_state=16, head_dim=16, angles=8, device="cuda", seed=9)
    y1, s1, g1 = _grads(ops.mamba3_scan, args, kw, leaves(args, kw))
    full = {key: kw.get(key) for key in _KW}
    y0, s0, g0 = _grads(ops._scan_torch, args, full, leaves(args, kw))
    assert rel_err(y1, y0) < 1e-4 and rel_err(s1, s0) < 1e-4
    for a, b in zip(g1, g0):
        assert rel_err(a, b) < 1e-4


@pytest.mark.parametrize("rank", [1, 4])
def test_model_training_step_matches_the_pytorch_formulation(monkeypatch, rank):
    torch.manual_seed(0)
    model = Mamba3(128, d_state=128, depth=2, mimo_rank=rank).cuda().train()
    x = torch.randn(2, 96, 128, device="cuda")
    target = torch.randn(2, 96, 128, device="cuda")

    def step():
        model.zero_grad(set_to_none=True)
        loss = torch.nn.functional.mse_loss(model(x), target)
        loss.backward()
        return loss.detach(), {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}

    loss1, grads1 = step()
    assert ops.LAST_SCAN_DISPATCH
    monkeypatch.setattr(ops, "_train_kernel_eligible", lambda q, value: False)
    loss0, grads0 = step()
    assert not ops.LAST_SCAN_DISPATCH
    assert abs(float(loss1) - float(loss0)) <= 1e-5 * abs(float(loss0))
    assert grads1.keys() == grads0.keys()
    for name in grads0:
        assert rel_err(grads1[name], grads0[name]) < 1e-4, name

"""Operator-level checks of ``mamba3_b200.ops`` on CPU (the PyTorch formulation), mirroring
tests/test_scan.py of jreoka/mamba3 and pinned to the reference's golden outputs."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from mamba3_b200.ops import heavy_tail_activation, mamba3_scan, mamba3_step, rotate_qk
from oracle import mamba3_oracle as O

SCANS = ["scan_small_r1", "scan_small_r4", "scan_small_r4_c5", "scan_cont_r1", "scan_kernel_r1",
         "scan_kernel_r4", "scan_kernel_r2", "scan_n16_r1"]


def scan_kwargs(f: dict, device="cpu", dtype=None) -> tuple[tuple, dict]:
    def t(key, low=False):
        if key not in f:
            return None
        x = torch.from_numpy(f[key]).to(device)
        return x.to(dtype) if (low and dtype is not None) else x
    args = (t("q", True), t("k", True), t("value", True), t("gate", True), t("adt"), t("dt"), t("trap", True),
            t("D"))
    kw = dict(mimo_x=t("mimo_x"), mimo_z=t("mimo_z"), mimo_out=t("mimo_out"), chunk_size=int(f["chunk"]),
              initial_state=t("initial_state"), initial_k=t("initial_k", True), initial_value=t("initial_value", True),
              phase=t("phase"), mimo_rotation=f["q"].shape[3] > 1,
              q_bias=t("q_bias"), k_bias=t("k_bias"))
    return args, kw


def test_heavy_tail_and_gradient():
    x = torch.tensor([-3.0, -0.5, 0.0, 0.5, 3.0], requires_grad=True)
    expected = torch.where(x >= 0, 1.0 + x, 1.0 / (1.0 - x))
    out = heavy_tail_activation(x)
    torch.testing.assert_close(out, expected)
    out.sum().backward()
    torch.testing.assert_close(x.grad, torch.where(x >= 0, torch.ones_like(x), expected.square()))


def test_rotation_golden_vectors():
    f = load_golden("rotation")
    siso, _ = rotate_qk(torch.from_numpy(f["siso_in"]), torch.from_numpy(f["siso_in"]),
                        torch.from_numpy(f["phase"]), mimo=False)
    mimo, _ = rotate_qk(torch.from_numpy(f["mimo_in"]), torch.from_numpy(f["mimo_in"]),
                        torch.from_numpy(f["phase"]), mimo=True)
    torch.testing.assert_close(siso, torch.from_numpy(f["siso"]), atol=1e-6, rtol=0)
    torch.testing.assert_close(mimo, torch.from_numpy(f["mimo"]), atol=1e-6, rtol=0)
    t, ph = torch.from_numpy(f["rand_in"]), torch.from_numpy(f["rand_phase"])
    torch.testing.assert_close(rotate_qk(t, t, ph, mimo=False)[0], torch.from_numpy(f["rand_siso"]), atol=1e-6, rtol=0)
    torch.testing.assert_close(rotate_qk(t, t, ph, mimo=True)[0], torch.from_numpy(f["rand_mimo"]), atol=1e-6, rtol=0)


@pytest.mark.parametrize("name", SCANS)
def test_scan_matches_reference_fixture(name):
    f = load_golden(name)
    args, kw = scan_kwargs(f)
    y, s = mamba3_scan(*args, **kw)
    assert rel_err(y, f["y"]) < 2e-5
    assert rel_err(s, f["state"]) < 2e-5


@pytest.mark.parametrize("chunk", [1, 3, 16, 512])
def test_scan_is_chunk_invariant(chunk):
    f = load_golden("scan_kernel_r4")
    args, kw = scan_kwargs(f)
    kw["chunk_size"] = chunk
    y, s = mamba3_scan(*args, **kw)
    assert rel_err(y, f["y"]) < 2e-5 and rel_err(s, f["state"]) < 2e-5


@pytest.mark.parametrize("rank", [1, 4])
def test_scan_gradients_match_oracle_finite_differences(rank):
    """Autograd through the PyTorch formulation equals the recurrence's gradient (float64)."""
    f = load_golden("scan_small_r4" if rank > 1 else "scan_small_r1")
    args, kw = scan_kwargs(f)
    args = tuple(a.double().requires_grad_(True) for a in args)
    kw = {k: (v.double().requires_grad_(True) if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
    y, s = mamba3_scan(*args, **kw)
    g = torch.Generator().manual_seed(0)
    wy = torch.randn(y.shape, generator=g, dtype=torch.float64)
    ws = torch.randn(s.shape, generator=g, dtype=torch.float64)
    ((y * wy).sum() + (s * ws).sum()).backward()
    # directional derivative check on q against the oracle recurrence
    dq = torch.randn(args[0].shape, generator=g, dtype=torch.float64)
    eps = 1e-6
    def loss(qv):
        heads = args[2].shape[2]
        qe = O.expand_heads(qv, heads)
        ke = O.expand_heads(args[1].detach().numpy(), heads)
        mx = kw["mimo_x"].detach().numpy() if kw["mimo_x"] is not None else None
        mz = kw["mimo_z"].detach().numpy() if kw["mimo_z"] is not None else None
        mo = kw["mimo_out"].detach().numpy() if kw["mimo_out"] is not None else None
        yy, ss = O.scan_recurrent(qe, ke, *(a.detach().numpy() for a in args[2:]), mimo_x=mx, mimo_z=mz, mimo_out=mo)
        return float((yy * wy.numpy()).sum() + (ss * ws.numpy()).sum())
    q0 = args[0].detach().numpy()
    fd = (loss(q0 + eps * dq.numpy()) - loss(q0 - eps * dq.numpy())) / (2 * eps)
    ad = float((args[0].grad * dq).sum())
    assert abs(fd - ad) <= 1e-6 * max(1.0, abs(fd))


@pytest.mark.parametrize("rank", [1, 4])
def test_scan_continuation(rank):
    f = load_golden("scan_small_r4" if rank > 1 else "scan_small_r1")
    args, kw = scan_kwargs(f)
    full, full_state = mamba3_scan(*args, **kw)
    split = 4
    first = tuple(a[:, :split] if i < 7 else a for i, a in enumerate(args))
    y1, s1 = mamba3_scan(*first, **kw)
    second = tuple(a[:, split:] if i < 7 else a for i, a in enumerate(args))
    heads = args[2].shape[2]
    kw2 = dict(kw, initial_state=s1, initial_k=args[1][:, split - 1].expand(-1, heads, -1, -1),
               initial_value=args[2][:, split - 1])
    y2, s2 = mamba3_scan(*second, **kw2)
    torch.testing.assert_close(torch.cat((y1, y2), 1), full, rtol=2e-5, atol=2e-6)
    torch.testing.assert_close(s2, full_state, rtol=2e-5, atol=2e-6)


def test_empty_scan_preserves_state():
    q = torch.empty(2, 0, 3, 1, 8)
    v = torch.empty(2, 0, 3, 4, requires_grad=True)
    state = torch.randn(2, 3, 4, 8)
    e = torch.empty(2, 0, 3)
    y, s = mamba3_scan(q, q, v, v, e, e, e, torch.ones(3), initial_state=state,
                       initial_k=torch.randn(2, 3, 1, 8), initial_value=torch.randn(2, 3, 4))
    assert y.shape == v.shape
    torch.testing.assert_close(s, state)
    y.sum().backward()
    assert v.grad is not None


def test_scan_validation_messages():
    q = torch.randn(1, 3, 1, 1, 8)
    v = torch.randn(1, 3, 2, 4)
    s = torch.randn(1, 3, 2)
    with pytest.raises(ValueError, match="matching"):
        mamba3_scan(q, q[:, :2], v, v, s, s, s, torch.ones(2))
    with pytest.raises(ValueError, match="D must"):
        mamba3_scan(q, q, v, v, s, s, s, torch.ones(3))
    with pytest.raises(ValueError, match="SISO"):
        mamba3_scan(q, q, v, v, s, s, s, torch.ones(2), mimo_x=torch.ones(2, 1, 4))
    with pytest.raises(ValueError, match="chunk_size"):
        mamba3_scan(q, q, v, v, s, s, s, torch.ones(2), chunk_size=0)


@pytest.mark.parametrize("rank", [1, 4])
def test_step_matches_reference_fixture(rank):
    f = load_golden(f"step_r{rank}")
    t = {key: torch.from_numpy(val) for key, val in f.items()}
    inc = torch.fmod(math.pi * torch.tanh(t["angle_rate"]).unsqueeze(1) * t["dt"].unsqueeze(-1), 2 * math.pi)
    phase = torch.fmod(t["phase0"] + inc, 2 * math.pi)
    q, k = rotate_qk(t["q"][:, None], t["k"][:, None], phase[:, None], mimo=rank > 1)
    y, (ph, s, k1, _) = mamba3_step(q[:, 0], k[:, 0], t["value"], t["gate"], t["adt"], t["dt"], t["trap"], t["D"],
                                    (phase, t["state0"], t["k0"], t["v0"]), mimo_x=t.get("mimo_x"),
                                    mimo_z=t.get("mimo_z"), mimo_out=t.get("mimo_out"))
    assert rel_err(y, f["y"]) < 2e-5 and rel_err(s, f["state1"]) < 2e-5
    assert rel_err(k1, f["k1"]) < 2e-5 and rel_err(ph, f["phase1"]) < 2e-5

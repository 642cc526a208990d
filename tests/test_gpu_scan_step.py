"""GPU parity of the sm_100a scan and step kernels against the oracle / reference fixtures.

Tolerances (normwise: max|a-e| / max|e|):
  float32 activations: outputs and states <= 1e-4 (north-star fp32 bound)
  bf16 / fp16 activations: outputs <= 2e-2, FP32 states <= 1e-2 (bf16) / 5e-3 (fp16), against
  the float64 oracle run on the same low-precision-rounded inputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import load_golden, rel_err
from mamba3_b200 import _ext, ops
from oracle import mamba3_oracle as O
from test_ops_cpu import SCANS, scan_kwargs
from test_oracle_golden import oracle_scan_inputs

pytestmark = pytest.mark.gpu

LOW = [torch.bfloat16, torch.float16]
STATE_TOL = {torch.bfloat16: 1e-2, torch.float16: 5e-3, torch.float32: 1e-4}


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert _ext.device_error(clear=True) == 0


@pytest.mark.parametrize("name", SCANS)
def test_scan_fp32_matches_reference(name):
    f = load_golden(name)
    args, kw = scan_kwargs(f, device="cuda")
    with torch.inference_mode():
        y, s = ops.mamba3_scan(*args, **kw)
    assert ops.LAST_SCAN_DISPATCH
    assert rel_err(y, f["y"]) < 1e-4
    assert rel_err(s, f["state"]) < 1e-4


def _rounded(f: dict, dtype) -> dict:
    """Round the activation-dtype inputs to `dtype` (what the GPU sees) for the oracle."""
    g = dict(f)
    for key in ("q", "k", "value", "gate", "trap", "initial_k", "initial_value"):
        if key in g:
            g[key] = torch.from_numpy(g[key]).to(dtype).float().numpy()
    return g


@pytest.mark.parametrize("name", SCANS)
@pytest.mark.parametrize("dtype", LOW)
def test_scan_low_precision_matches_oracle(name, dtype):
    f = _rounded(load_golden(name), dtype)
    args, kw = scan_kwargs(f, device="cuda", dtype=dtype)
    with torch.inference_mode():
        y, s = ops.mamba3_scan(*args, **kw)
    assert ops.LAST_SCAN_DISPATCH and y.dtype == dtype and s.dtype == torch.float32
    q, k, okw = oracle_scan_inputs(f)
    ye, se = O.scan_recurrent(q, k, f["value"], f["gate"], f["adt"], f["dt"], f["trap"], f["D"], **okw)
    assert rel_err(y.float(), ye) < 2e-2
    assert rel_err(s, se) < STATE_TOL[dtype]


def _random_scan(batch, length, heads, rank, n, p, s_angles, seed, device="cuda", cache=True, groups=1):
    g = torch.Generator().manual_seed(seed)
    t = lambda *shape: torch.randn(*shape, generator=g)
    out = dict(q=t(batch, length, groups, rank, n), k=t(batch, length, groups, rank, n),
               value=t(batch, length, heads, p), gate=t(batch, length, heads, p),
               adt=-torch.rand(batch, length, heads, generator=g) * 0.2,
               dt=torch.rand(batch, length, heads, generator=g) * 0.1 + 0.001,
               trap=t(batch, length, heads), D=t(heads))
    kw = dict(mimo_x=None, mimo_z=None, mimo_out=None, chunk_size=64, initial_state=None, initial_k=None,
              initial_value=None, phase=None, mimo_rotation=rank > 1, q_bias=None, k_bias=None)
    if rank > 1:
        kw.update(mimo_x=t(heads, rank, p) / rank, mimo_z=t(heads, rank, p), mimo_out=t(heads, rank, p) / rank)
    if s_angles:
        kw.update(phase=(torch.rand(batch, length, heads, s_angles, generator=g) * 4 - 2) * np.pi,
                  q_bias=1 + 0.1 * t(heads, rank, n), k_bias=1 + 0.1 * t(heads, rank, n))
    if cache:
        kw.update(initial_state=0.1 * t(batch, heads, p, n), initial_k=t(batch, heads, rank, n),
                  initial_value=t(batch, heads, p))
    args = tuple(out[key].to(device) for key in ("q", "k", "value", "gate", "adt", "dt", "trap", "D"))
    kw = {key: (val.to(device) if isinstance(val, torch.Tensor) else val) for key, val in kw.items()}
    return args, kw


@pytest.mark.parametrize("rank,length", [(1, 1), (1, 129), (1, 1000), (2, 77), (4, 33), (4, 513), (8, 40)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_scan_ragged_lengths_against_oracle(rank, length, dtype):
    args, kw = _random_scan(2, length, 2, rank, 128, 64, 32, seed=length * 10 + rank)
    low = tuple(a.to(dtype) if i in (0, 1, 2, 3, 6) else a for i, a in enumerate(args))
    kwl = dict(kw, initial_k=kw["initial_k"].to(dtype), initial_value=kw["initial_value"].to(dtype))
    with torch.inference_mode():
        y, s = ops.mamba3_scan(*low, **kwl)
    to_np = lambda x: x.float().cpu().numpy() if isinstance(x, torch.Tensor) else x
    f = {key: to_np(val) for key, val in zip(("q", "k", "value", "gate", "adt", "dt", "trap", "D"), low)}
    f.update({key: to_np(val) for key, val in kwl.items() if isinstance(val, torch.Tensor)})
    q, k, okw = oracle_scan_inputs(f)
    ye, se = O.scan_chunked(q, k, f["value"], f["gate"], f["adt"], f["dt"], f["trap"], f["D"], chunk_size=64, **okw)
    tol_y, tol_s = (1e-4 if dtype == torch.float32 else 2e-2), STATE_TOL[dtype]
    assert rel_err(y.float(), ye) < tol_y
    assert rel_err(s, se) < tol_s


@pytest.mark.parametrize("rank", [1, 4])
def test_scan_continuation_at_length_4096(rank):
    """Size-independent property at a long length: scanning [0, L) equals scanning [0, m) and then
    [m, L) from the returned state plus the endpoint cache (bf16, kernel on both sides)."""
    args, kw = _random_scan(1, 4096, 4, rank, 128, 64, 32, seed=7 + rank, cache=False)
    args = tuple(a.bfloat16() if i in (0, 1, 2, 3, 6) else a for i, a in enumerate(args))
    with torch.inference_mode():
        full, full_s = ops.mamba3_scan(*args, **kw)
        m = 1500
        part = lambda a, sl: a[:, sl]
        first = tuple(part(a, slice(0, m)) if i < 7 else a for i, a in enumerate(args))
        k1 = dict(kw, phase=kw["phase"][:, :m])
        y1, s1 = ops.mamba3_scan(*first, **k1)
        # endpoint cache: biased + rotated k and raw value of token m-1 (what prefill stores)
        qx, kx = ops.rotate_qk(args[0][:, m - 1:m].expand(-1, -1, 4, -1, -1) + kw["q_bias"].bfloat16(),
                               args[1][:, m - 1:m].expand(-1, -1, 4, -1, -1) + kw["k_bias"].bfloat16(),
                               kw["phase"][:, m - 1:m], mimo=rank > 1)
        second = tuple(part(a, slice(m, None)) if i < 7 else a for i, a in enumerate(args))
        k2 = dict(kw, phase=kw["phase"][:, m:], initial_state=s1, initial_k=kx[:, 0], initial_value=args[2][:, m - 1])
        y2, s2 = ops.mamba3_scan(*second, **k2)
    assert rel_err(torch.cat((y1, y2), 1).float(), full.float()) < 2e-2
    assert rel_err(s2, full_s) < STATE_TOL[torch.bfloat16]


@pytest.mark.parametrize("rank", [1, 4])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_step_matches_reference_fixture(rank, dtype):
    f = load_golden(f"step_r{rank}")
    t = {key: torch.from_numpy(val).cuda() for key, val in f.items()}
    act = lambda x: x.to(dtype)
    cache = (t["phase0"], t["state0"], act(t["k0"]), act(t["v0"]))
    with torch.inference_mode():
        out = ops.fused_step(act(t["q"]), act(t["k"]), act(t["value"]), act(t["gate"]), t["adt"], t["dt"],
                             act(t["trap"]), act(t["angle_rate"]), t["D"], cache, mimo_x=t.get("mimo_x"),
                             mimo_z=t.get("mimo_z"), mimo_out=t.get("mimo_out"))
    assert out is not None and ops.LAST_STEP_DISPATCH
    y, (ph, s, k1, v1) = out
    if dtype == torch.float32:
        torch.testing.assert_close(y, t["y"], rtol=2e-4, atol=2e-5)
        torch.testing.assert_close(s, t["state1"], rtol=2e-4, atol=2e-5)
        torch.testing.assert_close(k1, t["k1"], rtol=2e-4, atol=2e-5)
        torch.testing.assert_close(ph, t["phase1"], rtol=2e-4, atol=2e-5)
        return
    # low precision: oracle on the rounded inputs
    g = {key: (val.to(dtype).float().cpu().numpy() if key in ("q", "k", "value", "gate", "trap", "angle_rate",
                                                              "k0", "v0") else val.cpu().numpy())
         for key, val in t.items()}
    ye, (phe, se, ke, _) = O.fused_step(g["q"], g["k"], g["value"], g["gate"], g["adt"], g["dt"], g["trap"],
                                        g["angle_rate"], g["D"], (g["phase0"], g["state0"], g["k0"], g["v0"]),
                                        mimo_x=g.get("mimo_x"), mimo_z=g.get("mimo_z"), mimo_out=g.get("mimo_out"))
    assert rel_err(y.float(), ye) < 2e-2
    assert rel_err(s, se) < STATE_TOL[dtype]
    assert rel_err(k1.float(), ke) < 2e-2
    assert rel_err(ph, phe) < 1e-5


def test_step_writes_state_in_place_only_when_asked():
    f = load_golden("step_r1")
    t = {key: torch.from_numpy(val).cuda() for key, val in f.items()}
    state = t["state0"].clone()
    cache = (t["phase0"], state, t["k0"], t["v0"])
    with torch.inference_mode():
        y, nxt = ops._step_device(t["q"], t["k"], t["value"], t["gate"], t["adt"], t["dt"], t["trap"],
                                  t["angle_rate"], t["D"], cache, mimo_x=None, mimo_z=None, mimo_out=None)
        torch.testing.assert_close(state, t["state0"], rtol=0, atol=0)  # input cache untouched
        y2, nxt2 = ops._step_device(t["q"], t["k"], t["value"], t["gate"], t["adt"], t["dt"], t["trap"],
                                    t["angle_rate"], t["D"], cache, mimo_x=None, mimo_z=None, mimo_out=None,
                                    out_state=state)
    assert nxt2[1].data_ptr() == state.data_ptr()
    torch.testing.assert_close(state, nxt[1], rtol=0, atol=0)
    torch.testing.assert_close(y2, y, rtol=0, atol=0)


@pytest.mark.parametrize("batch,heads", [(1, 80), (64, 80), (3, 5)])
def test_step_large_batches_against_oracle(batch, heads):
    g = torch.Generator().manual_seed(batch * 100 + heads)
    n, p, s = 128, 64, 32
    t = lambda *shape: torch.randn(*shape, generator=g)
    q, k = t(batch, heads, 1, n), t(batch, heads, 1, n)
    v, z = t(batch, heads, p), t(batch, heads, p)
    adt, dt = -torch.rand(batch, heads, generator=g) * 0.3, torch.rand(batch, heads, generator=g) * 0.1
    tr, ang, D = t(batch, heads), t(batch, s), t(heads)
    cache = (torch.rand(batch, heads, s, generator=g) * 6 - 3, 0.1 * t(batch, heads, p, n), t(batch, heads, 1, n),
             t(batch, heads, p))
    cu = lambda x: x.cuda()
    with torch.inference_mode():
        y, (ph, st, kr, _) = ops.fused_step(cu(q), cu(k), cu(v), cu(z), cu(adt), cu(dt), cu(tr), cu(ang), cu(D),
                                            tuple(map(cu, cache)))
    npy = lambda x: x.numpy()
    ye, (phe, se, ke, _) = O.fused_step(npy(q), npy(k), npy(v), npy(z), npy(adt), npy(dt), npy(tr), npy(ang),
                                        npy(D), tuple(map(npy, cache)))
    assert rel_err(y, ye) < 1e-4 and rel_err(st, se) < 1e-4 and rel_err(kr, ke) < 1e-4


@pytest.mark.parametrize("rank", [1, 4])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("two_pass", [True, False])
def test_step_model_mode_matches_preprocessed_inputs(rank, dtype, two_pass):
    """Raw projection rows + norm weights + dt_bias in the kernel == the same math done first in torch."""
    g = torch.Generator().manual_seed(7 + rank)
    # 64 x 6 = 384 (batch, head) pairs reach the two-pass kernels (>= 2 per SM); 5 x 6 the single pass
    batch, heads, n, p, s = (64 if two_pass else 5), 6, 128, 64, 32
    t = lambda *shape: torch.randn(*shape, generator=g).cuda()
    C, B = t(batch, 1, rank, n).to(dtype) * 3, t(batch, 1, rank, n).to(dtype)
    wq, wk = 1 + 0.1 * t(n), 1 + 0.1 * t(n)
    qb, kb = 1 + 0.1 * t(heads, rank, n), 1 + 0.1 * t(heads, rank, n)
    v, z = t(batch, heads, p).to(dtype), t(batch, heads, p).to(dtype)
    delta, decay, bias = t(batch, heads).to(dtype), t(batch, heads).to(dtype), 0.5 * t(heads)
    tr, ang, D = t(batch, heads).to(dtype), t(batch, s).to(dtype), t(heads)
    mimo = {}
    if rank > 1:
        mimo = dict(mimo_x=t(heads, rank, p) / rank, mimo_z=t(heads, rank, p), mimo_out=t(heads, rank, p) / rank)
    else:
        mimo = dict(mimo_x=None, mimo_z=None, mimo_out=None)
    state = 0.1 * t(batch, heads, p, n)
    if not two_pass:  # a state with a non-unit inner stride runs the single-pass kernel
        state = state.transpose(2, 3).contiguous().transpose(2, 3)
    cache = (t(batch, heads, s) * 2, state, t(batch, heads, rank, n).to(dtype), t(batch, heads, p).to(dtype))
    eps = 1e-5
    with torch.inference_mode():
        qn = F.rms_norm(C, (n,), wq.to(dtype), eps).to(dtype)
        kn = F.rms_norm(B, (n,), wk.to(dtype), eps).to(dtype)
        dt = F.softplus(delta.float() + bias)
        adt = (-ops.heavy_tail_activation(decay.float())).clamp(max=-1e-4) * dt
        ex = lambda x: x.expand(-1, heads, -1, -1)
        y0, c0 = ops._step_device(ex(qn), ex(kn), v, z, adt, dt, tr, ang, D, cache, q_bias=qb, k_bias=kb, **mimo)
        y1, c1 = ops._step_device(ex(C), ex(B), v, z, decay, delta, tr, ang, D, cache, q_bias=qb, k_bias=kb,
                                  q_norm_w=wq, k_norm_w=wk, dt_bias=bias, norm_eps=eps, **mimo)
    if two_pass:
        assert _ext.last_step_kernel() == ("two_pass_mma" if rank > 1 and dtype != torch.float32 else "two_pass")
    else:
        assert _ext.last_step_kernel() == "single"
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel_err(y1.float(), y0.float()) < tol
    assert rel_err(c1[1], c0[1]) < tol
    assert rel_err(c1[2].float(), c0[2].float()) < tol
    torch.testing.assert_close(c1[0], c0[0], rtol=1e-5, atol=1e-5)

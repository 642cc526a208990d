"""GPU parity of every kernel variant the benchmark times, on the benchmark's own shapes.

Each test names the kernel variant it reaches (``m3_last_scan_kernel`` / ``m3_last_step_kernel``)
and compares it with the float64 oracle (``oracle/mamba3_oracle.py``) fed the same low-precision
inputs the GPU saw. Tolerances (normwise: max|a-e| / max|e|), the north-star bounds:

  float32:           outputs and states <= 1e-4
  bf16 / fp16:       outputs <= 2e-2; FP32 states compared separately, <= 1e-2 (bf16) / 5e-3 (fp16)
  phase (float32):   <= 1e-5 against the oracle; circular error <= 2e-3 at L = 131,072
                     (the reference's own long-context bound, tests/test_model.py:252-273)

Cases (reference tests they mirror: tests/test_scan.py:285-312, 385-435; tests/test_model.py:382-476):
  * model-mode tensor-core scan (raw in_proj columns, in-kernel norm / softplus / phase) at the
    SISO (d_model 1024), MIMO-4 (2048) and bidirectional (768, both directions) shapes, depth 1;
  * the non-factorised decay branch (tiles whose cumulative decay spans more than 16-bit operand
    factors can carry) in bf16 and fp16, alone and mixed with factorised tiles;
  * the in-kernel blocked phase carried across 2,048 blocks (L = 131,072), rank 1 and rank 4;
  * the two-pass decode kernels at B*H >= 296 in bf16 / fp16, rank 1 and rank 4 (rank 4 takes the
    16-byte-row prep and the reduce-scatter stream pass), in model mode as the decoder runs them;
  * the CPU-reference configuration in full: fp32 Mamba3(256, depth=4), [2, 1024, 256], forward -> prefill ->
    64 steps.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err
from mamba3_b200 import Mamba3, _ext, ops
from oracle import mamba3_oracle as O

pytestmark = pytest.mark.gpu

STATE_TOL = {torch.bfloat16: 1e-2, torch.float16: 5e-3, torch.float32: 1e-4}


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert _ext.device_error(clear=True) == 0


def _cfg(model: Mamba3) -> O.ModelConfig:
    return O.ModelConfig(model.d_model, model.d_state, model.depth, model.mimo_rank, model.causal)


def _layer0(model: Mamba3) -> dict:
    sd = {key: val.detach().float().cpu().numpy() for key, val in model.state_dict().items()}
    return O._layer_params(sd, 0)


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().double().cpu().numpy()


# ---------------------------------------------------------------------------------------------
# Model-mode tensor-core scan on the benchmark shapes
# ---------------------------------------------------------------------------------------------

@pytest.mark.parametrize("d_model,rank,causal", [(1024, 1, True), (2048, 4, True), (768, 1, False)],
                         ids=["siso-1024", "mimo4-2048", "bidir-768"])
def test_model_mode_tensor_core_scan_on_benchmark_shapes(d_model, rank, causal):
    torch.manual_seed(0)
    model = Mamba3(d_model, d_state=128, depth=1, mimo_rank=rank, causal=causal).cuda().eval()
    mixer = model.layers[0].mixer
    cfg, lp = _cfg(model), _layer0(model)
    x = torch.randn(1, 1024, d_model, device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        hidden = model.layers[0].norm(x)
        projected = mixer._project_linear("in_proj", hidden)
        assert projected.dtype == torch.bfloat16
        directions = (False, True) if not causal else (False,)
        for reverse in directions:
            y, state, phase, k_last, _ = mixer._scan_fused(projected, None, reverse=reverse, want_cache=not reverse)
            assert _ext.last_scan_kernel() == "umma"
            torch.cuda.synchronize()
            proj = _np(projected)
            if reverse:
                proj = np.ascontiguousarray(proj[:, ::-1])
            ye, se, phe, ke, _ = O.scan_projection(cfg, lp, proj)
            if reverse:
                ye = np.ascontiguousarray(ye[:, ::-1])
            assert rel_err(y.float(), ye) < 2e-2, reverse
            assert rel_err(state, se) < STATE_TOL[torch.bfloat16], reverse
            if not reverse:
                assert rel_err(phase, phe[:, -1]) < 1e-5
                assert rel_err(k_last.float(), ke[:, -1]) < 2e-2


def _scan_inputs(batch, length, heads, rank, adt, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    t = lambda *shape: torch.randn(*shape, generator=g)
    n, p, s = 128, 64, 32
    f = dict(q=t(batch, length, 1, rank, n), k=t(batch, length, 1, rank, n), value=t(batch, length, heads, p),
             gate=t(batch, length, heads, p), adt=adt, dt=torch.rand(batch, length, heads, generator=g) * 0.1 + 0.001,
             trap=t(batch, length, heads), D=t(heads),
             phase=(torch.rand(batch, length, heads, s, generator=g) * 4 - 2) * math.pi,
             q_bias=1 + 0.1 * t(heads, rank, n), k_bias=1 + 0.1 * t(heads, rank, n),
             initial_state=0.1 * t(batch, heads, p, n), initial_k=t(batch, heads, rank, n),
             initial_value=t(batch, heads, p))
    if rank > 1:
        f.update(mimo_x=t(heads, rank, p) / rank, mimo_z=t(heads, rank, p), mimo_out=t(heads, rank, p) / rank)
    for key in ("q", "k", "value", "gate", "trap", "initial_k", "initial_value"):
        f[key] = f[key].to(dtype)
    return f


def _run_scan_vs_oracle(f, dtype, rank):
    dev = {key: val.cuda() for key, val in f.items()}
    with torch.inference_mode():
        y, s = ops.mamba3_scan(dev["q"], dev["k"], dev["value"], dev["gate"], dev["adt"], dev["dt"], dev["trap"],
                               dev["D"], mimo_x=dev.get("mimo_x"), mimo_z=dev.get("mimo_z"),
                               mimo_out=dev.get("mimo_out"), chunk_size=64, initial_state=dev["initial_state"],
                               initial_k=dev["initial_k"], initial_value=dev["initial_value"], phase=dev["phase"],
                               mimo_rotation=rank > 1, q_bias=dev["q_bias"], k_bias=dev["k_bias"])
    assert ops.LAST_SCAN_DISPATCH and _ext.last_scan_kernel() == "umma"
    g = {key: _np(val) for key, val in f.items()}
    heads = g["value"].shape[2]
    mimo = rank > 1
    q = O.rotate(O.expand_heads(g["q"], heads) + g["q_bias"], g["phase"], mimo)
    k = O.rotate(O.expand_heads(g["k"], heads) + g["k_bias"], g["phase"], mimo)
    ye, se = O.scan_recurrent(q, k, g["value"], g["gate"], g["adt"], g["dt"], g["trap"], g["D"],
                              mimo_x=g.get("mimo_x"), mimo_z=g.get("mimo_z"), mimo_out=g.get("mimo_out"),
                              initial_state=g["initial_state"], initial_k=g["initial_k"],
                              initial_value=g["initial_value"])
    assert rel_err(y.float(), ye) < 2e-2
    assert rel_err(s, se) < STATE_TOL[dtype]


@pytest.mark.parametrize("rank,dtype,top", [(1, torch.bfloat16, 8.0), (4, torch.bfloat16, 30.0),
                                            (1, torch.float16, 1.0), (4, torch.float16, 4.0)])
def test_non_factorised_decay_tiles(rank, dtype, top):
    """adt ~ -U(0, top): the cumulative decay across a 64-row tile (64 tokens at rank 1, 16 at rank
    4) spans more than +-80 (bf16) / +-8 (fp16) around its middle, so every full tile takes the
    per-element exp2 branch with the explicitly decayed V2 operand."""
    batch, length, heads = 2, 300, 3
    g = torch.Generator().manual_seed(40 + rank)
    adt = -torch.rand(batch, length, heads, generator=g) * top
    f = _scan_inputs(batch, length, heads, rank, adt, seed=41 + rank, dtype=dtype)
    _run_scan_vs_oracle(f, dtype, rank)


@pytest.mark.parametrize("rank", [1, 4])
def test_factorised_and_non_factorised_tiles_mixed(rank):
    """Strong decay on some stretches and weak decay on others: both branches in one sequence, the
    state handed from one kind of tile to the other."""
    batch, length, heads = 2, 700, 2
    g = torch.Generator().manual_seed(50 + rank)
    adt = -torch.rand(batch, length, heads, generator=g) * 0.05
    adt[:, 100:260] = -torch.rand(batch, 160, heads, generator=g) * 30.0
    adt[:, 500:540] = -torch.rand(batch, 40, heads, generator=g) * 40.0
    f = _scan_inputs(batch, length, heads, rank, adt, seed=51 + rank, dtype=torch.bfloat16)
    _run_scan_vs_oracle(f, torch.bfloat16, rank)


# ---------------------------------------------------------------------------------------------
# In-kernel phase at long context
# ---------------------------------------------------------------------------------------------

@pytest.mark.parametrize("rank", [1, 4])
@pytest.mark.parametrize("target", [-1e-4, 2.5], ids=["tiny-negative", "wrapping"])
def test_in_kernel_phase_at_length_131072(rank, target):
    """The tensor-core kernel's blocked phase (64-token blocks, fmod carry, model.py:215-256) over
    131,072 tokens, read back through the prefill cache's last phase. Every token gets the same
    increment per head, so the exact phase is L * inc mod 2 pi."""
    torch.manual_seed(2)
    model = Mamba3(256, d_state=128, depth=1, mimo_rank=rank).cuda().to(torch.bfloat16).eval()
    mixer = model.layers[0].mixer
    length, heads, angles = 131_072, mixer.nheads, mixer.num_angles
    width = mixer.in_proj.out_features
    proj = torch.randn(1, length, width, device="cuda", dtype=torch.bfloat16) * 0.5
    di, bc = mixer.d_inner, mixer.d_state * mixer.mimo_rank
    o_delta = 2 * di + 2 * bc
    o_ang = o_delta + 3 * heads
    # dt = softplus(delta + dt_bias) = 1 for every head
    delta = (math.log(math.e - 1.0) - mixer.dt_bias.float()).to(torch.bfloat16)
    proj[..., o_delta:o_delta + heads] = delta
    raw = torch.tensor(math.atanh(target / math.pi), dtype=torch.bfloat16)
    proj[..., o_ang:o_ang + angles] = raw
    with torch.inference_mode():
        _, _, phase, _, _ = mixer._scan_fused(proj, None, reverse=False, want_cache=True)
    assert _ext.last_scan_kernel() == "umma"
    dt = F.softplus(delta.double().cpu() + mixer.dt_bias.double().cpu())  # [H]
    inc = torch.fmod(math.pi * math.tanh(float(raw)) * dt, 2 * math.pi)  # [H]
    expected = torch.remainder(length * inc, 2 * math.pi)[None, :, None].expand(1, heads, angles)
    circ = torch.remainder(phase.double().cpu() - expected + math.pi, 2 * math.pi) - math.pi
    # Each token's increment is rounded to float32 (tanhf, the product with dt, the fmod), so an
    # exact carry still drifts by up to ~2 ulp of |inc| per token; a broken carry or a missed block
    # reduction would be off by O(1) radians.
    bound = 2e-3 + length * float(inc.detach().abs().max()) * 2.0 ** -22
    assert circ.abs().max() < bound


# ---------------------------------------------------------------------------------------------
# Two-pass decode kernels (B * H >= 296), model mode as the decoder runs them
# ---------------------------------------------------------------------------------------------

@pytest.mark.parametrize("rank", [1, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_two_pass_decode_kernels_against_oracle(rank, dtype):
    g = torch.Generator().manual_seed(60 + rank)
    batch, heads, n, p, s = 64, 80, 128, 64, 32
    t = lambda *shape: torch.randn(*shape, generator=g)
    C, B = (t(batch, 1, rank, n) * 3).to(dtype), t(batch, 1, rank, n).to(dtype)
    wq, wk = 1 + 0.1 * t(n), 1 + 0.1 * t(n)
    qb, kb = 1 + 0.1 * t(heads, rank, n), 1 + 0.1 * t(heads, rank, n)
    v, z = t(batch, heads, p).to(dtype), t(batch, heads, p).to(dtype)
    delta, decay, bias = t(batch, heads).to(dtype), t(batch, heads).to(dtype), 0.5 * t(heads)
    tr, ang, D = t(batch, heads).to(dtype), t(batch, s).to(dtype), t(heads)
    mimo = dict(mimo_x=None, mimo_z=None, mimo_out=None)
    if rank > 1:
        mimo = dict(mimo_x=t(heads, rank, p) / rank, mimo_z=t(heads, rank, p), mimo_out=t(heads, rank, p) / rank)
    cache = (t(batch, heads, s) * 2, 0.1 * t(batch, heads, p, n), t(batch, heads, rank, n).to(dtype),
             t(batch, heads, p).to(dtype))
    cu = lambda x: None if x is None else x.cuda()
    ex = lambda x: cu(x).expand(-1, heads, -1, -1)
    with torch.inference_mode():
        y, (ph, st, kr, _) = ops._step_device(
            ex(C), ex(B), cu(v), cu(z), cu(decay), cu(delta), cu(tr), cu(ang), cu(D), tuple(map(cu, cache)),
            q_bias=cu(qb), k_bias=cu(kb), q_norm_w=cu(wq), k_norm_w=cu(wk), dt_bias=cu(bias), norm_eps=1e-5,
            **{key: cu(val) for key, val in mimo.items()})
    assert _ext.last_step_kernel() == ("two_pass_mma" if rank > 1 else "two_pass")
    d = lambda x: None if x is None else x.double().numpy()
    qn = O.rms_norm(d(C)[:, 0], d(wq))  # [B, R, N]
    kn = O.rms_norm(d(B)[:, 0], d(wk))
    dtv = O.softplus(d(delta) + d(bias))
    adt = np.minimum(-O.heavy_tail(d(decay)), -1e-4) * dtv
    qh = qn[:, None] + d(qb)[None]
    kh = kn[:, None] + d(kb)[None]
    ye, (phe, se, ke, _) = O.fused_step(qh, kh, d(v), d(z), adt, dtv, d(tr), d(ang), d(D),
                                        tuple(map(d, cache)), **{key: d(val) for key, val in mimo.items()})
    assert rel_err(y.float(), ye) < 2e-2
    assert rel_err(st, se) < STATE_TOL[dtype]
    assert rel_err(kr.float(), ke) < 2e-2
    assert rel_err(ph, phe) < 1e-5


@pytest.mark.parametrize("rank", [1, 4])
@pytest.mark.parametrize("batch", [1, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_small_batch_graph_decoder_against_oracle(rank, batch, dtype):
    """The small-batch decode path under the CUDA-graph decoder: projections on the few-row GEMV,
    block boundaries on the fused residual + RMSNorm kernel, the chain of dependent launches, the
    single-pass step kernel; against the oracle on the same 16-bit parameters and inputs."""
    torch.manual_seed(1)
    model = Mamba3(512, d_state=128, depth=2, mimo_rank=rank).cuda().to(dtype).eval()
    cfg = _cfg(model)
    sd = {key: val.detach().float().cpu().numpy() for key, val in model.state_dict().items()}
    prefix, steps = 24, 4
    x = torch.randn(batch, prefix + steps, 512, device="cuda", dtype=dtype)
    decoder = model.cuda_graph(batch_size=batch)
    with torch.inference_mode():
        _, cache = model.prefill(x[:, :prefix])
        for mine, theirs in zip(decoder.cache, cache):
            for dst, src in zip(mine, theirs):
                dst.copy_(src)
        outs = [decoder(x[:, t:t + 1]).clone() for t in range(prefix, prefix + steps)]
    torch.cuda.synchronize()
    assert _ext.last_step_kernel() == "single"
    xn = _np(x)
    _, caches = O.model_prefill(cfg, sd, xn[:, :prefix])
    expected = []
    for t in range(prefix, prefix + steps):
        o, caches = O.model_step(cfg, sd, xn[:, t:t + 1], caches)
        expected.append(o)
    assert rel_err(torch.cat(outs, 1).float(), np.concatenate(expected, 1)) < 2e-2
    for layer in range(2):
        assert rel_err(decoder.cache[layer][1], caches[layer][1]) < STATE_TOL[dtype]


@pytest.mark.parametrize("rank", [1, 4])
def test_bf16_graph_decoder_at_batch_64_against_oracle(rank):
    """The decode benchmark's path: Mamba3(2560) bf16 parameters, CUDA-graph decoder at batch 64
    (two-pass kernels, state updated in place), after a kernel prefill; against the oracle run on
    the same bf16 parameters and inputs."""
    torch.manual_seed(0)
    model = Mamba3(2560, d_state=128, depth=1, mimo_rank=rank).cuda().to(torch.bfloat16).eval()
    cfg = _cfg(model)
    sd = {key: val.detach().float().cpu().numpy() for key, val in model.state_dict().items()}
    batch, prefix, steps = 64, 40, 3
    x = torch.randn(batch, prefix + steps, 2560, device="cuda", dtype=torch.bfloat16)
    decoder = model.cuda_graph(batch_size=batch)
    with torch.inference_mode():
        _, cache = model.prefill(x[:, :prefix])
        for dst, src in zip(decoder.cache[0], cache[0]):
            dst.copy_(src)
        outs = [decoder(x[:, t:t + 1]).clone() for t in range(prefix, prefix + steps)]
    torch.cuda.synchronize()
    assert _ext.last_step_kernel() == ("two_pass_mma" if rank > 1 else "two_pass")
    xn = _np(x)
    _, caches = O.model_prefill(cfg, sd, xn[:, :prefix])
    expected = []
    for t in range(prefix, prefix + steps):
        o, caches = O.model_step(cfg, sd, xn[:, t:t + 1], caches)
        expected.append(o)
    assert rel_err(torch.cat(outs, 1).float(), np.concatenate(expected, 1)) < 2e-2
    assert rel_err(decoder.cache[0][1], caches[0][1]) < STATE_TOL[torch.bfloat16]
    # the phase follows the bf16-rounded angle columns of the in_proj output, which the oracle
    # computes unrounded; the op-level test above pins the phase arithmetic itself at 1e-5
    assert rel_err(decoder.cache[0][0], caches[0][0]) < 2e-2


# ---------------------------------------------------------------------------------------------
# The CPU-reference configuration in full
# ---------------------------------------------------------------------------------------------

def test_config1_forward_prefill_and_64_steps_fp32():
    """Mamba3(256, depth=4, d_state=128) fp32 with torch.manual_seed(0) default init, x ~ N(0,1)
    [2, 1024, 256]: forward, then prefill of the same x and 64 step() calls with fresh N(0,1)
    [2, 1, 256] inputs, all against the float64 oracle at the fp32 bound."""
    torch.manual_seed(0)
    model = Mamba3(256, d_state=128, depth=4, mimo_rank=1).eval()
    cfg = _cfg(model)
    sd = {key: val.detach().numpy() for key, val in model.state_dict().items()}
    x = torch.randn(2, 1024, 256)
    steps = torch.randn(64, 2, 1, 256)
    model = model.cuda()
    with torch.inference_mode():
        y = model(x.cuda())
        assert ops.LAST_SCAN_DISPATCH
        yp, cache = model.prefill(x.cuda())
        outs = []
        for i in range(64):
            o, cache = model.step(steps[i].cuda(), cache)
            outs.append(o)
        assert ops.LAST_STEP_DISPATCH
    torch.cuda.synchronize()
    ye = O.model_forward(cfg, sd, x.numpy())
    assert rel_err(y, ye) < 1e-4
    assert rel_err(yp, ye) < 1e-4
    _, caches = O.model_prefill(cfg, sd, x.numpy())
    expected = []
    for i in range(64):
        o, caches = O.model_step(cfg, sd, steps[i].numpy(), caches)
        expected.append(o)
    assert rel_err(torch.cat(outs, 1), np.concatenate(expected, 1)) < 1e-4
    for got, want in zip(cache, caches):
        for a, b in zip(got, want):
            assert rel_err(a, b) < 2e-4


# ---------------------------------------------------------------------------------------------
# Bidirectional mixer: both directions in one launch, blend folded into one out_proj GEMM
# ---------------------------------------------------------------------------------------------

def test_two_direction_scan_equals_two_launches_and_the_blend(monkeypatch):
    # one segment everywhere: the two-direction launch never splits, the one-direction reference
    # calls would split this small batch (the same result up to rounding, but not bit for bit)
    monkeypatch.setenv("MAMBA3_B200_SEGMENTS", "1")
    torch.manual_seed(0)
    model = Mamba3(768, d_state=128, depth=1, causal=False).cuda().eval()
    with torch.no_grad():
        model.layers[0].mixer.direction_logit.normal_()
    mixer = model.layers[0].mixer
    x = torch.randn(2, 1000, 768, device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        proj = mixer._project_linear("in_proj", model.layers[0].norm(x))
        fwd = mixer._scan_fused(proj, None, reverse=False, want_cache=False)
        bwd = mixer._scan_fused(proj, None, reverse=True, want_cache=False)
        sizes, tensors, kw = mixer._scan_arguments(proj, None)
        both = torch.empty(2, 1000, 2, mixer.nheads, mixer.headdim, device="cuda", dtype=proj.dtype)
        state = torch.empty_like(fwd[1])
        tensors.update(y=both[:, :, 0], y_reverse=both[:, :, 1], final_state=state)
        _ext.scan_forward(sizes=sizes, tensors=tensors, reverse="both", **kw)
        assert _ext.last_scan_kernel() == "umma"
        fused = mixer._forward_bidirectional_kernels(proj)
        out = mixer._project_linear("out_proj", fwd[0].flatten(-2))
        back = mixer._project_linear("out_proj", bwd[0].flatten(-2))
        blend = torch.sigmoid(mixer.direction_logit).to(out.dtype)
        unfused = out * blend + back * (1.0 - blend)
    torch.testing.assert_close(both[:, :, 0], fwd[0], rtol=0, atol=0)
    torch.testing.assert_close(both[:, :, 1], bwd[0], rtol=0, atol=0)
    torch.testing.assert_close(state, fwd[1], rtol=0, atol=0)
    assert rel_err(fused.float(), unfused.float()) < 2e-2

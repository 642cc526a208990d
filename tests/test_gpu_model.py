"""GPU parity of the whole ``Mamba3`` drop-in (forward / prefill / step / cuda_graph) against the
reference's golden outputs, and of the kernel path against the PyTorch formulation.

Tolerances (normwise): float32 models <= 1e-4 against the reference outputs; bf16 autocast
<= 2e-2 against the PyTorch formulation under the same autocast (the reference's portable path
semantics) and <= 5e-2 against the float32 reference outputs.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden, rel_err
from mamba3_b200 import Mamba3, _ext, ops
from test_model_cpu import golden_model

pytestmark = pytest.mark.gpu

MODELS = ["model_r1", "model_r4", "model_n16_r1", "model_n16_r4", "model_bidir"]


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert _ext.device_error(clear=True) == 0


def run_continued(model, x, split):
    prefix, cache = model.prefill(x[:, :split])
    outs = [prefix]
    for t in range(split, x.shape[1]):
        o, cache = model.step(x[:, t:t + 1], cache)
        outs.append(o)
    return torch.cat(outs, dim=1), cache


@pytest.mark.parametrize("name", MODELS)
def test_fp32_model_matches_reference(name):
    model, f = golden_model(name, device="cuda")
    x = torch.from_numpy(f["x"]).cuda()
    with torch.inference_mode():
        y = model(x)
        assert ops.LAST_SCAN_DISPATCH
        assert rel_err(y, f["y"]) < 1e-4
        if not model.causal:
            return
        cont, cache = run_continued(model, x, int(f["split"]))
        assert ops.LAST_STEP_DISPATCH
    assert rel_err(cont, f["continued"]) < 1e-4
    for i, layer in enumerate(cache):
        for j, tensor in enumerate(layer):
            assert rel_err(tensor, f[f"cache{i}_{j}"]) < 2e-4, (i, j)


@pytest.mark.parametrize("name", MODELS)
def test_bf16_autocast_model(name):
    model, f = golden_model(name, device="cuda")
    x = torch.from_numpy(f["x"]).cuda()
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = model(x)
    with torch.autocast("cuda", dtype=torch.bfloat16):  # grad mode on: the PyTorch formulation
        for p in model.parameters():
            p.requires_grad_(True)
        y_torch = model(x).detach()
    assert rel_err(y.float(), y_torch.float()) < 2e-2
    assert rel_err(y.float(), f["y"]) < 5e-2
    if model.causal:
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            cont, _ = run_continued(model, x, int(f["split"]))
        assert rel_err(cont.float(), f["continued"]) < 5e-2


@pytest.mark.parametrize("rank", [1, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_low_precision_model_kernels_vs_pytorch(rank, dtype):
    """Counterpart of the reference's fused-vs-portable test (tests/test_scan.py:385-435)."""
    torch.manual_seed(11 + rank)
    model = Mamba3(64, d_state=16, depth=1, mimo_rank=rank).cuda().to(dtype).eval()
    x = torch.randn(2, 37, 64, device="cuda", dtype=dtype)
    with torch.inference_mode():
        actual = model(x)
        cont, cache = run_continued(model, x, 9)
    for p in model.parameters():
        p.requires_grad_(True)
    expected = model(x).detach()
    torch.testing.assert_close(actual, expected, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(cont, expected, rtol=3e-2, atol=3e-2)


def _layer_by_layer(model, x, want_cache=False):
    """The block loop of the reference (`hidden + mixer(norm(hidden))`, then norm_f), op by op."""
    caches = []
    for layer in model.layers:
        if want_cache:
            x, c = layer(x, return_cache=True)
            caches.append(c)
        else:
            x = layer(x)
    return (model.norm_f(x), caches) if want_cache else model.norm_f(x)


@pytest.mark.parametrize("autocast", [False, True])
def test_fused_residual_stream_matches_block_loop(autocast):
    """Mamba3.forward / prefill on CUDA run the residual add and the next RMSNorm as one kernel
    (m3_residual_rmsnorm); the result must equal the reference block loop."""
    torch.manual_seed(3)
    model = Mamba3(256, d_state=128, depth=3).cuda().eval()
    for layer in model.layers:  # non-trivial norm weights
        layer.norm.weight.data.uniform_(0.5, 1.5)
    model.norm_f.weight.data.uniform_(0.5, 1.5)
    x = torch.randn(2, 200, 256, device="cuda")
    x_copy = x.clone()
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        fused = model(x)
        expected = _layer_by_layer(model, x)
        out_p, caches = model.prefill(x)
        exp_p, exp_caches = _layer_by_layer(model, x, want_cache=True)
    tol = 2e-2 if autocast else 1e-5
    assert fused.dtype == expected.dtype == torch.float32
    assert rel_err(fused, expected) < tol
    assert rel_err(out_p, exp_p) < tol
    for got, want in zip(caches, exp_caches):
        assert rel_err(got[1], want[1]) < (1e-2 if autocast else 1e-5)
    torch.testing.assert_close(x, x_copy, rtol=0, atol=0)  # the input is not written


def test_residual_rmsnorm_kernel_against_torch():
    torch.manual_seed(4)
    x = torch.randn(37, 1024, device="cuda")
    m = torch.randn(37, 1024, device="cuda", dtype=torch.bfloat16)
    w = torch.rand(1024, device="cuda") + 0.5
    out_x = torch.empty_like(x)
    n = _ext.residual_rmsnorm(x, m, w, 1e-5, out_dtype=torch.bfloat16, out_x=out_x)
    r = x + m.float()
    torch.testing.assert_close(out_x, r, rtol=0, atol=0)
    ref = torch.nn.functional.rms_norm(r, (1024,), w, 1e-5)
    torch.testing.assert_close(n.float(), ref, rtol=1e-2, atol=1e-2)
    # generic path: odd width, strided rows, fp32 output, in place residual
    x2 = torch.randn(5, 300, device="cuda")[:, :200]
    expect = torch.nn.functional.rms_norm(x2 + 1.0, (200,), w[:200], 1e-5)
    n2 = _ext.residual_rmsnorm(x2, torch.ones(5, 200, device="cuda"), w[:200], 1e-5, out_dtype=torch.float32,
                               out_x=x2)
    torch.testing.assert_close(n2, expect, rtol=1e-5, atol=1e-5)


def test_cuda_graph_decoder_matches_forward_and_resets():
    torch.manual_seed(5)
    model = Mamba3(64, d_state=128, depth=1).cuda().eval()
    x = torch.randn(2, 5, 64, device="cuda")
    ref_cache, ref_out = None, []
    with torch.inference_mode():
        for t in range(5):
            o, ref_cache = model.step(x[:, t:t + 1], ref_cache)
            ref_out.append(o)
    decoder = model.cuda_graph(batch_size=2)
    with torch.inference_mode():
        expected = model(x)
        actual = torch.cat([decoder(x[:, t:t + 1]).clone() for t in range(5)], dim=1)
    torch.testing.assert_close(actual, expected, rtol=2e-4, atol=2e-5)
    torch.testing.assert_close(actual, torch.cat(ref_out, 1), rtol=2e-4, atol=2e-5)
    for graph_layer, ref_layer in zip(decoder.cache, ref_cache):
        for a, b in zip(graph_layer, ref_layer):
            torch.testing.assert_close(a, b, rtol=2e-4, atol=2e-5)
    decoder.reset()
    with torch.inference_mode():
        again = decoder(x[:, :1]).clone()
    torch.testing.assert_close(again, expected[:, :1], rtol=2e-4, atol=2e-5)
    with torch.no_grad():
        model.layers[0].mixer.D.add_(0.1)
    with pytest.raises(RuntimeError, match="recreate"):
        decoder.validate()
    with pytest.raises(ValueError, match="gradient"):
        decoder(x[:, :1].requires_grad_())


@pytest.mark.parametrize("rank", [1, 4])
def test_bf16_cuda_graph_decoder_matches_eager_steps(rank):
    torch.manual_seed(21)
    model = Mamba3(128, d_state=128, depth=2, mimo_rank=rank).cuda().to(torch.bfloat16).eval()
    x = torch.randn(3, 6, 128, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        _, cache = model.prefill(x[:, :2])
        eager = []
        for t in range(2, 6):
            o, cache = model.step(x[:, t:t + 1], cache)
            eager.append(o)
    decoder = model.cuda_graph(batch_size=3)
    with torch.inference_mode():
        graph = [decoder(x[:, t:t + 1]).clone() for t in range(6)]
        _, ref = model.prefill(x)
    torch.testing.assert_close(torch.cat(graph, 1), model(x), rtol=3e-2, atol=3e-2)
    for a, b in zip(decoder.cache, ref):
        torch.testing.assert_close(a[1], b[1], rtol=3e-2, atol=3e-2)


def test_autocast_dtypes_and_training_path_on_cuda():
    torch.manual_seed(4)
    model = Mamba3(64, d_state=16, depth=1).cuda()
    x = torch.randn(2, 33, 64, device="cuda", requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = model(x)
    out.float().square().mean().backward()
    assert out.dtype == torch.float32 and torch.isfinite(out).all()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())
    model.eval()
    cache, steps = None, []
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        expected, prefill_cache = model.prefill(x.detach())
        for t in range(x.shape[1]):
            o, cache = model.step(x[:, t:t + 1].detach(), cache)
            steps.append(o)
    torch.testing.assert_close(torch.cat(steps, 1), expected, rtol=3e-2, atol=3e-2)
    for a_layer, b_layer in zip(prefill_cache, cache):
        for a, b in zip(a_layer, b_layer):
            torch.testing.assert_close(a.float(), b.float(), rtol=3e-2, atol=3e-2)


def test_negative_phase_increments_do_not_drift_at_long_context():
    """The in-kernel blocked phase stays exact at L=131072 (tests/test_model.py:252-273)."""
    import math
    torch.manual_seed(0)
    model = Mamba3(16, d_state=8, depth=1).cuda().eval()
    mixer = model.layers[0].mixer
    length = 131_072
    raw = math.atanh(-1e-4 / math.pi)
    angles = torch.full((1, length, mixer.num_angles), raw, device="cuda")
    dt = torch.ones(1, length, mixer.nheads, device="cuda")
    phase = mixer._phase(angles, dt, None)
    inc = math.pi * math.tanh(raw)
    pos = torch.arange(1, length + 1, device="cuda", dtype=torch.float64)
    expected = torch.remainder(pos * inc, 2 * math.pi).float()[None, :, None, None].expand_as(phase)
    circ = torch.remainder(phase - expected + math.pi, 2 * math.pi) - math.pi
    assert circ.abs().max() < 2e-3


def test_autocast_weight_cast_cache_is_exact_and_invalidated():
    """The kernel path keeps bf16 copies of in_proj/out_proj across autocast regions; the output
    equals a fresh autocast cast bit for bit and follows in-place weight updates."""
    torch.manual_seed(8)
    model = Mamba3(128, d_state=64, depth=2).cuda().eval()
    x = torch.randn(2, 70, 128, device="cuda")

    def run():
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            return model(x)

    def fresh():
        for layer in model.layers:
            layer.mixer._weight_casts.clear()
        return run()

    first = run()
    torch.testing.assert_close(run(), first, rtol=0, atol=0)
    torch.testing.assert_close(fresh(), first, rtol=0, atol=0)
    with torch.no_grad():
        model.layers[1].mixer.in_proj.weight.mul_(1.5)
        model.layers[0].mixer.out_proj.weight.add_(0.01)
    updated = run()
    assert rel_err(updated, first) > 1e-3
    torch.testing.assert_close(fresh(), updated, rtol=0, atol=0)


@pytest.mark.parametrize("rank,causal", [(1, True), (4, True), (1, False)])
def test_head_range_scans_match_the_full_scan(rank, causal):
    """Head sharding on the kernel path: the tensor-core scan restricted to head ranges (sliced
    per-head columns and parameters, shared q/k/angles) reproduces the full scan's heads bit for bit."""
    torch.manual_seed(12)
    model = Mamba3(256, d_state=128, depth=1, mimo_rank=rank, causal=causal).cuda().eval()
    mixer = model.layers[0].mixer
    x = torch.randn(1, 300, 256, device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        hidden = model.layers[0].norm(x)
        projected = mixer._project_linear("in_proj", hidden)
        for reverse in ((False, True) if not causal else (False,)):
            full = mixer._scan_fused(projected, None, reverse=reverse, want_cache=False)[0]
            assert _ext.last_scan_kernel() == "umma"
            parts = torch.cat([mixer.mixed_heads(hidden, 0, 3, reverse=reverse),
                               mixer.mixed_heads(hidden, 3, mixer.nheads, reverse=reverse)], dim=2)
            torch.testing.assert_close(parts, full, rtol=0, atol=0)

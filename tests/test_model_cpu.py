"""Host-side API behaviour of ``mamba3_b200.Mamba3`` (CPU path), mirroring the reference suite
(tests/test_model.py of jreoka/mamba3) and checked against the golden fixtures."""

from __future__ import annotations

import inspect
import math

import numpy as np
import pytest
import torch
from torch.nn import functional as F

import mamba3_b200
from conftest import load_golden, rel_err
from mamba3_b200 import Mamba3


def golden_model(name: str, device="cpu", dtype=torch.float32):
    f = load_golden(name)
    torch.manual_seed(0)
    model = Mamba3(int(f["d_model"]), d_state=int(f["d_state"]), depth=int(f["depth"]), mimo_rank=int(f["rank"]),
                   causal=bool(f["causal"]))
    sd = {key[3:]: torch.from_numpy(f[key]) for key in f if key.startswith("sd.")}
    model.load_state_dict(sd)
    return model.to(device=device, dtype=dtype).eval(), f


def test_public_surface_and_constructor():
    assert mamba3_b200.__all__ == ["Mamba3"]
    assert list(inspect.signature(Mamba3).parameters) == ["d_model", "d_state", "depth", "mimo_rank", "causal"]
    for kwargs, match in [(dict(d_model=0), "d_model"), (dict(d_model=16, d_state=2), "at least 4"),
                          (dict(d_model=16, d_state=10, mimo_rank=4), "divisible by 4"),
                          (dict(d_model=16, depth=0), "depth"), (dict(d_model=16, mimo_rank=0), "mimo_rank")]:
        with pytest.raises(ValueError, match=match):
            Mamba3(**kwargs)


@pytest.mark.parametrize("name", ["model_r1", "model_r4", "model_bidir"])
def test_seeded_init_and_state_dict_match_reference(name):
    """Parameter names, shapes and seeded initial values equal the reference's (same creation order)."""
    f = load_golden(name)
    torch.manual_seed(0)
    model = Mamba3(int(f["d_model"]), d_state=int(f["d_state"]), depth=int(f["depth"]), mimo_rank=int(f["rank"]),
                   causal=bool(f["causal"]))
    sd = model.state_dict()
    ref = {key[3:]: f[key] for key in f if key.startswith("sd.")}
    assert list(sd) == list(ref)
    for key, val in ref.items():
        np.testing.assert_array_equal(sd[key].numpy(), val)


@pytest.mark.parametrize("rank", [1, 4])
def test_canonical_parameters(rank):
    model = Mamba3(64, depth=1, mimo_rank=rank)
    mixer = model.layers[0].mixer
    assert (mixer.d_state, mixer.d_inner, mixer.headdim, mixer.nheads, mixer.num_angles) == (128, 128, 64, 2, 32)
    assert mixer.in_proj.weight.shape == (2 * 128 + 2 * 128 * rank + 6 + 32, 64)
    assert mixer.B_bias.shape == mixer.C_bias.shape == (2, rank, 128)
    q, k, *_ = mixer._project(torch.randn(1, 3, 64))
    assert q.shape == k.shape == (1, 3, 1, rank, 128)
    dt = F.softplus(mixer.dt_bias)
    assert (dt >= 0.001).all() and (dt <= 0.1).all()


@pytest.mark.parametrize("name", ["model_r1", "model_r4", "model_n16_r1", "model_n16_r4", "model_bidir"])
def test_cpu_forward_prefill_step_match_reference(name):
    model, f = golden_model(name)
    x = torch.from_numpy(f["x"])
    with torch.no_grad():
        assert rel_err(model(x), f["y"]) < 2e-5
        if not model.causal:
            return
        split = int(f["split"])
        prefix, cache = model.prefill(x[:, :split])
        outs = [prefix]
        for t in range(split, x.shape[1]):
            o, cache = model.step(x[:, t:t + 1], cache)
            outs.append(o)
    assert rel_err(torch.cat(outs, dim=1), f["continued"]) < 2e-5
    for i, layer in enumerate(cache):
        for j, tensor in enumerate(layer):
            assert rel_err(tensor, f[f"cache{i}_{j}"]) < 5e-5


def test_shapes_empty_inputs_and_backward():
    model = Mamba3(24, d_state=8, depth=2)
    x = torch.randn(2, 17, 24)
    assert model(x).shape == x.shape
    assert model(torch.empty(0, 5, 24)).shape == (0, 5, 24)
    assert model(torch.empty(2, 0, 24)).shape == (2, 0, 24)
    with pytest.raises(ValueError, match="expected"):
        model(torch.empty(2, 5, 7))
    model.zero_grad(set_to_none=True)
    model(torch.empty(2, 0, 24)).sum().backward()
    assert all(p.grad is not None for p in model.parameters())


@pytest.mark.parametrize("rank", [1, 4])
@pytest.mark.parametrize("causal", [True, False])
def test_backward_reaches_every_parameter(rank, causal):
    model = Mamba3(16, d_state=8, depth=2, mimo_rank=rank, causal=causal)
    x = torch.randn(2, 9, 16, requires_grad=True)
    model(x).square().mean().backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())


def test_causality_and_bidirectional_dependence():
    torch.manual_seed(0)
    model = Mamba3(16, d_state=8, depth=2).eval()
    a = torch.randn(1, 12, 16)
    b = a.clone()
    b[:, 7:] = torch.randn_like(b[:, 7:])
    with torch.no_grad():
        torch.testing.assert_close(model(a)[:, :7], model(b)[:, :7], rtol=0, atol=1e-7)
    bi = Mamba3(16, d_state=8, depth=1, causal=False).eval()
    torch.testing.assert_close(bi.layers[0].mixer.direction_logit, torch.zeros(16))
    with torch.no_grad():
        assert not torch.allclose(bi(a)[:, 0], bi(b)[:, 0], rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError, match="causal"):
        bi.prefill(torch.randn(1, 4, 16))
    with pytest.raises(ValueError, match="causal"):
        bi.step(torch.randn(1, 1, 16))
    with pytest.raises(ValueError, match="causal"):
        bi.layers[0].mixer(torch.randn(1, 4, 16), return_cache=True)


@pytest.mark.parametrize("rank", [1, 4])
def test_cached_steps_match_forward(rank):
    torch.manual_seed(2)
    model = Mamba3(16, d_state=8, depth=2, mimo_rank=rank).eval()
    x = torch.randn(2, 11, 16)
    cache = None
    outs = []
    with torch.no_grad():
        expected = model(x)
        for t in range(x.shape[1]):
            o, cache = model.step(x[:, t:t + 1], cache)
            outs.append(o)
    torch.testing.assert_close(torch.cat(outs, dim=1), expected, rtol=2e-5, atol=2e-6)
    mixer = model.layers[0].mixer
    phase, state, prev_k, prev_v = cache[0]
    assert phase.shape == (2, mixer.nheads, mixer.num_angles)
    assert state.shape == (2, mixer.nheads, mixer.headdim, mixer.d_state) and state.dtype == torch.float32
    assert prev_k.shape == (2, mixer.nheads, rank, mixer.d_state)
    assert prev_v.shape == (2, mixer.nheads, mixer.headdim)


def test_prefill_cache_is_compact():
    model = Mamba3(32, d_state=16, depth=1).eval()
    with torch.inference_mode():
        _, cache = model.prefill(torch.randn(2, 257, 32))
    for tensor in (cache[0][0], cache[0][2], cache[0][3]):
        assert tensor.untyped_storage().nbytes() == tensor.numel() * tensor.element_size()


def test_phase_bounded_per_block_matches_sequential():
    mixer = Mamba3(16, d_state=8, depth=1).layers[0].mixer
    length = 2048
    q = torch.zeros(1, length, mixer.nheads, 1, mixer.d_state)
    angles = torch.full((1, length, mixer.num_angles), 3.0)
    dt = torch.full((1, length, mixer.nheads), 100.0)
    _, _, phase = mixer._phase_and_rotate(q, q, angles, dt, None)
    inc = torch.fmod(math.pi * torch.tanh(angles[:, 0]).unsqueeze(1) * dt[:, 0].unsqueeze(-1), 2 * math.pi)
    state = torch.zeros_like(phase[:, 0])
    expected = []
    for _ in range(length):
        state = torch.fmod(state + inc, 2 * math.pi)
        expected.append(state)
    circ = torch.remainder(phase - torch.stack(expected, 1) + math.pi, 2 * math.pi) - math.pi
    assert circ.abs().max() < 2e-3
    assert phase.abs().max() < 2 * math.pi


def test_phase_matches_reference_fixture():
    f = load_golden("phase")
    torch.manual_seed(0)
    mixer = Mamba3(64, d_state=128, depth=1).layers[0].mixer
    phase = mixer._phase(torch.from_numpy(f["angles"]), torch.from_numpy(f["dt"]), torch.from_numpy(f["initial"]))
    circ = torch.remainder(phase.double() - torch.from_numpy(f["phase"]).double() + math.pi, 2 * math.pi) - math.pi
    assert circ.abs().max() < 1e-4


def test_step_validation_and_chunk_api():
    model = Mamba3(16, d_state=8, depth=2)
    with pytest.raises(ValueError, match="batch, 1"):
        model.step(torch.randn(2, 3, 16))
    with pytest.raises(ValueError, match="cache for 2"):
        model.step(torch.randn(2, 1, 16), cache=[])
    _, cache = model.step(torch.randn(2, 1, 16))
    bad = list(cache)
    bad[0] = (bad[0][0], bad[0][1], bad[0][2][:1], bad[0][3])
    with pytest.raises(ValueError, match="cache shapes"):
        model.step(torch.randn(2, 1, 16), bad)
    with pytest.raises(ValueError, match="non-empty"):
        model.prefill(torch.empty(2, 0, 16))
    assert model.set_chunk_sizes(training=8, inference=16) is model
    assert model.layers[0].mixer.chunk_size == 8 and model.layers[0].mixer.inference_chunk_size == 16
    with pytest.raises(ValueError, match="positive"):
        model.set_chunk_sizes(inference=0)


def test_chunk_size_env_override(monkeypatch):
    monkeypatch.setenv("MAMBA3_CHUNK_SIZE", "5")
    mixer = Mamba3(16, d_state=8, depth=1).layers[0].mixer
    assert mixer.chunk_size == mixer.inference_chunk_size == 5
    monkeypatch.setenv("MAMBA3_CHUNK_SIZE", "-1")
    with pytest.raises(ValueError, match="positive integer"):
        Mamba3(16, d_state=8, depth=1)


def test_cuda_graph_requires_cuda_model():
    with pytest.raises(ValueError, match="CUDA"):
        Mamba3(16, d_state=8, depth=1).eval().cuda_graph(1)

"""Pin the numpy oracle to the golden fixtures produced by running the reference itself."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden, rel_err
from oracle import mamba3_oracle as O

SCANS = ["scan_small_r1", "scan_small_r4", "scan_small_r4_c5", "scan_cont_r1", "scan_kernel_r1",
         "scan_kernel_r4", "scan_kernel_r2", "scan_n16_r1"]
MODELS = ["model_r1", "model_r4", "model_n16_r1", "model_n16_r4", "model_bidir"]


def oracle_scan_inputs(f: dict):
    """Expand + bias + rotate q/k exactly as mamba3/ops.py:698-714 does before the chunk loop."""
    heads = f["value"].shape[2]
    rank = f["q"].shape[3]
    q = O.expand_heads(f["q"].astype(np.float64), heads)
    k = O.expand_heads(f["k"].astype(np.float64), heads)
    if "q_bias" in f:
        q = q + f["q_bias"]
        k = k + f["k_bias"]
    if "phase" in f:
        q = O.rotate(q, f["phase"], rank > 1)
        k = O.rotate(k, f["phase"], rank > 1)
    kwargs = {key: f.get(key) for key in ("mimo_x", "mimo_z", "mimo_out", "initial_state", "initial_k",
                                          "initial_value")}
    return q, k, kwargs


@pytest.mark.parametrize("name", SCANS)
@pytest.mark.parametrize("form", ["recurrent", "chunked"])
def test_oracle_scan_matches_reference(name, form):
    f = load_golden(name)
    q, k, kw = oracle_scan_inputs(f)
    args = (q, k, f["value"], f["gate"], f["adt"], f["dt"], f["trap"], f["D"])
    if form == "recurrent":
        y, s = O.scan_recurrent(*args, **kw)
    else:
        y, s = O.scan_chunked(*args, chunk_size=int(f["chunk"]), **kw)
    assert rel_err(y, f["y"]) < 2e-6
    assert rel_err(s, f["state"]) < 2e-6


def test_oracle_rotation_known_answers():
    f = load_golden("rotation")
    # tests/test_scan.py:155-168 golden vectors
    np.testing.assert_allclose(O.rotate(f["siso_in"][0, 0, 0], f["phase"][0, 0, 0], False), f["siso"][0, 0, 0],
                               atol=1e-6)
    np.testing.assert_allclose(O.rotate(f["mimo_in"][0, 0, 0], f["phase"][0, 0, 0], True), f["mimo"][0, 0, 0],
                               atol=1e-6)
    np.testing.assert_allclose(O.rotate(f["rand_in"], f["rand_phase"], False), f["rand_siso"], atol=2e-6)
    np.testing.assert_allclose(O.rotate(f["rand_in"], f["rand_phase"], True), f["rand_mimo"], atol=2e-6)
    np.testing.assert_allclose(O.heavy_tail(f["heavy_in"]), f["heavy"], rtol=1e-6)


def test_oracle_phase_matches_reference():
    f = load_golden("phase")
    ph = O.phase_scheme(f["angles"], f["dt"], f["initial"])
    circ = np.remainder(ph - f["phase"] + np.pi, 2 * np.pi) - np.pi
    assert np.abs(circ).max() < 1e-4


@pytest.mark.parametrize("rank", [1, 4])
def test_oracle_step_matches_reference(rank):
    f = load_golden(f"step_r{rank}")
    y, (ph, s, k1, _) = O.fused_step(f["q"], f["k"], f["value"], f["gate"], f["adt"], f["dt"], f["trap"],
                                     f["angle_rate"], f["D"], (f["phase0"], f["state0"], f["k0"], f["v0"]),
                                     mimo_x=f.get("mimo_x"), mimo_z=f.get("mimo_z"), mimo_out=f.get("mimo_out"))
    assert rel_err(y, f["y"]) < 2e-6
    assert rel_err(s, f["state1"]) < 2e-6
    assert rel_err(k1, f["k1"]) < 2e-6
    assert rel_err(ph, f["phase1"]) < 2e-6


def model_from_golden(f: dict):
    cfg = O.ModelConfig(int(f["d_model"]), int(f["d_state"]), int(f["depth"]), int(f["rank"]), bool(f["causal"]))
    sd = {key[3:]: f[key] for key in f if key.startswith("sd.")}
    return cfg, sd


@pytest.mark.parametrize("name", MODELS)
def test_oracle_model_matches_reference(name):
    f = load_golden(name)
    cfg, sd = model_from_golden(f)
    assert rel_err(O.model_forward(cfg, sd, f["x"]), f["y"]) < 2e-6
    if not cfg.causal:
        return
    split = int(f["split"])
    y, caches = O.model_prefill(cfg, sd, f["x"][:, :split])
    outs = [y]
    for t in range(split, f["x"].shape[1]):
        o, caches = O.model_step(cfg, sd, f["x"][:, t:t + 1], caches)
        outs.append(o)
    assert rel_err(np.concatenate(outs, axis=1), f["continued"]) < 2e-6
    for i in range(cfg.depth):
        for j in range(4):
            assert rel_err(caches[i][j], f[f"cache{i}_{j}"]) < 5e-6


def test_oracle_recurrent_equals_chunked_on_random_inputs():
    rng = np.random.default_rng(3)
    b, l, h, r, n, p = 2, 23, 2, 2, 8, 4
    q = rng.standard_normal((b, l, h, r, n))
    k = rng.standard_normal((b, l, h, r, n))
    v = rng.standard_normal((b, l, h, p))
    z = rng.standard_normal((b, l, h, p))
    adt = -rng.random((b, l, h)) * 0.3
    dt = rng.random((b, l, h)) * 0.2 + 0.01
    tr = rng.standard_normal((b, l, h))
    D = rng.standard_normal(h)
    mx, mz, mo = (rng.standard_normal((h, r, p)) for _ in range(3))
    kw = dict(mimo_x=mx, mimo_z=mz, mimo_out=mo)
    y1, s1 = O.scan_recurrent(q, k, v, z, adt, dt, tr, D, **kw)
    for chunk in (1, 4, 7, 64):
        y2, s2 = O.scan_chunked(q, k, v, z, adt, dt, tr, D, chunk_size=chunk, **kw)
        assert rel_err(y2, y1) < 1e-12 and rel_err(s2, s1) < 1e-12

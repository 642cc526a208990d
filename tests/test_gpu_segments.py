"""GPU parity of the segmented scan: a sequence split into segments scanned in parallel (state pass,
FP32 scan over the segment records, main pass from each segment's initial cache).

The split must not change the result beyond rounding: every case compares the segmented kernel with
the float64 oracle and with the unsplit kernel (segments = 1). Tolerances (normwise) as elsewhere:
bf16 outputs <= 2e-2, FP32 states <= 1e-2, phase <= 1e-5; the segmented and unsplit kernels agree
to <= 1e-2 on outputs (they round at different points) and the phase bit for bit up to fmod rounding.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import rel_err
from mamba3_b200 import Mamba3, _ext, ops
from oracle import mamba3_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert _ext.device_error(clear=True) == 0


def _np(t):
    return t.detach().double().cpu().numpy()


def _mixer_scan(mixer, projected, reverse, segments, cache=None):
    old = _ext._segments
    _ext._segments = lambda s: segments
    try:
        return mixer._scan_fused(projected, cache, reverse=reverse, want_cache=not reverse)
    finally:
        _ext._segments = old


@pytest.mark.parametrize("rank,reverse", [(1, False), (4, False), (1, True)], ids=["siso", "mimo4", "reverse"])
@pytest.mark.parametrize("segments", [0, 3, 7])
def test_segmented_model_mode_scan_matches_oracle_and_unsplit(rank, reverse, segments):
    torch.manual_seed(5 + rank)
    model = Mamba3(256, d_state=128, depth=1, mimo_rank=rank, causal=not reverse).cuda().eval()
    mixer = model.layers[0].mixer
    cfg = O.ModelConfig(256, 128, 1, rank, not reverse)
    lp = O._layer_params({k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}, 0)
    length = 2000  # not a multiple of the 64-token segment granule
    x = torch.randn(1, length, 256, device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        projected = mixer._project_linear("in_proj", model.layers[0].norm(x))
        y1, s1, ph1, k1, _ = _mixer_scan(mixer, projected, reverse, 1)
        ys, ss, phs, ks, _ = _mixer_scan(mixer, projected, reverse, segments)
        assert _ext.last_scan_kernel() == "umma"
    torch.cuda.synchronize()
    proj = _np(projected)
    if reverse:
        proj = np.ascontiguousarray(proj[:, ::-1])
    ye, se, phe, ke, _ = O.scan_projection(cfg, lp, proj)
    if reverse:
        ye = np.ascontiguousarray(ye[:, ::-1])
    assert rel_err(ys.float(), ye) < 2e-2
    assert rel_err(ss, se) < 1e-2
    assert rel_err(ys.float(), y1.float()) < 1e-2
    assert rel_err(ss, s1) < 1e-2
    if not reverse:
        assert rel_err(phs, phe[:, -1]) < 1e-5
        assert rel_err(ks.float(), ke[:, -1]) < 2e-2
        circ = torch.remainder(phs - ph1 + math.pi, 2 * math.pi) - math.pi
        assert circ.abs().max() < 1e-4


@pytest.mark.parametrize("rank", [1, 4])
def test_segmented_scan_continues_a_prefill_cache(rank):
    """Segments after an initial cache (state, phase, endpoint k/value): the first segment folds the
    caller's endpoint term, later ones the combined records."""
    torch.manual_seed(9)
    model = Mamba3(256, d_state=128, depth=1, mimo_rank=rank).cuda().eval()
    mixer = model.layers[0].mixer
    x = torch.randn(2, 1500 + 1300, 256, device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        hidden = model.layers[0].norm(x)
        proj = mixer._project_linear("in_proj", hidden)
        full = _mixer_scan(mixer, proj, False, 1)
        first = _mixer_scan(mixer, proj[:, :1500], False, 1)
        cache = (first[2], first[1], first[3], first[4][:, -1])
        second = _mixer_scan(mixer, proj[:, 1500:], False, 5, cache=cache)
    y = torch.cat((first[0], second[0]), 1)
    assert rel_err(y.float(), full[0].float()) < 2e-2
    assert rel_err(second[1], full[1]) < 1e-2
    circ = torch.remainder(second[2] - full[2] + math.pi, 2 * math.pi) - math.pi
    assert circ.abs().max() < 1e-4


def test_automatic_segments_on_a_batch_one_prefill_match_the_oracle():
    """Batch 1 of the SISO benchmark width: the automatic plan splits the sequence (32 heads leave
    most SMs idle) and the whole forward still matches the oracle on the same bf16 projection."""
    torch.manual_seed(0)
    model = Mamba3(1024, d_state=128, depth=1).cuda().eval()
    mixer = model.layers[0].mixer
    cfg = O.ModelConfig(1024, 128, 1, 1, True)
    lp = O._layer_params({k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}, 0)
    x = torch.randn(1, 4096, 1024, device="cuda")
    lib = _ext.load()
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        projected = mixer._project_linear("in_proj", model.layers[0].norm(x))
        y, s, ph, k, _ = mixer._scan_fused(projected, None, reverse=False, want_cache=True)
    torch.cuda.synchronize()
    ye, se, phe, ke, _ = O.scan_projection(cfg, lp, _np(projected))
    assert rel_err(y.float(), ye) < 2e-2
    assert rel_err(s, se) < 1e-2
    assert rel_err(ph, phe[:, -1]) < 1e-5
    # the plan did split: the workspace holds the segment records beyond the per-token rows
    args = _ext.ScanArgs()
    args.batch, args.length, args.groups, args.heads, args.rank = 1, 4096, 1, 32, 1
    args.d_state, args.head_dim, args.num_angles, args.chunk_hint = 128, 64, 32, 256
    assert lib.m3_scan_segments(args) > 1
    args.segments = 1
    assert lib.m3_scan_segments(args) == 1

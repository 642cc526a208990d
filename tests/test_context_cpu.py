"""Host-side check of the context-parallel fold (``mamba3_b200.context.fold_prefix``) on CPU.

Slices of a sequence are summarised with the PyTorch formulation (each slice scanned from a zero
state and zero phase, exactly what ``m3_scan_summary`` computes on the GPU), folded, and the next
slice is scanned as a continuation from the folded cache. The result must equal the scan of the
whole sequence (float32, normwise <= 1e-4; the phase compared on the circle).
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import rel_err
from mamba3_b200 import Mamba3
from mamba3_b200.context import _slice_summary_torch, fold_prefix


@pytest.mark.parametrize("rank", [1, 4])
def test_fold_of_slice_summaries_continues_the_full_scan(rank):
    torch.manual_seed(17 + rank)
    model = Mamba3(64, d_state=16, depth=1, mimo_rank=rank).eval()
    mixer = model.layers[0].mixer
    bounds = [0, 192, 320, 448, 498]  # slices of 192, 128, 128 and a 50-token tail
    hidden = torch.randn(2, bounds[-1], 64)
    with torch.no_grad():
        full_mixed, full_state, full_phase, _, _, _ = mixer._scan_torch_direction(hidden, None)
        summaries = []
        for j in range(len(bounds) - 1):
            part = hidden[:, bounds[j]: bounds[j + 1]]
            if summaries:
                cache = fold_prefix(summaries, mimo=rank > 1, mimo_x=mixer.mimo_x)
                mixed, state, phase, _, _, _ = mixer._scan_torch_direction(part, cache)
                assert rel_err(mixed, full_mixed[:, bounds[j]: bounds[j + 1]]) < 1e-4, j
                circ = torch.remainder(phase[:, -1] - full_phase[:, bounds[j + 1] - 1] + math.pi,
                                       2 * math.pi) - math.pi
                assert circ.abs().max() < 1e-4, j
                if j == len(bounds) - 2:
                    assert rel_err(state, full_state) < 1e-4
            summaries.append(_slice_summary_torch(mixer, part))

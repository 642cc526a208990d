"""GPU parity of context-parallel prefill (``mamba3_b200.context``): a sequence split along its
length, each slice summarised by ``m3_scan_summary`` (the state pass from zeros), the summaries
folded, each slice scanned as a continuation.

One process emulates the ranks (slices in order, the fold over the earlier slices' summaries), so
the kernel path is checked on one GPU; with two or more GPUs a second test runs the real
``forward_context_parallel`` over NCCL, one process per GPU. Tolerances (normwise): bf16 outputs
<= 2e-2 against the unsplit kernel scan and the float64 oracle, FP32 end state <= 1e-2.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import rel_err
from mamba3_b200 import Mamba3, _ext
from mamba3_b200.context import _slice_summary, fold_prefix
from oracle import mamba3_oracle as O

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert _ext.device_error(clear=True) == 0


@pytest.mark.parametrize("rank", [1, 4])
def test_slice_summaries_fold_into_the_unsplit_scan(rank):
    torch.manual_seed(3 + rank)
    d_model = 1024 if rank == 1 else 2048
    model = Mamba3(d_model, d_state=128, depth=1, mimo_rank=rank).cuda().eval()
    mixer = model.layers[0].mixer
    bounds = [0, 1024, 1536, 2560, 3000]
    x = torch.randn(2, bounds[-1], d_model, device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        proj = mixer._project_linear("in_proj", model.layers[0].norm(x))
        full_y, full_s, full_ph, _, _ = mixer._scan_fused(proj, None, reverse=False, want_cache=True)
        ys, summaries = [], []
        for j in range(len(bounds) - 1):
            part = proj[:, bounds[j]: bounds[j + 1]]
            cache = None
            if summaries:
                phase, state, k, x_last = fold_prefix(summaries, mimo=rank > 1, mimo_x=mixer.mimo_x)
                cache = (phase, state, k.to(part.dtype), x_last.to(part.dtype))
            y, s, ph, _, _ = mixer._scan_fused(part, cache, reverse=False, want_cache=True)
            ys.append(y)
            if j + 1 < len(bounds) - 1:
                summaries.append(_slice_summary(mixer, part))
    torch.cuda.synchronize()
    y = torch.cat(ys, 1)
    assert rel_err(y.float(), full_y.float()) < 2e-2
    assert rel_err(s, full_s) < 1e-2
    circ = torch.remainder(ph - full_ph + np.pi, 2 * np.pi) - np.pi
    assert circ.abs().max() < 1e-3
    cfg = O.ModelConfig(d_model, 128, 1, rank, True)
    lp = O._layer_params({k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}, 0)
    ye, se, _, _, _ = O.scan_projection(cfg, lp, proj.double().cpu().numpy())
    assert rel_err(y.float(), ye) < 2e-2
    assert rel_err(s, se) < 1e-2


def test_summary_of_a_slice_equals_the_scan_from_zeros():
    """The record's end state and rotated last k equal an ordinary scan of the slice from zeros."""
    torch.manual_seed(8)
    model = Mamba3(1024, d_state=128, depth=1).cuda().eval()
    mixer = model.layers[0].mixer
    x = torch.randn(2, 768, 1024, device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        proj = mixer._project_linear("in_proj", model.layers[0].norm(x))
        _, s, _, k, _ = mixer._scan_fused(proj, None, reverse=False, want_cache=True)
        summ = _slice_summary(mixer, proj)
    assert rel_err(summ["state"], s) < 1e-2
    assert rel_err(summ["k"], k.float()) < 1e-2


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _nccl_worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from mamba3_b200.context import forward_context_parallel

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        torch.manual_seed(0)
        model = Mamba3(1024, d_state=128, depth=2).cuda().eval()
        x = torch.randn(1, 1024 * world, 1024, generator=torch.Generator().manual_seed(1)).cuda()
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            y = forward_context_parallel(model, x[:, 1024 * rank: 1024 * (rank + 1)])
        torch.save(y.float().cpu(), Path(out_dir) / f"y{rank}.pt")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_context_parallel_forward_equals_one_gpu(tmp_path):
    world = 2
    mp.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    torch.manual_seed(0)
    model = Mamba3(1024, d_state=128, depth=2).cuda().eval()
    x = torch.randn(1, 1024 * world, 1024, generator=torch.Generator().manual_seed(1)).cuda()
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        expected = model(x).float().cpu()
    got = torch.cat([torch.load(tmp_path / f"y{r}.pt") for r in range(world)], dim=1)
    assert rel_err(got, expected) < 2e-2

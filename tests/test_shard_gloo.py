"""Multi-process batch and head sharding on CPU (gloo, world size 2): outputs equal the
single-process forward, uneven batches / head counts work, and a rank that dies before the gather
makes the survivor's collective fail within its timeout instead of hanging."""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]

from mamba3_b200.shard import shard_bounds  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(mode):
    """Model and input of a test mode; head modes use 3 heads (d_model 96) and batch 1."""
    from mamba3_b200 import Mamba3

    torch.manual_seed(0)
    if mode.startswith("context"):  # one sequence of 150 tokens, split 128 + 22 along its length
        model = Mamba3(32, d_state=16, depth=2, mimo_rank=4 if mode == "context_mimo" else 1).eval()
        return model, torch.randn(2, 150, 32, generator=torch.Generator().manual_seed(1))
    if mode.startswith("heads"):
        model = Mamba3(96, d_state=16, depth=2, mimo_rank=2 if mode == "heads_mimo" else 1,
                       causal=mode != "heads_bidir").eval()
        return model, torch.randn(1, 21, 96, generator=torch.Generator().manual_seed(1))
    model = Mamba3(32, d_state=16, depth=2, mimo_rank=2 if mode == "mimo" else 1).eval()
    return model, torch.randn(3, 21, 32, generator=torch.Generator().manual_seed(1))


def _worker(rank, world, port, mode, out_dir):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from mamba3_b200.context import forward_context_parallel
    from mamba3_b200.shard import forward_head_sharded, forward_sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    model, x = _case(mode)
    try:
        if mode == "fail" and rank == 1:
            raise SystemExit(3)  # this rank dies before the gather
        with torch.no_grad():
            if mode.startswith("context"):
                y = forward_context_parallel(model, x[:, :128] if rank == 0 else x[:, 128:])
            else:
                y = (forward_head_sharded if mode.startswith("heads") else forward_sharded)(model, x)
        torch.save(y, Path(out_dir) / f"y{rank}.pt")
    except RuntimeError as error:  # the survivor's collective timed out / saw the peer close
        (Path(out_dir) / f"err{rank}.txt").write_text(str(error))
    finally:
        if not (mode == "fail" and rank == 1):
            dist.destroy_process_group()


def test_shard_bounds_cover_the_batch_once():
    for batch in (0, 1, 3, 8, 17):
        for world in (1, 2, 4, 8):
            spans = [shard_bounds(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


@pytest.mark.parametrize("mode", ["siso", "mimo", "heads", "heads_mimo", "heads_bidir", "context", "context_mimo"])
def test_two_rank_sharded_forward_equals_single_process(tmp_path, mode):
    """Batch sharding, (modes "heads*") head sharding of a batch-1 input over 3 heads, and (modes
    "context*") context parallelism: each rank holds a slice of the sequence length."""
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, mode, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    model, x = _case(mode)
    assert not mode.startswith("heads") or model.layers[0].mixer.nheads == 3
    with torch.no_grad():
        expected = model(x)
    for rank in range(2):
        got = torch.load(tmp_path / f"y{rank}.pt")
        if mode.startswith("context"):
            want = expected[:, :128] if rank == 0 else expected[:, 128:]
            torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5)
        else:
            torch.testing.assert_close(got, expected, rtol=1e-5, atol=1e-6)


def test_dead_rank_fails_the_gather_instead_of_hanging(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_worker, args=(2, port, "fail", str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    assert all(not p.is_alive() for p in ctx.processes)
    assert ctx.processes[1].exitcode == 3
    assert (tmp_path / "err0.txt").exists() and not (tmp_path / "y0.pt").exists()


def test_mixed_heads_partition_equals_the_full_mixer():
    """Concatenating the per-range SSD outputs of a mixer gives the mixer's output (single process)."""
    model, x = _case("heads_bidir")
    mixer = model.layers[0].mixer
    hidden = model.layers[0].norm(x)
    with torch.no_grad():
        for reverse in (False, True):
            parts = torch.cat([mixer.mixed_heads(hidden, 0, 2, reverse=reverse),
                               mixer.mixed_heads(hidden, 2, 3, reverse=reverse)], dim=2)
            assert parts.shape == (1, 21, 3, mixer.headdim)
            blend = torch.sigmoid(mixer.direction_logit)
            if reverse:
                rev = parts
            else:
                fwd = parts
        out = mixer.out_proj(fwd.flatten(-2)) * blend + mixer.out_proj(rev.flatten(-2)) * (1 - blend)
        torch.testing.assert_close(out, mixer(hidden), rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError, match="head range"):
        mixer.mixed_heads(hidden, 2, 4)

"""Multi-process batch sharding on CPU (gloo, world size 2): outputs equal the single-process
forward, uneven batches work, and a rank that dies before the gather makes the survivor's
collective fail within its timeout instead of hanging."""

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


def _worker(rank, world, port, mode, out_dir):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from mamba3_b200 import Mamba3
    from mamba3_b200.shard import forward_sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    torch.manual_seed(0)
    model = Mamba3(32, d_state=16, depth=2, mimo_rank=2 if mode == "mimo" else 1).eval()
    x = torch.randn(3, 21, 32, generator=torch.Generator().manual_seed(1))
    try:
        if mode == "fail" and rank == 1:
            raise SystemExit(3)  # this rank dies before the gather
        with torch.no_grad():
            y = forward_sharded(model, x)
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


@pytest.mark.parametrize("mode", ["siso", "mimo"])
def test_two_rank_sharded_forward_equals_single_process(tmp_path, mode):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, mode, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    from mamba3_b200 import Mamba3

    torch.manual_seed(0)
    model = Mamba3(32, d_state=16, depth=2, mimo_rank=2 if mode == "mimo" else 1).eval()
    x = torch.randn(3, 21, 32, generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        expected = model(x)
    for rank in range(2):
        got = torch.load(tmp_path / f"y{rank}.pt")
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

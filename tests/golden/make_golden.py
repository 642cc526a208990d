"""Generate the golden fixtures in this folder by running the reference package.

Run once in a container that holds the reference checkout (it is not needed
afterwards, and the GPU box never runs this script):

    MAMBA3_REFERENCE=/path/to/jreoka-mamba3 python tests/golden/make_golden.py

The reference is imported from ``$MAMBA3_REFERENCE`` with its Triton path
disabled, so every number comes from its portable PyTorch implementation on
CPU in float32 (``mamba3/ops.py`` mamba3_scan / mamba3_step / rotate_qk and
``mamba3/model.py`` Mamba3). Each fixture is one ``.npz`` file of float32
arrays plus a few integer scalars describing the case.
"""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _import_reference():
    root = os.environ.get("MAMBA3_REFERENCE")
    if not root:
        raise SystemExit("set MAMBA3_REFERENCE to the reference checkout")
    os.environ["MAMBA3_DISABLE_TRITON"] = "1"
    sys.path.insert(0, root)
    import mamba3  # noqa: F401
    import mamba3.ops as ops
    from mamba3 import Mamba3
    return ops, Mamba3


def _np(t):
    if t is None:
        return None
    return t.detach().float().cpu().numpy()


def _save(name: str, **arrays) -> None:
    clean = {k: (np.asarray(v) if not isinstance(v, np.ndarray) else v) for k, v in arrays.items() if v is not None}
    np.savez_compressed(HERE / f"{name}.npz", **clean)
    size = (HERE / f"{name}.npz").stat().st_size
    print(f"{name}.npz  {size / 1024:.1f} KiB  keys={sorted(clean)}")


def scan_inputs(rank, batch, length, heads, head_dim, d_state, seed, groups=1, angles=0, with_cache=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, length, groups, rank, d_state, generator=g)
    k = torch.randn(batch, length, groups, rank, d_state, generator=g)
    value = torch.randn(batch, length, heads, head_dim, generator=g)
    gate = torch.randn(batch, length, heads, head_dim, generator=g)
    adt = -torch.rand(batch, length, heads, generator=g) * 0.2
    dt = torch.rand(batch, length, heads, generator=g) * 0.1 + 0.001
    trap = torch.randn(batch, length, heads, generator=g)
    D = torch.randn(heads, generator=g)
    out = dict(q=q, k=k, value=value, gate=gate, adt=adt, dt=dt, trap=trap, D=D)
    if rank > 1:
        out["mimo_x"] = torch.randn(heads, rank, head_dim, generator=g) / rank
        out["mimo_z"] = torch.randn(heads, rank, head_dim, generator=g)
        out["mimo_out"] = torch.randn(heads, rank, head_dim, generator=g) / rank
    if angles:
        out["phase"] = (torch.rand(batch, length, heads, angles, generator=g) * 4 - 2) * math.pi
        out["q_bias"] = 1.0 + 0.1 * torch.randn(heads, rank, d_state, generator=g)
        out["k_bias"] = 1.0 + 0.1 * torch.randn(heads, rank, d_state, generator=g)
    if with_cache:
        out["initial_state"] = 0.1 * torch.randn(batch, heads, head_dim, d_state, generator=g)
        out["initial_k"] = torch.randn(batch, heads, rank, d_state, generator=g)
        out["initial_value"] = torch.randn(batch, heads, head_dim, generator=g)
    return out


def make_scans(ops) -> None:
    cases = [
        # name, rank, B, L, H, P, N, groups, angles, cache, chunk
        ("scan_small_r1", 1, 2, 7, 3, 4, 8, 1, 0, False, 3),
        ("scan_small_r4", 4, 2, 7, 3, 4, 8, 1, 0, False, 2),
        ("scan_small_r4_c5", 4, 2, 7, 3, 4, 8, 1, 0, False, 5),
        ("scan_cont_r1", 1, 2, 9, 3, 4, 8, 3, 0, True, 3),
        ("scan_kernel_r1", 1, 1, 300, 2, 64, 128, 1, 32, True, 256),
        ("scan_kernel_r4", 4, 1, 90, 2, 64, 128, 1, 32, True, 32),
        ("scan_kernel_r2", 2, 1, 100, 2, 64, 128, 2, 32, False, 64),
        ("scan_n16_r1", 1, 2, 37, 2, 64, 16, 1, 4, True, 256),
    ]
    for name, rank, b, l, h, p, n, groups, angles, cache, chunk in cases:
        inp = scan_inputs(rank, b, l, h, p, n, seed=1000 + len(name) * 7 + rank, groups=groups,
                          angles=angles, with_cache=cache)
        kwargs = {key: inp.get(key) for key in ("mimo_x", "mimo_z", "mimo_out", "initial_state", "initial_k",
                                                "initial_value", "phase", "q_bias", "k_bias")}
        y, state = ops.mamba3_scan(inp["q"], inp["k"], inp["value"], inp["gate"], inp["adt"], inp["dt"],
                                   inp["trap"], inp["D"], chunk_size=chunk, mimo_rotation=rank > 1, **kwargs)
        _save(name, chunk=chunk, **{key: _np(val) for key, val in inp.items()}, y=_np(y), state=_np(state))


def make_rotation(ops) -> None:
    q = torch.tensor([[[[[1.0, 0.0, 2.0, 0.0, 5.0, 6.0, 7.0, 8.0]]]]])
    phase = torch.tensor([[[[math.pi / 2, 0.0]]]])
    siso, _ = ops.rotate_qk(q, q, phase, mimo=False)
    qm = torch.tensor([[[[[1.0, 2.0, 3.0, 4.0, 0.0, 5.0, 6.0, 7.0]]]]])
    mimo, _ = ops.rotate_qk(qm, qm, phase, mimo=True)
    g = torch.Generator().manual_seed(7)
    t = torch.randn(2, 3, 2, 4, 128, generator=g)
    ph = torch.rand(2, 3, 2, 32, generator=g) * 12 - 6
    rs, _ = ops.rotate_qk(t, t, ph, mimo=False)
    rm, _ = ops.rotate_qk(t, t, ph, mimo=True)
    x = torch.tensor([-3.0, -0.5, 0.0, 0.5, 3.0])
    _save("rotation", siso_in=_np(q), mimo_in=_np(qm), phase=_np(phase), siso=_np(siso), mimo=_np(mimo),
          rand_in=_np(t), rand_phase=_np(ph), rand_siso=_np(rs), rand_mimo=_np(rm),
          heavy_in=_np(x), heavy=_np(ops.heavy_tail_activation(x)))


def make_steps(ops) -> None:
    for rank in (1, 4):
        g = torch.Generator().manual_seed(50 + rank)
        b, h, p, n, s = 2, 3, 64, 128, 32
        q = torch.randn(b, h, rank, n, generator=g)
        k = torch.randn(b, h, rank, n, generator=g)
        value = torch.randn(b, h, p, generator=g)
        gate = torch.randn(b, h, p, generator=g)
        adt = -torch.rand(b, h, generator=g) * 0.3
        dt = torch.rand(b, h, generator=g) * 0.1 + 0.001
        trap = torch.randn(b, h, generator=g)
        angle_rate = torch.randn(b, s, generator=g) * 3
        D = torch.randn(h, generator=g)
        cache = ((torch.rand(b, h, s, generator=g) * 4 - 2) * math.pi, 0.1 * torch.randn(b, h, p, n, generator=g),
                 torch.randn(b, h, rank, n, generator=g), torch.randn(b, h, p, generator=g))
        mimo = {}
        if rank > 1:
            mimo = dict(mimo_x=torch.randn(h, rank, p, generator=g) / rank,
                        mimo_z=torch.randn(h, rank, p, generator=g),
                        mimo_out=torch.randn(h, rank, p, generator=g) / rank)
        # The portable decode path of mamba3/model.py:460-484.
        inc = torch.fmod(math.pi * torch.tanh(angle_rate).unsqueeze(1) * dt.unsqueeze(-1), 2.0 * math.pi)
        phase = torch.fmod(cache[0] + inc, 2.0 * math.pi)
        qr, kr = ops.rotate_qk(q[:, None], k[:, None], phase[:, None], mimo=rank > 1)
        y, nxt = ops.mamba3_step(qr[:, 0], kr[:, 0], value, gate, adt, dt, trap, D,
                                 (phase, cache[1], cache[2], cache[3]), **mimo)
        _save(f"step_r{rank}", q=_np(q), k=_np(k), value=_np(value), gate=_np(gate), adt=_np(adt), dt=_np(dt),
              trap=_np(trap), angle_rate=_np(angle_rate), D=_np(D), phase0=_np(cache[0]), state0=_np(cache[1]),
              k0=_np(cache[2]), v0=_np(cache[3]), **{key: _np(val) for key, val in mimo.items()}, y=_np(y),
              phase1=_np(nxt[0]), state1=_np(nxt[1]), k1=_np(nxt[2]), v1=_np(nxt[3]))


def make_models(Mamba3) -> None:
    cases = [
        # name, d_model, d_state, depth, rank, causal, batch, length, split
        ("model_r1", 64, 128, 2, 1, True, 2, 40, 25),
        ("model_r4", 64, 128, 1, 4, True, 2, 40, 25),
        ("model_n16_r1", 64, 16, 1, 1, True, 2, 37, 9),
        ("model_n16_r4", 64, 16, 1, 4, True, 2, 37, 9),
        ("model_bidir", 64, 128, 1, 1, False, 2, 33, 0),
    ]
    for name, d_model, d_state, depth, rank, causal, batch, length, split in cases:
        torch.manual_seed(0)
        model = Mamba3(d_model, d_state=d_state, depth=depth, mimo_rank=rank, causal=causal).eval()
        g = torch.Generator().manual_seed(99)
        x = torch.randn(batch, length, d_model, generator=g)
        extra = {}
        with torch.inference_mode():
            y = model(x)
            if causal:
                prefix, cache = model.prefill(x[:, :split])
                outs = [prefix]
                for t in range(split, length):
                    o, cache = model.step(x[:, t:t + 1], cache)
                    outs.append(o)
                extra["continued"] = _np(torch.cat(outs, dim=1))
                for i, layer in enumerate(cache):
                    for j, tensor in enumerate(layer):
                        extra[f"cache{i}_{j}"] = _np(tensor)
        sd = {f"sd.{key}": _np(val) for key, val in model.state_dict().items()}
        _save(name, d_model=d_model, d_state=d_state, depth=depth, rank=rank, causal=int(causal), split=split,
              x=_np(x), y=_np(y), **extra, **sd)


def make_phase(Mamba3) -> None:
    torch.manual_seed(0)
    mixer = Mamba3(64, d_state=128, depth=1).layers[0].mixer
    g = torch.Generator().manual_seed(5)
    angles = torch.randn(2, 300, mixer.num_angles, generator=g) * 2
    dt = torch.rand(2, 300, mixer.nheads, generator=g) * 3
    initial = (torch.rand(2, mixer.nheads, mixer.num_angles, generator=g) * 4 - 2) * math.pi
    phase = mixer._phase(angles, dt, initial)
    _save("phase", angles=_np(angles), dt=_np(dt), initial=_np(initial), phase=_np(phase))


def main() -> None:
    ops, Mamba3 = _import_reference()
    torch.set_num_threads(4)
    make_rotation(ops)
    make_scans(ops)
    make_steps(ops)
    make_phase(Mamba3)
    make_models(Mamba3)


if __name__ == "__main__":
    main()

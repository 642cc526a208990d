"""Seeded inputs of the chunked SSD for the training-path tests (shared by the CPU and GPU files)."""

from __future__ import annotations

import torch


def scan_case(rank: int, *, batch=2, length=45, heads=4, groups=1, d_state=32, head_dim=16, angles=4,
              cache=True, seed=0, dtype=torch.float32, device="cpu"):
    """(args, kwargs) of ``mamba3_scan`` with every optional input present; float tensors that can
    carry gradients are leaves with ``requires_grad``."""
    g = torch.Generator().manual_seed(seed)
    t = lambda *s, scale=1.0: (torch.randn(*s, generator=g) * scale)
    leaf = lambda x, low=False: (x.to(dtype) if low else x).to(device).requires_grad_(True)
    q = leaf(t(batch, length, groups, rank, d_state), True)
    k = leaf(t(batch, length, groups, rank, d_state), True)
    value = leaf(t(batch, length, heads, head_dim), True)
    gate = leaf(t(batch, length, heads, head_dim), True)
    adt = leaf(-torch.rand(batch, length, heads, generator=g) * 0.5)
    dt = leaf(torch.rand(batch, length, heads, generator=g) * 0.5 + 0.05)
    trap = leaf(t(batch, length, heads), True)
    D = leaf(t(heads))
    kw = dict(chunk_size=16, mimo_rotation=rank > 1)
    if rank > 1:
        kw.update(mimo_x=leaf(t(heads, rank, head_dim, scale=0.5)), mimo_z=leaf(t(heads, rank, head_dim)),
                  mimo_out=leaf(t(heads, rank, head_dim, scale=0.5)))
    kw.update(q_bias=leaf(t(heads, rank, d_state, scale=0.3)), k_bias=leaf(t(heads, rank, d_state, scale=0.3)),
              phase=leaf(t(batch, length, heads, angles, scale=2.0)))
    if cache:
        kw.update(initial_state=leaf(t(batch, heads, head_dim, d_state, scale=0.2)),
                  initial_k=leaf(t(batch, heads, rank, d_state), True),
                  initial_value=leaf(t(batch, heads, head_dim), True))
    return (q, k, value, gate, adt, dt, trap, D), kw


def leaves(args, kw):
    out = [a for a in args] + [v for v in kw.values() if isinstance(v, torch.Tensor)]
    return [x for x in out if x.requires_grad]

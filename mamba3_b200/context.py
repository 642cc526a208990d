"""Context-parallel prefill: one long sequence split along its length across ranks.

Rank r holds the slice ``[r * Ls, (r + 1) * Ls)`` of every sequence (``Ls`` a multiple of the
64-token phase block; the last rank may hold a shorter tail). Per layer each rank

1. projects its slice (``in_proj``) and runs the scan's state pass over it from a zero state and
   zero phase (``m3_scan_summary``): end state, biased last k rotated by the slice's own phases,
   endpoint weight ``dt (1 - sigmoid(trap))`` of its first token, total log-decay and the sum of its
   64-token block phase totals;
2. all-gathers those summaries (one NCCL collective of ``B * H * (P * N + ...)`` floats per rank,
   independent of the slice length);
3. folds the summaries of the ranks before it into its initial cache (:func:`fold_prefix`) and runs
   the ordinary scan on its slice as a continuation from that cache.

The fold is the chunked state carry of mamba3/ops.py:804-816 applied to whole slices, with the
exp-trapezoidal endpoint term of each slice boundary added as in a prefill continuation
(ops.py:679-686), and every slice's local state and k rotated by the phase its slice started from
(rotating every k of a slice by one angle rotates its whole state contribution by that angle; pair
layout of mamba3/ops.py:35-84).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _ext
from .ops import rotate_qk

_P, _N, _PHASE_SLOTS = 64, 128, 32


def unpack_records(record: torch.Tensor, rank: int):
    """(end state [B,H,P,N], last rotated k [B,H,R,N], endpoint weight c0 [B,H], log-decay [B,H]) of
    ``m3_scan_summary`` records ``[B, H, floats]``."""
    b, h = record.shape[:2]
    state = record[..., : _P * _N].reshape(b, h, _P, _N)
    k0 = _P * _N + _PHASE_SLOTS
    k = record[..., k0: k0 + rank * _N].reshape(b, h, rank, _N)
    c0 = record[..., k0 + rank * _N]
    decay = record[..., k0 + rank * _N + 1]
    return state, k, c0, decay


def rotate_rows(t: torch.Tensor, phase: torch.Tensor, mimo: bool) -> torch.Tensor:
    """Rotate the last (N) axis of ``t [B, H, M, N]`` by ``phase [B, H, S]`` with the rotation pairs
    of the scan (SISO (2i, 2i+1), MIMO (i, 2S + i))."""
    x = t.unsqueeze(1)
    ph = phase.unsqueeze(1)
    out, _ = rotate_qk(x, x, ph, mimo=mimo)
    return out[:, 0]


def fold_prefix(summaries: list[dict], *, mimo: bool, mimo_x: torch.Tensor | None,
                initial_phase: torch.Tensor | None = None):
    """Initial cache (phase, state, rotated k, value) of the slice that follows ``summaries``.

    Each summary (in slice order) holds ``state`` [B,H,P,N], ``k`` [B,H,R,N] (rotated by the
    slice's own phases), ``c0`` [B,H], ``decay`` [B,H], ``phase_total`` [B,H,S] (the slice's summed
    block phase totals) and ``x_last`` [B,H,P] (its last value row). The first slice's summary was
    taken from the true initial cache (state, k already true); later ones from zeros.
    """
    first = summaries[0]
    b, h = first["state"].shape[:2]
    s_count = first["phase_total"].shape[-1]
    phase = (torch.zeros(b, h, s_count, device=first["state"].device, dtype=torch.float64)
             if initial_phase is None else initial_phase.double())
    state, k = first["state"].float(), first["k"].float()
    phase = torch.fmod(phase + first["phase_total"].double(), 2.0 * math.pi)
    x_last = first["x_last"].float()
    for summ in summaries[1:]:
        ph = phase.float()
        xr = x_last.unsqueeze(2) if mimo_x is None else x_last.unsqueeze(2) * mimo_x.float()[None]  # [B,H,R,P]
        outer = torch.einsum("bhrp,bhrn->bhpn", xr, k)
        local = rotate_rows(summ["state"].float(), ph, mimo)
        state = torch.exp(summ["decay"].float())[..., None, None] * (state + summ["c0"].float()[..., None, None] * outer)
        state = state + local
        k = rotate_rows(summ["k"].float(), ph, mimo)
        phase = torch.fmod(phase + summ["phase_total"].double(), 2.0 * math.pi)
        x_last = summ["x_last"].float()
    return phase.float(), state, k, x_last


def _slice_summary(mixer, projected: torch.Tensor) -> dict:
    """Summary of this rank's slice for one mixer (model mode: raw in_proj columns)."""
    sizes, tensors, kw = mixer._scan_arguments(projected, None)
    record, blocks = _ext.scan_summary(sizes=sizes, tensors=tensors, **kw)
    state, k, c0, decay = unpack_records(record, mixer.mimo_rank)
    total = (blocks.double().sum(dim=2) if blocks is not None else
             torch.zeros(*record.shape[:2], _PHASE_SLOTS, device=record.device, dtype=torch.float64))
    x = projected[..., mixer.d_inner: 2 * mixer.d_inner].unflatten(-1, (mixer.nheads, mixer.headdim))
    return dict(state=state, k=k, c0=c0, decay=decay, phase_total=total[..., : mixer.num_angles].float(),
                x_last=x[:, -1].float())


def _slice_summary_torch(mixer, hidden: torch.Tensor) -> dict:
    """The same summary with the PyTorch formulation (CPU tensors and autograd calls)."""
    _, state, phase, q, k, x = mixer._scan_torch_direction(hidden, None)
    _, _, _, _, adt, dt, trap, angles = mixer._project(hidden)
    q_last, k_last = mixer._expand_qk(q[:, -1:], k[:, -1:])
    _, k_rot = rotate_qk(q_last, k_last, phase[:, -1:], mimo=mixer.mimo_rank > 1)
    inc = torch.fmod(math.pi * torch.tanh(angles.double()).unsqueeze(2) * dt.double().unsqueeze(-1), 2 * math.pi)
    c0 = dt[:, 0].float() * (1.0 - torch.sigmoid(trap[:, 0].float()))
    return dict(state=state.float(), k=k_rot[:, 0].float(), c0=c0, decay=adt.float().sum(dim=1),
                phase_total=inc.sum(dim=1).float(), x_last=x[:, -1].float())


def _pack(summary: dict) -> torch.Tensor:
    return torch.cat([summary[key].reshape(summary[key].shape[0], summary[key].shape[1], -1).float()
                      for key in ("state", "k", "c0", "decay", "phase_total", "x_last")], dim=-1)


def _unpack(flat: torch.Tensor, like: dict) -> dict:
    out, off = {}, 0
    for key in ("state", "k", "c0", "decay", "phase_total", "x_last"):
        shape = like[key].shape
        width = 1 if len(shape) == 2 else int(torch.tensor(shape[2:]).prod())
        out[key] = flat[..., off: off + width].reshape(shape)
        off += width
    return out


def mixer_context_parallel(mixer, hidden: torch.Tensor, group=None) -> torch.Tensor:
    """One causal mixer on this rank's slice ``hidden [B, Ls, D]`` of a sequence split across the
    ranks of ``group`` in rank order; returns the mixer output for the slice."""
    if not mixer.causal:
        raise ValueError("context-parallel prefill needs a causal mixer")
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    kernels = mixer._use_kernels(hidden)
    projected = mixer._project_linear("in_proj", hidden) if kernels else None
    cache = None
    if world > 1:
        summ = _slice_summary(mixer, projected) if kernels else _slice_summary_torch(mixer, hidden)
        flat = _pack(summ).contiguous()
        parts = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(parts, flat, group=group)
        if rank > 0:
            prefix = [_unpack(p, summ) for p in parts[:rank]]
            phase, state, k, x_last = fold_prefix(prefix, mimo=mixer.mimo_rank > 1, mimo_x=mixer.mimo_x)
            act = projected.dtype if kernels else hidden.dtype
            cache = (phase, state, k.to(act), x_last.to(act))
    if not kernels:  # the PyTorch formulation (CPU tensors, autograd)
        return mixer(hidden, cache=cache)
    mixed = mixer._scan_fused(projected, cache, reverse=False, want_cache=False)[0]
    return mixer._project_linear("out_proj", mixed.flatten(-2))


def forward_context_parallel(model, x_local: torch.Tensor, group=None) -> torch.Tensor:
    """``Mamba3.forward`` of a sequence whose length is split across the ranks of ``group``: every
    rank passes its slice ``x_local [B, Ls, D]`` (rank order = sequence order; every slice but the
    last a multiple of 64 tokens) and receives the output of its slice. One all-gather of the slice
    summaries per layer; no activations cross ranks."""
    x = x_local
    for layer in model.layers:
        x = x + mixer_context_parallel(layer.mixer, layer.norm(x), group)
    return model.norm_f(x)

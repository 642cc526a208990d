"""Batch sharding of Mamba3 over one process per GPU.

Every (sequence, head) scan is independent, so the sequences of a batch split across ranks with no
exchange during the layers: each rank runs the whole model on its contiguous slice of the batch and
one all-gather at the end assembles the full output (over NCCL/NVLink on GPUs; gloo in CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous near-equal split: the first ``batch % world`` ranks get one extra sequence."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def all_gather_batch(local: torch.Tensor, batch: int, group=None) -> torch.Tensor:
    """All-gather the per-rank batch shards ``local`` (this rank's ``shard_bounds`` share of a batch of
    ``batch``) into the full batch on every rank. Shards are padded to the widest share so one
    fixed-size NCCL all-gather moves them."""
    world = dist.get_world_size(group)
    widest = -(-batch // world)
    padded = local if local.shape[0] == widest else torch.cat(
        (local, local.new_zeros((widest - local.shape[0], *local.shape[1:]))))
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    pieces = []
    for r, part in enumerate(parts):
        s, e = shard_bounds(batch, world, r)
        pieces.append(part[: e - s])
    return torch.cat(pieces, dim=0)


def forward_local_gather(model, x_local: torch.Tensor, batch: int, group=None) -> torch.Tensor:
    """``model`` on this rank's shard ``x_local`` of a batch of ``batch`` sequences, then the all-gather
    of the outputs: the full ``model(x)`` on every rank, each rank having read only its own inputs."""
    if x_local.shape[0] > 0:
        local = model(x_local)
    else:  # an empty share still joins the gather
        local = x_local.new_empty((0, *x_local.shape[1:]))
    return all_gather_batch(local, batch, group)


def forward_sharded(model, x: torch.Tensor, group=None) -> torch.Tensor:
    """Run ``model`` on this rank's share of the batch of ``x`` and all-gather the full output.

    ``x`` is the full batch (every rank passes the same tensor, or at least the same shape); the
    result is the full ``model(x)`` on every rank. Ranks with an empty share still take part in
    the gather.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    batch = x.shape[0]
    start, stop = shard_bounds(batch, world, rank)
    return forward_local_gather(model, x[start:stop], batch, group)


def _gather_heads(local: torch.Tensor, heads: int, world: int, group) -> torch.Tensor:
    """All-gather ``[B, L, h_r, P]`` head shards (near-equal split of ``heads``) into ``[B, L, heads, P]``."""
    widest = -(-heads // world)
    padded = local.new_zeros((*local.shape[:2], widest, local.shape[3]))
    padded[:, :, : local.shape[2]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    pieces = []
    for r, part in enumerate(parts):
        s, e = shard_bounds(heads, world, r)
        pieces.append(part[:, :, : e - s])
    return torch.cat(pieces, dim=2)


def forward_head_sharded(model, x: torch.Tensor, group=None) -> torch.Tensor:
    """``model(x)`` with the heads of every mixer split across ranks: the fallback when the batch is
    smaller than the number of GPUs (batch 1 prefill).

    Each rank computes the replicated parts (norms, in_proj, out_proj, residual) in full and the scan
    of its contiguous share of the heads; one all-gather of the mixer output ``[B, L, H, P]`` along
    heads per layer and direction precedes out_proj. Every rank passes the same ``x`` and receives
    the full output.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    for layer in model.layers:
        mixer = layer.mixer
        h0, h1 = shard_bounds(mixer.nheads, world, rank)
        hidden = layer.norm(x)

        def direction(reverse: bool) -> torch.Tensor:
            if h1 > h0:
                local = mixer.mixed_heads(hidden, h0, h1, reverse=reverse)
            else:  # more ranks than heads: an empty share still joins the gather
                local = hidden.new_empty((*hidden.shape[:2], 0, mixer.headdim))
            mixed = _gather_heads(local, mixer.nheads, world, group)
            return mixer._project_linear("out_proj", mixed.flatten(-2))

        out = direction(False)
        if not mixer.causal:
            blend = torch.sigmoid(mixer.direction_logit).to(out.dtype)
            out = out * blend + direction(True) * (1.0 - blend)
        x = x + out
    return model.norm_f(x)

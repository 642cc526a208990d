"""Mamba-3 SSD operators: the B200 kernels on CUDA, a differentiable PyTorch form elsewhere.

Public operator surface (same names, arguments, shapes and errors as ``mamba3/ops.py`` of
jreoka/mamba3): :func:`heavy_tail_activation`, :func:`rotate_qk`, :func:`fused_step`,
:func:`mamba3_scan`, :func:`mamba3_step`.

Dispatch rule. Inference calls on CUDA tensors (no tensor that requires grad while grad mode is
on) run the sm_100a kernels of ``csrc/`` through the C ABI — there is no other GPU path and no
silent fallback: if the library is missing the call raises. Calls on CUDA tensors that need
autograd (training) run the chunked core on the training kernels (``m3_ssd_train_fwd/bwd``) with
the elementwise prelude and epilogue as PyTorch ops (d_state <= 128 and head_dim <= 64; other shapes
take the PyTorch formulation). Calls on CPU tensors run the PyTorch formulation below (the CPU
device path, as in the reference, ``mamba3/ops.py:659-822``).
"""

from __future__ import annotations

import math

import torch
from torch.nn import functional as F

from . import _ext

TWO_PI = 2.0 * math.pi

# Set by every call: True when the last scan / step ran through the CUDA library.
LAST_SCAN_DISPATCH = False
LAST_STEP_DISPATCH = False


def heavy_tail_activation(x: torch.Tensor) -> torch.Tensor:
    """Positive heavy-tail map: 1 + x for x >= 0 and 1 / (1 - x) below (mamba3/ops.py:28-32)."""
    below = 1.0 / (1.0 - torch.clamp(x, max=0.0))
    return torch.where(x >= 0, x + 1.0, below)


def rotate_qk(q: torch.Tensor, k: torch.Tensor, phase: torch.Tensor, *, mimo: bool):
    """Rotate q/k ``[B, L, H, R, N]`` by ``phase`` ``[B, L, H, S]`` in real coordinates.

    SISO rotates adjacent pairs (2i, 2i+1); MIMO rotates (i, 2S+i) (the split-half checkpoint
    layout), leaving the other coordinates unchanged (mamba3/ops.py:35-84). cos/sin are cast to
    the q dtype before use, as in the reference.
    """
    if q.ndim != 5 or q.shape != k.shape:
        raise ValueError("q and k must have matching [B, L, H, R, N] shapes")
    if phase.ndim != 4 or phase.shape[:3] != q.shape[:3]:
        raise ValueError("phase must have shape [B, L, H, S]")
    count = phase.shape[-1]
    if (4 if mimo else 2) * count > q.shape[-1]:
        raise ValueError("phase has too many angles for the Q/K state width")
    cos = torch.cos(phase).unsqueeze(3).to(q.dtype)
    sin = torch.sin(phase).unsqueeze(3).to(q.dtype)

    def turn(t: torch.Tensor) -> torch.Tensor:
        if mimo:
            a = t[..., :count]
            b = t[..., 2 * count:3 * count]
            return torch.cat((a * cos - b * sin, t[..., count:2 * count], a * sin + b * cos, t[..., 3 * count:]),
                             dim=-1)
        pairs = t[..., :2 * count].unflatten(-1, (count, 2))
        a, b = pairs[..., 0], pairs[..., 1]
        turned = torch.stack((a * cos - b * sin, a * sin + b * cos), dim=-1).flatten(-2)
        return torch.cat((turned, t[..., 2 * count:]), dim=-1)

    return turn(q), turn(k)


def _needs_autograd(*tensors) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _kernel_eligible(*tensors) -> bool:
    """CUDA inference call: the kernels own it."""
    first = tensors[0]
    return first.is_cuda and not _needs_autograd(*tensors)


def _rank_values(value: torch.Tensor, projection: torch.Tensor | None) -> torch.Tensor:
    """[..., H, P] -> [..., H, R, P] (mamba3/ops.py:193-199), in float32."""
    value = value.float()
    if projection is None:
        return value.unsqueeze(-2)
    return value.unsqueeze(-2) * projection.float()


def _expand_groups(t: torch.Tensor, heads: int) -> torch.Tensor:
    groups = t.shape[2]
    if groups == heads:
        return t
    if groups == 1:
        return t.expand(-1, -1, heads, -1, -1)
    return t.repeat_interleave(heads // groups, dim=2)


# ---------------------------------------------------------------------------
# Chunked scan
# ---------------------------------------------------------------------------


def _validate_scan(q, k, value, gate, adt, dt, trap_logits, D, mimo_x, mimo_z, mimo_out, chunk_size,
                   initial_state, initial_k, initial_value, phase, q_bias, k_bias):
    """Argument checks of mamba3/ops.py:574-631 (same messages)."""
    if q.ndim != 5 or q.shape != k.shape:
        raise ValueError("q and k must have matching [B, L, G, R, N] shapes")
    batch, length, groups, rank, d_state = q.shape
    if value.ndim != 4 or gate.shape != value.shape:
        raise ValueError("value and gate must have matching [B, L, H, P] shapes")
    if value.shape[:2] != (batch, length):
        raise ValueError("value dimensions must match q and k")
    heads, head_dim = value.shape[2], value.shape[3]
    if heads % groups != 0:
        raise ValueError("value heads must be divisible by Q/K groups")
    if adt.shape != (batch, length, heads):
        raise ValueError("adt must have shape [B, L, H]")
    if dt.shape != adt.shape or trap_logits.shape != adt.shape:
        raise ValueError("dt and trap_logits must match adt")
    if D.shape != (heads,):
        raise ValueError("D must have shape [H]")
    if (q_bias is None) != (k_bias is None):
        raise ValueError("q_bias and k_bias must be provided together")
    if q_bias is not None:
        want = (heads, rank, d_state)
        if q_bias.shape != want or k_bias.shape != want:
            raise ValueError(f"Q/K biases must have shape {want}")
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive")
    if phase is not None and (phase.ndim != 4 or phase.shape[:3] != (batch, length, heads)):
        raise ValueError("phase must have shape [B, L, H, S]")
    want_state = (batch, heads, head_dim, d_state)
    if initial_state is not None and initial_state.shape != want_state:
        raise ValueError(f"initial_state must have shape {want_state}")
    projections = (mimo_x, mimo_z, mimo_out)
    if rank == 1:
        if any(p is not None for p in projections):
            raise ValueError("SISO inputs must not provide MIMO projections")
    else:
        want = (heads, rank, head_dim)
        if any(p is None or p.shape != want for p in projections):
            raise ValueError(f"MIMO projections must have shape {want}")
    if initial_k is not None or initial_value is not None:
        want_k = (batch, heads, rank, d_state)
        want_v = (batch, heads, head_dim)
        if initial_k is None or initial_k.shape != want_k:
            raise ValueError(f"initial_k must have shape {want_k}")
        if initial_value is None or initial_value.shape != want_v:
            raise ValueError(f"initial_value must have shape {want_v}")


def _scalar_prelude(adt, dt, trap_logits):
    """sigma, gamma, scale, diag of mamba3/ops.py:659-671 (float32)."""
    sig = torch.sigmoid(trap_logits.float())
    dtf = dt.float()
    gamma = dtf * sig
    nxt = F.pad(dtf[:, 1:] * (1.0 - sig[:, 1:]), (0, 0, 0, 1))
    scale = gamma + nxt
    return sig, gamma, scale, gamma / scale


def _scan_torch(q, k, value, gate, adt, dt, trap_logits, D, *, mimo_x, mimo_z, mimo_out, chunk_size,
                initial_state, initial_k, initial_value, phase, mimo_rotation, q_bias, k_bias):
    """Differentiable chunked SSD with the reference's rounding schedule (mamba3/ops.py:659-822).

    Per chunk: inter-chunk term e^{cum} (Q S^T), masked decayed scores (Q (K*scale)^T) o L with
    the gamma/scale diagonal, D skip, SiLU gate, MIMO rank sum; then the state carry
    S <- e^{cum_last} S + V^T (K*scale*e^{cum_last - cum}).

    With bf16/fp16 activations the operands are rounded where the reference rounds them: ``scale``,
    the biased/rotated q/k, ``k*scale``, ``v*mimo_x`` and ``z*mimo_z`` in the activation dtype
    (ops.py:665-676, 719-745), the state read as ``state.to(q.dtype)`` (ops.py:754), the weighted
    scores as ``.to(value.dtype)`` (ops.py:787), ``k_scaled * end_decay.to(act)`` (ops.py:807);
    every product is accumulated in float32 and the state stays float32. With float32 activations
    every rounding is the identity.
    """
    batch, length, _, rank, d_state = q.shape
    heads, head_dim = value.shape[2], value.shape[3]
    act = value.dtype
    qf = _expand_groups(q, heads)
    kf = _expand_groups(k, heads)
    if q_bias is not None:
        qf = qf + q_bias.to(q.dtype)
        kf = kf + k_bias.to(k.dtype)
    if phase is not None:
        qf, kf = rotate_qk(qf, kf, phase, mimo=mimo_rotation)
    sig, _, scale, diag = _scalar_prelude(adt, dt, trap_logits)
    scale_act = scale.to(k.dtype)
    adtf = adt.float()
    dtf = dt.float()

    def rank_act(t, proj):  # [..., H, P] -> [..., H, R, P] in the activation dtype (ops.py:193-199)
        return t.unsqueeze(-2) if proj is None else t.unsqueeze(-2) * proj.to(t.dtype)

    rv = rank_act(value, mimo_x)  # [B, L, H, R, P]
    rz = rank_act(gate, mimo_z)
    state = (torch.zeros(batch, heads, head_dim, d_state, device=value.device, dtype=torch.float32)
             if initial_state is None else initial_state.float())
    if initial_k is not None:
        prev = rank_act(initial_value, mimo_x).float()
        coef = dtf[:, 0] * (1.0 - sig[:, 0])
        state = state + coef[..., None, None] * torch.einsum("bhrp,bhrn->bhpn", prev, initial_k.float())
    Dv = D.float()[None, :, None, None]
    mo = mimo_out.float()[None, :, None] if mimo_out is not None else None
    outputs = []
    for start in range(0, length, chunk_size):
        end = min(start + chunk_size, length)
        w = end - start
        rows = w * rank
        cum = torch.cumsum(adtf[:, start:end], dim=1).transpose(1, 2)  # [B, H, w]
        Qc = qf[:, start:end].permute(0, 2, 1, 3, 4).reshape(batch, heads, rows, d_state)
        Kc = (kf[:, start:end] * scale_act[:, start:end, :, None, None]).permute(0, 2, 1, 3, 4).reshape(
            batch, heads, rows, d_state)
        Vc = rv[:, start:end].permute(0, 2, 1, 3, 4).reshape(batch, heads, rows, head_dim)
        row_cum = cum.repeat_interleave(rank, dim=-1)  # [B, H, rows]
        inter = torch.matmul(Qc.float(), state.to(q.dtype).float().transpose(-1, -2)) * torch.exp(
            row_cum).unsqueeze(-1)
        scores = torch.matmul(Qc.float(), Kc.float().transpose(-1, -2))
        lower = torch.ones(w, w, dtype=torch.bool, device=q.device).tril(-1)
        gap = (cum.unsqueeze(-1) - cum.unsqueeze(-2)).masked_fill(~lower, -torch.inf)
        decay = torch.exp(gap) + torch.diag_embed(diag[:, start:end].transpose(1, 2))
        decay = decay.repeat_interleave(rank, dim=-1).repeat_interleave(rank, dim=-2)
        weighted = (scores * decay).to(act).float()
        y = inter + torch.matmul(weighted, Vc.float()) + Dv * Vc.float()
        y = y.reshape(batch, heads, w, rank, head_dim) * F.silu(rz[:, start:end].permute(0, 2, 1, 3, 4).float())
        y = y.sum(dim=3) if mo is None else (y * mo).sum(dim=3)
        outputs.append(y.transpose(1, 2).to(act))
        tail = torch.exp(row_cum[..., -1:] - row_cum).unsqueeze(-1)
        state_k = (Kc * tail.to(Kc.dtype)).float()
        state = torch.exp(cum[..., -1])[..., None, None] * state + torch.matmul(Vc.float().transpose(-1, -2), state_k)
    return torch.cat(outputs, dim=1), state


class _SSDCore(torch.autograd.Function):
    """The chunked SSD core on the training kernels (``m3_ssd_train_fwd`` / ``m3_ssd_train_bwd``):
    ``(q, k*scale, rank values, adt, diag, initial state) -> (pre-gate output [B,L,H,R,P], final
    state)``, float32. The forward keeps the state at every chunk start for the backward."""

    @staticmethod
    def forward(ctx, q, k, v, adt, diag, initial_state):
        y, final, chunks = _ext.ssd_train_forward(q, k, v, adt, diag, initial_state)
        ctx.save_for_backward(q, k, v, adt, diag, chunks)
        return y, final

    @staticmethod
    def backward(ctx, dy, dfinal):
        q, k, v, adt, diag, chunks = ctx.saved_tensors
        dy = torch.zeros_like(v) if dy is None else dy.float().contiguous()
        dfinal = None if dfinal is None else dfinal.float().contiguous()
        dq, dk, dv, dadt, ddiag, dinit = _ext.ssd_train_backward(q, k, v, adt, diag, chunks, dy, dfinal,
                                                                 want_initial=ctx.needs_input_grad[5])
        return dq, dk, dv, dadt, ddiag, dinit


class _Prelude(torch.autograd.Function):
    """Group expansion, bias, rotation and trapezoid scale of q / k on the prelude kernels
    (``m3_ssd_prelude_fwd`` / ``_bwd``): ``(q, k, q_bias, k_bias, phase, scale) -> (qf, k*scale)``
    as float32 ``[B,L,H,R,N]``."""

    @staticmethod
    def forward(ctx, q, k, q_bias, k_bias, phase, scale, heads, mimo_rotation):
        phase32 = None if phase is None else phase.float()
        qf, kc = _ext.ssd_prelude_forward(q, k, q_bias, k_bias, phase32, scale, heads, mimo_rotation)
        ctx.save_for_backward(q, k, q_bias, k_bias, phase32, scale)
        ctx.heads, ctx.mimo = heads, mimo_rotation
        ctx.phase_dtype = None if phase is None else phase.dtype
        return qf, kc

    @staticmethod
    def backward(ctx, dqf, dkc):
        q, k, q_bias, k_bias, phase, scale = ctx.saved_tensors
        shape = (*q.shape[:2], ctx.heads, *q.shape[3:])
        dqf = q.new_zeros(shape, dtype=torch.float32) if dqf is None else dqf.float().contiguous()
        dkc = torch.zeros_like(dqf) if dkc is None else dkc.float().contiguous()
        dqb, dkb, dphase, dscale = _ext.ssd_prelude_backward(q, k, q_bias, k_bias, phase, scale, ctx.heads, ctx.mimo,
                                                             dqf, dkc, want_phase=ctx.needs_input_grad[4])
        batch, length, groups, rank, n = q.shape
        per = ctx.heads // groups
        dq = dqb.view(batch, length, groups, per, rank, n).sum(3).to(q.dtype) if ctx.needs_input_grad[0] else None
        dk = dkb.view(batch, length, groups, per, rank, n).sum(3).to(k.dtype) if ctx.needs_input_grad[1] else None
        dqbias = dqb.sum((0, 1)).to(q_bias.dtype) if (q_bias is not None and ctx.needs_input_grad[2]) else None
        dkbias = dkb.sum((0, 1)).to(k_bias.dtype) if (k_bias is not None and ctx.needs_input_grad[3]) else None
        if dphase is not None:
            dphase = dphase.to(ctx.phase_dtype)
        return dq, dk, dqbias, dkbias, dphase, dscale, None, None


def _prelude_kernel_eligible(q, phase, mimo_rotation) -> bool:
    """CUDA calls whose shapes the prelude kernels serve (d_state <= 128, a multiple of 4; MIMO
    angle counts a multiple of 4)."""
    n = q.shape[-1]
    if not q.is_cuda or n > 128 or n % 4 or q.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        return False
    return phase is None or not mimo_rotation or phase.shape[-1] % 4 == 0


def _train_kernel_eligible(q, value) -> bool:
    """CUDA autograd calls whose shapes the training kernels serve (d_state <= 128, head_dim <= 64)."""
    return q.is_cuda and q.shape[-1] <= 128 and value.shape[-1] <= 64


def _scan_train(q, k, value, gate, adt, dt, trap_logits, D, *, mimo_x, mimo_z, mimo_out, chunk_size,
                initial_state, initial_k, initial_value, phase, mimo_rotation, q_bias, k_bias):
    """Differentiable chunked SSD for CUDA training: the same prelude as :func:`_scan_torch` (group
    expansion, bias, rotation, trapezoid scale, rank values, endpoint-cache term) as PyTorch ops,
    the chunked core and its backward on the training kernels, then D skip, SiLU gate and rank sum.
    The core runs in float32 from the activation-dtype operands (no intermediate 16-bit rounding)."""
    heads = value.shape[2]
    act = value.dtype
    sig, _, scale, diag = _scalar_prelude(adt, dt, trap_logits)
    if _prelude_kernel_eligible(q, phase, mimo_rotation):
        qf, kc = _Prelude.apply(q, k, q_bias, k_bias, phase, scale, heads, mimo_rotation)
    else:
        qf = _expand_groups(q, heads)
        kf = _expand_groups(k, heads)
        if q_bias is not None:
            qf = qf + q_bias.to(q.dtype)
            kf = kf + k_bias.to(k.dtype)
        if phase is not None:
            qf, kf = rotate_qk(qf, kf, phase, mimo=mimo_rotation)
        kc = kf * scale.to(k.dtype)[..., None, None]

    def rank_act(t, proj):  # [..., H, P] -> [..., H, R, P] in the activation dtype (ops.py:193-199)
        return t.unsqueeze(-2) if proj is None else t.unsqueeze(-2) * proj.to(t.dtype)

    rv = rank_act(value, mimo_x)
    rz = rank_act(gate, mimo_z)
    state = None if initial_state is None else initial_state.float()
    if initial_k is not None:
        prev = rank_act(initial_value, mimo_x).float()
        coef = dt.float()[:, 0] * (1.0 - sig[:, 0])
        outer = coef[..., None, None] * torch.einsum("bhrp,bhrn->bhpn", prev, initial_k.float())
        state = outer if state is None else state + outer
    # the kernels compute in float32 (a float64 caller off the GPU keeps float64: host-logic checks)
    cdt = torch.float32 if q.is_cuda else torch.promote_types(act, torch.float32)
    rvf = rv.to(cdt)
    if state is not None:
        state = state.to(cdt)
    y, final = _SSDCore.apply(qf.to(cdt).contiguous(), kc.to(cdt).contiguous(), rvf.contiguous(),
                              adt.to(cdt).contiguous(), diag.to(cdt).contiguous(), state)
    y = (y + D.to(cdt)[:, None, None] * rvf) * F.silu(rz.to(cdt))
    y = y.sum(dim=3) if mimo_out is None else (y * mimo_out.to(cdt)).sum(dim=3)
    return y.to(act), final


def _scan_device(q, k, value, gate, adt, dt, trap_logits, D, *, mimo_x, mimo_z, mimo_out, chunk_size,
                 initial_state, initial_k, initial_value, phase, mimo_rotation, q_bias, k_bias):
    batch, length, groups, rank, d_state = q.shape
    heads, head_dim = value.shape[2], value.shape[3]
    act = value.dtype
    if act not in (torch.float32, torch.float16, torch.bfloat16):
        raise TypeError(f"unsupported activation dtype {act}")
    q, k, gate = q.to(act), k.to(act), gate.to(act)
    y = torch.empty(batch, length, heads, head_dim, device=value.device, dtype=act)
    state = torch.empty(batch, heads, head_dim, d_state, device=value.device, dtype=torch.float32)
    if initial_k is not None:
        initial_k = initial_k.to(act)
        initial_value = initial_value.to(act)
    tensors = dict(q=q, k=k, value=value, gate=gate, adt=adt.float(), dt=dt.float(), trap=trap_logits, D=D,
                   mimo_x=mimo_x, mimo_z=mimo_z, mimo_out=mimo_out, initial_state=initial_state,
                   initial_k=initial_k, initial_value=initial_value, phase=None if phase is None else phase.float(),
                   q_bias=q_bias, k_bias=k_bias, y=y, final_state=state)
    sizes = dict(batch=batch, length=length, groups=groups, heads=heads, rank=rank, d_state=d_state,
                 head_dim=head_dim, num_angles=0 if phase is None else phase.shape[-1])
    _ext.scan_forward(sizes=sizes, tensors=tensors, mimo_rotation=mimo_rotation, chunk_hint=chunk_size)
    return y, state


def mamba3_scan(q, k, value, gate, adt, dt, trap_logits, D, *, mimo_x=None, mimo_z=None, mimo_out=None,
                chunk_size: int = 64, initial_state=None, initial_k=None, initial_value=None, phase=None,
                mimo_rotation: bool = False, q_bias=None, k_bias=None):
    """Parallel chunked Mamba-3 SSD with FP32 recurrent state (mamba3/ops.py:544-822).

    ``q/k: [B,L,G,R,N]``, ``value/gate: [B,L,H,P]``, ``adt/dt/trap_logits: [B,L,H]``. Returns
    ``(y [B,L,H,P], final state [B,H,P,N] float32)``. CUDA inference calls run the sm_100a kernel;
    the kernel tiles the sequence itself, so ``chunk_size`` only has to be positive there (the
    result does not depend on the chunk length beyond rounding).
    """
    global LAST_SCAN_DISPATCH
    LAST_SCAN_DISPATCH = False
    _validate_scan(q, k, value, gate, adt, dt, trap_logits, D, mimo_x, mimo_z, mimo_out, chunk_size,
                   initial_state, initial_k, initial_value, phase, q_bias, k_bias)
    batch, length, _, _, d_state = q.shape
    if length == 0:
        heads, head_dim = value.shape[2], value.shape[3]
        state = (torch.zeros(batch, heads, head_dim, d_state, device=value.device, dtype=torch.float32)
                 if initial_state is None else initial_state.float())
        return value.clone(), state
    kwargs = dict(mimo_x=mimo_x, mimo_z=mimo_z, mimo_out=mimo_out, chunk_size=chunk_size,
                  initial_state=initial_state, initial_k=initial_k, initial_value=initial_value, phase=phase,
                  mimo_rotation=mimo_rotation, q_bias=q_bias, k_bias=k_bias)
    tensors = (q, k, value, gate, adt, dt, trap_logits, D, mimo_x, mimo_z, mimo_out, initial_state, initial_k,
               initial_value, phase, q_bias, k_bias)
    if _kernel_eligible(*tensors):
        out = _scan_device(q, k, value, gate, adt, dt, trap_logits, D, **kwargs)
        LAST_SCAN_DISPATCH = True
        return out
    if _train_kernel_eligible(q, value) and _needs_autograd(*tensors):
        out = _scan_train(q, k, value, gate, adt, dt, trap_logits, D, **kwargs)
        LAST_SCAN_DISPATCH = True
        return out
    return _scan_torch(q, k, value, gate, adt, dt, trap_logits, D, **kwargs)


# ---------------------------------------------------------------------------
# Decode step
# ---------------------------------------------------------------------------


def mamba3_step(q, k, value, gate, adt, dt, trap_logits, D, cache, *, mimo_x=None, mimo_z=None, mimo_out=None):
    """One exact recurrent update on already-rotated q/k (mamba3/ops.py:825-879).

    ``cache`` is (phase, FP32 state, previous rotated k, previous value); the phase is passed
    through unchanged. Returns ``(y [B,H,P], (phase, new state, k, value))``.
    """
    phase, state, prev_k, prev_value = cache
    sig = torch.sigmoid(trap_logits.float())
    alpha = torch.exp(adt.float())
    beta = (1.0 - sig) * dt.float() * alpha
    gamma = sig * dt.float()
    rv = _rank_values(value, mimo_x)
    prv = _rank_values(prev_value, mimo_x)
    new_state = (alpha[..., None, None] * state.float()
                 + beta[..., None, None] * torch.einsum("bhrp,bhrn->bhpn", prv, prev_k.float())
                 + gamma[..., None, None] * torch.einsum("bhrp,bhrn->bhpn", rv, k.float()))
    read = new_state.to(q.dtype).float()
    y = torch.einsum("bhpn,bhrn->bhrp", read, q.float()) + D.float()[None, :, None, None] * rv
    y = y * F.silu(_rank_values(gate, mimo_z))
    y = y.sum(dim=2) if mimo_out is None else (y * mimo_out.float()).sum(dim=2)
    return y.to(value.dtype), (phase, new_state, k, value)


def _validate_fused_step(q, k, value, gate, adt, dt, trap_logits, angle_rate, D, cache, mimo_x, mimo_z, mimo_out):
    """Shape/dtype contract of mamba3/_triton.py:967-1044."""
    phase, state, prev_k, prev_value = cache
    if q.ndim != 4:
        raise ValueError("q must have shape [B, H, R, N]")
    batch, heads, rank, d_state = q.shape
    head_dim = value.shape[-1]
    count = angle_rate.shape[-1]
    if count <= 0 or count > d_state // 2:
        raise ValueError("angle width must be in [1, d_state / 2]")
    if rank > 1 and 4 * count != d_state:
        raise ValueError("fused MIMO step requires 4 * num_angles == d_state "
                         "(rope_fraction 0.5 and d_state divisible by 4)")
    expected = {
        "k": (k, (batch, heads, rank, d_state)), "value": (value, (batch, heads, head_dim)),
        "gate": (gate, (batch, heads, head_dim)), "adt": (adt, (batch, heads)), "dt": (dt, (batch, heads)),
        "trap_logits": (trap_logits, (batch, heads)), "angle_rate": (angle_rate, (batch, count)),
        "D": (D, (heads,)), "phase": (phase, (batch, heads, count)),
        "state": (state, (batch, heads, head_dim, d_state)), "previous_k": (prev_k, (batch, heads, rank, d_state)),
        "previous_value": (prev_value, (batch, heads, head_dim)),
    }
    for name, (tensor, shape) in expected.items():
        if tuple(tensor.shape) != shape:
            raise ValueError(f"invalid {name} shape: expected {shape}, got {tuple(tensor.shape)}")
    if not (q.dtype == k.dtype == value.dtype == gate.dtype):
        raise ValueError("q, k, value, and gate must have the same dtype")
    if prev_k.dtype != q.dtype or prev_value.dtype != value.dtype:
        raise ValueError("K/value cache dtypes must match current activations")
    if phase.dtype != torch.float32 or state.dtype != torch.float32:
        raise ValueError("phase and state must be float32")
    if rank > 1:
        if mimo_x is None or mimo_z is None or mimo_out is None:
            raise ValueError("fused MIMO step requires all three MIMO projections")
        for name, proj in (("mimo_x", mimo_x), ("mimo_z", mimo_z), ("mimo_out", mimo_out)):
            if tuple(proj.shape) != (heads, rank, head_dim):
                raise ValueError(f"invalid {name} shape: expected {(heads, rank, head_dim)}, "
                                 f"got {tuple(proj.shape)}")
    elif mimo_x is not None:
        raise ValueError("MIMO projections require rank > 1")


def _step_device(q, k, value, gate, adt, dt, trap_logits, angle_rate, D, cache, *, mimo_x, mimo_z, mimo_out,
                 q_bias=None, k_bias=None, out_state=None, q_norm_w=None, k_norm_w=None, dt_bias=None,
                 norm_eps=1e-5):
    """Launch ``m3_step_fwd``. With ``dt_bias`` given, ``adt``/``dt`` are the raw decay/delta
    logits and the kernel discretises them; with ``q_norm_w``/``k_norm_w`` given, ``q``/``k``
    are the raw C/B rows and the kernel RMS-normalises them (model mode)."""
    phase, state, prev_k, prev_value = cache
    batch, heads, rank, d_state = q.shape
    y = torch.empty(value.shape, device=value.device, dtype=value.dtype)
    out_phase = torch.empty(phase.shape, device=phase.device, dtype=torch.float32)
    out_k = torch.empty(batch, heads, rank, d_state, device=q.device, dtype=q.dtype)
    if out_state is None:
        out_state = torch.empty(state.shape, device=state.device, dtype=torch.float32)
    if dt_bias is None:
        adt, dt = adt.float(), dt.float()
    tensors = dict(q=q, k=k, q_bias=q_bias, k_bias=k_bias, value=value, gate=gate, adt=adt,
                   dt=dt, trap=trap_logits, angle_rate=angle_rate, D=D, mimo_x=mimo_x, mimo_z=mimo_z,
                   mimo_out=mimo_out, phase=phase, state=state, prev_k=prev_k, prev_value=prev_value, y=y,
                   out_phase=out_phase, out_state=out_state, out_k=out_k, q_norm_w=q_norm_w,
                   k_norm_w=k_norm_w, dt_bias=dt_bias)
    sizes = dict(batch=batch, heads=heads, rank=rank, d_state=d_state, head_dim=value.shape[-1],
                 num_angles=angle_rate.shape[-1])
    _ext.step_forward(sizes=sizes, tensors=tensors, norm_eps=norm_eps)
    global LAST_STEP_DISPATCH
    LAST_STEP_DISPATCH = True
    return y, (out_phase, out_state, out_k, value)


def fused_step(q, k, value, gate, adt, dt, trap_logits, angle_rate, D, cache, *, mimo_x=None, mimo_z=None,
               mimo_out=None):
    """Fused decode step on unrotated q/k (contract of mamba3/ops.py:87-190).

    Returns ``(y [B,H,P], (new phase, new state, rotated k, value))`` from the CUDA kernel, or
    ``None`` when the call is not a CUDA inference call (CPU tensors, or autograd needed) — the
    caller then runs the PyTorch step, exactly like the reference's dispatch contract.
    """
    global LAST_STEP_DISPATCH
    LAST_STEP_DISPATCH = False
    tensors = (q, k, value, gate, adt, dt, trap_logits, angle_rate, D, *cache, mimo_x, mimo_z, mimo_out)
    if not _kernel_eligible(*tensors):
        return None
    _validate_fused_step(q, k, value, gate, adt, dt, trap_logits, angle_rate, D, cache, mimo_x, mimo_z, mimo_out)
    if any(t is not None and t.device != q.device for t in tensors):
        raise ValueError("fused step tensors must be on the same CUDA device")
    return _step_device(q, k, value, gate, adt, dt, trap_logits, angle_rate, D, cache, mimo_x=mimo_x,
                        mimo_z=mimo_z, mimo_out=mimo_out)

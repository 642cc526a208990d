"""CPU oracle for the Mamba-3 chunked SSD and decode step (numpy, float64).

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this module;
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
use it, and only as the checker or as the timed CPU baseline.

It restates the reference algorithm of jreoka/mamba3 in plain numpy so that the
CUDA kernels can be checked against an implementation that shares no code with
them. Every function names the reference lines it follows (paths are relative
to the reference project root). Parity of this restatement is pinned by the
golden fixtures in ``tests/golden/`` that were produced by running the
reference itself (see ``tests/golden/make_golden.py``) and by the reference
test suite's own known-answer vectors (rotation, heavy-tail).

Shapes follow the reference: q/k ``[B, L, H, R, N]`` (already expanded to the
value heads), value/gate ``[B, L, H, P]``, adt/dt/trap ``[B, L, H]``, state
``[B, H, P, N]``, phase ``[B, L, H, S]``.
"""

from __future__ import annotations

import math

import numpy as np

TWO_PI = 2.0 * math.pi
PHASE_BLOCK = 64  # mamba3/model.py:25 (_PHASE_CHUNK)
A_FLOOR = 1e-4  # mamba3/model.py:22
EXPANSION = 2  # mamba3/model.py:19
CANONICAL_HEAD_DIM = 64  # mamba3/model.py:20


# ---------------------------------------------------------------------------
# Elementwise maps
# ---------------------------------------------------------------------------

def heavy_tail(x: np.ndarray) -> np.ndarray:
    """1 + x for x >= 0, 1 / (1 - x) below zero (mamba3/ops.py:28-32)."""
    x = np.asarray(x, dtype=np.float64)
    return np.where(x >= 0, 1.0 + x, 1.0 / (1.0 - np.minimum(x, 0.0)))


def sigmoid(x: np.ndarray) -> np.ndarray:
    return 0.5 * (1.0 + np.tanh(0.5 * np.asarray(x, dtype=np.float64)))


def softplus(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    return np.logaddexp(0.0, x)


def silu(x: np.ndarray) -> np.ndarray:
    return x * sigmoid(x)


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """RMS normalisation over the last axis (mamba3/model.py:42-55)."""
    x = np.asarray(x, dtype=np.float64)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * inv * weight


# ---------------------------------------------------------------------------
# Rotation and phase
# ---------------------------------------------------------------------------

def rotate(t: np.ndarray, phase: np.ndarray, mimo: bool) -> np.ndarray:
    """Real-coordinate complex rotation of the state axis (mamba3/ops.py:35-84).

    ``t`` is ``[..., R, N]`` and ``phase`` is ``[..., S]`` (broadcast over R).
    SISO rotates adjacent pairs (2i, 2i+1); MIMO rotates (i, 2S+i).
    """
    t = np.array(t, dtype=np.float64, copy=True)
    s = phase.shape[-1]
    c = np.cos(phase)[..., None, :]
    sn = np.sin(phase)[..., None, :]
    if mimo:
        a = t[..., :s].copy()
        b = t[..., 2 * s:3 * s].copy()
        t[..., :s] = a * c - b * sn
        t[..., 2 * s:3 * s] = a * sn + b * c
    else:
        a = t[..., 0:2 * s:2].copy()
        b = t[..., 1:2 * s:2].copy()
        t[..., 0:2 * s:2] = a * c - b * sn
        t[..., 1:2 * s:2] = a * sn + b * c
    return t


def phase_increments(angles: np.ndarray, dt: np.ndarray) -> np.ndarray:
    """fmod(pi * tanh(angle) * dt, 2 pi), ``[B, L, H, S]`` (mamba3/model.py:225-230)."""
    inc = math.pi * np.tanh(np.asarray(angles, np.float64))[:, :, None, :] * np.asarray(dt, np.float64)[..., None]
    return np.fmod(inc, TWO_PI)


def phase_scheme(angles: np.ndarray, dt: np.ndarray, initial_phase: np.ndarray | None) -> np.ndarray:
    """Blocked phase accumulation of mamba3/model.py:215-256.

    Within each 64-token block the increments are summed from the block
    start; the block offset is carried sequentially and reduced mod 2 pi
    after every block, and each token's phase is fmod(local + offset).
    """
    inc = phase_increments(angles, dt)
    batch, length, heads, count = inc.shape
    out = np.empty_like(inc)
    offset = (np.zeros((batch, heads, count)) if initial_phase is None
              else np.asarray(initial_phase, np.float64).copy())
    for start in range(0, length, PHASE_BLOCK):
        end = min(start + PHASE_BLOCK, length)
        local = np.cumsum(inc[:, start:end], axis=1)
        out[:, start:end] = np.fmod(local + offset[:, None], TWO_PI)
        offset = np.fmod(offset + local[:, -1], TWO_PI)
    return out


def phase_sequential(angles: np.ndarray, dt: np.ndarray) -> np.ndarray:
    """Token-by-token phase, fmod after every token (tests/test_model.py:213-249)."""
    inc = phase_increments(angles, dt)
    out = np.empty_like(inc)
    state = np.zeros_like(inc[:, 0])
    for t in range(inc.shape[1]):
        state = np.fmod(state + inc[:, t], TWO_PI)
        out[:, t] = state
    return out


# ---------------------------------------------------------------------------
# Scan
# ---------------------------------------------------------------------------

def _rank_values(value: np.ndarray, proj: np.ndarray | None) -> np.ndarray:
    """value [..., H, P] -> [..., H, R, P] (mamba3/ops.py:193-199)."""
    if proj is None:
        return value[..., None, :]
    return value[..., None, :] * proj


def expand_heads(q: np.ndarray, heads: int) -> np.ndarray:
    """[B, L, G, R, N] -> [B, L, H, R, N] by repeating each group (mamba3/ops.py:700-709)."""
    groups = q.shape[2]
    if groups == heads:
        return q
    return np.repeat(q, heads // groups, axis=2)


def scan_recurrent(q, k, value, gate, adt, dt, trap_logits, D, *, mimo_x=None, mimo_z=None,
                   mimo_out=None, initial_state=None, initial_k=None, initial_value=None):
    """Token-by-token Mamba-3 recurrence (tests/test_scan.py:21-98).

    S_t = alpha_t S_{t-1} + beta_t U_{t-1} + gamma_t U_t with U_t = sum_r v_{t,r} k_{t,r}^T,
    y_t = sum_r mo_r * silu(z_t mz_r) * (S_t q_{t,r} + D v_{t,r}).
    q/k are [B, L, H, R, N] and already carry bias and rotation.
    Returns (y [B, L, H, P], S [B, H, P, N]).
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    value = np.asarray(value, np.float64)
    gate = np.asarray(gate, np.float64)
    batch, length, heads, rank, n = q.shape
    p = value.shape[-1]
    rv = _rank_values(value, mimo_x)
    rg = _rank_values(gate, mimo_z)
    state = np.zeros((batch, heads, p, n)) if initial_state is None else np.asarray(initial_state, np.float64).copy()
    prev_k = np.zeros((batch, heads, rank, n)) if initial_k is None else np.asarray(initial_k, np.float64)
    prev_v = np.zeros((batch, heads, p)) if initial_value is None else np.asarray(initial_value, np.float64)
    prev_rv = _rank_values(prev_v, mimo_x)
    out = np.empty((batch, length, heads, p))
    for t in range(length):
        tr = sigmoid(trap_logits[:, t])
        alpha = np.exp(adt[:, t])
        beta = (1.0 - tr) * dt[:, t] * alpha
        gamma = tr * dt[:, t]
        prev_outer = np.einsum("bhrp,bhrn->bhpn", prev_rv, prev_k)
        cur_outer = np.einsum("bhrp,bhrn->bhpn", rv[:, t], k[:, t])
        state = alpha[..., None, None] * state + beta[..., None, None] * prev_outer + gamma[..., None, None] * cur_outer
        y = np.einsum("bhpn,bhrn->bhrp", state, q[:, t])
        y = (y + np.asarray(D, np.float64)[None, :, None, None] * rv[:, t]) * silu(rg[:, t])
        out[:, t] = y.sum(axis=2) if mimo_out is None else (y * mimo_out).sum(axis=2)
        prev_k = k[:, t]
        prev_rv = rv[:, t]
    return out, state


def scan_chunked(q, k, value, gate, adt, dt, trap_logits, D, *, chunk_size=64, mimo_x=None, mimo_z=None,
                 mimo_out=None, initial_state=None, initial_k=None, initial_value=None):
    """Chunked (parallel-within-chunk) form of the same recurrence (mamba3/ops.py:659-822).

    Same inputs/outputs as :func:`scan_recurrent`. ``scale_t = gamma_t +
    dt_{t+1}(1 - sigma_{t+1})`` carries the next token's left trapezoid
    endpoint (0 after the last token) so that chunk states compose, and the
    same-token diagonal of the decay matrix is ``gamma_t / scale_t``.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    value = np.asarray(value, np.float64)
    gate = np.asarray(gate, np.float64)
    adt = np.asarray(adt, np.float64)
    dt = np.asarray(dt, np.float64)
    batch, length, heads, rank, n = q.shape
    p = value.shape[-1]
    tr = sigmoid(trap_logits)
    gamma = dt * tr
    nxt = np.zeros_like(dt)
    nxt[:, :-1] = dt[:, 1:] * (1.0 - tr[:, 1:])
    scale = gamma + nxt
    diag = gamma / scale
    state = np.zeros((batch, heads, p, n)) if initial_state is None else np.asarray(initial_state, np.float64).copy()
    if initial_k is not None:
        prv = _rank_values(np.asarray(initial_value, np.float64), mimo_x)
        state = state + (dt[:, 0] * (1.0 - tr[:, 0]))[..., None, None] * np.einsum(
            "bhrp,bhrn->bhpn", prv, np.asarray(initial_k, np.float64))
    rv = _rank_values(value, mimo_x)  # [B, L, H, R, P]
    rg = _rank_values(gate, mimo_z)
    Dv = np.asarray(D, np.float64)
    out = np.empty((batch, length, heads, p))
    for start in range(0, length, chunk_size):
        end = min(start + chunk_size, length)
        w = end - start
        cum = np.cumsum(adt[:, start:end], axis=1)  # [B, w, H]
        qc = q[:, start:end].transpose(0, 2, 1, 3, 4).reshape(batch, heads, w * rank, n)
        kc = (k[:, start:end] * scale[:, start:end, :, None, None]).transpose(0, 2, 1, 3, 4).reshape(
            batch, heads, w * rank, n)
        vc = rv[:, start:end].transpose(0, 2, 1, 3, 4).reshape(batch, heads, w * rank, p)
        cumh = cum.transpose(0, 2, 1)  # [B, H, w]
        # inter-chunk
        inter = np.einsum("bhin,bhpn->bhip", qc, state)
        inter = inter.reshape(batch, heads, w, rank, p) * np.exp(cumh)[..., None, None]
        # intra-chunk
        scores = np.einsum("bhin,bhjn->bhij", qc, kc).reshape(batch, heads, w, rank, w, rank)
        diff = cumh[..., :, None] - cumh[..., None, :]
        tri = np.tril(np.ones((w, w), dtype=bool), -1)
        decay = np.where(tri, np.exp(np.where(tri, diff, 0.0)), 0.0)
        decay = decay + np.eye(w) * diag[:, start:end].transpose(0, 2, 1)[..., None]
        wts = (scores * decay[:, :, :, None, :, None]).reshape(batch, heads, w * rank, w * rank)
        intra = np.einsum("bhij,bhjp->bhip", wts, vc).reshape(batch, heads, w, rank, p)
        y = inter + intra + Dv[None, :, None, None, None] * vc.reshape(batch, heads, w, rank, p)
        y = y * silu(rg[:, start:end].transpose(0, 2, 1, 3, 4))
        y = y.sum(axis=3) if mimo_out is None else (y * mimo_out[None, :, None]).sum(axis=3)
        out[:, start:end] = y.transpose(0, 2, 1, 3)
        # state carry
        end_decay = np.exp(cumh[..., -1:] - cumh)  # [B, H, w]
        ks = kc.reshape(batch, heads, w, rank, n) * end_decay[..., None, None]
        state = np.exp(cumh[..., -1])[..., None, None] * state + np.einsum(
            "bhip,bhin->bhpn", vc, ks.reshape(batch, heads, w * rank, n))
    return out, state


def step_recurrence(q, k, value, gate, adt, dt, trap_logits, D, cache, *, mimo_x=None, mimo_z=None,
                    mimo_out=None):
    """One exact recurrent update on rotated q/k (mamba3/ops.py:825-879).

    q/k ``[B, H, R, N]``; cache = (phase, state, previous rotated k, previous value).
    Returns (y [B, H, P], (phase, new state, k, value)).
    """
    phase, state, prev_k, prev_v = cache
    y, new_state = scan_recurrent(q[:, None], k[:, None], value[:, None], gate[:, None], adt[:, None],
                                  dt[:, None], trap_logits[:, None], D, mimo_x=mimo_x, mimo_z=mimo_z,
                                  mimo_out=mimo_out, initial_state=state, initial_k=prev_k,
                                  initial_value=prev_v)
    return y[:, 0], (phase, new_state, np.asarray(k, np.float64), np.asarray(value, np.float64))


def fused_step(q, k, value, gate, adt, dt, trap_logits, angle_rate, D, cache, *, mimo_x=None, mimo_z=None,
               mimo_out=None):
    """Decode step on unrotated q/k (mamba3/ops.py:87-105 contract; math of mamba3/model.py:460-484).

    The phase advances by fmod(pi tanh(angle) dt, 2 pi) and is reduced mod 2 pi;
    q/k are rotated by the new phase; then :func:`step_recurrence`.
    ``angle_rate`` is ``[B, S]`` (shared across heads), ``dt`` is ``[B, H]``.
    """
    phase0, state, prev_k, prev_v = cache
    inc = np.fmod(math.pi * np.tanh(np.asarray(angle_rate, np.float64))[:, None, :] * np.asarray(dt, np.float64)[..., None],
                  TWO_PI)
    phase = np.fmod(np.asarray(phase0, np.float64) + inc, TWO_PI)
    mimo = q.shape[2] > 1
    qr = rotate(q, phase, mimo)
    kr = rotate(k, phase, mimo)
    y, (_, new_state, k_out, v_out) = step_recurrence(qr, kr, value, gate, adt, dt, trap_logits, D,
                                                       (phase, state, prev_k, prev_v), mimo_x=mimo_x,
                                                       mimo_z=mimo_z, mimo_out=mimo_out)
    return y, (phase, new_state, kr, v_out)


# ---------------------------------------------------------------------------
# Whole model from a state_dict (mamba3/model.py)
# ---------------------------------------------------------------------------

class ModelConfig:
    """Derived sizes of mamba3/model.py:74-113."""

    def __init__(self, d_model: int, d_state: int = 128, depth: int = 4, mimo_rank: int = 1,
                 causal: bool = True) -> None:
        self.d_model = d_model
        self.d_state = d_state
        self.depth = depth
        self.mimo_rank = mimo_rank
        self.causal = causal
        self.d_inner = EXPANSION * d_model
        self.headdim = math.gcd(self.d_inner, CANONICAL_HEAD_DIM)
        self.nheads = self.d_inner // self.headdim
        self.num_angles = int(d_state * 0.5) // 2


def _layer_params(sd: dict, i: int) -> dict:
    pre = f"layers.{i}."
    return {key[len(pre):]: np.asarray(val, np.float64) for key, val in sd.items() if key.startswith(pre)}


def _project(cfg: ModelConfig, lp: dict, h: np.ndarray):
    """in_proj split + B/C norm + dt/adt (mamba3/model.py:147-199)."""
    return split_projection(cfg, lp, h @ lp["mixer.in_proj.weight"].T)


def split_projection(cfg: ModelConfig, lp: dict, proj: np.ndarray):
    """Split of an in_proj output [B, L, W] + B/C norm + dt/adt (mamba3/model.py:147-199)."""
    proj = np.asarray(proj, np.float64)
    di, n, r, nh, s = cfg.d_inner, cfg.d_state, cfg.mimo_rank, cfg.nheads, cfg.num_angles
    sizes = [di, di, n * r, n * r, nh, nh, nh, s]
    offs = np.cumsum([0] + sizes)
    z, x, B, C, dl, al, trap, ang = [proj[..., offs[j]:offs[j + 1]] for j in range(8)]
    bsz, length = proj.shape[:2]
    z = z.reshape(bsz, length, nh, cfg.headdim)
    x = x.reshape(bsz, length, nh, cfg.headdim)
    B = rms_norm(B.reshape(bsz, length, r, n), lp["mixer.B_norm.weight"])
    C = rms_norm(C.reshape(bsz, length, r, n), lp["mixer.C_norm.weight"])
    dt = softplus(dl + lp["mixer.dt_bias"])
    adt = np.minimum(-heavy_tail(al), -A_FLOOR) * dt
    return C[:, :, None], B[:, :, None], x, z, adt, dt, trap, ang


def _mimo(lp: dict):
    return lp.get("mixer.mimo_x"), lp.get("mixer.mimo_z"), lp.get("mixer.mimo_out")


def _scan_direction(cfg, lp, h, cache, chunked: bool):
    return scan_projection(cfg, lp, h @ lp["mixer.in_proj.weight"].T, cache, chunked)


def scan_projection(cfg, lp, proj, cache=None, chunked: bool = True):
    """One mixer direction from its in_proj output: (y [B,L,H,P] before out_proj, final state,
    phase [B,L,H,S], rotated biased k [B,L,H,R,N], x [B,L,H,P]) (mamba3/model.py:270-327)."""
    q, k, x, z, adt, dt, trap, ang = split_projection(cfg, lp, proj)
    phase = phase_scheme(ang, dt, None if cache is None else cache[0])
    q = expand_heads(q, cfg.nheads) + lp["mixer.C_bias"]
    k = expand_heads(k, cfg.nheads) + lp["mixer.B_bias"]
    mimo = cfg.mimo_rank > 1
    q = rotate(q, phase, mimo)
    k = rotate(k, phase, mimo)
    mx, mz, mo = _mimo(lp)
    kwargs = dict(mimo_x=mx, mimo_z=mz, mimo_out=mo)
    if cache is not None:
        kwargs.update(initial_state=cache[1], initial_k=cache[2], initial_value=cache[3])
    fn = scan_chunked if chunked else scan_recurrent
    y, state = fn(q, k, x, z, adt, dt, trap, lp["mixer.D"], **kwargs)
    return y, state, phase, k, x


def mixer_forward(cfg, lp, h, cache=None, return_cache=False, chunked=True):
    """_Mamba3Mixer.forward (mamba3/model.py:270-362)."""
    y, state, phase, k, x = _scan_direction(cfg, lp, h, cache, chunked)
    out = y.reshape(*y.shape[:2], -1) @ lp["mixer.out_proj.weight"].T
    if cfg.causal:
        if not return_cache:
            return out
        return out, (phase[:, -1].copy(), state, k[:, -1].copy(), x[:, -1].copy())
    yr, _, _, _, _ = _scan_direction(cfg, lp, h[:, ::-1], None, chunked)
    back = yr[:, ::-1].reshape(*yr.shape[:2], -1) @ lp["mixer.out_proj.weight"].T
    blend = sigmoid(lp["mixer.direction_logit"])
    return out * blend + back * (1.0 - blend)


def model_forward(cfg, sd, x, chunked=True):
    """Mamba3.forward (mamba3/model.py:585-591)."""
    h = np.asarray(x, np.float64)
    for i in range(cfg.depth):
        lp = _layer_params(sd, i)
        h = h + mixer_forward(cfg, lp, rms_norm(h, lp["norm.weight"]), chunked=chunked)
    return rms_norm(h, np.asarray(sd["norm_f.weight"], np.float64))


def model_prefill(cfg, sd, x, chunked=True):
    """Mamba3.prefill (mamba3/model.py:593-607)."""
    h = np.asarray(x, np.float64)
    caches = []
    for i in range(cfg.depth):
        lp = _layer_params(sd, i)
        out, cache = mixer_forward(cfg, lp, rms_norm(h, lp["norm.weight"]), return_cache=True, chunked=chunked)
        h = h + out
        caches.append(cache)
    return rms_norm(h, np.asarray(sd["norm_f.weight"], np.float64)), caches


def empty_cache(cfg, batch):
    """allocate_cache zeros (mamba3/model.py:364-402)."""
    return (np.zeros((batch, cfg.nheads, cfg.num_angles)), np.zeros((batch, cfg.nheads, cfg.headdim, cfg.d_state)),
            np.zeros((batch, cfg.nheads, cfg.mimo_rank, cfg.d_state)), np.zeros((batch, cfg.nheads, cfg.headdim)))


def model_step(cfg, sd, x, caches=None):
    """Mamba3.step (mamba3/model.py:609-630, mixer step 422-484). x is [B, 1, D]."""
    h = np.asarray(x, np.float64)
    batch = h.shape[0]
    caches = [empty_cache(cfg, batch) for _ in range(cfg.depth)] if caches is None else caches
    new = []
    for i in range(cfg.depth):
        lp = _layer_params(sd, i)
        q, k, xv, z, adt, dt, trap, ang = _project(cfg, lp, rms_norm(h, lp["norm.weight"]))
        q = expand_heads(q, cfg.nheads)[:, 0] + lp["mixer.C_bias"]
        k = expand_heads(k, cfg.nheads)[:, 0] + lp["mixer.B_bias"]
        mx, mz, mo = _mimo(lp)
        y, cache = fused_step(q, k, xv[:, 0], z[:, 0], adt[:, 0], dt[:, 0], trap[:, 0], ang[:, 0], lp["mixer.D"],
                              caches[i], mimo_x=mx, mimo_z=mz, mimo_out=mo)
        h = h + (y.reshape(batch, -1) @ lp["mixer.out_proj.weight"].T)[:, None]
        new.append(cache)
    return rms_norm(h, np.asarray(sd["norm_f.weight"], np.float64)), new

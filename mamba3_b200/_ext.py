"""ctypes binding of the C-ABI library ``_lib/libmamba3_b200.so`` (see ``include/mamba3_b200.h``).

This module only marshals torch tensors into the plain-pointer argument structs and enqueues the
kernels on the current torch stream. It never falls back to another implementation: a missing or
unloadable library raises ``RuntimeError`` when a CUDA call needs it.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libmamba3_b200.so"

M3_F32, M3_F16, M3_BF16 = 0, 1, 2
_DTYPES = {torch.float32: M3_F32, torch.float16: M3_F16, torch.bfloat16: M3_BF16}
ABI_VERSION = 3


class M3Tensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("stride", ctypes.c_int64 * 6),
    ]


_SCAN_TENSORS = (
    "q", "k", "q_norm_w", "k_norm_w", "q_bias", "k_bias",
    "value", "gate",
    "adt", "dt", "trap", "dt_bias",
    "phase", "angles", "initial_phase",
    "D", "mimo_x", "mimo_z", "mimo_out",
    "initial_state", "initial_k", "initial_value",
    "y", "final_state", "final_phase", "final_k",
    "workspace", "y_reverse",
)

_STEP_TENSORS = (
    "q", "k", "q_bias", "k_bias", "value", "gate",
    "adt", "dt", "trap", "angle_rate", "D", "mimo_x", "mimo_z", "mimo_out",
    "phase", "state", "prev_k", "prev_value",
    "y", "out_phase", "out_state", "out_k",
    "workspace",
    "q_norm_w", "k_norm_w", "dt_bias",
)


class ScanArgs(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "batch", "length", "groups", "heads", "rank", "d_state", "head_dim", "num_angles",
        "reverse", "mimo_rotation", "chunk_hint", "device")] + [
        ("norm_eps", ctypes.c_float), ("segments", ctypes.c_int32)] + [
        (name, M3Tensor) for name in _SCAN_TENSORS]


class GemvArgs(ctypes.Structure):
    _fields_ = [("out_dim", ctypes.c_int64), ("in_dim", ctypes.c_int64), ("rows", ctypes.c_int32),
                ("device", ctypes.c_int32)] + [(name, M3Tensor) for name in ("x", "w", "y")]


class NormArgs(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("dim", ctypes.c_int32), ("device", ctypes.c_int32),
                ("eps", ctypes.c_float), ("reserved", ctypes.c_int32)] + [
        (name, M3Tensor) for name in ("x", "m", "w", "out_x", "out_n")]


class StepArgs(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "batch", "heads", "rank", "d_state", "head_dim", "num_angles", "device")] + [
        ("norm_eps", ctypes.c_float)] + [
        (name, M3Tensor) for name in _STEP_TENSORS]


_SSD_TENSORS = (
    "q", "k", "v", "adt", "diag", "initial_state",
    "y", "final_state", "chunk_states",
    "dy", "dfinal",
    "dq", "dk", "dv", "dadt", "ddiag", "dinitial",
    "workspace",
)


_PRELUDE_TENSORS = ("q", "k", "q_bias", "k_bias", "phase", "scale", "qf", "kc",
                    "dqf", "dkc", "dqb", "dkb", "dphase", "dscale")


class PreludeArgs(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "batch", "length", "groups", "heads", "rank", "d_state", "num_angles", "mimo_rotation", "device",
        "reserved")] + [(name, M3Tensor) for name in _PRELUDE_TENSORS]


class SSDArgs(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "batch", "length", "heads", "rank", "d_state", "head_dim", "device", "reserved")] + [
        (name, M3Tensor) for name in _SSD_TENSORS]


_lib = None
_lock = threading.Lock()


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the CUDA library once; raise RuntimeError if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise RuntimeError(
                f"mamba3_b200 CUDA library not built ({_LIB_PATH}); run `python -m mamba3_b200._build`")
        lib = ctypes.CDLL(str(_LIB_PATH))
        lib.m3_scan_fwd.argtypes = [ctypes.POINTER(ScanArgs), ctypes.c_void_p]
        lib.m3_scan_fwd.restype = ctypes.c_int
        lib.m3_step_fwd.argtypes = [ctypes.POINTER(StepArgs), ctypes.c_void_p]
        lib.m3_step_fwd.restype = ctypes.c_int
        lib.m3_last_error.argtypes = []
        lib.m3_last_error.restype = ctypes.c_char_p
        lib.m3_abi_version.argtypes = []
        lib.m3_abi_version.restype = ctypes.c_int
        lib.m3_device_error.argtypes = [ctypes.c_int]
        lib.m3_device_error.restype = ctypes.c_int
        lib.m3_scan_workspace_bytes.argtypes = [ctypes.POINTER(ScanArgs)]
        lib.m3_scan_workspace_bytes.restype = ctypes.c_int64
        lib.m3_step_workspace_bytes.argtypes = [ctypes.POINTER(StepArgs)]
        lib.m3_step_workspace_bytes.restype = ctypes.c_int64
        lib.m3_gemv.argtypes = [ctypes.POINTER(GemvArgs), ctypes.c_void_p]
        lib.m3_gemv.restype = ctypes.c_int
        lib.m3_residual_rmsnorm.argtypes = [ctypes.POINTER(NormArgs), ctypes.c_void_p]
        lib.m3_residual_rmsnorm.restype = ctypes.c_int
        lib.m3_last_scan_kernel.argtypes = []
        lib.m3_last_scan_kernel.restype = ctypes.c_char_p
        lib.m3_scan_segments.argtypes = [ctypes.POINTER(ScanArgs)]
        lib.m3_scan_segments.restype = ctypes.c_int
        lib.m3_scan_summary.argtypes = [ctypes.POINTER(ScanArgs), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.m3_scan_summary.restype = ctypes.c_int
        lib.m3_scan_summary_floats.argtypes = [ctypes.c_int]
        lib.m3_scan_summary_floats.restype = ctypes.c_int
        lib.m3_last_step_kernel.argtypes = []
        lib.m3_last_step_kernel.restype = ctypes.c_char_p
        lib.m3_ssd_chunk_rows.argtypes = []
        lib.m3_ssd_chunk_rows.restype = ctypes.c_int
        lib.m3_ssd_prelude_fwd.argtypes = [ctypes.POINTER(PreludeArgs), ctypes.c_void_p]
        lib.m3_ssd_prelude_fwd.restype = ctypes.c_int
        lib.m3_ssd_prelude_bwd.argtypes = [ctypes.POINTER(PreludeArgs), ctypes.c_void_p]
        lib.m3_ssd_prelude_bwd.restype = ctypes.c_int
        lib.m3_ssd_workspace_bytes.argtypes = [ctypes.POINTER(SSDArgs), ctypes.c_int]
        lib.m3_ssd_workspace_bytes.restype = ctypes.c_int64
        lib.m3_ssd_train_fwd.argtypes = [ctypes.POINTER(SSDArgs), ctypes.c_void_p]
        lib.m3_ssd_train_fwd.restype = ctypes.c_int
        lib.m3_ssd_train_bwd.argtypes = [ctypes.POINTER(SSDArgs), ctypes.c_void_p]
        lib.m3_ssd_train_bwd.restype = ctypes.c_int
        if lib.m3_abi_version() != ABI_VERSION:
            raise RuntimeError("mamba3_b200 library ABI mismatch; rebuild it")
        _lib = lib
    return _lib


def _desc(t: torch.Tensor | None) -> M3Tensor:
    d = M3Tensor()
    if t is None:
        return d
    if t.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {t.dtype}")
    if t.dim() > 6:
        raise ValueError("at most 6 dimensions")
    d.data = t.data_ptr()
    d.dtype = _DTYPES[t.dtype]
    d.ndim = t.dim()
    for i, s in enumerate(t.stride()):
        d.stride[i] = s
    return d


def _cuda_device(tensors: dict) -> torch.device:
    device = tensors["value"].device
    for name, t in tensors.items():
        if t is not None and t.device != device:
            raise ValueError(f"{name} is on {t.device}, expected {device}")
    if device.type != "cuda":
        raise ValueError(f"the mamba3_b200 kernels need CUDA tensors, got {device}")
    return device


def _check(rc: int, lib) -> None:
    if rc != 0:
        msg = lib.m3_last_error().decode()
        raise RuntimeError(f"mamba3_b200 kernel error {rc}: {msg}")


def _segments(segments: int | None) -> int:
    if segments is None:
        segments = int(os.environ.get("MAMBA3_B200_SEGMENTS", "0") or 0)
    if segments < 0:
        raise ValueError("segments must be >= 0")
    return int(segments)


@torch.compiler.disable
def scan_forward(*, sizes: dict, tensors: dict, reverse: bool = False, mimo_rotation: bool = False,
                 chunk_hint: int = 64, norm_eps: float = 1e-5, segments: int | None = None) -> None:
    """Enqueue ``m3_scan_fwd`` on the current stream of the tensors' device. ``segments``: 0 / None =
    automatic sequence split, 1 = never split, n >= 2 = n segments (``MAMBA3_B200_SEGMENTS`` sets
    the default)."""
    lib = load()
    args = ScanArgs()
    args.segments = _segments(segments)
    for key, val in sizes.items():
        setattr(args, key, int(val))
    args.reverse = 2 if reverse == "both" else int(reverse)
    args.mimo_rotation = int(mimo_rotation)
    args.chunk_hint = int(chunk_hint)
    args.norm_eps = float(norm_eps)
    device = _cuda_device(tensors)
    args.device = device.index if device.index is not None else torch.cuda.current_device()
    for name in _SCAN_TENSORS:
        setattr(args, name, _desc(tensors.get(name)))
    need = lib.m3_scan_workspace_bytes(ctypes.byref(args))
    if need < 0:
        _check(int(-need), lib)
    workspace = None
    if need > 0:
        workspace = torch.empty((need + 3) // 4, device=device, dtype=torch.float32)
        args.workspace = _desc(workspace)
    stream = torch.cuda.current_stream(device).cuda_stream
    _check(lib.m3_scan_fwd(ctypes.byref(args), ctypes.c_void_p(stream)), lib)


@torch.compiler.disable
def step_forward(*, sizes: dict, tensors: dict, norm_eps: float = 1e-5) -> None:
    """Enqueue ``m3_step_fwd`` on the current stream of the tensors' device."""
    lib = load()
    args = StepArgs()
    for key, val in sizes.items():
        setattr(args, key, int(val))
    args.norm_eps = float(norm_eps)
    device = _cuda_device(tensors)
    args.device = device.index if device.index is not None else torch.cuda.current_device()
    for name in _STEP_TENSORS:
        setattr(args, name, _desc(tensors.get(name)))
    need = lib.m3_step_workspace_bytes(ctypes.byref(args))
    if need < 0:
        _check(int(-need), lib)
    workspace = None
    if need > 0:
        workspace = torch.empty((need + 3) // 4, device=device, dtype=torch.float32)
        args.workspace = _desc(workspace)
    stream = torch.cuda.current_stream(device).cuda_stream
    _check(lib.m3_step_fwd(ctypes.byref(args), ctypes.c_void_p(stream)), lib)


@torch.compiler.disable
def residual_rmsnorm(x: torch.Tensor, m: torch.Tensor | None, w: torch.Tensor, eps: float, *,
                     out_dtype: torch.dtype, out_x: torch.Tensor | None = None) -> torch.Tensor:
    """Enqueue ``m3_residual_rmsnorm`` over the rows of x (+ m): writes the updated residual into
    ``out_x`` when given and returns the normalised rows in ``out_dtype``."""
    lib = load()
    d = x.shape[-1]
    x2 = x.reshape(-1, d)
    out_n = torch.empty(x2.shape, device=x.device, dtype=out_dtype)
    args = NormArgs()
    args.rows, args.dim, args.eps = x2.shape[0], d, float(eps)
    args.device = x.device.index if x.device.index is not None else torch.cuda.current_device()
    args.x, args.w, args.out_n = _desc(x2), _desc(w), _desc(out_n)
    args.m = _desc(m.reshape(-1, d) if m is not None else None)
    args.out_x = _desc(out_x.reshape(-1, d) if out_x is not None else None)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _check(lib.m3_residual_rmsnorm(ctypes.byref(args), ctypes.c_void_p(stream)), lib)
    return out_n.view(x.shape)


@torch.compiler.disable
def scan_summary(*, sizes: dict, tensors: dict, mimo_rotation: bool = False, chunk_hint: int = 64,
                 norm_eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Enqueue ``m3_scan_summary`` (the state pass of a whole slice, for context-parallel prefill).
    Returns the records ``[B, H, m3_scan_summary_floats(R)]`` and, with in-kernel phases, the block
    phase totals ``[B, H, L / 64, 32]`` (float32, on the tensors' device)."""
    lib = load()
    args = ScanArgs()
    for key, val in sizes.items():
        setattr(args, key, int(val))
    args.segments = 1
    args.mimo_rotation = int(mimo_rotation)
    args.chunk_hint = int(chunk_hint)
    args.norm_eps = float(norm_eps)
    device = _cuda_device(tensors)
    args.device = device.index if device.index is not None else torch.cuda.current_device()
    for name in _SCAN_TENSORS:
        setattr(args, name, _desc(tensors.get(name)))
    need = lib.m3_scan_workspace_bytes(ctypes.byref(args))
    if need < 0:
        _check(int(-need), lib)
    workspace = None
    if need > 0:
        workspace = torch.empty((need + 3) // 4, device=device, dtype=torch.float32)
        args.workspace = _desc(workspace)
    floats = lib.m3_scan_summary_floats(int(sizes["rank"]))
    if floats < 0:
        _check(int(-floats), lib)
    batch, heads, length = int(sizes["batch"]), int(sizes["heads"]), int(sizes["length"])
    record = torch.empty(batch, heads, floats, device=device, dtype=torch.float32)
    blocks = None
    if tensors.get("angles") is not None:
        blocks = torch.empty(batch, heads, length // 64, 32, device=device, dtype=torch.float32)
    stream = torch.cuda.current_stream(device).cuda_stream
    _check(lib.m3_scan_summary(ctypes.byref(args), ctypes.c_void_p(record.data_ptr()),
                               ctypes.c_void_p(blocks.data_ptr() if blocks is not None else 0),
                               ctypes.c_void_p(stream)), lib)
    return record, blocks


def last_scan_kernel() -> str:
    return load().m3_last_scan_kernel().decode()


def last_step_kernel() -> str:
    return load().m3_last_step_kernel().decode()


def device_error(clear: bool = True) -> int:
    return load().m3_device_error(int(clear))


@torch.compiler.disable
def scan_forward_noalloc(*, sizes: dict, tensors: dict, reverse: bool = False, mimo_rotation: bool = False,
                         chunk_hint: int = 64, norm_eps: float = 1e-5, segments: int | None = None) -> None:
    """Enqueue ``m3_scan_fwd_noalloc``: the scan with the library's fixed scratch array instead of a
    caller workspace, for hosts that cannot allocate device memory at the call site (see the
    header). Nothing is allocated here either."""
    lib = load()
    lib.m3_scan_fwd_noalloc.argtypes = [ctypes.POINTER(ScanArgs), ctypes.c_void_p]
    lib.m3_scan_fwd_noalloc.restype = ctypes.c_int
    args = ScanArgs()
    args.segments = _segments(segments)
    for key, val in sizes.items():
        setattr(args, key, int(val))
    args.reverse = 2 if reverse == "both" else int(reverse)
    args.mimo_rotation = int(mimo_rotation)
    args.chunk_hint = int(chunk_hint)
    args.norm_eps = float(norm_eps)
    device = _cuda_device(tensors)
    args.device = device.index if device.index is not None else torch.cuda.current_device()
    for name in _SCAN_TENSORS:
        setattr(args, name, _desc(tensors.get(name)))
    stream = torch.cuda.current_stream(device).cuda_stream
    _check(lib.m3_scan_fwd_noalloc(ctypes.byref(args), ctypes.c_void_p(stream)), lib)


def _ssd_args(q: torch.Tensor, tensors: dict, backward: bool) -> SSDArgs:
    """Argument struct of the training kernels, with the scratch they need allocated on q's device."""
    lib = load()
    batch, length, heads, rank, d_state = q.shape
    args = SSDArgs()
    args.batch, args.length, args.heads, args.rank, args.d_state = batch, length, heads, rank, d_state
    args.head_dim = tensors["v"].shape[-1]
    args.device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    for name in _SSD_TENSORS:
        setattr(args, name, _desc(tensors.get(name)))
    need = lib.m3_ssd_workspace_bytes(ctypes.byref(args), int(backward))
    if need < 0:
        _check(int(-need), lib)
    workspace = torch.empty((need + 3) // 4, device=q.device, dtype=torch.float32)
    args.workspace = _desc(workspace)
    args._keep = workspace  # alive until the launch is enqueued (stream-ordered reuse after that)
    return args


@torch.compiler.disable
def ssd_train_forward(q, k, v, adt, diag, initial_state):
    """``m3_ssd_train_fwd``: the SSD core for training on float32 tensors ``q, k [B,L,H,R,N]``,
    ``v [B,L,H,R,P]``, ``adt, diag [B,L,H]``, ``initial_state [B,H,P,N]`` (or None). Returns
    ``(y [B,L,H,R,P], final_state [B,H,P,N], chunk_states)`` (float32)."""
    lib = load()
    batch, length, heads, rank, d_state = q.shape
    head_dim = v.shape[-1]
    rows = lib.m3_ssd_chunk_rows()
    nchunk = (length * rank + rows - 1) // rows
    dev = q.device
    y = torch.empty(batch, length, heads, rank, head_dim, device=dev, dtype=torch.float32)
    final = torch.empty(batch, heads, head_dim, d_state, device=dev, dtype=torch.float32)
    chunks = torch.empty(batch, heads, nchunk, head_dim, d_state, device=dev, dtype=torch.float32)
    args = _ssd_args(q, dict(q=q, k=k, v=v, adt=adt, diag=diag, initial_state=initial_state, y=y,
                             final_state=final, chunk_states=chunks), backward=False)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _check(lib.m3_ssd_train_fwd(ctypes.byref(args), ctypes.c_void_p(stream)), lib)
    return y, final, chunks


@torch.compiler.disable
def ssd_train_backward(q, k, v, adt, diag, chunk_states, dy, dfinal, want_initial: bool):
    """``m3_ssd_train_bwd``: gradients ``(dq, dk, dv, dadt, ddiag, dinitial or None)`` of the SSD
    core from ``dy [B,L,H,R,P]`` and ``dfinal [B,H,P,N]`` (or None), float32."""
    lib = load()
    batch, length, heads, rank, d_state = q.shape
    head_dim = v.shape[-1]
    dev = q.device
    dq, dk = torch.empty_like(q), torch.empty_like(k)
    dv = torch.empty_like(v)
    dadt = torch.empty(batch, length, heads, device=dev, dtype=torch.float32)
    ddiag = torch.empty_like(dadt)
    dinit = (torch.empty(batch, heads, head_dim, d_state, device=dev, dtype=torch.float32)
             if want_initial else None)
    args = _ssd_args(q, dict(q=q, k=k, v=v, adt=adt, diag=diag, chunk_states=chunk_states, dy=dy, dfinal=dfinal,
                             dq=dq, dk=dk, dv=dv, dadt=dadt, ddiag=ddiag, dinitial=dinit), backward=True)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _check(lib.m3_ssd_train_bwd(ctypes.byref(args), ctypes.c_void_p(stream)), lib)
    return dq, dk, dv, dadt, ddiag, dinit


def _prelude_args(q, heads, tensors, num_angles, mimo_rotation) -> PreludeArgs:
    batch, length, groups, rank, d_state = q.shape
    args = PreludeArgs()
    args.batch, args.length, args.groups, args.heads, args.rank = batch, length, groups, heads, rank
    args.d_state, args.num_angles, args.mimo_rotation = d_state, num_angles, int(mimo_rotation)
    args.device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    for name in _PRELUDE_TENSORS:
        setattr(args, name, _desc(tensors.get(name)))
    return args


@torch.compiler.disable
def ssd_prelude_forward(q, k, q_bias, k_bias, phase, scale, heads: int, mimo_rotation: bool):
    """``m3_ssd_prelude_fwd``: float32 core operands ``(qf, kc)`` ``[B,L,H,R,N]`` from the raw
    ``[B,L,G,R,N]`` q / k, biases, phase ``[B,L,H,S]`` (float32 or None) and scale ``[B,L,H]``."""
    lib = load()
    batch, length, _, rank, d_state = q.shape
    qf = torch.empty(batch, length, heads, rank, d_state, device=q.device, dtype=torch.float32)
    kc = torch.empty_like(qf)
    args = _prelude_args(q, heads, dict(q=q, k=k, q_bias=q_bias, k_bias=k_bias, phase=phase, scale=scale, qf=qf,
                                        kc=kc), 0 if phase is None else phase.shape[-1], mimo_rotation)
    _check(lib.m3_ssd_prelude_fwd(ctypes.byref(args), ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)),
           lib)
    return qf, kc


@torch.compiler.disable
def ssd_prelude_backward(q, k, q_bias, k_bias, phase, scale, heads: int, mimo_rotation: bool, dqf, dkc,
                         want_phase: bool):
    """``m3_ssd_prelude_bwd``: ``(dqb, dkb, dphase or None, dscale)``, float32."""
    lib = load()
    dqb, dkb = torch.empty_like(dqf), torch.empty_like(dkc)
    batch, length = q.shape[:2]
    dphase = torch.empty_like(phase, dtype=torch.float32) if (want_phase and phase is not None) else None
    dscale = torch.empty(batch, length, heads, device=q.device, dtype=torch.float32)
    args = _prelude_args(q, heads, dict(q=q, k=k, q_bias=q_bias, k_bias=k_bias, phase=phase, scale=scale, dqf=dqf,
                                        dkc=dkc, dqb=dqb, dkb=dkb, dphase=dphase, dscale=dscale),
                         0 if phase is None else phase.shape[-1], mimo_rotation)
    _check(lib.m3_ssd_prelude_bwd(ctypes.byref(args), ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)),
           lib)
    return dqb, dkb, dphase, dscale


def gemv_eligible(x: torch.Tensor, w: torch.Tensor) -> bool:
    """Few-row projections ``m3_gemv`` serves: 1..4 rows, one 16-bit dtype, contiguous aligned rows."""
    if not (x.is_cuda and w.is_cuda) or x.dtype != w.dtype or x.dtype not in (torch.bfloat16, torch.float16):
        return False
    rows = x.numel() // max(x.shape[-1], 1)
    i = x.shape[-1]
    return (1 <= rows <= 4 and i % 8 == 0 and i <= 16384 and w.dim() == 2 and w.shape[1] == i and w.stride(1) == 1
            and w.stride(0) % 8 == 0 and w.data_ptr() % 16 == 0)


@torch.compiler.disable
def gemv(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` on ``m3_gemv`` for a few rows of x (decode-step projections)."""
    lib = load()
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    y = torch.empty(x2.shape[0], w.shape[0], device=x.device, dtype=x.dtype)
    args = GemvArgs()
    args.out_dim, args.in_dim, args.rows = w.shape[0], w.shape[1], x2.shape[0]
    args.device = x.device.index if x.device.index is not None else torch.cuda.current_device()
    args.x, args.w, args.y = _desc(x2), _desc(w), _desc(y)
    _check(lib.m3_gemv(ctypes.byref(args), ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)), lib)
    return y.view(*x.shape[:-1], w.shape[0])

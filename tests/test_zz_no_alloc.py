"""GPU check of m3_scan_fwd_noalloc, the scan entry point for callers that cannot allocate.

Hosts such as a runtime that owns all device memory through its own pool, or a plugin that must not
use its host process's allocator, cannot hand the scan a freshly allocated workspace. This entry
point uses the library's fixed device scratch array instead. The test runs it twice in a row through
the C ABI and compares with m3_scan_fwd (caller workspace) on the same inputs: both run the same
kernel, so every output must be bit-identical. The file is named
to be collected last, so a run that stops at the first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from mamba3_b200 import Mamba3, _ext

pytestmark = pytest.mark.gpu


def _model_mode_tensors(mixer, projected):
    z, x, B, C, delta, decay, trap, angles = mixer._views(projected)
    batch, length = projected.shape[:2]
    dev = projected.device
    out = dict(
        q=C, k=B, q_norm_w=mixer.C_norm.weight, k_norm_w=mixer.B_norm.weight, q_bias=mixer.C_bias,
        k_bias=mixer.B_bias, value=x, gate=z, adt=decay, dt=delta, trap=trap, dt_bias=mixer.dt_bias, angles=angles,
        D=mixer.D, mimo_x=mixer.mimo_x, mimo_z=mixer.mimo_z, mimo_out=mixer.mimo_out,
        y=torch.empty(batch, length, mixer.nheads, mixer.headdim, device=dev, dtype=projected.dtype),
        final_state=torch.empty(batch, mixer.nheads, mixer.headdim, mixer.d_state, device=dev, dtype=torch.float32),
        final_phase=torch.empty(batch, mixer.nheads, mixer.num_angles, device=dev, dtype=torch.float32),
        final_k=torch.empty(batch, mixer.nheads, mixer.mimo_rank, mixer.d_state, device=dev, dtype=projected.dtype),
    )
    sizes = dict(batch=batch, length=length, groups=mixer.ngroups, heads=mixer.nheads, rank=mixer.mimo_rank,
                 d_state=mixer.d_state, head_dim=mixer.headdim, num_angles=mixer.num_angles)
    return sizes, out


@pytest.mark.parametrize("rank", [1, 4])
def test_noalloc_scan_matches_workspace_scan_twice(rank):
    torch.manual_seed(3 + rank)
    model = Mamba3(256, depth=1, mimo_rank=rank).cuda().to(torch.bfloat16).eval()
    mixer = model.layers[0].mixer
    x = torch.randn(2, 700, 256, device="cuda", dtype=torch.bfloat16)
    kw = dict(mimo_rotation=rank > 1, chunk_hint=mixer.inference_chunk_size, norm_eps=mixer.C_norm.eps)
    with torch.inference_mode():
        projected = mixer.in_proj(x)
        sizes, ref = _model_mode_tensors(mixer, projected)
        _ext.scan_forward(sizes=sizes, tensors=ref, **kw)
        assert _ext.last_scan_kernel() == "umma"  # the variant that uses scratch memory
        for _ in range(2):
            _, got = _model_mode_tensors(mixer, projected)
            _ext.scan_forward_noalloc(sizes=sizes, tensors=got, **kw)
            torch.cuda.synchronize()
            # the same kernel on the same inputs: only the scratch address differs, so the results
            # must agree bit for bit (stale or aliased scratch would show up here)
            for key in ("y", "final_state", "final_phase", "final_k"):
                assert torch.equal(got[key], ref[key]), key
    assert _ext.device_error(clear=True) == 0


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch():
    lib = _ext.load()
    lib.m3_scan_fwd_noalloc.argtypes = [ctypes.POINTER(_ext.ScanArgs), ctypes.c_void_p]
    lib.m3_scan_fwd_noalloc.restype = ctypes.c_int
    args = _ext.ScanArgs()
    args.batch, args.length, args.groups, args.heads, args.rank = 64, 100_000, 1, 8, 1
    args.d_state, args.head_dim, args.num_angles, args.chunk_hint, args.device = 128, 64, 32, 256, 0
    # Descriptors only (nothing is launched): aligned, contiguous-row layouts of the shapes above.
    def desc(nd, dtype=_ext.M3_BF16):
        t = _ext.M3Tensor(data=256, dtype=dtype, ndim=nd)
        for i in range(nd):
            t.stride[i] = 1 if i == nd - 1 else 1024
        return t
    args.q, args.k, args.value, args.gate = desc(5), desc(5), desc(4), desc(4)
    args.dt, args.adt, args.trap = desc(3), desc(3), desc(3)  # per-token scalar columns [B, L, H]
    args.q_norm_w = desc(1, _ext.M3_F32)
    assert lib.m3_scan_workspace_bytes(ctypes.byref(args)) > 8 * 1024 * 1024
    assert lib.m3_scan_fwd_noalloc(ctypes.byref(args), None) == 1  # M3_ERR_SHAPE, nothing launched
    assert b"fixed limit" in lib.m3_last_error()

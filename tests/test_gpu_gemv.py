"""Few-row projection kernel of the decode step (``m3_gemv``) against torch's linear of the same
16-bit operands, and the decode step that uses it against the step without it."""

from __future__ import annotations

import pytest
import torch

from conftest import rel_err
from mamba3_b200 import Mamba3, _ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows", [1, 2, 3, 4])
@pytest.mark.parametrize("shape", [(10768, 2560), (2560, 5120), (37, 264)])
def test_gemv_matches_linear(dtype, rows, shape):
    g = torch.Generator(device="cuda").manual_seed(rows)
    out_dim, in_dim = shape
    w = torch.randn(out_dim, in_dim, device="cuda", generator=g).to(dtype) * 0.05
    x = torch.randn(rows, 1, in_dim, device="cuda", generator=g).to(dtype)
    assert _ext.gemv_eligible(x, w)
    y = _ext.gemv(x, w)
    ref = (x.float() @ w.float().T)  # exact products, FP32 sums: the library GEMM's arithmetic
    assert y.shape == (rows, 1, out_dim) and y.dtype == dtype
    # one rounding of an FP32 sum to the 16-bit output
    assert rel_err(y.float(), ref) < (4e-3 if dtype == torch.bfloat16 else 1e-3)
    torch.testing.assert_close(y, torch.nn.functional.linear(x, w), rtol=1e-2, atol=1e-2)


def test_decode_step_with_fused_stream_and_gemv_matches_layerwise_step(monkeypatch):
    """Mamba3.step on CUDA (fused residual stream, few-row projections on m3_gemv) against the same
    step with both turned off (block-by-block, torch linear)."""
    torch.manual_seed(0)
    model = Mamba3(512, d_state=128, depth=3).cuda().to(torch.bfloat16).eval()
    x = torch.randn(2, 40, 512, device="cuda", dtype=torch.bfloat16)
    xs = torch.randn(2, 1, 512, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        _, cache = model.prefill(x)
        y1, c1 = model.step(xs, cache)
        monkeypatch.setattr(_ext, "gemv_eligible", lambda *args: False)
        monkeypatch.setattr(type(model), "_fused_stream", lambda self, t: False)
        y0, c0 = model.step(xs, cache)
    assert rel_err(y1.float(), y0.float()) < 2e-2
    for a, b in zip(c1, c0):
        assert rel_err(a[1], b[1]) < 1e-2  # FP32 states

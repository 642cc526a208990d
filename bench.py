"""Benchmark: Mamba-3 chunked-SSD prefill on B200 (tokens/s), every other configuration of the
scope table as sub-records, and the reference's own code timed beside it.

Headline workload: Mamba3(d_model=1024, depth=24, d_state=128, mimo_rank=1), FP32 master
weights, bf16 autocast, inference_mode, x ~ N(0,1) [8, 8192, 1024] per GPU. A step is one full
forward over that batch (24 x {in_proj GEMM, chunked-SSD kernel, out_proj GEMM} plus the fused
residual/RMSNorm kernels). Synthetic data and seeded random-init weights (no datasets or
checkpoints on the box).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload siso|mimo|bidir]

Multi-GPU: one process per GPU (torchrun). The global batch is 8 x N sequences; every rank runs
``shard.forward_sharded`` on it: its contiguous share of the batch, then the NCCL all-gather of the
outputs, inside the timed region (weak scaling: per-GPU work is fixed). Time = max over ranks of
CUDA-event time bracketed by barrier + synchronize.

Sub-records of the default run (fewer steps each): ``configs.mimo`` (MIMO-4 prefill),
``configs.bidir`` (bidirectional prefill), ``configs.decode_b{1,64,256}`` and ``configs.decode_r4_b64``
(CUDA-graph decode), each with its own roofline, and ``configs.train`` (forward + backward of one
layer's scan under autograd, beside the reference's training path). At N = 1, ``reference_gpu`` times the reference's
own Triton path (``baseline/_ref``, installed unmodified) on the same GPU, the kernel bar, and
``cpu_baseline`` times the reference's portable PyTorch path on the host cores.

--impl reference times the reference's own CPU implementation (its portable PyTorch path from
``baseline/_ref`` on CPU tensors, fp32, all host threads) on a bounded sample of the same
workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
REF_DIR = ROOT / "baseline" / "_ref"

import numpy as np  # noqa: E402
import torch  # noqa: E402

WORKLOADS = {
    # name: (d_model, depth, mimo_rank, causal, batch, length)
    "siso": (1024, 24, 1, True, 8, 8192),
    "mimo": (2048, 24, 4, True, 16, 4096),
    "bidir": (768, 12, 1, False, 32, 2048),
}
DECODE = dict(d_model=2560, depth=32, batch=64, prefix=2048)
# DRAM bytes (read + write) per token of one scan-kernel launch, from one ncu capture of the same
# kernel on a smaller case of the workload (dram__bytes_read.sum + dram__bytes_write.sum = 192.33 MB
# over 2 x 8192 tokens, d_model 1024, rank 1). Traffic grows with tokens, so the bench scales it.
SCAN_TRAFFIC_PER_TOKEN = {"siso": 192.33e6 / 16384,
                          # d_model 2048, rank 4: 156.67 + 47.51 MB over 2 x 4096 tokens
                          "mimo": 204.18e6 / 8192}


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}, "fallback"


# ---------------------------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------------------------

class ClockSampler:
    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 8:
                    rows.append(parts)
        finally:
            Path(self.path).unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][1]) if rows[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------------------------

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # NCCL prints its version banner on stdout when the communicator comes up; send it to
        # stderr so that stdout carries only the JSON line.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(fn, steps, world):
    """Mean ms per call of `fn` over `steps` calls: CUDA events on the current stream, bracketed by a
    barrier and a synchronize on both sides; max over ranks."""
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(end) / steps, world)


# ---------------------------------------------------------------------------------------------
# Roofline arithmetic
# ---------------------------------------------------------------------------------------------

def build_model(d_model, depth, rank, causal, seed=0):
    """Seeded random-init model, built on the GPU (same architecture and init distributions as the
    reference's constructor; the weights come from the CUDA generator)."""
    from mamba3_b200 import Mamba3
    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = Mamba3(d_model, d_state=128, depth=depth, mimo_rank=rank, causal=causal)
    return model.eval()


def scan_bytes_per_token_layer(model) -> int:
    """Algorithmic HBM bytes of the chunked-SSD kernel per (token, layer): it reads the in_proj
    columns it needs once (z, x, B, C, delta, decay, trap, angles; bf16) and writes y (bf16)."""
    m = model.layers[0].mixer
    read = 2 * (2 * m.d_inner + 2 * m.d_state * m.mimo_rank + 3 * m.nheads + m.num_angles)
    write = 2 * m.d_inner
    return read + write


def scan_flops_per_token_layer(model) -> float:
    """Causal-counted SSD FLOPs per (token, layer) at the reference's inference chunk C (256 at rank 1,
    32 at rank 4): per (b, h, chunk) (CR)(CR+1)(N+P) + 4 C R N P, divided by the C tokens of a chunk
    (82,112 per token-head for SISO, 230,144 for MIMO-4)."""
    m = model.layers[0].mixer
    chunk = m.inference_chunk_size
    cr = chunk * m.mimo_rank
    per_chunk = cr * (cr + 1) * (m.d_state + m.headdim) + 4 * cr * m.d_state * m.headdim
    return m.nheads * per_chunk / chunk


def scan_roofline(model, kernel_ms, tokens, workload, kernel_name):
    pk, pk_kind = peaks()
    bytes_launch = scan_bytes_per_token_layer(model) * tokens
    flops_launch = scan_flops_per_token_layer(model) * tokens
    gbs = bytes_launch / (kernel_ms / 1e3) / 1e9
    tflops = flops_launch / (kernel_ms / 1e3) / 1e12
    traffic = SCAN_TRAFFIC_PER_TOKEN[workload] * tokens if workload in SCAN_TRAFFIC_PER_TOKEN else None
    common = {"peak_kind": pk_kind, "kernel": f"m3 scan ({kernel_name})", "kernel_ms": kernel_ms,
              "algorithmic_bytes_per_launch": bytes_launch, "algorithmic_flops_per_launch": flops_launch}
    if model.mimo_rank > 1:  # arithmetic intensity above the ridge: graded on the tensor pipe
        return {"bound": "tensor", "achieved": tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": tflops / pk["bf16_tflops"], "traffic": traffic, **common,
                "hbm_gbs": gbs, "hbm_frac": gbs / pk["hbm_gbs"]}
    return {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": gbs / pk["hbm_gbs"], "traffic": traffic, **common,
            "tensor_tflops": tflops, "tensor_frac": tflops / pk["bf16_tflops"]}


# ---------------------------------------------------------------------------------------------
# Prefill
# ---------------------------------------------------------------------------------------------

def run_prefill(args, world, rank, local, workload, steps, warmup, full=True):
    """One prefill configuration. `full` adds the e2e, clock and all-gather measurements of the
    headline line; sub-records skip them."""
    from mamba3_b200 import _ext, ops, shard
    d_model, depth, mrank, causal, batch, length = WORKLOADS[workload]
    if full:
        batch = args.batch or batch
        length = args.seq_len or length
        depth = args.depth or depth
    model = build_model(d_model, depth, mrank, causal)
    global_batch = batch * world
    g = torch.Generator(device="cuda").manual_seed(1234)
    x = torch.randn(global_batch, length, d_model, device="cuda", generator=g)
    if world > 1:
        import torch.distributed as dist
        start, stop = shard.shard_bounds(global_batch, world, rank)

        def step():
            with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
                return shard.forward_sharded(model, x)
    else:
        start, stop = 0, batch

        def step():
            with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
                return model(x)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    assert ops.LAST_SCAN_DISPATCH, "scan did not dispatch to the CUDA library"
    with ClockSampler(local) as clocks:
        ms = timed(step, steps, world)
    tokens = global_batch * length
    result = {"value": tokens / (ms / 1e3), "ms_per_step": ms, "steps": steps, "warmup": warmup,
              "config": {"workload": f"{workload}: Mamba3(d_model={d_model}, depth={depth}, d_state=128, "
                                     f"mimo_rank={mrank}, causal={causal}) x[{batch},{length},{d_model}] per GPU, "
                                     "bf16 autocast, full forward",
                         "global_batch": global_batch, "seq_len": length,
                         "parallelism": f"batch-shard x{world}" + (" + NCCL all-gather of the outputs"
                                                                   if world > 1 else ""),
                         "l2": "inputs larger than L2 (per-layer projections 0.5+ GB)"}}
    if full:
        result["clocks"] = clocks.summary()
        if world > 1:
            # the gather alone, on an output of the same shape: its share of the step
            local_out = torch.empty(stop - start, length, d_model, device="cuda")
            gather_ms = timed(lambda: shard.all_gather_batch(local_out, global_batch), steps, world)
            result["all_gather_ms"] = gather_ms
            result["all_gather_share"] = gather_ms / ms

        # End to end through the public API: this rank's share of the pinned host input -> device,
        # forward (+ the all-gather at N > 1), this rank's output -> pinned host.
        host_x = x[start:stop].cpu().pin_memory()
        out_host = torch.empty(stop - start, length, d_model, dtype=torch.float32).pin_memory()

        def e2e_step():
            with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
                xd = host_x.to("cuda", non_blocking=True)
                if world > 1:
                    y = shard.forward_local_gather(model, xd, global_batch)[start:stop]
                else:
                    y = model(xd)
                out_host.copy_(y, non_blocking=True)

        for _ in range(max(1, warmup)):
            e2e_step()
        e2e_ms = timed(e2e_step, steps, world)
        result["e2e"] = {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                         "h2d_bytes_per_step": world * host_x.numel() * host_x.element_size(),
                         "d2h_bytes_per_step": world * out_host.numel() * out_host.element_size()}

    # Kernel roofline: the scan kernel alone on layer 0's projections (CUDA events on its stream).
    mixer = model.layers[0].mixer
    xl = x[start:stop]
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        proj = mixer._project_linear("in_proj", model.layers[0].norm(xl))
        for _ in range(3):
            mixer._scan_fused(proj, None, reverse=False, want_cache=False)
        kernel_ms = timed(lambda: mixer._scan_fused(proj, None, reverse=False, want_cache=False),
                          max(steps, 5), world)
    result["roofline"] = scan_roofline(model, kernel_ms, xl.shape[0] * length, workload, _ext.last_scan_kernel())
    result["layer_ms"] = ms / depth
    # per layer and direction: the token pre-pass and the chunked-SSD kernel; per block boundary one
    # fused residual add + RMSNorm kernel
    result["gpu_launches"] = (depth * 2 * (1 if causal else 2) + depth + 1) * steps
    del model, x, proj
    torch.cuda.empty_cache()
    return result


# ---------------------------------------------------------------------------------------------
# Decode
# ---------------------------------------------------------------------------------------------

def run_decode(world, rank, batch, drank, depth=DECODE["depth"], steps=64, prefix=DECODE["prefix"]):
    """CUDA-graph decode of Mamba3(2560, depth) with bf16 parameters and FP32 state at `batch`: a
    kernel prefill of an N(0,1) prefix, then `steps` timed graph steps (µs per step). The step
    kernels of one layer are also timed alone (as a graph replay, in place) against the state bytes."""
    from mamba3_b200 import _ext, ops
    model = build_model(DECODE["d_model"], depth, drank, True).to(torch.bfloat16)
    decoder = model.cuda_graph(batch_size=batch)
    g = torch.Generator(device="cuda").manual_seed(99 + rank)
    with torch.inference_mode():
        pre = torch.randn(batch, prefix, DECODE["d_model"], device="cuda", dtype=torch.bfloat16, generator=g)
        _, cache = model.prefill(pre)
        for mine, theirs in zip(decoder.cache, cache):
            for dst, src in zip(mine, theirs):
                dst.copy_(src)
        del pre, cache
    xs = torch.randn(16, batch, 1, DECODE["d_model"], device="cuda", dtype=torch.bfloat16, generator=g)
    for i in range(5):
        decoder(xs[i % 16])
    it = iter(range(10 ** 9))
    us = timed(lambda: decoder(xs[next(it) % 16]), steps, world) * 1e3
    step_kernel = _ext.last_step_kernel()
    mixer = model.layers[0].mixer
    cache = mixer.allocate_cache(batch, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        z, xv, B, C, delta, decay, trap, ang = mixer._views(mixer.in_proj(model.layers[0].norm(xs[0])))
        heads = mixer.nheads
        qh, kh = C[:, 0].expand(-1, heads, -1, -1), B[:, 0].expand(-1, heads, -1, -1)

        def kern():
            ops._step_device(qh, kh, xv[:, 0], z[:, 0], decay[:, 0], delta[:, 0], trap[:, 0], ang[:, 0], mixer.D,
                             cache, mimo_x=mixer.mimo_x, mimo_z=mixer.mimo_z, mimo_out=mixer.mimo_out,
                             q_bias=mixer.C_bias, k_bias=mixer.B_bias, out_state=cache[1],
                             q_norm_w=mixer.C_norm.weight, k_norm_w=mixer.B_norm.weight, dt_bias=mixer.dt_bias,
                             norm_eps=mixer.C_norm.eps)
        for _ in range(3):
            kern()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            kern()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            kern()
        kus = timed(graph.replay, 50, world) * 1e3
    pk, pk_kind = peaks()
    state_bytes = 2 * batch * mixer.nheads * mixer.headdim * mixer.d_state * 4
    gbs = state_bytes / (kus / 1e6) / 1e9
    launches = 2 if step_kernel.startswith("two_pass") else 1
    out = {"us_per_step": us, "batch": batch, "steps": steps, "prefix": prefix,
           "model": f"Mamba3(2560, depth={depth}, mimo_rank={drank}) bf16, FP32 state, cuda_graph",
           # per layer: the step kernels, the fused residual + RMSNorm, and (batch <= 4) the two
           # projections on m3_gemv; plus the first norm of a step
           "gpu_launches": (launches + 1 + (2 if batch <= 4 else 0)) * depth * steps + steps,
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": gbs / pk["hbm_gbs"], "peak_kind": pk_kind,
                        "kernel": f"m3 step ({step_kernel})", "kernel_us": kus,
                        "algorithmic_bytes_per_launch": state_bytes,
                        # one layer's state below the 126 MB L2 stays cached between replays
                        "l2_resident": state_bytes < 126e6}}
    del model, decoder, graph
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------------------------
# Training path
# ---------------------------------------------------------------------------------------------

TRAIN = dict(batch=4, length=2048, heads=32, d_state=128, head_dim=64, angles=16)
# Nominal FP32 CUDA-core peak of a B200 (148 SMs x 128 FMA/clock x 2 x 1.965 GHz); no measured
# figure exists for it, so the training kernels' fraction is labelled nominal.
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def train_flops(batch, length, heads, rank, n, p):
    """FP32 flops of the training kernels (forward + backward) as they compute them: per chunk of 32
    rows the full 32 x 32 score blocks, the inter / intra products, the chunk-state products."""
    rows = 32
    chunks = batch * heads * -(-length * rank // rows)
    fwd = rows * rows * n + rows * p * (n + rows) + rows * p * n
    bwd = rows * p * n + rows * rows * (n + p) + 2 * rows * n * (p + rows) + rows * p * n + rows * p * (n + rows)
    return 2.0 * chunks * (fwd + bwd)


def run_train(world, steps=5):
    """Forward + backward of one layer's chunked SSD under autograd (``mamba3_scan`` with every
    optional input, bf16 operands, SISO layer width, [4, 2048] tokens): ours (training kernels +
    PyTorch prelude / epilogue) beside the reference's own training path on the same inputs; and
    the training kernels alone against the nominal FP32 CUDA-core peak."""
    from mamba3_b200 import _ext, ops
    B, L, H, N, P, S = (TRAIN[k] for k in ("batch", "length", "heads", "d_state", "head_dim", "angles"))
    g = torch.Generator(device="cuda").manual_seed(5)

    def mk(*shape, dtype=torch.bfloat16, scale=1.0, shift=0.0):
        return (torch.randn(*shape, generator=g, device="cuda") * scale + shift).to(dtype).requires_grad_(True)

    q, k = mk(B, L, 1, 1, N), mk(B, L, 1, 1, N)
    v, z, trap = mk(B, L, H, P), mk(B, L, H, P), mk(B, L, H)
    adt = (-torch.rand(B, L, H, generator=g, device="cuda") * 0.5).requires_grad_(True)
    dt = (torch.rand(B, L, H, generator=g, device="cuda") * 0.5 + 0.05).requires_grad_(True)
    D = mk(H, dtype=torch.float32)
    kw = dict(chunk_size=512, phase=mk(B, L, H, S, dtype=torch.float32, scale=2.0),
              q_bias=mk(H, 1, N, dtype=torch.float32, scale=0.3), k_bias=mk(H, 1, N, dtype=torch.float32, scale=0.3))

    def step(fn):
        y, st = fn(q, k, v, z, adt, dt, trap, D, **kw)
        (y.float().square().mean() + st.square().mean()).backward()

    for _ in range(2):
        step(ops.mamba3_scan)
    ours_ms = timed(lambda: step(ops.mamba3_scan), steps, world)
    # the kernels alone on float32 core operands
    with torch.no_grad():
        cq = torch.randn(B, L, H, 1, N, device="cuda", generator=g)
        ck = torch.randn(B, L, H, 1, N, device="cuda", generator=g)
        cv = torch.randn(B, L, H, 1, P, device="cuda", generator=g)
        cadt = -torch.rand(B, L, H, device="cuda", generator=g) * 0.5
        cdiag = torch.rand(B, L, H, device="cuda", generator=g)
        cdy = torch.randn(B, L, H, 1, P, device="cuda", generator=g)

    def kernels():
        _, _, chunks = _ext.ssd_train_forward(cq, ck, cv, cadt, cdiag, None)
        _ext.ssd_train_backward(cq, ck, cv, cadt, cdiag, chunks, cdy, None, want_initial=False)

    for _ in range(3):
        kernels()
    kern_ms = timed(kernels, steps, world)
    flops = train_flops(B, L, H, 1, N, P)
    out = {"ms": ours_ms, "shape": f"mamba3_scan fwd+bwd, x[{B},{L}] x {H} heads, N {N}, P {P}, bf16 operands",
           "kernels_ms": kern_ms,
           "kernels_roofline": {"bound": "fp32 CUDA cores", "achieved": flops / (kern_ms / 1e3) / 1e12,
                                "peak": FP32_NOMINAL_TFLOPS, "unit": "TFLOP/s",
                                "frac": flops / (kern_ms / 1e3) / 1e12 / FP32_NOMINAL_TFLOPS,
                                "peak_kind": "nominal", "flops_per_launch_pair": flops},
           "gpu_launches": 8 * (steps + 2)}
    if world == 1:
        try:
            import_reference()
            import importlib
            rops = importlib.import_module("mamba3.ops")
            for _ in range(2):
                step(rops.mamba3_scan)
            ref_ms = timed(lambda: step(rops.mamba3_scan), steps, world)
            out["reference_ms"] = ref_ms
            out["speedup"] = ref_ms / ours_ms
            out["reference_impl"] = "reference training path (baseline/_ref mamba3_scan under autograd, same GPU)"
        except Exception as exc:  # reported, not hidden
            out["reference_error"] = f"{type(exc).__name__}: {exc}"
    del q, k, v, z, cq, ck, cv, cdy
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------------------------
# The reference's own code: Triton path on the GPU, portable PyTorch path on the host cores
# ---------------------------------------------------------------------------------------------

def import_reference():
    """The unmodified reference package installed into baseline/_ref (pip --target)."""
    if not (REF_DIR / "mamba3" / "__init__.py").exists():
        raise RuntimeError("baseline/_ref is not installed")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import mamba3
    return mamba3


def reference_gpu(workload, kernel_ms, layer_ms, steps=5):
    """The reference's Triton path (MAMBA3_DISABLE_TRITON unset) on this GPU, same per-GPU shape:
    its mamba3_scan per layer (Python chunk loop of Triton launches, expanded rotated q/k) on its own
    layer-0 projections, and one whole block (projection, phase loop, scan, out_proj)."""
    d_model, depth, mrank, causal, batch, length = WORKLOADS[workload]
    try:
        ref = import_reference()
        torch.manual_seed(0)
        with torch.device("cuda"):
            model = ref.Mamba3(d_model, d_state=128, depth=1, mimo_rank=mrank, causal=causal).eval()
        x = torch.randn(batch, length, d_model, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7))
        mixer = model.layers[0].mixer
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            q, k, xv, z, adt, dt, trap, ang = mixer._project(model.layers[0].norm(x))
            phase = mixer._phase(ang, dt, None)

            def scan():
                return ref.ops.mamba3_scan(q, k, xv, z, adt, dt, trap, mixer.D, mimo_x=mixer.mimo_x,
                                           mimo_z=mixer.mimo_z, mimo_out=mixer.mimo_out,
                                           chunk_size=mixer.inference_chunk_size, phase=phase,
                                           mimo_rotation=mrank > 1, q_bias=mixer.C_bias, k_bias=mixer.B_bias)
            scan()
            triton = bool(ref.ops._TRITON_LAST_SCAN_DISPATCH)
            scan_ms = timed(scan, steps, 1)
            block = lambda: model.layers[0](x)
            block()
            block_ms = timed(block, steps, 1)
        del model, x, q, k, xv, z, phase
        torch.cuda.empty_cache()
        return {"impl": "reference Triton path (baseline/_ref, unmodified)" if triton else
                        "reference portable PyTorch path on CUDA (Triton declined the call)",
                "triton_dispatch": triton, "triton_ms": scan_ms, "kernel_ms": kernel_ms,
                "scan_speedup": scan_ms / kernel_ms, "reference_layer_ms": block_ms, "layer_ms": layer_ms,
                "layer_speedup": block_ms / layer_ms,
                "shape": f"Mamba3({d_model}, mimo_rank={mrank}, causal={causal}) one layer, x[{batch},{length}]"}
    except Exception as exc:  # recorded in the line, never a fallback for our own numbers
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}


def reference_gpu_all(configs: dict, head_workload: str, head: dict) -> dict:
    """The reference Triton bar for every prefill configuration measured in this run (one layer
    each, same per-GPU shape), beside our per-layer and scan-kernel times."""
    out = {head_workload: reference_gpu(head_workload, head["roofline"]["kernel_ms"], head["layer_ms"])}
    for wl, sub in configs.items():
        if wl in WORKLOADS:
            out[wl] = reference_gpu(wl, sub["roofline"]["kernel_ms"], sub["layer_ms"], steps=2)
    return out


def reference_gpu_decode(batch, our_us_per_layer, steps=64):
    """The reference's CUDA-graph decoder (its Triton step kernel) at the decode shape, depth 4,
    per layer beside ours."""
    try:
        ref = import_reference()
        torch.manual_seed(0)
        depth = 4
        with torch.device("cuda"):
            model = ref.Mamba3(DECODE["d_model"], d_state=128, depth=depth).to(torch.bfloat16).eval()
        decoder = model.cuda_graph(batch_size=batch)
        xs = torch.randn(16, batch, 1, DECODE["d_model"], device="cuda", dtype=torch.bfloat16)
        for i in range(5):
            decoder(xs[i % 16])
        it = iter(range(10 ** 9))
        us = timed(lambda: decoder(xs[next(it) % 16]), steps, 1) * 1e3
        triton = bool(getattr(ref.ops, "_TRITON_LAST_DISPATCH", False))
        del model, decoder
        torch.cuda.empty_cache()
        return {"reference_us_per_layer": us / depth, "us_per_layer": our_us_per_layer,
                "layer_speedup": us / depth / our_us_per_layer, "triton_dispatch": triton, "batch": batch}
    except Exception as exc:
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}


def cpu_config1() -> dict:
    """The CPU-reference configuration in full on the host cores with the reference's portable
    PyTorch path: Mamba3(256, depth=4), fp32, manual_seed(0), x ~ N(0,1) [2, 1024, 256]: forward,
    then prefill of the same x and 64 step() calls with fresh N(0,1) [2, 1, 256] inputs."""
    try:
        ref = import_reference()
    except RuntimeError as exc:
        return {"unavailable": str(exc)}
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    torch.manual_seed(0)
    model = ref.Mamba3(256, d_state=128, depth=4, mimo_rank=1).eval()
    x = torch.randn(2, 1024, 256)
    steps = torch.randn(64, 2, 1, 256)
    with torch.inference_mode():
        model(x)
        t0 = time.perf_counter()
        model(x)
        t1 = time.perf_counter()
        _, cache = model.prefill(x)
        t2 = time.perf_counter()
        for i in range(64):
            _, cache = model.step(steps[i], cache)
        t3 = time.perf_counter()
    return {"forward_ms": (t1 - t0) * 1e3, "forward_tokens_per_s": 2048 / (t1 - t0), "prefill_ms": (t2 - t1) * 1e3,
            "step_ms": (t3 - t2) * 1e3 / 64, "cores": cores,
            "impl": "reference mamba3 (baseline/_ref) portable PyTorch path on CPU tensors, fp32"}


def gpu_config1() -> dict:
    """The same CPU-reference configuration through this package on the GPU (fp32: the CUDA-core
    scan kernel)."""
    from mamba3_b200 import Mamba3
    torch.manual_seed(0)
    model = Mamba3(256, d_state=128, depth=4, mimo_rank=1).eval().cuda()
    x = torch.randn(2, 1024, 256).cuda()
    steps = torch.randn(64, 2, 1, 256).cuda()
    with torch.inference_mode():
        for _ in range(3):
            model(x)
        fwd = timed(lambda: model(x), 10, 1)
        pre = timed(lambda: model.prefill(x), 10, 1)
        _, cache = model.prefill(x)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record()
        for i in range(64):
            _, cache = model.step(steps[i], cache)
        ev1.record()
        torch.cuda.synchronize()
    return {"forward_ms": fwd, "forward_tokens_per_s": 2048 / (fwd / 1e3), "prefill_ms": pre,
            "step_ms": ev0.elapsed_time(ev1) / 64, "dtype": "f32"}


def cpu_sample(workload, tokens=None) -> dict:
    """The reference's portable PyTorch path on CPU tensors (fp32, all host threads) on a bounded
    sample: one layer of the workload's model on one sequence; reported as whole-model tokens/s
    (per-layer rate / depth). Falls back to the numpy port only when baseline/_ref is absent."""
    d_model, depth, mrank, causal, _, length = WORKLOADS[workload]
    tokens = tokens or (length if mrank == 1 else 1024)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    x = torch.randn(1, tokens, d_model, generator=torch.Generator().manual_seed(0))
    try:
        ref = import_reference()
    except RuntimeError:
        ref = None
    if ref is not None:
        torch.manual_seed(0)
        model = ref.Mamba3(d_model, d_state=128, depth=1, mimo_rank=mrank, causal=causal).eval()
        with torch.inference_mode():
            t0 = time.perf_counter()
            model(x)
            sec = time.perf_counter() - t0
        return {"value": tokens / sec / depth, "unit": "tokens/s", "cores": cores, "kind": "reference",
                "sample": f"reference mamba3 (baseline/_ref) portable PyTorch path on CPU tensors, fp32, "
                          f"{cores} threads: 1 of {depth} layers of the {workload} config on 1 x {tokens} "
                          f"tokens; rate / depth"}
    from oracle import mamba3_oracle as O
    from mamba3_b200 import Mamba3
    torch.manual_seed(0)
    layer = Mamba3(d_model, d_state=128, depth=1, mimo_rank=mrank, causal=causal)
    sd = {k: v.numpy() for k, v in layer.state_dict().items()}
    t0 = time.perf_counter()
    O.model_forward(O.ModelConfig(d_model, 128, 1, mrank, causal), sd, x.numpy())
    sec = time.perf_counter() - t0
    return {"value": tokens / sec / depth, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"numpy port (float64) of the reference algorithm, {cores} threads, 1 of {depth} layers, "
                      f"1 x {tokens} tokens of the {workload} config; rate / depth (baseline/_ref absent)"}


# ---------------------------------------------------------------------------------------------
# Main
# ---------------------------------------------------------------------------------------------

def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="siso")
    p.add_argument("--no-extras", action="store_true", help="headline line only (profiling)")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-ref-gpu", action="store_true")
    p.add_argument("--only", choices=["prefill", "decode", "train"], default=None,
                   help="run one part (profiling cases)")
    p.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (profiling cases)")
    p.add_argument("--seq-len", type=int, default=0, help="override the sequence length (profiling cases)")
    p.add_argument("--depth", type=int, default=0, help="override the depth (profiling cases)")
    p.add_argument("--decode-rank", type=int, default=1, help="MIMO rank of the decode model (--only decode)")
    args = p.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        samples = [cpu_sample(args.workload) for _ in range(max(0, args.warmup) + max(1, min(args.steps, 3)))]
        timed_samples = samples[max(0, args.warmup):] or samples
        value = statistics.median(s["value"] for s in timed_samples)
        base = dict(timed_samples[0], value=value)
        print(json.dumps({
            "impl": "reference", "metric": "prefill_tokens_per_s", "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,1) inputs, seeded random-init weights",
            "config": {"workload": f"{args.workload} (bounded CPU sample, see cpu_baseline.sample)"},
            "cpu_baseline": base,
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    world, rank, local = dist_setup()
    if args.only == "train":
        result = {"train": run_train(world, steps=max(args.steps, 2))}
        if rank == 0:
            print(json.dumps(result))
        return
    if args.only == "decode":
        result = {"decode": run_decode(world, rank, args.batch or DECODE["batch"], args.decode_rank,
                                       depth=args.depth or DECODE["depth"], steps=max(args.steps, 16))}
        if rank == 0:
            print(json.dumps(result))
        return
    head = run_prefill(args, world, rank, local, args.workload, args.steps, args.warmup, full=True)
    result = {
        "metric": "prefill_tokens_per_s", "value": head["value"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1) inputs, seeded random-init weights", "config": head["config"],
        "e2e": head["e2e"], "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
        "roofline": head["roofline"], "layer_ms": head["layer_ms"],
    }
    for key in ("all_gather_ms", "all_gather_share"):
        if key in head:
            result[key] = head[key]
    if not args.no_extras and args.only is None:
        extra_steps = max(2, args.steps // 5)
        configs = {}
        for wl in WORKLOADS:
            if wl == args.workload:
                continue
            sub = run_prefill(args, world, rank, local, wl, extra_steps, 2, full=False)
            configs[wl] = sub
        for name, batch, drank in (("decode_b1", 1, 1), ("decode_b64", 64, 1), ("decode_b256", 256, 1),
                                   ("decode_r4_b64", 64, 4)):
            configs[name] = run_decode(world, rank, batch, drank, steps=64 if batch < 256 else 32)
        configs["train"] = run_train(world)
        result["configs"] = configs
        result["gpu_launches"] += sum(c.get("gpu_launches", 0) for c in configs.values())
    if rank == 0 and world == 1 and not args.no_ref_gpu and args.only is None:
        if "configs" in result:
            result["reference_gpu"] = reference_gpu_all(result["configs"], args.workload, head)
        else:
            result["reference_gpu"] = {args.workload: reference_gpu(args.workload, head["roofline"]["kernel_ms"],
                                                                    head["layer_ms"])}
        if "configs" in result:
            ours = result["configs"]["decode_b64"]["us_per_step"] / DECODE["depth"]
            result["reference_gpu_decode"] = reference_gpu_decode(64, ours)
    if rank == 0 and world == 1 and not args.no_cpu and args.only is None:
        result["cpu_baseline"] = cpu_sample(args.workload)
        if not args.no_extras:
            result["config1"] = {"gpu": gpu_config1(), "cpu_reference": cpu_config1()}
    if rank == 0:
        print(json.dumps(result))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

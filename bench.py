"""Benchmark: Mamba-3 chunked-SSD prefill on B200 (tokens/s), plus the decode step (us/step).

Default workload: Mamba3(d_model=1024, depth=24, d_state=128, mimo_rank=1),
FP32 master weights, bf16 autocast, inference_mode, x ~ N(0,1) [8, 8192, 1024] per GPU.
A step is one full forward over that batch (24 x {in_proj GEMM, chunked-SSD kernel, out_proj
GEMM}). Synthetic data and seeded random-init weights (no datasets/checkpoints on the box).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload siso|mimo|bidir]

Multi-GPU: one process per GPU (torchrun), each rank runs its own batch of 8 sequences (weak
scaling, batch sharding); there is no data-path collective. Time = max over ranks of CUDA-event
time bracketed by barrier + synchronize.

--impl reference times the reference algorithm's CPU implementation (the numpy port in oracle/,
the only CPU code here) on a bounded sample of the same workload with all host threads; rank 0
only.
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

import numpy as np  # noqa: E402
import torch  # noqa: E402

WORKLOADS = {
    # name: (d_model, depth, mimo_rank, causal, batch, length)
    "siso": (1024, 24, 1, True, 8, 8192),
    "mimo": (2048, 24, 4, True, 16, 4096),
    "bidir": (768, 12, 1, False, 32, 2048),
}
DECODE = dict(d_model=2560, depth=32, batch=64)
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


# ---------------------------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------------------------

def build_model(d_model, depth, rank, causal, seed=0):
    from mamba3_b200 import Mamba3
    torch.manual_seed(seed)
    return Mamba3(d_model, d_state=128, depth=depth, mimo_rank=rank, causal=causal).cuda().eval()


def timed(fn, steps, world):
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


def scan_bytes_per_token_layer(model) -> int:
    """Algorithmic HBM bytes of the chunked-SSD kernel per (token, layer): it reads the in_proj
    columns it needs once (z, x, B, C, delta, decay, trap, angles; bf16) and writes y (bf16)."""
    m = model.layers[0].mixer
    read = 2 * (2 * m.d_inner + 2 * m.d_state * m.mimo_rank + 3 * m.nheads + m.num_angles)
    write = 2 * m.d_inner
    return read + write


def scan_flops_per_token_layer(model, chunk) -> float:
    """Causal-counted SSD FLOPs per (token, layer): per (b, h, chunk of C tokens, R ranks)
    (CR)(CR+1)(N+P) + 4 CR N P, divided by C tokens."""
    m = model.layers[0].mixer
    cr = chunk * m.mimo_rank
    per_chunk = cr * (cr + 1) * (m.d_state + m.headdim) + 4 * cr * m.d_state * m.headdim
    return m.nheads * per_chunk / chunk


def run_prefill(args, world, rank, local):
    from mamba3_b200 import _ext, ops
    d_model, depth, mrank, causal, batch, length = WORKLOADS[args.workload]
    batch = args.batch or batch
    length = args.seq_len or length
    depth = args.depth or depth
    model = build_model(d_model, depth, mrank, causal)
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    x = torch.randn(batch, length, d_model, device="cuda", generator=g)

    def step():
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            return model(x)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert ops.LAST_SCAN_DISPATCH, "scan did not dispatch to the CUDA library"
    with ClockSampler(local) as clocks:
        ms = timed(step, args.steps, world)
    tokens = batch * length * world
    value = tokens / (ms / 1e3)

    # End to end through the public API: pinned host input -> device, forward, output -> host.
    host_x = x.cpu().pin_memory()
    out_host = torch.empty(batch, length, d_model, dtype=torch.float32).pin_memory()

    def e2e_step():
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            xd = host_x.to("cuda", non_blocking=True)
            y = model(xd)
            out_host.copy_(y, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    e2e_ms = timed(e2e_step, args.steps, world)

    # Kernel roofline: the scan kernel alone on layer 0's projections (CUDA events on its stream).
    mixer = model.layers[0].mixer
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        proj = mixer.in_proj(model.layers[0].norm(x))
        for _ in range(3):
            mixer._scan_fused(proj, None, reverse=False, want_cache=False)
        kernel_ms = timed(lambda: mixer._scan_fused(proj, None, reverse=False, want_cache=False), args.steps, world)
    kernel_name = _ext.last_scan_kernel()
    pk, pk_kind = peaks()
    bytes_launch = scan_bytes_per_token_layer(model) * batch * length
    flops_launch = scan_flops_per_token_layer(model, 128 // mrank if mrank > 1 else 128) * batch * length
    achieved = bytes_launch / (kernel_ms / 1e3) / 1e9
    tflops = flops_launch / (kernel_ms / 1e3) / 1e12
    # per layer and direction: the token pre-pass and the chunked-SSD kernel; per block boundary one
    # fused residual add + RMSNorm
    launches_per_step = depth * 2 * (1 if causal else 2) + depth + 1  # + residual add / RMSNorm kernels
    traffic = (SCAN_TRAFFIC_PER_TOKEN[args.workload] * batch * length
               if args.workload in SCAN_TRAFFIC_PER_TOKEN else None)
    common = {"peak_kind": pk_kind, "kernel": f"m3 scan ({kernel_name})", "kernel_ms": kernel_ms,
              "algorithmic_bytes_per_launch": bytes_launch, "algorithmic_flops_per_launch": flops_launch}
    if mrank > 1:  # arithmetic intensity above the ridge: graded on the tensor pipe
        roofline = {"bound": "tensor", "achieved": tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": tflops / pk["bf16_tflops"], "traffic": traffic, **common,
                    "hbm_gbs": achieved, "hbm_frac": achieved / pk["hbm_gbs"]}
    else:
        roofline = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / pk["hbm_gbs"], "traffic": traffic, **common,
                    "tensor_tflops": tflops, "tensor_frac": tflops / pk["bf16_tflops"]}
    result = {
        "metric": "prefill_tokens_per_s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic N(0,1) inputs, seeded random-init weights",
        "config": {"workload": f"{args.workload}: Mamba3(d_model={d_model}, depth={depth}, d_state=128, "
                               f"mimo_rank={mrank}, causal={causal}) x[{batch},{length},{d_model}] per GPU, "
                               "bf16 autocast, full forward",
                   "global_batch": batch * world, "seq_len": length, "parallelism": f"batch-shard x{world}",
                   "l2": "inputs larger than L2 (per-layer projections 0.5+ GB)"},
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": host_x.numel() * host_x.element_size(),
                "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
        "roofline": roofline,
    }
    return result


def run_decode(args, world, rank):
    """CUDA-graph decode step of Mamba3(2560, depth=32) at batch 64 (bf16 params, FP32 state);
    `--only decode` with `--batch` / `--depth` / `--decode-rank` measures the other decode cases."""
    from mamba3_b200 import ops
    batch = (args.batch if args.only == "decode" and args.batch else DECODE["batch"])
    depth = (args.depth if args.only == "decode" and args.depth else DECODE["depth"])
    drank = args.decode_rank
    model = build_model(DECODE["d_model"], depth, drank, True).to(torch.bfloat16)
    decoder = model.cuda_graph(batch_size=batch)
    g = torch.Generator(device="cuda").manual_seed(99 + rank)
    xs = torch.randn(16, batch, 1, DECODE["d_model"], device="cuda", dtype=torch.bfloat16, generator=g)
    for i in range(5):
        decoder(xs[i % 16])
    n = max(args.steps * 10, 50)
    it = iter(range(10 ** 9))
    us = timed(lambda: decoder(xs[next(it) % 16]), n, world) * 1e3
    # step-kernel roofline: one layer's step kernel alone, in place (as in the graph)
    mixer = model.layers[0].mixer
    cache = mixer.allocate_cache(batch, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        q, k, xv, z, adt, dt, trap, ang = mixer._project(mixer_input := model.layers[0].norm(xs[0]))
        qh = q[:, 0].expand(-1, mixer.nheads, -1, -1)
        kh = k[:, 0].expand(-1, mixer.nheads, -1, -1)

        def kern():
            ops._step_device(qh, kh, xv[:, 0], z[:, 0], adt[:, 0], dt[:, 0], trap[:, 0], ang[:, 0], mixer.D, cache,
                             mimo_x=mixer.mimo_x, mimo_z=mixer.mimo_z, mimo_out=mixer.mimo_out,
                             q_bias=mixer.C_bias, k_bias=mixer.B_bias,
                             out_state=cache[1])
        for _ in range(3):
            kern()
        # Timed as a graph replay, as the decoder runs it: at small batch a Python-launched call
        # measures the host, not the kernels.
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            kern()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            kern()
        kus = timed(graph.replay, 50, world) * 1e3
    del mixer_input
    pk, _ = peaks()
    state_bytes = 2 * batch * mixer.nheads * mixer.headdim * mixer.d_state * 4
    return {"us_per_step": us, "batch": batch, "model": f"Mamba3(2560, depth={depth}, mimo_rank={drank}) bf16",
            "step_kernel_us": kus, "step_kernel_state_gbs": state_bytes / (kus / 1e6) / 1e9,
            "step_kernel_frac": state_bytes / (kus / 1e6) / 1e9 / pk["hbm_gbs"],
            "state_bytes_per_layer": state_bytes,
            # one layer's state below the 126 MB L2 stays cached between replays of the kernel alone
            "step_kernel_l2_resident": state_bytes < 126e6}


def cpu_baseline(args, sample_tokens=None) -> dict:
    """The numpy port of the reference algorithm on the host cores, on a bounded sample:
    one layer of the same model config, one sequence of `sample_tokens` tokens; reported as
    whole-model tokens/s (per-layer rate / depth)."""
    from oracle import mamba3_oracle as O
    from mamba3_b200 import Mamba3
    d_model, depth, mrank, causal, _, length = WORKLOADS[args.workload]
    sample_tokens = sample_tokens or (2048 if mrank == 1 else 512)
    torch.manual_seed(0)
    layer = Mamba3(d_model, d_state=128, depth=1, mimo_rank=mrank, causal=causal)
    sd = {k: v.numpy() for k, v in layer.state_dict().items()}
    cfg = O.ModelConfig(d_model, 128, 1, mrank, causal)
    x = np.random.default_rng(0).standard_normal((1, sample_tokens, d_model))
    t0 = time.perf_counter()
    O.model_forward(cfg, sd, x)
    sec = time.perf_counter() - t0
    cores = os.cpu_count() or 1
    return {"value": sample_tokens / sec / depth, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"numpy oracle (float64, BLAS on {cores} threads), 1 of {depth} layers, "
                      f"1 x {sample_tokens} tokens of the {args.workload} config; rate / depth"}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="siso")
    p.add_argument("--no-decode", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--only", choices=["prefill", "decode"], default=None,
                   help="run one part (profiling); the default run measures both")
    p.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (profiling cases)")
    p.add_argument("--seq-len", type=int, default=0, help="override the sequence length (profiling cases)")
    p.add_argument("--depth", type=int, default=0, help="override the depth (profiling cases)")
    p.add_argument("--decode-rank", type=int, default=1, help="MIMO rank of the decode model")
    args = p.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        samples = [cpu_baseline(args)["value"] for _ in range(max(1, args.warmup) + max(1, min(args.steps, 3)))]
        base = cpu_baseline(args)
        value = statistics.median(samples[max(1, args.warmup):] or samples)
        base["value"] = value
        d_model, depth, mrank, causal, batch, length = WORKLOADS[args.workload]
        print(json.dumps({
            "impl": "reference", "metric": "prefill_tokens_per_s", "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic N(0,1) inputs, seeded random-init weights",
            "config": {"workload": f"{args.workload} (bounded CPU sample, see cpu_baseline.sample)"},
            "cpu_baseline": base,
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    world, rank, local = dist_setup()
    if args.only == "decode":
        result = {"decode": run_decode(args, world, rank)}
    else:
        result = run_prefill(args, world, rank, local)
        if not args.no_decode and args.only != "prefill":
            result["decode"] = run_decode(args, world, rank)
    if rank == 0 and world == 1 and not args.no_cpu and args.only is None:
        result["cpu_baseline"] = cpu_baseline(args)
    if rank == 0:
        print(json.dumps(result))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

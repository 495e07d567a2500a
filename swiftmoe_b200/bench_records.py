"""Benchmark records in the reference's schema, on this package's layers.

The reference's driver (experiments/benchmark_suite.py:79-164) times a layer with 10
warm-up forwards and 100 forwards each bracketed by torch.cuda.synchronize() and CUDA
events (:44-77), then writes one record per configuration (:134-152) and a
``<name>_ws<N>.json`` file per world size (:205-219).  ``run_single_config`` does the
same for ``swiftmoe_b200.StandardMoE`` ("baseline") and ``UltimateMoE`` ("ultimate"),
with identical keys, so the reference's analysis scripts read these results unchanged.

    torchrun --nproc-per-node 8 -m swiftmoe_b200.bench_records --out results/comprehensive

runs the reference's grid (d_model 1024; 64, 128 and 256 experts; batch 512..8192 per
rank; linear experts, fp16, top-2; :166-200).
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
from typing import Dict, List

import numpy as np
import torch
import torch.distributed as dist

from .baseline_moe import StandardMoE
from .ultimate_moe import UltimateMoE


@torch.no_grad()
def measure_latency(model, x, iterations: int = 100):
    """Per-iteration CUDA-event latency with a synchronize on both sides (:50-77); the
    forward runs as inference (no gradient recording)."""
    times = []
    for _ in range(iterations):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        model(x)
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return float(np.mean(times)), float(np.std(times)), times


def run_single_config(model_type: str, num_experts: int, d_model: int, batch_size: int, *, device,
                      world_size: int = 1, use_triton: bool = True, use_nccl_opt: bool = True,
                      enable_profiling: bool = False, warmup: int = 10, iterations: int = 100,
                      **layer_kwargs) -> Dict:
    if model_type == "baseline":
        model = StandardMoE(num_experts=num_experts, d_model=d_model, use_fp16=True, device=device,
                            **layer_kwargs)
    elif model_type == "ultimate":
        model = UltimateMoE(num_experts=num_experts, d_model=d_model, use_fp16=True, use_triton=use_triton,
                            use_nccl_opt=use_nccl_opt, enable_profiling=enable_profiling, device=device,
                            **layer_kwargs)
    else:
        raise ValueError(f"unknown model type {model_type}")
    x = torch.randn(batch_size, d_model, device=device, dtype=torch.float16)
    with torch.no_grad():
        for _ in range(warmup):
            model(x)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    if enable_profiling:
        model.reset_profiling()
    mean, std, times = measure_latency(model, x, iterations)
    breakdown = model.get_profile_summary() if enable_profiling else {}
    return {
        "model_type": model_type, "world_size": world_size, "batch_size": batch_size,
        "num_experts": num_experts, "d_model": d_model, "use_triton": use_triton, "use_nccl_opt": use_nccl_opt,
        "latency_mean_ms": mean, "latency_std_ms": std, "latency_min_ms": float(np.min(times)),
        "latency_max_ms": float(np.max(times)), "latency_p50_ms": float(np.percentile(times, 50)),
        "latency_p95_ms": float(np.percentile(times, 95)), "latency_p99_ms": float(np.percentile(times, 99)),
        "throughput_tokens_per_sec": batch_size * world_size / (mean / 1000.0),
        "max_memory_gb": torch.cuda.max_memory_allocated(device) / 1e9,
        **breakdown,
    }


def reference_grid() -> List[tuple]:
    return [(e, b) for e in (64, 128, 256) for b in (512, 1024, 2048, 4096, 8192)]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="results/comprehensive")
    ap.add_argument("--name", default="comprehensive_benchmark")
    ap.add_argument("--iterations", type=int, default=100)
    ap.add_argument("--grid", default="reference", choices=["reference", "quick"])
    args = ap.parse_args(argv)
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    rank = dist.get_rank() if ws > 1 else 0
    grid = reference_grid() if args.grid == "reference" else [(128, 2048)]
    results = []
    for (E, bs) in grid:
        for kind, prof in (("baseline", False), ("ultimate", True)):
            r = run_single_config(kind, E, 1024, bs, device=dev, world_size=ws, enable_profiling=prof,
                                  iterations=args.iterations)
            results.append(r)
            if rank == 0:
                print(f"{kind:8s} E={E:3d} BS={bs:5d} ws={ws}: {r['latency_mean_ms']:.3f} ms, "
                      f"{r['throughput_tokens_per_sec']:.0f} tok/s", flush=True)
        if ws > 1:
            dist.barrier()
    if rank == 0:
        out = Path(args.out)
        out.mkdir(parents=True, exist_ok=True)
        path = out / f"{args.name}_ws{ws}.json"
        path.write_text(json.dumps(results, indent=2))
        print(f"results saved to {path}")
    if ws > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

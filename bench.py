#!/usr/bin/env python
"""MoE-layer forward benchmark (tokens/s) on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl swiftmoe|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload: the Mixtral-shaped MoE layer, bf16: d_model=4096, 8 experts, top-2 softmax
gating, SwiGLU d_ff=14336, 16384 tokens per GPU ~ N(0,1), weights N(0, 0.02), no
router bias, no capacity limit (synthetic, seeded; no dataset is involved).  At N GPUs
the experts are split 8/N per GPU (expert parallelism, all-to-all over NCCL) and every
GPU routes its own 16384 tokens (weak scaling).

One step = one forward of the layer over one batch.  `value` is the whole-job
throughput with the input already resident in HBM; `e2e` is the same forward through
the public module API with the input copied from pinned host memory and the output
copied back inside the timed region.  `--impl reference` times the reference algorithm
on the host CPU (the numpy restatement in oracle/, since the reference is pure Python
torch with no SwiGLU expert) on a bounded token sample of the same layer.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer fwd tokens/sec at 1/2/4/8 B200; exposed all-to-all ms; % of roofline"
# Workloads (tokens are per GPU).  "mixtral" is the default and the headline line; the
# others are the remaining layer shapes of the benchmark configurations, measured with
# the same harness.
WORKLOADS = {
    "mixtral": dict(d=4096, E=8, k=2, F=14336, T=16384, dtype="bf16", cf=None, shared=0, bias_std=0.0,
                    name="mixtral-moe-layer-fwd: d_model 4096, 8 experts top-2 softmax, SwiGLU d_ff 14336, "
                         "16384 tok/GPU, bf16"),
    "ep-capacity": dict(d=4096, E=64, k=2, F=4096, T=8192, dtype="bf16", cf=1.25, shared=0, bias_std=0.0,
                        name="ep-moe-layer-fwd: d_model 4096, 64 experts top-2, SwiGLU d_ff 4096, 8192 tok/GPU, "
                             "capacity factor 1.25 (overflow dropped in index order), bf16"),
    "fine-grained": dict(d=2048, E=128, k=8, F=1024, T=32768, dtype="bf16", cf=None, shared=1, bias_std=1.5,
                         name="fine-grained-moe-layer-fwd: d_model 2048, 128 experts + 1 shared, top-8, SwiGLU "
                              "d_ff 1024, 32768 tok/GPU, router offsets ~N(0,1.5), bf16"),
    "cpu-runnable-fp32": dict(d=512, E=8, k=2, F=2048, T=4096, dtype="fp32", cf=None, shared=0, bias_std=0.0,
                              name="small-moe-layer-fwd: d_model 512, 8 experts top-2, SwiGLU d_ff 2048, "
                                   "4096 tok, fp32"),
}
WL = WORKLOADS["mixtral"]     # the selected workload (main() sets it from --workload)
D_MODEL, N_EXPERTS, TOP_K, D_FF, TOKENS = WL["d"], WL["E"], WL["k"], WL["F"], WL["T"]
WORKLOAD = WL["name"]
# dram__bytes_read.sum + dram__bytes_write.sum of one grouped SwiGLU (gate/up) GEMM launch
# of the default workload at full size (2.906 GB read + 0.929 GB written), from the ncu
# capture summarised in profiles/grouped_gemm_mixtral_T16384_dram.md
GEMM1_DRAM_BYTES_PER_LAUNCH = 3834612224


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="swiftmoe", choices=["swiftmoe", "reference"])
    ap.add_argument("--tokens", type=int, default=None, help="tokens per GPU (default: the workload's)")
    ap.add_argument("--workload", default="mixtral", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ep-chunks", type=int, default=None, help="token chunks of the EP exchange")
    ap.add_argument("--ep-transport", default=None, choices=["p2p", "collective"])
    ap.add_argument("--ep-schedule", default=None, choices=["local_first", "chunked"],
                    help="overlap schedule of the p2p exchange")
    ap.add_argument("--ep-return", default=None, choices=["fused", "copy"],
                    help="local-first return: GEMM epilogue stores to the peers, or copies")
    ap.add_argument("--ep-dedup", default=None, choices=["auto", "on", "off"],
                    help="local first: send each token once per destination rank")
    ap.add_argument("--ep-split-min-ws", type=int, default=None,
                    help="local first: split the own rows in two halves from this world size on")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 100 ms in a background reader; samples are host-stamped so
    that only those taken inside the timed region are summarised."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.samples = []
        self.window = (0.0, float("inf"))

    def start(self):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self

        def reader():
            for line in self.proc.stdout:
                if line.strip():
                    self.samples.append((time.time(), line.strip()))
        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        t0 = time.time()
        while not self.samples and time.time() - t0 < 5:   # wait for the first sample
            time.sleep(0.02)
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lo, hi = self.window
        sel = [l for (t, l) in self.samples if lo <= t <= hi]
        if not sel:   # region shorter than the sampling period: take the sample right after it
            sel = [l for (t, l) in self.samples if t >= lo][:1]
        for l in sel:
            parts = [p.strip() for p in l.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------- CPU arm
def _host_threads():
    """All host threads this process may run on.  torchrun sets OMP_NUM_THREADS=1 for its
    workers, so the BLAS pool is raised back to the affinity mask before timing."""
    from threadpoolctl import threadpool_limits
    return threadpool_limits(limits=len(os.sched_getaffinity(0)))


def _oracle_layer(rng, sample_tokens: int):
    """The selected workload's layer as the oracle's fp32 parameters (seeded; shared
    expert and router offsets when the workload has them) and a sample input batch."""
    import numpy as np

    from oracle import moe_oracle as O
    E, d, F = N_EXPERTS, D_MODEL, D_FF

    def w(shape):
        return rng.standard_normal(shape, dtype=np.float32) * 0.02

    p = O.MoEParams(gate=w((E, d)), expert_type="swiglu", w1=w((E, F, d)), w3=w((E, F, d)), w2=w((E, d, F)))
    if WL["shared"]:
        p.sw1, p.sw3, p.sw2 = w((1, F, d)), w((1, F, d)), w((1, d, F))
    if WL["bias_std"]:
        p.logit_bias = rng.standard_normal(E).astype(np.float32) * WL["bias_std"]
    return p, rng.standard_normal((sample_tokens, d), dtype=np.float32)


def _oracle_forward(p, x):
    """One layer forward of the numpy restatement (capacity scaled to the batch)."""
    from oracle import moe_oracle as O
    return O.moe_forward([x], p, k=TOP_K, capacity_factor=WL["cf"])


def cpu_reference(tokens_budget_s: float, sample_tokens: int = 64, seed: int = 0):
    """Time the numpy restatement of the reference forward on this host's cores."""
    import numpy as np
    from threadpoolctl import threadpool_info

    p, x = _oracle_layer(np.random.default_rng(seed), sample_tokens)
    with _host_threads():
        _oracle_forward(p, x[:8])  # warm BLAS
        done, t0 = 0, time.perf_counter()
        while True:
            _oracle_forward(p, x)
            done += sample_tokens
            el = time.perf_counter() - t0
            if el >= tokens_budget_s:
                break
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    return {"value": done / el, "unit": "tokens/s", "cores": int(threads), "kind": "port",
            "sample": f"{done} tokens in batches of {sample_tokens} through the full layer "
                      f"(numpy fp32, oracle/moe_oracle.py), {el:.1f} s"}, p, x


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from threadpoolctl import threadpool_info

    sample = 64
    p, x = _oracle_layer(np.random.default_rng(0), sample)
    with _host_threads():
        for _ in range(args.warmup):
            _oracle_forward(p, x)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _oracle_forward(p, x)
        el = time.perf_counter() - t0
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    v = sample * args.steps / el
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "parallelism": "host CPU", "sample_tokens_per_step": sample},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": int(threads), "kind": "port",
                             "sample": f"{sample} tokens per step through the full layer (numpy fp32 "
                                       f"restatement of the reference forward, oracle/moe_oracle.py)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- GPU arm
def _cpulist(text: str):
    cpus = set()
    for part in text.strip().split(","):
        if part:
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
    return cpus


def bind_near_gpu(index: int):
    """Run this process on the host CPUs of the GPU's NUMA node (PCI local_cpulist), so
    the pinned host buffers of the end-to-end leg are allocated in that node's memory.
    Returns (the CPUs bound, the previous mask), or None if the topology is unknown."""
    import torch
    try:
        p = torch.cuda.get_device_properties(index)
        path = f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0/local_cpulist"
        with open(path) as f:
            local = _cpulist(f.read())
        before = os.sched_getaffinity(0)
        sel = local & before
        if not sel or sel == before:
            return None
        os.sched_setaffinity(0, sel)
        return sel, before
    except (OSError, ValueError, AttributeError, RuntimeError):
        return None


def count_launches(fn):
    """Kernels of libswiftmoe (namespace smoe) launched by fn(), from a CUPTI trace."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return sum(1 for e in prof.events() if e.device_type.name == "CUDA" and "smoe" in e.name)


def main():
    args = parse()
    global D_MODEL, N_EXPERTS, TOP_K, D_FF, WORKLOAD, WL
    wl = WL = WORKLOADS[args.workload]
    D_MODEL, N_EXPERTS, TOP_K, D_FF, WORKLOAD = wl["d"], wl["E"], wl["k"], wl["F"], wl["name"]
    if args.tokens is None:
        args.tokens = wl["T"]
    if args.impl == "reference":
        run_reference_arm(args)
        return
    import torch
    import torch.distributed as dist

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ws}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    binding = bind_near_gpu(local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import swiftmoe_b200 as S
    from swiftmoe_b200 import _lib as L

    T = args.tokens
    torch.manual_seed(1234)
    cdtype = torch.float32 if wl["dtype"] == "fp32" else torch.bfloat16
    model = S.UltimateMoE(N_EXPERTS, D_MODEL, use_fp16=False, use_nccl_opt=False, dtype=cdtype,
                          top_k=TOP_K, expert_type="swiglu", d_ff=D_FF, device=dev,
                          enable_profiling=(ws > 1), capacity_factor=wl["cf"],
                          num_shared_experts=wl["shared"], d_ff_shared=D_FF)
    if wl["bias_std"]:
        model.set_logit_bias(torch.randn(N_EXPERTS, generator=torch.Generator().manual_seed(2)) * wl["bias_std"])
    with torch.no_grad():
        g = torch.Generator(device=dev).manual_seed(7)   # identical gate on every rank
        model.gate_weight.copy_(torch.randn(model.gate_weight.shape, generator=g, device=dev) * 0.02)
    if ws > 1:
        if args.ep_chunks:
            model.comm.chunks = args.ep_chunks
        if args.ep_transport:
            model.comm.transport = args.ep_transport
        if args.ep_schedule:
            model.comm.schedule = args.ep_schedule
        if args.ep_return:
            model.comm.return_mode = args.ep_return
        if args.ep_split_min_ws:
            model.comm.split_min_ws = args.ep_split_min_ws
        if args.ep_dedup:
            model.comm.dedup = args.ep_dedup
    x = torch.randn((T, D_MODEL), device=dev, dtype=cdtype, generator=torch.Generator(device=dev).manual_seed(100 + rank))
    out = torch.empty_like(x)

    def barrier():
        if ws > 1:
            dist.barrier(device_ids=[local])

    def step(events=None):
        if ws == 1:
            return model._forward_fused(x, events, out=out)
        return model(x)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    model.reset_profiling()
    barrier()
    torch.cuda.synchronize()
    evs = [L.StageEvents() for _ in range(args.steps)] if ws == 1 else None
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local).start()
    h0 = time.time()
    t_start.record()
    for i in range(args.steps):
        step(evs[i] if evs else None)
    t_end.record()
    torch.cuda.synchronize()
    clk.window = (h0, time.time())
    barrier()
    ms = t_start.elapsed_time(t_end) / args.steps
    if ws > 1:
        tm = torch.tensor([ms], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    value = T * ws / (ms / 1e3)

    # per-stage / per-kernel times from the events recorded in the timed region
    if ws == 1:
        st = {"Router": [], "Dispatch_Comm": [], "Expert_GEMM1": [], "Expert_GEMM2": [], "Combine_Comm": []}
        for e in evs:
            st["Router"].append(e.elapsed(0, 1))
            st["Dispatch_Comm"].append(e.elapsed(1, 2))
            st["Expert_GEMM1"].append(e.elapsed(2, 3))
            st["Expert_GEMM2"].append(e.elapsed(3, 4))
            st["Combine_Comm"].append(e.elapsed(4, 5))
        stage_ms = {k: statistics.mean(v) for k, v in st.items()}
        exposed = 0.0
        spans = None
    else:
        s = model.get_profile_summary()
        stage_ms = {k: v for k, v in s.items()}
        exposed = s.get("Exposed_A2A", 0.0)
        spans = {k: round(v, 4) for k, v in model.get_profile_spans().items()}
    burst, sustained, hbm, src = peaks()
    # routed rows this rank computed (capacity drops included), from the plan / exchange
    if ws == 1:
        S_rows = T * TOP_K if wl["cf"] is None else None
    else:
        S_rows = model.comm.last_rows
    if S_rows is None:  # one GPU with a capacity: kept rows = sum of the plan's kept counts
        from swiftmoe_b200._core import capacity_rows
        from swiftmoe_b200 import kernels as KK
        cap = capacity_rows(wl["cf"], T, 1, TOP_K, N_EXPERTS)
        idx_, _ = KK.router(x, model.gate_weight, TOP_K, model.logit_bias)
        S_rows = int(torch.clamp(torch.bincount(idx_.flatten().long(), minlength=N_EXPERTS), max=cap).sum())
    if ws == 1:
        gemm1_ms = stage_ms["Expert_GEMM1"]
        flops = 2.0 * S_rows * D_MODEL * 2 * D_FF
        kname = "grouped SwiGLU gate/up GEMM (tcgen05)" if cdtype != torch.float32 else \
            "grouped SwiGLU gate/up GEMM (fp32 FFMA)"
    else:
        gemm1_ms = stage_ms["Expert_Compute"]
        flops = 6.0 * S_rows * D_MODEL * D_FF
        kname = "expert FFN (both grouped GEMMs, tcgen05), routed rows of this rank"
    if wl["shared"]:
        flops_shared = 6.0 * T * D_MODEL * D_FF
    else:
        flops_shared = 0.0
    achieved = flops / (gemm1_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "kernel": kname, "achieved": achieved, "peak": sustained,
                "peak_kind": f"bf16_tflops_sustained ({src})", "unit": "TFLOP/s", "frac": achieved / sustained,
                "traffic": GEMM1_DRAM_BYTES_PER_LAUNCH if args.workload == "mixtral" and ws == 1 else None,
                "algorithmic_flops_per_launch": flops, "launch_ms": gemm1_ms}
    layer_flops = 6.0 * S_rows * D_MODEL * D_FF + flops_shared + 2.0 * T * D_MODEL * N_EXPERTS
    layer_frac = layer_flops / (ms / 1e3) / 1e12 / sustained

    # end-to-end through the public API: every step copies its input from pinned host
    # memory, runs UltimateMoE.forward and copies its output back to pinned host memory.
    # Double-buffered across steps: the H2D copy of step i+1 and the D2H copy of step i-1
    # run on their own streams while step i computes.
    xh = x.cpu().pin_memory()
    ohs = [torch.empty_like(xh).pin_memory() for _ in range(2)]
    xds = [torch.empty_like(x) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)

    def e2e_run(n):
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_done = [torch.cuda.Event() for _ in range(2)]
        s_in.wait_stream(comp)
        with torch.cuda.stream(s_in):
            xds[0].copy_(xh, non_blocking=True)
            ev_in[0].record(s_in)
        for i in range(n):
            cur, nxt = i % 2, (i + 1) % 2
            comp.wait_event(ev_in[cur])
            o = model(xds[cur])
            ev_done[cur].record(comp)
            if i + 1 < n:
                if i > 0:
                    s_in.wait_event(ev_done[nxt])      # step i-1 no longer reads xds[nxt]
                with torch.cuda.stream(s_in):
                    xds[nxt].copy_(xh, non_blocking=True)
                    ev_in[nxt].record(s_in)
            s_out.wait_event(ev_done[cur])
            with torch.cuda.stream(s_out):
                ohs[cur].copy_(o, non_blocking=True)
            o.record_stream(s_out)
        comp.wait_stream(s_out)

    e2e_run(2)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    e2e_run(args.steps)
    e1.record(comp)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    if ws > 1:
        tm = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms_e2e = float(tm.item())
    e2e = {"value": T * ws / (ms_e2e / 1e3), "unit": "tokens/s", "ms_per_step": ms_e2e,
           "h2d_bytes_per_step": xh.numel() * xh.element_size(),
           "d2h_bytes_per_step": ohs[0].numel() * ohs[0].element_size(),
           "mode": "UltimateMoE.forward; pinned host input/output copied every step, double-buffered "
                   "so copies of neighbouring steps overlap the forward"}

    # this library's kernels in one forward, counted from the CUDA activity trace of an
    # untimed forward (every rank runs it: the forward holds collectives)
    try:
        launches_per_step, launches_src = count_launches(lambda: model(x)), "CUPTI trace of one forward"
    except Exception as e:  # no activity trace on this host: the static count of the path
        launches_per_step = 8 if ws == 1 else (16 if ws >= 4 else 14)
        launches_src = f"static count (trace failed: {type(e).__name__})"
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        try:
            if binding is not None:     # the CPU baseline uses every host thread again
                os.sched_setaffinity(0, binding[1])
            cpu, _, _ = cpu_reference(args.cpu_seconds)
        except Exception as ex:  # reported, never fatal
            cpu = {"value": None, "error": repr(ex)}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": wl["dtype"],
                "data": "synthetic: x ~ N(0,1), weights N(0,0.02), seeded",
                "config": {"workload": WORKLOAD, "d_model": D_MODEL, "num_experts": N_EXPERTS, "top_k": TOP_K,
                           "d_ff": D_FF, "tokens_per_gpu": T, "parallelism": f"ep{ws}",
                           "capacity_factor": wl["cf"], "shared_experts": wl["shared"],
                           "host_cpus": None if binding is None else
                           f"{len(binding[0])} CPUs of the GPU's NUMA node (of {len(binding[1])})",
                           "ep_exchange": None if ws == 1 else
                           f"{model.comm.transport} transport, " + (
                               f"{model.comm.schedule} schedule, {model.comm.return_mode} return, "
                               f"token dedup {model.comm.dedup}"
                               if model.comm.schedule == "local_first"
                               else f"{model.comm.n_chunks(T)} token chunks"),
                           "l2": f"inputs larger than L2: x {x.numel() * x.element_size() / 2**20:.0f} MiB and "
                                 f"{3 * model.exp_per_rank * D_FF * D_MODEL * x.element_size() / 1e9:.2f} GB of "
                                 f"expert weights read every step"},
                "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
                "gpu_launches_per_step": launches_per_step, "gpu_launches_source": launches_src,
                "roofline": roofline,
                "layer_tensor_frac": layer_frac, "stage_ms": stage_ms, "exposed_a2a_ms": exposed,
                "rank0_timeline_ms": spans,
                "cpu_baseline": cpu, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    clk.stop()
    if ws > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

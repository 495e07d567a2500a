#!/usr/bin/env python
"""MoE-layer forward benchmark (tokens/s) on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl swiftmoe|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload: the Mixtral-shaped MoE layer, bf16: d_model=4096, 8 experts, top-2 softmax
gating, SwiGLU d_ff=14336, 16384 tokens per GPU ~ N(0,1), weights N(0, 0.02), no
router bias, no capacity limit (synthetic, seeded; no dataset is involved).  At N GPUs
the experts are split 8/N per GPU (expert parallelism) and every GPU routes its own
16384 tokens (weak scaling).

One step = one forward of the layer over one batch.  `value` is the whole-job
throughput with the input already resident in HBM; `e2e` is the same forward through
the public module API with the input copied from pinned host memory and the output
copied back inside the timed region.  After the timed region every rank checks a
sample of its output rows against a float32 evaluation of the same layer (`parity`),
and the other layer shapes of the benchmark set are measured briefly
(`extra_workloads`).  `--impl reference` times the reference algorithm on the host CPU
(the numpy restatement in oracle/: the reference is pure-Python torch, which does not
travel with this repository) on a bounded token sample of the same layer.
"""
from __future__ import annotations

import argparse
import json
import math
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
DECODE_TOKENS = (1, 8, 64, 256)
WL = WORKLOADS["mixtral"]     # the selected workload (main() sets it from --workload)
D_MODEL, N_EXPERTS, TOP_K, D_FF, TOKENS = WL["d"], WL["E"], WL["k"], WL["F"], WL["T"]
WORKLOAD = WL["name"]
# dram__bytes_read.sum + dram__bytes_write.sum of one grouped SwiGLU (gate/up) GEMM launch
# of the default workload at full size (2.906 GB read + 0.929 GB written), from the ncu
# capture summarised in profiles/grouped_gemm_mixtral_T16384_dram.md
GEMM1_DRAM_BYTES_PER_LAUNCH = 3834612224
# a timed region at least this long runs at the clock the power cap settles at, so its
# GEMM fraction is taken against the sustained cuBLAS peak; shorter ones against the burst
SUSTAINED_REGION_S = 2.0


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
    ap.add_argument("--extras", default="auto", choices=["auto", "none"],
                    help="auto: also measure the other layer shapes and the decode sweep")
    ap.add_argument("--parity-sample", type=int, default=64, help="tokens per rank checked after timing")
    ap.add_argument("--mode", default="forward", choices=["forward", "backward"],
                    help="backward: time the layer's backward pass alone (one GPU; profiling cases)")
    ap.add_argument("--ep-chunks", type=int, default=None, help="token chunks of the EP exchange")
    ap.add_argument("--ep-transport", default=None, choices=["p2p", "collective"])
    ap.add_argument("--ep-schedule", default=None, choices=["device", "local_first", "chunked"],
                    help="schedule of the p2p exchange (default: device)")
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
        return dict(burst=d.get("bf16_tflops", 1590.0), sustained=d.get("bf16_tflops_sustained", 1400.0),
                    hbm=d.get("hbm_gbs", 6650.0), src="measured")
    return dict(burst=1590.0, sustained=1400.0, hbm=6650.0, src="fallback")


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
CPU_SAMPLE_TOKENS = 512


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


def cpu_reference(tokens_budget_s: float, sample_tokens: int = CPU_SAMPLE_TOKENS, seed: int = 0):
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

    sample = CPU_SAMPLE_TOKENS
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
                                       f"restatement of the reference forward, oracle/moe_oracle.py; the "
                                       f"reference itself is Python that does not travel to this host)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- GPU arm helpers
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


class Ranks:
    """World size, rank and device of this process, and the collectives the harness uses."""

    def __init__(self, ws, rank, local, dev):
        self.ws, self.rank, self.local, self.dev = ws, rank, local, dev

    def barrier(self):
        if self.ws > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[self.local])

    def max(self, v: float) -> float:
        if self.ws == 1:
            return v
        import torch
        import torch.distributed as dist
        t = torch.tensor([v], device=self.dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def min(self, v: float) -> float:
        return -self.max(-v)


def make_layer(wl, R: Ranks, T: int, profiling: bool):
    """The workload's layer on this rank (random-init weights; identical gate and router
    offsets on every rank) and this rank's seeded input batch."""
    import torch
    import swiftmoe_b200 as S
    cdtype = torch.float32 if wl["dtype"] == "fp32" else torch.bfloat16
    torch.manual_seed(1234 + R.rank)
    model = S.UltimateMoE(wl["E"], wl["d"], use_fp16=False, use_nccl_opt=False, dtype=cdtype,
                          top_k=wl["k"], expert_type="swiglu", d_ff=wl["F"], device=R.dev,
                          enable_profiling=profiling, capacity_factor=wl["cf"],
                          num_shared_experts=wl["shared"], d_ff_shared=wl["F"])
    if wl["bias_std"]:
        model.set_logit_bias(torch.randn(wl["E"], generator=torch.Generator().manual_seed(2)) * wl["bias_std"])
    with torch.no_grad():
        g = torch.Generator(device=R.dev).manual_seed(7)   # identical gate on every rank
        model.gate_weight.copy_(torch.randn(model.gate_weight.shape, generator=g, device=R.dev) * 0.02)
        if wl["shared"]:                                    # the shared expert is replicated too
            for i, p in enumerate((model.shared_w1, model.shared_w3, model.shared_w2)):
                gs = torch.Generator(device=R.dev).manual_seed(11 + i)
                p.copy_(torch.randn(p.shape, generator=gs, device=R.dev) * 0.02)
    x = torch.randn((T, wl["d"]), device=R.dev, dtype=cdtype,
                    generator=torch.Generator(device=R.dev).manual_seed(100 + R.rank))
    return model, x


def time_steps(step, steps: int, warmup: int, R: Ranks, clk=None):
    """W untimed steps, then K steps bracketed by a barrier and a synchronize on both
    sides, timed with CUDA events on the launching stream; max over ranks (ms/step)."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    R.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    h0 = time.time()
    t0.record()
    for i in range(steps):
        step(i)
    t1.record()
    torch.cuda.synchronize()
    if clk is not None:
        clk.window = (h0, time.time())
    R.barrier()
    return R.max(t0.elapsed_time(t1) / steps)


def full_expert_weights(model, R: Ranks):
    """Every expert's (w1, w3, w2) on every rank: the ranks' contiguous blocks gathered."""
    import torch
    import torch.distributed as dist
    ws = (model.w1, model.w3, model.w2)
    if R.ws == 1:
        return ws
    out = []
    for w in ws:
        full = torch.empty((R.ws * w.shape[0],) + tuple(w.shape[1:]), dtype=w.dtype, device=w.device)
        dist.all_gather_into_tensor(full, w.detach().contiguous())
        out.append(full)
    return tuple(out)


def parity_check(model, x, out, wl, R: Ranks, sample: int):
    import torch
    with torch.no_grad():
        return _parity_check(model, x, out, wl, R, sample)


def _parity_check(model, x, out, wl, R: Ranks, sample: int):
    """A sample of this rank's output rows against a float32 torch evaluation of the same
    layer (full-precision matmuls of the bf16 inputs and weights), on the routing the
    layer itself chose; capacity drops follow the (source rank, token, slot) order over
    every rank's routing.  Reports max|out - ref| / max|ref| (bar 2e-2), the element-wise
    form floored at 1e-3 max|ref|, and how many sampled tokens route exactly as the
    float32 logits do (the rest are near-ties)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as Fn
    from swiftmoe_b200 import kernels as K
    from swiftmoe_b200._core import capacity_rows
    torch.backends.cuda.matmul.allow_tf32 = False
    T, k, E = x.shape[0], wl["k"], wl["E"]
    n = min(sample, T)
    w1, w3, w2 = full_expert_weights(model, R)            # collective: every rank joins
    bias = model.logit_bias
    idx_all, _ = K.router(x, model.gate_weight, k, bias)
    kept = torch.ones((T, k), dtype=torch.bool, device=R.dev)
    cap = capacity_rows(wl["cf"], T, R.ws, k, E)
    if cap > 0:
        flat = idx_all.reshape(-1).long()
        counts = torch.bincount(flat, minlength=E).to(torch.int64)
        if R.ws > 1:
            allc = torch.empty((R.ws, E), dtype=torch.int64, device=R.dev)
            dist.all_gather_into_tensor(allc.view(-1), counts)
            base = allc[:R.rank].sum(0)
        else:
            base = torch.zeros(E, dtype=torch.int64, device=R.dev)
        oh = Fn.one_hot(flat, E).to(torch.int32)
        pos = (torch.cumsum(oh, 0) - oh).gather(1, flat.view(-1, 1)).view(-1)
        kept = ((base[flat] + pos) < cap).view(T, k)
    if n == 0:
        return {"rows_checked": 0}
    sel = torch.linspace(0, T - 1, n, device=R.dev).round().long()
    xs = x[sel].float()
    idx = idx_all[sel].long()
    logits = xs @ model.gate_weight.float().T
    if bias is not None:
        logits = logits + bias.float()
    ref_idx = torch.topk(logits, k, dim=1).indices
    agree = float((torch.sort(ref_idx, 1).values == torch.sort(idx, 1).values).all(1).float().mean())
    wts = torch.softmax(logits.gather(1, idx), dim=1) * kept[sel].float()
    ref = torch.zeros_like(xs)

    def swiglu(a, W1, W3, W2):
        return (Fn.silu(a @ W1.float().T) * (a @ W3.float().T)) @ W2.float().T

    for e in torch.unique(idx).tolist():
        rows, slots = torch.nonzero(idx == e, as_tuple=True)
        y = swiglu(xs[rows], w1[e], w3[e], w2[e])
        ref.index_add_(0, rows, y * wts[rows, slots].view(-1, 1))
    if wl["shared"]:
        ref += swiglu(xs, model.shared_w1, model.shared_w3, model.shared_w2)
    o = out[sel].float()
    err = (o - ref).abs()
    mx = float(ref.abs().max())
    elem = float((err / torch.clamp(ref.abs(), min=1e-3 * mx)).max())
    res = {"max_rel": float(err.max()) / max(mx, 1e-30), "elementwise_rel": elem,
           "routed_agree": agree, "rows_checked": n, "tolerance": 2e-2}
    res = {k_: (R.max(v) if k_ in ("max_rel", "elementwise_rel") else
                (R.min(v) if k_ == "routed_agree" else v)) for k_, v in res.items()}
    res["rows_checked"] = n * R.ws
    res["reference"] = "float32 torch matmuls of the bf16 inputs/weights on the GPU, the layer's own routing"
    return res


def host_link(R: Ranks, nbytes: int):
    """Host<->device bandwidth with every rank copying at once (pinned host memory, one
    H2D and one D2H stream in flight together): the bound of the end-to-end leg."""
    import torch
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d_in = torch.empty(nbytes, dtype=torch.uint8, device=R.dev)
    d_out = torch.empty(nbytes, dtype=torch.uint8, device=R.dev)
    s1, s2 = torch.cuda.Stream(R.dev), torch.cuda.Stream(R.dev)
    res = []
    for it in range(3):
        torch.cuda.synchronize()
        R.barrier()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        with torch.cuda.stream(s1):
            e[0].record(s1)
            d_in.copy_(src, non_blocking=True)
            e[1].record(s1)
        with torch.cuda.stream(s2):
            e[2].record(s2)
            dst.copy_(d_out, non_blocking=True)
            e[3].record(s2)
        torch.cuda.synchronize()
        res.append((e[0].elapsed_time(e[1]), e[2].elapsed_time(e[3])))
    h2d_ms, d2h_ms = min(r[0] for r in res), min(r[1] for r in res)
    return R.min(nbytes / h2d_ms / 1e6), R.min(nbytes / d2h_ms / 1e6)


def rows_routed(model, x, wl, R: Ranks):
    """Expert rows this rank computed in the last forward (after any capacity cut)."""
    import torch
    from swiftmoe_b200 import kernels as K
    from swiftmoe_b200._core import capacity_rows
    if R.ws > 1:
        return model.comm.last_rows
    if wl["cf"] is None:
        return x.shape[0] * wl["k"]
    cap = capacity_rows(wl["cf"], x.shape[0], 1, wl["k"], wl["E"])
    idx, _ = K.router(x, model.gate_weight, wl["k"], model.logit_bias)
    return int(torch.clamp(torch.bincount(idx.flatten().long(), minlength=wl["E"]), max=cap).sum())


def release(model, R: Ranks):
    import torch
    if R.ws > 1 and model.comm is not None:
        model.comm.close()
    del model
    torch.cuda.empty_cache()


def backward_timing(model, T: int, R: Ranks, pk, steps: int, warmup: int):
    """The layer's backward (``smoe_layer_bwd``: gradients of x, the gate and every expert
    weight) for a seeded upstream gradient, CUDA-event timed; FLOPs counted as the GEMMs
    it runs (gate/up recompute, dout W2, dgrad, two weight gradients)."""
    import torch
    d, F = model.d_model, model.d_ff
    x = torch.randn((T, d), device=R.dev, dtype=torch.bfloat16, generator=torch.Generator(R.dev).manual_seed(300))
    dout = torch.randn((T, d), device=R.dev, dtype=torch.bfloat16, generator=torch.Generator(R.dev).manual_seed(301))
    ms = time_steps(lambda i=None: model._backward_fused(x, dout), steps, warmup, R)
    S = T * model.top_k      # routed rows per rank (under expert parallelism: on average)
    flops = 2.0 * S * d * 2 * F * 3 + 2.0 * S * d * F * 2
    return {"ms_per_backward": ms, "tokens_per_gpu": T, "gemm_tflops": flops / (ms / 1e3) / 1e12,
            "frac_of_burst_peak": flops / (ms / 1e3) / 1e12 / pk["burst"], "gemm_flops": flops,
            "what": "gradients of x, gate, w1, w3, w2 (bf16 layer, fp32 weight gradients); one GPU: "
                    "smoe_layer_bwd, N > 1: the expert-parallel backward (max over ranks)"}


def extra_workloads(R: Ranks, pk, steps: int, warmup: int, decode_model=None, sample: int = 32):
    """The other layer shapes of the benchmark set, a few seconds each: the fp32 layer
    (one GPU), the capacity-limited and fine-grained expert-parallel layers (every N),
    and the decode sweep of the Mixtral layer (1 and 8 GPUs).  Throughput, expert-FLOP
    fraction of the burst bf16 peak (not claimed for fp32, whose GEMMs run three tf32
    products per fp32 product), exposed exchange time and a sampled parity check each."""
    import torch
    res = {}
    names = ["ep-capacity", "fine-grained"] + (["cpu-runnable-fp32"] if R.ws == 1 else [])
    for name in names:
        wl = WORKLOADS[name]
        model, x = make_layer(wl, R, wl["T"], profiling=R.ws > 1)
        out = torch.empty_like(x)

        def step(i=None, model=model, x=x, out=out):
            if R.ws == 1:
                return model._forward_fused(x, out=out)
            out.copy_(model(x))
        ms = time_steps(step, steps, warmup, R)
        rows = rows_routed(model, x, wl, R)
        flops = 6.0 * rows * wl["d"] * wl["F"] + (6.0 * x.shape[0] * wl["d"] * wl["F"] if wl["shared"] else 0.0)
        ent = {"tokens_per_s": x.shape[0] * R.ws / (ms / 1e3), "ms_per_step": ms, "steps": steps,
               "tokens_per_gpu": x.shape[0], "workload": wl["name"]}
        if wl["dtype"] != "fp32":
            ent["expert_tflops_rank0"] = flops / (ms / 1e3) / 1e12
            ent["expert_frac_of_burst_peak"] = ent["expert_tflops_rank0"] / pk["burst"]
        if R.ws > 1:
            ent["exposed_a2a_ms"] = R.max(model.get_profile_summary()["Exposed_A2A"])
        if R.ws == 1:
            model._forward_fused(x, out=out)
        else:
            out = model(x)
        ent["parity"] = parity_check(model, x, out, wl, R, sample)
        res[name] = ent
        release(model, R)
    if decode_model is not None and R.ws == 1:
        res["backward"] = backward_timing(decode_model, WORKLOADS["mixtral"]["T"], R, pk, steps=5, warmup=2)
    if decode_model is not None and R.ws in (1, 8):
        wl = WORKLOADS["mixtral"]
        for T in DECODE_TOKENS:
            x = torch.randn((T, wl["d"]), device=R.dev, dtype=torch.bfloat16,
                            generator=torch.Generator(device=R.dev).manual_seed(500 + R.rank))

            def step(i=None, x=x):
                return decode_model(x)
            ms = time_steps(step, max(steps, 20), warmup, R)
            from swiftmoe_b200 import kernels as K
            idx, _ = K.router(x, decode_model.gate_weight, wl["k"])
            hit = torch.zeros(wl["E"], dtype=torch.int32, device=R.dev)
            hit[idx.flatten().long()] = 1
            if R.ws > 1:
                import torch.distributed as dist
                dist.all_reduce(hit, op=dist.ReduceOp.MAX)
            El = decode_model.exp_per_rank
            mine = int(hit[R.rank * El:(R.rank + 1) * El].sum())
            wbytes = mine * 3 * wl["d"] * wl["F"] * 2
            res[f"decode-T{T}"] = {"tokens_per_s": T * R.ws / (ms / 1e3), "ms_per_step": ms,
                                   "tokens_per_gpu": T, "expert_weight_bytes_rank0": wbytes,
                                   "weight_stream_frac_of_hbm_rank0": wbytes / (ms / 1e3) / 1e9 / pk["hbm"]}
    return res


# --------------------------------------------------------------------- GPU arm
def main():
    import torch
    with torch.no_grad():      # a forward (inference) benchmark: no autograd graph is recorded
        _main()


def _main():
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
    if args.mode == "backward":
        # one GPU: smoe_layer_bwd; under torchrun: the expert-parallel backward on every rank
        bws = int(os.environ.get("WORLD_SIZE", "1"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        if bws > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        R = Ranks(bws, int(os.environ.get("RANK", "0")), local, dev)
        model, _ = make_layer(wl, R, 1, profiling=False)
        res = backward_timing(model, args.tokens, R, peaks(), args.steps, args.warmup)
        if bws > 1:
            model.comm.close()
        if R.rank == 0:
            print(json.dumps({"mode": "backward", "workload": WORKLOAD, "n_gpus": bws, **res}), flush=True)
        if bws > 1:
            dist.barrier(device_ids=[local])
            dist.destroy_process_group()
        return

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
    from swiftmoe_b200 import _lib as L
    R = Ranks(ws, rank, local, dev)
    pk = peaks()

    T = args.tokens
    model, x = make_layer(wl, R, T, profiling=ws > 1)
    cdtype = x.dtype
    if ws > 1:
        for attr, val in (("chunks", args.ep_chunks), ("transport", args.ep_transport),
                          ("schedule", args.ep_schedule), ("return_mode", args.ep_return),
                          ("split_min_ws", args.ep_split_min_ws), ("dedup", args.ep_dedup)):
            if val:
                setattr(model.comm, attr, val)
    out = torch.empty_like(x)
    evs = [L.StageEvents() for _ in range(args.steps)] if ws == 1 else None

    def step(i=None):
        if ws == 1:
            return model._forward_fused(x, None if i is None else evs[i], out=out)
        return model(x)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    model.reset_profiling()
    clk = ClockSampler(local).start()
    ms = time_steps(step, args.steps, 0, R, clk)
    value = T * ws / (ms / 1e3)
    region_s = ms * args.steps / 1e3

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
        exposed = R.max(s.get("Exposed_A2A", 0.0))
        spans = {k: round(v, 4) for k, v in model.get_profile_spans().items()}
    S_rows = rows_routed(model, x, wl, R)
    if ws == 1:
        gemm1_ms = stage_ms["Expert_GEMM1"]
        flops = 2.0 * S_rows * D_MODEL * 2 * D_FF
        kname = "grouped SwiGLU gate/up GEMM (tcgen05)" if cdtype != torch.float32 else \
            "grouped SwiGLU gate/up GEMM (fp32 as split tf32 operands on tcgen05)"
    else:
        gemm1_ms = stage_ms["Expert_Compute"]
        flops = 6.0 * S_rows * D_MODEL * D_FF
        kname = "expert FFN (both grouped GEMMs, tcgen05), routed rows of this rank"
    flops_shared = 6.0 * T * D_MODEL * D_FF if wl["shared"] else 0.0
    sustained_ok = region_s >= SUSTAINED_REGION_S
    peak = pk["sustained"] if sustained_ok else pk["burst"]
    peak_kind = (f"bf16_tflops_sustained ({pk['src']}): timed region {region_s:.2f} s >= {SUSTAINED_REGION_S} s"
                 if sustained_ok else
                 f"bf16_tflops burst ({pk['src']}): timed region {region_s:.2f} s < {SUSTAINED_REGION_S} s")
    achieved = flops / (gemm1_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "kernel": kname, "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": GEMM1_DRAM_BYTES_PER_LAUNCH if args.workload == "mixtral" and ws == 1 else None,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one full-size launch "
                                  "(profiles/grouped_gemm_mixtral_T16384_dram.md)",
                "algorithmic_flops_per_launch": flops, "launch_ms": gemm1_ms,
                "frac_of_sustained_peak": achieved / pk["sustained"]}
    layer_flops = 6.0 * S_rows * D_MODEL * D_FF + flops_shared + 2.0 * T * D_MODEL * N_EXPERTS
    layer_frac = layer_flops / (ms / 1e3) / 1e12 / peak

    # correctness of what was timed: a sample of every rank's rows against float32
    o_last = step()
    if ws == 1:
        o_last = out
    parity = parity_check(model, x, o_last, wl, R, args.parity_sample)

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
    R.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    e2e_run(args.steps)
    e1.record(comp)
    torch.cuda.synchronize()
    R.barrier()
    ms_e2e = R.max(e0.elapsed_time(e1) / args.steps)
    nb = xh.numel() * xh.element_size()
    h2d_gbs, d2h_gbs = host_link(R, nb)
    e2e = {"value": T * ws / (ms_e2e / 1e3), "unit": "tokens/s", "ms_per_step": ms_e2e,
           "h2d_bytes_per_step": nb, "d2h_bytes_per_step": ohs[0].numel() * ohs[0].element_size(),
           "mode": "UltimateMoE.forward; pinned host input/output copied every step, double-buffered "
                   "so copies of neighbouring steps overlap the forward",
           "host_link": {"h2d_gbs": h2d_gbs, "d2h_gbs": d2h_gbs,
                         "bound_ms_per_step": max(nb / h2d_gbs / 1e6, nb / d2h_gbs / 1e6),
                         "how": f"all {ws} ranks copying {nb >> 20} MiB each way at once (slowest rank)"}}

    # this library's kernels in one forward, counted from the CUDA activity trace of an
    # untimed forward (every rank runs it: the forward holds collectives)
    try:
        launches_per_step, launches_src = count_launches(lambda: model(x)), "CUPTI trace of one forward"
    except Exception as e:  # no activity trace on this host: the static count of the path
        launches_per_step = 8 if ws == 1 else 16
        launches_src = f"static count (trace failed: {type(e).__name__})"

    extras = None
    if args.extras == "auto" and args.workload == "mixtral":
        extras = extra_workloads(R, pk, steps=10, warmup=3, decode_model=model)
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
                           "ep_exchange": None if ws == 1 else model.comm.describe(),
                           "l2": f"inputs larger than L2: x {x.numel() * x.element_size() / 2**20:.0f} MiB and "
                                 f"{3 * model.exp_per_rank * D_FF * D_MODEL * x.element_size() / 1e9:.2f} GB of "
                                 f"expert weights read every step"},
                "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
                "gpu_launches_per_step": launches_per_step, "gpu_launches_source": launches_src,
                "roofline": roofline,
                "layer_tensor_frac": layer_frac, "stage_ms": stage_ms, "exposed_a2a_ms": exposed,
                "parity": parity, "rank0_timeline_ms": spans, "extra_workloads": extras,
                "cpu_baseline": cpu, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    clk.stop()
    if ws > 1:
        model.comm.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the EXL3 routed-expert MoE layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--tokens T]

Workload (the decode config): one routed-MoE layer,
128 experts, top-8 softmax routing, hidden 2048, expert intermediate 768,
uniform K=4 MCG, T=64 tokens per step (the largest decode batch of the
config; T = 1, 8, 32 are reported in `decode_sweep`).  Weights and inputs are
seeded synthetic (exl3_b200.synthetic).  A step is one layer forward over
one batch; 8 different routings/batches rotate across steps.

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier
and torch.cuda.synchronize(); every step is timed with CUDA events on the
launching stream around the layer only, after an untimed 256 MB L2 flush.
`value` = tokens of all ranks / max-over-ranks device time (CUDA graph of the
layer, inputs resident in HBM).  `e2e` = the same metric through the public
API (exl3_b200.moe.Exl3RoutedExperts.apply, eager) with pinned-host inputs
copied in and the output copied back inside the timed region.

N > 1: expert parallelism (exl3_b200.ep): rank g holds experts
[g*128/N, (g+1)*128/N) and T tokens of its own (weak scaling); a step is
dispatch (the library's kernels store each pair row straight into its
owner's IPC-mapped window over NVLink; --ep-transport nccl uses NCCL
instead), the local fused forward, the partial rows stored back, and the
per-token combine, one CUDA graph per step, timed per step and taken as the
max over ranks.
--workload ep: configs[4] (256 experts, H7168 I2048, 8192 tokens split over
the ranks: strong scaling), same EP step at any N.  --workload prefill:
configs[2] on one GPU (tcgen05 grouped GEMM path).  --impl reference: rank 0 times the
reference's CPU path (dequant_trellis compiled from the reference's own
csrc/bindings.cpp, oracle/_ref; else the oracle port) on a bounded sample of
each step's experts, scaled to the step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vllm-exl3_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

H, I, E, TOPK, KBITS = 2048, 768, 128, 8, 4

# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu
# capture of this workload (dram__bytes_read.sum + dram__bytes_write.sum).
# ncu cannot run inside the timed bench, so the capture's figure is reported
# with its source; it belongs to the kernel build named there, not
# necessarily to the build being timed.
DRAM_TRAFFIC = {
    "decode": {"bytes": 241.6e6, "kernel": "gemv_kernel<2,GATEUP,MCG>, T=64",
               "source": "profiles/gemv_gateup_cfg2_T64.md"},
    "prefill": {"bytes": 695.5e6, "kernel": "tc_gemm_kernel gate/up launches (mean), T=2048",
                "source": "profiles/tc_gemm_cfg3_T2048.md"},
}
METRIC = "MoE layer decode tokens/s (128 experts top-8, H2048 I768, K4 MCG)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time the expert-parallel step eagerly")
    ap.add_argument("--ep-transport", default="nvlink", choices=["nvlink", "nccl"],
                    help="expert-parallel exchange: the library's NVLink peer-store kernels or NCCL")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "ep"],
                    help="decode = configs[1] (the default, reported line); prefill = configs[2]; "
                         "ep = configs[4]")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# CPU reference sample (reference arm and the cpu_baseline key)
# ---------------------------------------------------------------------------
_REF = None


def _ref_dequant():
    """dequant_trellis of the reference's own compiled CPU code, else the port."""
    global _REF
    if _REF is None:
        import torch  # noqa: F401
        sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))
        try:
            import vllm_exl3_ref_c
            _REF = ("reference", vllm_exl3_ref_c)
        except Exception:
            import cpu_oracle
            _REF = ("port", cpu_oracle)
    return _REF


def _slice_task(args):
    """One sampled slice of the eager loop (exl3.py:2377-2413): dequant_trellis
    of `rows` input rows of one expert projection per call (the CPU branch of
    exl3_gemv, bindings.cpp:144-146) and its routes' matmul.  Returns
    (seconds, weights decoded)."""
    import numpy as np
    import torch
    torch.set_num_threads(1)
    seed, which, rows, route_rows = args
    from exl3_b200 import synthetic
    rng = np.random.default_rng(seed)
    in_f, out_f = (H, I) if which < 2 else (I, H)
    rows = min(rows, in_f)
    p = synthetic.make_projection(rng, rows, out_f, KBITS, 1)
    h = torch.from_numpy(rng.normal(0, 1, (route_rows, rows)).astype(np.float32)).half()
    kind, mod = _ref_dequant()
    t0 = time.perf_counter()
    if kind == "reference":
        w = mod.dequant_trellis(torch.from_numpy(p.trellis), torch.from_numpy(p.suh),
                                torch.from_numpy(p.svh), KBITS, True)
    else:
        w = torch.from_numpy(mod.dequant(p.trellis, p.suh, p.svh, KBITS, True))
    y = h.float() @ w.float()
    _ = float(y.sum())
    return time.perf_counter() - t0, rows * out_f


def cpu_reference(tokens: int, steps: int, warmup: int, budget_s: float):
    """Time the reference CPU path on bounded samples; returns a dict.

    A full step decodes gate, up and down of every distinct routed expert
    (3 * H * I weights each) and runs their routes' matmuls.  Each sample runs
    `cores` slices in parallel (one process each) sized so a sample takes about
    `budget_s`; step time = full-step weights / sampled decode throughput."""
    import multiprocessing as mp
    import numpy as np
    from exl3_b200 import synthetic
    cores = max(1, min(os.cpu_count() or 1, 32))
    ctx = mp.get_context("spawn")
    kind = _ref_dequant()[0]
    rng = np.random.default_rng(5)
    ids, _ = synthetic.softmax_topk(rng, tokens, E, TOPK)
    uniq, counts = np.unique(ids, return_counts=True)
    n_distinct = len(uniq)
    step_weights = n_distinct * 3 * H * I
    per_step = []
    with ctx.Pool(cores) as pool:
        cal = pool.map(_slice_task, [(9000 + c, c % 3, 128, 1) for c in range(cores)])
        sec_per_w = statistics.median(t / n for t, n in cal)
        rows = int(max(128, min(2048, budget_s / sec_per_w / I)) // 128 * 128)
        for s in range(warmup + steps):
            tasks = [(s * 131 + c, c % 3, rows, int(counts[c % n_distinct])) for c in range(cores)]
            t0 = time.perf_counter()
            res = pool.map(_slice_task, tasks)
            wall = time.perf_counter() - t0
            if s >= warmup:
                per_step.append(wall * step_weights / sum(n for _, n in res))
    step_s = statistics.median(per_step)
    return {
        "value": tokens / step_s,
        "unit": "tokens/s",
        "cores": cores,
        "kind": kind,
        "step_seconds": step_s,
        "sample": (f"per sample {cores} parallel slices ({rows} input rows of one gate/up/down "
                   f"projection each: dequant_trellis + the routes' matmul), scaled to the "
                   f"{n_distinct} distinct experts x 3 projections of a T={tokens} step; median of "
                   f"{len(per_step)} samples"),
        "cpu": _cpu_model(),
    }


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML polled from a thread)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.stop_flag = [], 0, False
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self.stop_flag:
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self.stop_flag = True
        if self.nv is not None:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------
def run_b200(args, rank, local_rank, world):
    import numpy as np
    import torch
    import torch.distributed as dist
    from exl3_b200 import _native, moe, synthetic

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T = args.tokens
    pack = synthetic.make_moe_pack(0, E, H, I, synthetic.CB_MCG, (KBITS,))
    layer = moe.layer_from_pack(pack, dev)
    NB = 8
    batches = []
    for b in range(NB):
        rng = np.random.default_rng(100 + b)
        x = synthetic.activations(rng, T, H)
        ids, w = synthetic.softmax_topk(rng, T, E, TOPK)
        batches.append((torch.from_numpy(x).to(dev).to(torch.bfloat16), torch.from_numpy(ids).to(dev),
                        torch.from_numpy(w).to(dev)))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    sx = batches[0][0].clone()
    sid = batches[0][1].clone()
    sw = batches[0][2].clone()
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)

    def fwd():
        layer.apply(sx, sw, sid, out=out)

    def load(b):
        x, ids, w = batches[b % NB]
        sx.copy_(x)
        sid.copy_(ids)
        sw.copy_(w)

    # capture the layer once (5 kernels) in a CUDA graph
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(3):
            fwd()
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fwd()

    def timed_loop(n, record=True):
        evs = []
        for i in range(n):
            flush.zero_()
            load(i)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            evs.append((a, b))
        return evs

    timed_loop(args.warmup)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        evs = timed_loop(args.steps)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = world * T * args.steps / (total_ms / 1e3)

    # ---- per-kernel phase times (eager, library events, queued behind a spin)
    _native.profile_enable(True, 2_000_000)
    phases = []
    for i in range(12):
        flush.zero_()
        load(i)
        fwd()
        phases.append(_native.profile_read())
    _native.profile_enable(False)
    names = ["prep", "rotate", "gate_up", "down", "combine"]
    ph = {n: statistics.median(p[j] for p in phases[2:]) * 1e3 for j, n in enumerate(names)}

    # algorithmic bytes (per step average over the rotating batches)
    tile_b = KBITS * 32
    gu_bytes_e = 2 * (H // 16) * (I // 16) * tile_b + 2 * (H + I) * 2
    dn_bytes_e = (I // 16) * (H // 16) * tile_b + (I + H) * 2
    distinct = [len(np.unique(batches[b][1].cpu().numpy())) for b in range(NB)]
    routes = T * TOPK
    gu_bytes = np.mean([d * gu_bytes_e for d in distinct]) + routes * 2 * H * 2 + routes * I * 2
    layer_bytes = np.mean([d * (gu_bytes_e + dn_bytes_e) for d in distinct]) + T * H * 2 * 2
    peak, peak_kind = peaks()
    gu_s = ph["gate_up"] / 1e6
    roofline = {
        "kernel": "gemv_kernel<2,GATEUP> (gate+up decode GEMV)",
        "bound": "hbm", "unit": "GB/s",
        "achieved": gu_bytes / gu_s / 1e9, "peak": peak, "peak_kind": peak_kind,
        "frac": gu_bytes / gu_s / 1e9 / peak,
        "bytes_per_launch": gu_bytes, "us_per_launch": ph["gate_up"],
        "traffic": DRAM_TRAFFIC["decode"]["bytes"] if T == 64 else None,
        "traffic_source": DRAM_TRAFFIC["decode"]["source"] if T == 64 else None,
        "layer": {"bytes": layer_bytes, "us": total_ms / args.steps * 1e3,
                  "achieved": layer_bytes / (total_ms / args.steps / 1e3) / 1e9,
                  "frac": layer_bytes / (total_ms / args.steps / 1e3) / 1e9 / peak},
    }

    # ---- e2e through the public API with host buffers
    hx = [batches[b][0].cpu().pin_memory() for b in range(NB)]
    hid = [batches[b][1].cpu().pin_memory() for b in range(NB)]
    hw = [batches[b][2].cpu().pin_memory() for b in range(NB)]
    hout = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()

    def e2e_loop(n):
        evs = []
        for i in range(n):
            flush.zero_()
            b = i % NB
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            xd = hx[b].to(dev, non_blocking=True)
            idd = hid[b].to(dev, non_blocking=True)
            wd = hw[b].to(dev, non_blocking=True)
            y = layer.apply(xd, wd, idd)
            hout.copy_(y, non_blocking=True)
            a1.record()
            evs.append((a0, a1))
        return evs

    e2e_loop(args.warmup)
    torch.cuda.synchronize(dev)
    evs = e2e_loop(args.steps)
    torch.cuda.synchronize(dev)
    e2e_ms = sum(a.elapsed_time(b) for a, b in evs)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = T * H * 2 + T * TOPK * 8 + T * TOPK * 4
    d2h = T * H * 2

    # ---- decode sweep (graph per batch size), single rank
    sweep = {}
    for tt in (1, 8, 32, 64):
        sweep[str(tt)] = _sweep_point(layer, dev, tt, flush)

    result = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 MMA, fp32 accumulate (int trellis decode)", "data": "synthetic",
        "config": {"workload": f"configs[1] decode GEMV, T={T} tokens/step",
                   "experts": E, "topk": TOPK, "hidden": H, "intermediate": I, "K": KBITS,
                   "codebook": "MCG", "tokens_per_step_per_rank": T,
                   "parallelism": "replicas" if world > 1 else "single GPU",
                   "l2": "256 MB L2 flush before every step (untimed)",
                   "timing": "CUDA events per step around one CUDA-graph replay of the layer"},
        "us_per_layer": total_ms / args.steps * 1e3,
        "phases_us": ph,
        "roofline": roofline,
        "e2e": {"value": world * T * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "us_per_step": e2e_ms / args.steps * 1e3},
        "gpu_launches": 5 * args.steps,
        "clocks": clk.summary(),
        "decode_sweep_us_per_layer": sweep,
    }
    del graph
    return result


PREFILL = {
    # GLM-class mixed-K prefill, mul1, K in {2,3}
    "prefill": dict(cfg="cfg3", E=160, topk=8, H=5120, I=1536, tokens=2048,
                    name="configs[2] mixed-K prefill: 160 experts top-8, H5120 I1536, K2/3 mul1"),
}

# expert-parallel workloads: experts sharded evenly over the ranks, rows
# exchanged over NVLink peer memory or NCCL (exl3_b200.ep, fixed-capacity
# exchange)
EP_WORKLOADS = {
    # configs[1] decode layer at N > 1: T tokens per rank (weak scaling)
    "decode": dict(E=128, topk=8, H=2048, I=768, cb=1, k=(4,), kp=None, router="softmax", sigma=1.0,
                   name="configs[1] decode layer, 128 experts top-8, H2048 I768, K4 MCG, expert-parallel"),
    # 8192 tokens split over the ranks (strong scaling)
    "ep": dict(E=256, topk=8, H=7168, I=2048, cb=1, k=(2, 3, 4), kp=(0.3, 0.5, 0.2), router="sigmoid_zipf",
               tokens=8192, name="configs[4] EP layer: 256 experts top-8 sigmoid+Zipf, H7168 I2048, K2/3/4 MCG"),
}


def run_ep(args, rank, local_rank, world, which):
    """One expert-parallel layer step per rank: dispatch and exchange, local
    fused forward, partial rows back, combine (fixed-capacity exchange, no
    host synchronisation inside a step)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from exl3_b200 import _native, moe, synthetic
    from exl3_b200.ep import Exl3ExpertParallel

    c = EP_WORKLOADS[which]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    E_, H_, I_, k = c["E"], c["H"], c["I"], c["topk"]
    if which == "decode":
        Tr, scaling = args.tokens, "weak"
        Tt = Tr * world
    else:
        Tt = c["tokens"] if args.tokens == 64 else args.tokens
        Tr, scaling = Tt // world, "strong"
    epr = E_ // world
    lo, hi = rank * epr, (rank + 1) * epr
    pack = synthetic.make_moe_pack_slice(0, E_, H_, I_, c["cb"], c["k"], c["kp"], lo, hi)
    kbits = [e["gate"].K for e in pack.experts]
    layer = moe.layer_from_pack(pack, dev)
    del pack
    ep = Exl3ExpertParallel(layer, E_, capacity=Tr, transport=args.ep_transport)
    NB = 4 if which == "decode" else 2
    batches, local_routes, local_experts = [], [], []
    for b in range(NB):
        rng = np.random.default_rng([900 + b])  # routing of all tokens: identical on every rank
        if c["router"] == "softmax":
            ids, w = synthetic.softmax_topk(rng, Tt, E_, k, c["sigma"])
        else:
            ids, w = synthetic.sigmoid_zipf_topk(rng, Tt, E_, k)
        mine = (ids >= lo) & (ids < hi)
        local_routes.append(int(mine.sum()))
        local_experts.append(len(np.unique(ids[mine])))
        x = synthetic.activations(np.random.default_rng([900 + b, rank]), Tr, H_)
        sl = slice(rank * Tr, (rank + 1) * Tr)
        batches.append((torch.from_numpy(x).to(torch.bfloat16).to(dev), torch.from_numpy(ids[sl]).to(dev),
                        torch.from_numpy(w[sl]).to(dev)))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = torch.empty(Tr, H_, dtype=torch.bfloat16, device=dev)

    def step(i):
        x, ids, w = batches[i % NB]
        ep(x, w, ids, out=out)

    def max_over_ranks(v, op=None):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=op or dist.ReduceOp.MAX)
        return float(t.item())

    # decode-sized steps are launch-bound: capture the whole EP step (dispatch,
    # exchange, local forward, combine) in one CUDA graph; the fixed-
    # capacity exchange has no host synchronisation, so it is capturable.
    # Every rank must agree, so capture success is reduced over the ranks.
    graph = None
    sx, sid, sw = (t.clone() for t in batches[0])
    if which == "decode" and not args.no_graph:
        ok, why = 1.0, ""
        try:
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(2):
                    ep(sx, sw, sid, out=out)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                ep(sx, sw, sid, out=out)
        except Exception as ex:  # capture unsupported here: time the eager step
            ok, why, graph = 0.0, str(ex)[:200], None
        if max_over_ranks(ok, dist.ReduceOp.MIN if world > 1 else None) < 1.0:
            graph = None
            if why:
                print(f"[bench] EP graph capture failed: {why}", file=sys.stderr)

    def timed(n):
        evs = []
        for i in range(n):
            flush.zero_()
            if graph is not None:
                x, ids, w = batches[i % NB]
                sx.copy_(x)
                sid.copy_(ids)
                sw.copy_(w)
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            if graph is not None:
                graph.replay()
            else:
                step(i)
            a1.record()
            evs.append((a0, a1))
        return evs

    timed(args.warmup)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        evs = timed(args.steps)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in evs))
    step_s = total_ms / args.steps / 1e3

    # per-phase times: the EP step (CUDA events between phases; with a graph,
    # event nodes captured into a second graph of the same step, so the
    # phases are timed as the graph runs them) and, inside the local
    # forward, the library's kernel phases (eager)
    ep.profile = True
    ep_ph = []
    if graph is not None:
        pgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(pgraph):
            ep(sx, sw, sid, out=out)
        for i in range(4):
            flush.zero_()
            x, ids, w = batches[i % NB]
            sx.copy_(x)
            sid.copy_(ids)
            sw.copy_(w)
            pgraph.replay()
            ep_ph.append(ep.phase_ms())
        del pgraph
    else:
        for i in range(4):
            flush.zero_()
            step(i)
            ep_ph.append(ep.phase_ms())
    ep.profile = False
    _native.profile_enable(True, 2_000_000)
    loc = []
    for i in range(4):
        step(i)
        torch.cuda.synchronize(dev)
        loc.append(_native.profile_read())
    _native.profile_enable(False)
    eph = {n: statistics.median(p[n] for p in ep_ph[1:]) * 1e3 for n in ep.phases}
    nloc = len(loc[0])
    names = ["prep", "rotate", "gate_up", "act", "down", "combine"] if nloc == 6 else \
        ["prep", "rotate", "gate_up", "down", "combine"]
    lph = {n: statistics.median(p[j] for p in loc[1:]) * 1e3 for j, n in enumerate(names)}

    peak_b, kind_b = peaks()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpk, kind_t = float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        tpk, kind_t = 1590.0, "fallback"
    gu_s = lph["gate_up"] / 1e6
    routes = float(np.mean(local_routes))
    if which == "ep":
        flops = routes * 4.0 * H_ * I_
        roof = {"kernel": "tc_gemm_kernel x2 (gate, up) of the local forward, rank %d" % rank,
                "bound": "tensor", "unit": "TFLOP/s", "achieved": flops / gu_s / 1e12, "peak": tpk,
                "peak_kind": kind_t, "frac": flops / gu_s / 1e12 / tpk, "flops_per_launch": flops,
                "us_per_launch": lph["gate_up"], "traffic": None}
    else:
        kb = float(np.mean(kbits))
        per_e = 2 * (H_ // 16) * (I_ // 16) * kb * 32 + 2 * (H_ + I_) * 2
        byts = float(np.mean(local_experts)) * per_e + routes * 2 * H_ * 2
        roof = {"kernel": "gate+up phase of the local forward, rank %d" % rank, "bound": "hbm", "unit": "GB/s",
                "achieved": byts / gu_s / 1e9, "peak": peak_b, "peak_kind": kind_b,
                "frac": byts / gu_s / 1e9 / peak_b, "bytes_per_launch": byts, "us_per_launch": lph["gate_up"],
                "traffic": None}

    # e2e through the public API with pinned host buffers
    hb = [tuple(t.cpu().pin_memory() for t in b) for b in batches]
    hout = torch.empty(Tr, H_, dtype=torch.bfloat16).pin_memory()

    def e2e(n):
        evs = []
        for i in range(n):
            flush.zero_()
            hx, hid, hw = hb[i % NB]
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            y = ep(hx.to(dev, non_blocking=True), hw.to(dev, non_blocking=True), hid.to(dev, non_blocking=True))
            hout.copy_(y, non_blocking=True)
            a1.record()
            evs.append((a0, a1))
        return evs

    e2e(max(1, args.warmup))
    torch.cuda.synchronize(dev)
    evs = e2e(args.steps)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in evs))
    launches = (2 + nloc + 1) if args.ep_transport == "nccl" else (2 + 1 + nloc + 1 + 1 + 1)
    graph_used = graph is not None
    del graph
    torch.cuda.synchronize(dev)
    ep.close()
    return {
        "metric": METRIC if which == "decode" else f"MoE layer prefill tokens/s ({c['name']})",
        "value": Tt * args.steps / (total_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None,
        "dtype": "fp16 MMA, fp32 accumulate (int trellis decode); bf16 rows out, fp32 partials back", "data": "synthetic",
        "config": {"workload": f"{c['name']}, T={Tt} tokens/step ({Tr} per rank)", "experts": E_,
                   "experts_per_rank": epr, "topk": k, "hidden": H_, "intermediate": I_,
                   "parallelism": f"ep{world}",
                   "exchange": ("NVLink peer stores into IPC-mapped windows (library kernels), per-step flags"
                                if args.ep_transport == "nvlink" else "NCCL grouped send/recv")
                   + ", fixed capacity %d rows/rank" % Tr,
                   "l2": "256 MB L2 flush before every step (untimed)",
                   "timing": ("CUDA events per step around one CUDA-graph replay of the EP step" if graph_used
                              else "CUDA events per step around the eager EP step") + ", max over ranks"},
        "us_per_layer": step_s * 1e6, "phases_us": {"ep": eph, "local": lph}, "roofline": roof,
        "local_routes_per_rank": routes,
        "e2e": {"value": Tt * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": Tr * H_ * 2 + Tr * k * 8 + Tr * k * 4, "d2h_bytes_per_step": Tr * H_ * 2,
                "us_per_step": e2e_ms / args.steps * 1e3},
        "gpu_launches": launches * args.steps, "clocks": clk.summary(),
    }


def run_prefill(args, rank, local_rank, world):
    """Tensor-bound workloads (tcgen05 grouped GEMM path); single GPU."""
    import numpy as np
    import torch
    from exl3_b200 import _native, moe, synthetic

    w = PREFILL[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T = args.tokens if args.tokens != 64 else w["tokens"]
    pack, x, ids, wt = synthetic.make_config(w["cfg"], seed=0, tokens=T)
    layer = moe.layer_from_pack(pack, dev)
    NB = 2
    batches = [(torch.from_numpy(x).to(dev).to(torch.bfloat16), torch.from_numpy(ids).to(dev),
                torch.from_numpy(wt).to(dev))]
    rng = np.random.default_rng(1234)
    x2 = synthetic.activations(rng, T, w["H"])
    if w["cfg"] == "cfg5":
        ids2, w2 = synthetic.sigmoid_zipf_topk(rng, T, w["E"], w["topk"])
    else:
        ids2, w2 = synthetic.softmax_topk(rng, T, w["E"], w["topk"], 1.5)
    batches.append((torch.from_numpy(x2).to(dev).to(torch.bfloat16), torch.from_numpy(ids2).to(dev),
                    torch.from_numpy(w2).to(dev)))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    sx, sid, sw = (t.clone() for t in batches[0])
    out = torch.empty(T, w["H"], dtype=torch.bfloat16, device=dev)

    def fwd():
        layer.apply(sx, sw, sid, out=out)

    def load(b):
        sx.copy_(batches[b % NB][0])
        sid.copy_(batches[b % NB][1])
        sw.copy_(batches[b % NB][2])

    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(st):
        for _ in range(2):
            fwd()
    torch.cuda.current_stream(dev).wait_stream(st)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fwd()

    def timed(n):
        evs = []
        for i in range(n):
            flush.zero_()
            load(i)
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            graph.replay()
            a1.record()
            evs.append((a0, a1))
        return evs

    timed(args.warmup)
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        evs = timed(args.steps)
        torch.cuda.synchronize(dev)
    total_ms = sum(a.elapsed_time(b) for a, b in evs)

    _native.profile_enable(True, 2_000_000)
    phases = []
    for i in range(4):
        load(i)
        fwd()
        phases.append(_native.profile_read())
    _native.profile_enable(False)
    names = ["prep", "rotate", "gate_up", "act", "down", "combine"]
    ph = {n: statistics.median(p[j] for p in phases[1:]) * 1e3 for j, n in enumerate(names) if j < len(phases[0])}

    H_, I_, k = w["H"], w["I"], w["topk"]
    flops_layer = T * k * 6.0 * H_ * I_
    flops_gu = T * k * 4.0 * H_ * I_
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpk = float(json.load(f)["bf16_tflops"])
        tkind = "measured"
    except Exception:
        tpk, tkind = 1590.0, "fallback"
    gu_s = ph["gate_up"] / 1e6
    step_s = total_ms / args.steps / 1e3
    roofline = {"kernel": "tc_gemm_kernel x2 (gate, up: tcgen05 grouped GEMM)", "bound": "tensor",
                "unit": "TFLOP/s", "achieved": flops_gu / gu_s / 1e12, "peak": tpk, "peak_kind": tkind,
                "frac": flops_gu / gu_s / 1e12 / tpk, "flops_per_launch": flops_gu, "us_per_launch": ph["gate_up"],
                "traffic": DRAM_TRAFFIC["prefill"]["bytes"] if T == 2048 else None,
                "traffic_source": DRAM_TRAFFIC["prefill"]["source"] if T == 2048 else None,
                "layer": {"flops": flops_layer, "us": step_s * 1e6, "achieved": flops_layer / step_s / 1e12,
                          "frac": flops_layer / step_s / 1e12 / tpk}}
    del graph
    return {"metric": f"MoE layer prefill tokens/s ({w['name']})", "value": T * args.steps / (total_ms / 1e3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16 MMA (tcgen05), fp32 accumulate", "data": "synthetic",
            "config": {"workload": w["name"] + f", T={T}", "tokens_per_step": T,
                       "l2": "256 MB L2 flush before every step (untimed)"},
            "us_per_layer": step_s * 1e6, "phases_us": ph, "roofline": roofline,
            "gpu_launches": 7 * args.steps, "clocks": clk.summary()}


def _sweep_point(layer, dev, T, flush):
    import numpy as np
    import torch
    from exl3_b200 import synthetic
    rng = np.random.default_rng(7000 + T)
    bs = []
    for b in range(8):
        x = synthetic.activations(rng, T, H)
        ids, w = synthetic.softmax_topk(rng, T, E, TOPK)
        bs.append((torch.from_numpy(x).to(dev).to(torch.bfloat16), torch.from_numpy(ids).to(dev),
                   torch.from_numpy(w).to(dev)))
    sx, sid, sw = (t.clone() for t in bs[0])
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(3):
            layer.apply(sx, sw, sid, out=out)
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.apply(sx, sw, sid, out=out)
    ts = []
    for i in range(40):
        flush.zero_()
        sx.copy_(bs[i % 8][0])
        sid.copy_(bs[i % 8][1])
        sw.copy_(bs[i % 8][2])
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        ts.append((a, b))
    torch.cuda.synchronize(dev)
    del g
    vals = [a.elapsed_time(b) * 1e3 for a, b in ts[8:]]
    return statistics.median(vals)


def main():
    args = parse()
    rank, local_rank, world = env_rank()
    if args.impl == "reference":
        if rank != 0:
            return
        budget = max(0.05, min(2.0, 150.0 / max(1, args.steps + args.warmup)))
        r = cpu_reference(args.tokens, args.steps, args.warmup, budget)
        line = {"metric": METRIC, "value": r["value"], "unit": "tokens/s", "impl": "reference",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": r["step_seconds"] * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (CPU)", "data": "synthetic",
                "config": {"workload": f"configs[1] decode GEMV, T={args.tokens} tokens/step",
                           "experts": E, "topk": TOPK, "hidden": H, "intermediate": I, "K": KBITS},
                "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if args.workload == "prefill":
        print(json.dumps(run_prefill(args, rank, local_rank, world)), flush=True)
        return
    if world > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    # the CPU sample runs first, before CUDA is touched (spawned workers)
    cpu = None
    if rank == 0 and world == 1 and args.workload == "decode" and not args.no_cpu_baseline:
        cpu = cpu_reference(args.tokens, 5, 1, 2.0)
    if args.workload == "ep" or world > 1:
        res = run_ep(args, rank, local_rank, world, "ep" if args.workload == "ep" else "decode")
    else:
        res = run_b200(args, rank, local_rank, world)
    if cpu is not None:
        res["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

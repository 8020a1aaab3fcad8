"""Benchmark of the EXL3 routed-expert MoE layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--tokens T]
                    [--workload decode|prefill|ep] [--no-prefill] [--no-ep-cfg4] [--no-cpu-baseline]

Headline (the decode config): one routed-MoE layer,
128 experts, top-8 softmax routing, hidden 2048, expert intermediate 768,
uniform K=4 MCG, T=64 tokens per step (the config's largest decode batch;
T = 1, 8, 32 are reported in `decode_sweep_us_per_layer`).  Weights and inputs
are seeded synthetic (exl3_b200.synthetic).  A step is one layer forward over
one batch; 8 different routings/batches rotate across steps.

The same line carries, as sub-objects measured in the same run:
* `prefill`: configs[2] (160 experts, H5120 I1536, K2/3 mul1, T=2048), the
  tcgen05 grouped-GEMM path, one GPU;
* `dense`: configs[3] (8192x28672 then 28672x8192, K3 MCG, M = 1, 16, 256,
  4096 rows) through the dense layer API, one GPU;
* `ep_cfg4`: configs[4] (256 experts top-8 sigmoid+Zipf, H7168 I2048,
  K2/3/4 MCG, 8192 tokens split over the N ranks: strong scaling), the
  expert-parallel step with per-phase in-graph times and the per-rank
  local-route skew.

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier
and torch.cuda.synchronize(); every step is timed with CUDA events on the
launching stream around the layer only, after an untimed 256 MB L2 flush
(larger than the 126 MB L2).  `value` = tokens of all ranks / max-over-ranks
device time (CUDA graph of the layer, inputs resident in HBM).  `e2e` = the
same metric through the public API (exl3_b200.moe.Exl3RoutedExperts.apply,
eager) with pinned-host inputs copied in and the output copied back inside
the timed region.  Every line's outputs are checked against the CPU eager
loop (oracle/parity.py) outside the timed region: `parity`.

N > 1: expert parallelism (exl3_b200.ep): rank g holds experts
[g*E/N, (g+1)*E/N); the headline runs the decode layer with T tokens per rank
(weak scaling); a step is dispatch (the library's kernels store each pair row
straight into its owner's IPC-mapped window over NVLink; --ep-transport nccl
uses NCCL instead), the local fused forward, the partial rows stored back,
and the per-token combine, one CUDA graph per step, timed per step and taken
as the max over ranks.

--impl reference: rank 0 times the reference's CPU path (oracle/ref_loop.py:
the reference's eager loop apply_exl3_python_loop with dequant_trellis from
the reference's own csrc/bindings.cpp compiled into oracle/_ref) on this
box's host cores: each step runs the loop body of a sample of the batch's
distinct experts, one process per core; `ms_per_step` is that step's
measured time and `value` the equivalent tokens/s (tokens x the sampled
fraction of the step's experts / step time).  configs[0] is also timed as one
whole layer, serially as the reference runs it (median of 3).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
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
    "decode": {"bytes": 264.5e6, "kernel": "gemv_kernel<2,GATEUP,MCG>, T=64",
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
    ap.add_argument("--no-prefill", action="store_true", help="skip the configs[2] prefill sub-object")
    ap.add_argument("--no-ep-cfg4", action="store_true", help="skip the configs[4] expert-parallel sub-object")
    ap.add_argument("--no-dense", action="store_true", help="skip the configs[3] dense-linear sub-object")
    ap.add_argument("--no-parity", action="store_true", help="skip the output checks against the oracle")
    ap.add_argument("--no-graph", action="store_true", help="time the expert-parallel step eagerly")
    ap.add_argument("--ep-transport", default="nvlink", choices=["nvlink", "nccl"],
                    help="expert-parallel exchange: the library's NVLink peer-store kernels or NCCL")
    ap.add_argument("--ep-placement", default="balanced", choices=["balanced", "contiguous"],
                    help="configs[4] expert placement over the ranks: even 128-row route tiles per rank from "
                         "a calibration batch's counts, or contiguous blocks of E/G experts")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "ep"],
                    help="decode = configs[1] (the default, reported line, with the prefill and ep_cfg4 "
                         "sub-objects); prefill = configs[2] alone; ep = configs[4] alone")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, kind) from MEASURED_PEAKS.json, else the
    pool's earlier measurement."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def log(msg: str) -> None:
    print(f"[bench] {msg}", file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------
# the reference's CPU path (the reference arm and the cpu_baseline key)
# ---------------------------------------------------------------------------
def _decode_batches_np(T: int, NB: int = 8, seed0: int = 100):
    import numpy as np
    from exl3_b200 import synthetic
    out = []
    for b in range(NB):
        rng = np.random.default_rng(seed0 + b)
        x = synthetic.activations(rng, T, H)
        ids, w = synthetic.softmax_topk(rng, T, E, TOPK)
        out.append((x, ids, w))
    return out


def cpu_reference(tokens: int, steps: int, warmup: int, per_step: int | None = None, cfg0: bool = False):
    """Measured steps of the reference's eager loop on the host cores
    (oracle/ref_loop.py); see the module docstring for what a step is."""
    import numpy as np
    import ref_loop
    from exl3_b200 import synthetic
    pack = synthetic.make_moe_pack(0, E, H, I, synthetic.CB_MCG, (KBITS,))
    batches = _decode_batches_np(tokens)
    pool = ref_loop.ExpertPool(pack)
    try:
        n = pool.cores if per_step is None else per_step
        r = ref_loop.sampled_steps(pool, batches, steps, warmup, n)
    finally:
        pool.close()
    secs, fr = r["seconds"], r["fractions"]
    eq_tokens = [tokens * f for f in fr]
    value = sum(eq_tokens) / sum(secs)
    distinct = float(np.mean([np.unique(b[1]).size for b in batches]))
    res = {
        "value": value, "unit": "tokens/s", "cores": pool.cores, "kind": ref_loop.ref_module()[0],
        "ms_per_step": 1e3 * sum(secs) / len(secs),
        "sample": (f"each step: the reference eager loop (apply_exl3_python_loop, dequant_trellis of the "
                   f"reference's compiled csrc/bindings.cpp) over {n} of the batch's ~{distinct:.0f} distinct "
                   f"experts, one process per host core; value = T={tokens} x sampled fraction / measured "
                   f"step time, over {len(secs)} timed steps"),
        "equivalent_tokens_per_step": float(np.mean(eq_tokens)),
        "full_step_seconds_estimate": sum(secs) / sum(fr),
        "cpu": ref_loop.cpu_model(), "nproc": os.cpu_count(),
    }
    if cfg0:
        p0, x0, i0, w0 = synthetic.make_config("cfg1", seed=0)
        med, reps = ref_loop.time_layer_serial(p0, x0, i0, w0, reps=3, threads=os.cpu_count() or 1)
        res["cfg0_full_layer"] = {
            "workload": "configs[0]: 8 experts top-2, H1024 I512, K4 MCG, T=16, whole layer, serial loop",
            "seconds_median": med, "seconds": reps, "tokens_per_s": 16 / med,
            "torch_threads": os.cpu_count()}
    return res


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


def _capture(fn, dev, warm: int = 2):
    """fn captured in a CUDA graph after `warm` eager runs on a side stream."""
    import torch
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def _timed_replays(graph, n, flush, load):
    """CUDA events around each replay, after an untimed L2 flush and input load."""
    import torch
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


# ---------------------------------------------------------------------------
# the headline: configs[1] decode on one GPU
# ---------------------------------------------------------------------------
def run_decode(args, rank, local_rank, world):
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
    np_batches = _decode_batches_np(T, NB)
    batches = [(torch.from_numpy(x).to(dev).to(torch.bfloat16), torch.from_numpy(ids).to(dev),
                torch.from_numpy(w).to(dev)) for x, ids, w in np_batches]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    sx, sid, sw = (t.clone() for t in batches[0])
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)

    def fwd():
        layer.apply(sx, sw, sid, out=out)

    def load(b):
        x, ids, w = batches[b % NB]
        sx.copy_(x)
        sid.copy_(ids)
        sw.copy_(w)

    graph = _capture(fwd, dev, warm=3)
    _timed_replays(graph, args.warmup, flush, load)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        evs = _timed_replays(graph, args.steps, flush, load)
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

    # parity: batch 0, every token, against the eager loop.  The check runs on
    # fp32 output rows (the same kernels; only the final store differs):
    # rounding the output to bf16 alone moves elements beyond 8 x RMS by more
    # than 2e-2 x RMS, so the bf16 graph output is reported as information
    par = None
    if not args.no_parity:
        par = _parity_rows(layer, pack.experts, E, batches[0], np_batches[0], graph, out, load, None, None)

    # per-kernel phase times (eager, library events, queued behind a spin)
    _native.profile_enable(True, 2_000_000)
    phases = []
    for i in range(12):
        flush.zero_()
        load(i)
        fwd()
        phases.append(_native.profile_read())
    _native.profile_enable(False)
    names = ["prep", "rotate", "gate_up", "down", "combine"]
    n_ph = len(phases[0])
    if n_ph != len(names):
        names = [f"phase{j}" for j in range(n_ph)]
    ph = {n: statistics.median(p[j] for p in phases[2:]) * 1e3 for j, n in enumerate(names)}

    # algorithmic bytes (per step average over the rotating batches)
    tile_b = KBITS * 32
    gu_bytes_e = 2 * (H // 16) * (I // 16) * tile_b + 2 * (H + I) * 2
    dn_bytes_e = (I // 16) * (H // 16) * tile_b + (I + H) * 2
    distinct = [len(np.unique(b[1])) for b in np_batches]
    routes = T * TOPK
    gu_bytes = np.mean([d * gu_bytes_e for d in distinct]) + routes * 2 * H * 2 + routes * I * 2
    layer_bytes = np.mean([d * (gu_bytes_e + dn_bytes_e) for d in distinct]) + T * H * 2 * 2
    peak, _tpk, peak_kind = peaks()
    gu_us = ph.get("gate_up")
    roofline = {
        "kernel": "gemv_kernel<2,GATEUP> (gate+up decode GEMV)", "bound": "hbm", "unit": "GB/s",
        "peak": peak, "peak_kind": peak_kind, "bytes_per_launch": gu_bytes, "us_per_launch": gu_us,
        "traffic": DRAM_TRAFFIC["decode"]["bytes"] if T == 64 else None,
        "traffic_source": DRAM_TRAFFIC["decode"]["source"] if T == 64 else None,
        "layer": {"bytes": layer_bytes, "us": total_ms / args.steps * 1e3,
                  "achieved": layer_bytes / (total_ms / args.steps / 1e3) / 1e9,
                  "frac": layer_bytes / (total_ms / args.steps / 1e3) / 1e9 / peak},
    }
    if gu_us:
        roofline["achieved"] = gu_bytes / (gu_us / 1e6) / 1e9
        roofline["frac"] = roofline["achieved"] / peak

    # e2e through the public API with host buffers
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

    sweep = {str(tt): _sweep_point(layer, dev, tt, flush) for tt in (1, 8, 32, 64)}
    del graph
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
        "gpu_launches": n_ph * args.steps,
        "clocks": clk.summary(),
        "decode_sweep_us_per_layer": sweep,
    }
    if par is not None:
        result["parity"] = par
    del layer
    torch.cuda.empty_cache()
    return result


def _parity_rows(layer, experts, n_experts, batch_dev, batch_np, graph, out, load, sel, blocks):
    """Check one batch's rows (all, or the sampled `sel`) against the eager
    loop: fp32 output of an eager call (the pass/fail figure) and, for
    information, the captured graph's own output in its dtype."""
    import numpy as np
    import torch
    import parity
    xd, idd, wd = batch_dev
    _x, ids, w = batch_np
    dev = xd.device
    f32 = torch.empty(xd.shape[0], out.shape[1], dtype=torch.float32, device=dev)
    layer.apply(xd, wd, idd, out=f32)
    load(0)
    graph.replay()
    torch.cuda.synchronize(dev)
    rows = np.arange(xd.shape[0]) if sel is None else sel
    idx = torch.from_numpy(rows).to(dev)
    xb = xd.float().cpu().numpy()[rows]
    want = parity.expected_moe(xb, ids[rows], w[rows], lambda e: experts[e], n_experts, blocks)
    st = parity.compare(f32[idx].cpu().numpy(), want, blocks)
    st_out = parity.compare(out[idx].float().cpu().numpy(), want, blocks)
    st["tokens"] = int(len(rows))
    st["col_blocks"] = None if blocks is None else len(blocks)
    st["graph_output"] = {"dtype": str(out.dtype).replace("torch.", ""),
                          "max_abs_over_rms": st_out["max_abs_over_rms"], "cos": st_out["cos"]}
    st["note"] = ("fp32 rows of an eager call vs the eager loop (pass/fail); graph_output: the timed "
                  "graph's own output rows, rounded to their dtype, for information")
    return st


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

    def load(i):
        sx.copy_(bs[i % 8][0])
        sid.copy_(bs[i % 8][1])
        sw.copy_(bs[i % 8][2])

    g = _capture(lambda: layer.apply(sx, sw, sid, out=out), dev, warm=3)
    ts = _timed_replays(g, 40, flush, load)
    torch.cuda.synchronize(dev)
    del g
    return statistics.median(a.elapsed_time(b) * 1e3 for a, b in ts[8:])


# ---------------------------------------------------------------------------
# mixed-K prefill (tcgen05 grouped GEMM), one GPU
# ---------------------------------------------------------------------------
PREFILL = dict(cfg="cfg3", E=160, topk=8, H=5120, I=1536, tokens=2048,
               name="configs[2] mixed-K prefill: 160 experts top-8, H5120 I1536, K2/3 mul1")


def run_prefill(args, local_rank, steps, warmup, tokens=None):
    import numpy as np
    import torch
    from exl3_b200 import _native, moe, synthetic

    w = PREFILL
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T = tokens or w["tokens"]
    pack, x, ids, wt = synthetic.make_config(w["cfg"], seed=0, tokens=T)
    layer = moe.layer_from_pack(pack, dev)
    NB = 2
    batches = [(torch.from_numpy(x).to(dev).to(torch.bfloat16), torch.from_numpy(ids).to(dev),
                torch.from_numpy(wt).to(dev))]
    rng = np.random.default_rng(1234)
    x2 = synthetic.activations(rng, T, w["H"])
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

    graph = _capture(fwd, dev)
    _timed_replays(graph, warmup, flush, load)
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        evs = _timed_replays(graph, steps, flush, load)
        torch.cuda.synchronize(dev)
    total_ms = sum(a.elapsed_time(b) for a, b in evs)

    par = None
    if not args.no_parity:
        import parity
        par = _parity_rows(layer, pack.experts, w["E"], batches[0], (x, ids, wt), graph, out, load,
                           parity.sample_tokens(T, 8, seed=1), None)
    del graph

    _native.profile_enable(True, 2_000_000)
    phases = []
    for i in range(4):
        load(i)
        fwd()
        phases.append(_native.profile_read())
    _native.profile_enable(False)
    names = ["prep", "rotate", "gate_up", "act", "down", "combine"]
    n_ph = len(phases[0])
    ph = {n: statistics.median(p[j] for p in phases[1:]) * 1e3 for j, n in enumerate(names) if j < n_ph}

    H_, I_, k = w["H"], w["I"], w["topk"]
    flops_layer = T * k * 6.0 * H_ * I_
    flops_gu = T * k * 4.0 * H_ * I_
    _hbm, tpk, tkind = peaks()
    gu_s = ph["gate_up"] / 1e6
    step_s = total_ms / steps / 1e3
    roofline = {"kernel": "tc_gemm_kernel (gate and up: tcgen05 grouped GEMM)", "bound": "tensor",
                "unit": "TFLOP/s", "achieved": flops_gu / gu_s / 1e12, "peak": tpk, "peak_kind": tkind,
                "frac": flops_gu / gu_s / 1e12 / tpk, "flops_per_launch": flops_gu, "us_per_launch": ph["gate_up"],
                "traffic": DRAM_TRAFFIC["prefill"]["bytes"] if T == 2048 else None,
                "traffic_source": DRAM_TRAFFIC["prefill"]["source"] if T == 2048 else None,
                "layer": {"flops": flops_layer, "us": step_s * 1e6, "achieved": flops_layer / step_s / 1e12,
                          "frac": flops_layer / step_s / 1e12 / tpk}}
    res = {"metric": f"MoE layer prefill tokens/s ({w['name']})", "value": T * steps / (total_ms / 1e3),
           "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": warmup,
           "ms_per_step": total_ms / steps, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "fp16 MMA (tcgen05), fp32 accumulate", "data": "synthetic",
           "config": {"workload": w["name"] + f", T={T}", "tokens_per_step": T,
                      "l2": "256 MB L2 flush before every step (untimed)",
                      "timing": "CUDA events per step around one CUDA-graph replay of the layer"},
           "us_per_layer": step_s * 1e6, "phases_us": ph, "roofline": roofline,
           "gpu_launches": n_ph * steps, "clocks": clk.summary()}
    if par is not None:
        res["parity"] = par
    del layer
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------
# dense EXL3 linear, MLP-sized, one GPU
# ---------------------------------------------------------------------------
DENSE = dict(n=8192, f=28672, K=3, ms=(1, 16, 256, 4096),
             name="configs[3] dense EXL3 linear: 8192x28672 then 28672x8192, K3 MCG")


def run_dense(args, local_rank, steps, warmup):
    """The two projections of an MLP (x W1 then y W2) through the dense layer
    API (exl3_b200.linear.Exl3Linear) at each row count; per row count a step
    is both projections, bf16 in and out."""
    import numpy as np
    import torch
    from exl3_b200 import linear as lin
    from exl3_b200 import synthetic

    c = DENSE
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(4)
    p1 = synthetic.make_projection(rng, c["n"], c["f"], c["K"], synthetic.CB_MCG)
    p2 = synthetic.make_projection(rng, c["f"], c["n"], c["K"], synthetic.CB_MCG)
    l1 = lin.linear_from_projections([p1], dev)
    l2 = lin.linear_from_projections([p2], dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    hbm, tpk, kind = peaks()
    wbytes = 2 * (c["n"] // 16) * (c["f"] // 16) * 32 * c["K"] + 2 * (c["n"] + c["f"]) * 2
    out = {"workload": c["name"], "peak_kind": kind}
    for M in c["ms"]:
        x = torch.from_numpy(np.random.default_rng(10 + M).normal(0, 1, (M, c["n"])).astype(np.float32)).to(dev)
        x = x.to(torch.bfloat16)
        ys = {}

        def step():
            ys["y"] = l2(l1(x))

        g = _capture(step, dev)
        with ClockSampler(local_rank) as clk:
            evs = _timed_replays(g, warmup + steps, flush, lambda i: None)[warmup:]
            torch.cuda.synchronize(dev)
        us = statistics.median(a.elapsed_time(b) for a, b in evs) * 1e3
        # each projection timed alone (eager, events on the launching stream)
        t1, t2 = [], []
        for _ in range(5):
            flush.zero_()
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record()
            y1 = l1(x)
            e1.record()
            l2(y1)
            e2.record()
            torch.cuda.synchronize(dev)
            t1.append(e0.elapsed_time(e1) * 1e3)
            t2.append(e1.elapsed_time(e2) * 1e3)
        u1, u2 = statistics.median(t1[1:]), statistics.median(t2[1:])
        act_bytes = 2 * M * (c["n"] + c["f"]) * 2  # bf16 in and out of both projections
        flops = 2.0 * M * c["n"] * c["f"] * 2
        if M <= 16:
            ach = (wbytes + act_bytes) / (us / 1e6) / 1e9
            roof = {"bound": "hbm", "unit": "GB/s", "achieved": ach, "peak": hbm, "frac": ach / hbm,
                    "bytes_per_step": wbytes + act_bytes}
        else:
            ach = flops / (us / 1e6) / 1e12
            roof = {"bound": "tensor", "unit": "TFLOP/s", "achieved": ach, "peak": tpk, "frac": ach / tpk,
                    "flops_per_step": flops}
        r = {"us_per_step": us, "us_w1": u1, "us_w2": u2, "roofline": roof, "clocks": clk.summary()}
        if not args.no_parity:
            import parity
            rows = parity.sample_tokens(M, 8, seed=M)
            idx = torch.from_numpy(rows).to(dev)
            xh = x.float().cpu().numpy()[rows].astype(np.float16).astype(np.float32)
            y1f = l1._exl3_linears[0]
            import vllm_exl3_c
            f1 = vllm_exl3_c.exl3_linear(x, y1f.trellis, y1f.suh, y1f.svh, y1f.K, 1, out_dtype=torch.float32)
            b1 = parity.col_blocks(c["f"], 4, seed=M)
            st1 = parity.compare(f1[idx].cpu().numpy(), xh @ parity.projection_dense(p1, b1).astype(np.float32), b1)
            y1 = l1(x)
            y2f = l2._exl3_linears[0]
            f2 = vllm_exl3_c.exl3_linear(y1, y2f.trellis, y2f.suh, y2f.svh, y2f.K, 1, out_dtype=torch.float32)
            x2 = y1.float().cpu().numpy()[rows].astype(np.float16).astype(np.float32)
            b2 = parity.col_blocks(c["n"], 4, seed=M + 1)
            st2 = parity.compare(f2[idx].cpu().numpy(), x2 @ parity.projection_dense(p2, b2).astype(np.float32), b2)
            r["parity"] = {"w1": st1, "w2": st2, "pass": st1["pass"] and st2["pass"],
                           "note": f"fp32 rows of each projection vs the oracle's dequant matmul, {len(rows)} "
                                   "sampled rows x 4 128-column blocks"}
        out[f"M={M}"] = r
        del g
    del l1, l2
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# expert-parallel workloads
# ---------------------------------------------------------------------------
EP_WORKLOADS = {
    # configs[1] decode layer at N > 1: T tokens per rank (weak scaling)
    "decode": dict(E=128, topk=8, H=2048, I=768, cb=1, k=(4,), kp=None, router="softmax", sigma=1.0,
                   name="configs[1] decode layer, 128 experts top-8, H2048 I768, K4 MCG, expert-parallel"),
    # 8192 tokens split over the ranks (strong scaling)
    "ep": dict(E=256, topk=8, H=7168, I=2048, cb=1, k=(2, 3, 4), kp=(0.3, 0.5, 0.2), router="sigmoid_zipf",
               tokens=8192, name="configs[4] EP layer: 256 experts top-8 sigmoid+Zipf, H7168 I2048, K2/3/4 MCG"),
}


def run_ep(args, rank, local_rank, world, which, steps, warmup):
    """One expert-parallel layer step per rank: dispatch and exchange, local
    fused forward, partial rows back, combine (fixed-capacity exchange, no
    host synchronisation inside a step)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from exl3_b200 import _native, moe, synthetic
    from exl3_b200.ep import Exl3ExpertParallel, balanced_placement, experts_of_rank

    c = EP_WORKLOADS[which]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    E_, H_, I_, k = c["E"], c["H"], c["I"], c["topk"]
    if which == "decode":
        Tr, scaling = args.tokens, "weak"
        Tt = Tr * world
    else:
        Tt = c["tokens"]
        Tr, scaling = Tt // world, "strong"
    epr = E_ // world
    lo = rank * epr

    def make(a, b):
        return synthetic.make_moe_pack_slice(0, E_, H_, I_, c["cb"], c["k"], c["kp"], a, b)

    def expert_of(e):
        return make(e, e + 1).experts[0]

    # the router's per-expert Zipf bias is a property of the layer: every
    # batch of it uses the same popularity ranks
    zipf_ranks = np.random.default_rng([899]).permutation(E_) if c["router"] != "softmax" else None

    def route(seed):
        rng = np.random.default_rng(seed)
        if c["router"] == "softmax":
            return synthetic.softmax_topk(rng, Tt, E_, k, c["sigma"])
        return synthetic.sigmoid_zipf_topk(rng, Tt, E_, k, ranks=zipf_ranks)

    # load-aware placement (skewed routing only): slots from the routing
    # counts of a calibration batch that is not one of the timed batches
    slot = None
    if which == "ep" and world > 1 and args.ep_placement == "balanced":
        cal_ids, _ = route([950])
        slot = np.asarray(balanced_placement(np.bincount(cal_ids.ravel(), minlength=E_), world))
    if slot is None:
        layer = moe.layer_from_slices(lambda a, b: make(lo + a, lo + b), epr, H_, I_, dev)
    else:
        held = experts_of_rank(slot, world, rank)

        def make_held(a, b):
            pk = make(0, 0)
            pk.experts = [expert_of(e) for e in held[a:b]]
            return pk

        layer = moe.layer_from_slices(make_held, epr, H_, I_, dev)
    kbits = [int(inn["gate"].K) for inn in layer._exl3_inners]
    ep = Exl3ExpertParallel(layer, E_, capacity=Tr, transport=args.ep_transport,
                            placement=None if slot is None else slot.tolist())
    NB = 4 if which == "decode" else 2
    batches, np_batches, local_routes, local_experts, rank_routes = [], [], [], [], []
    for b in range(NB):
        ids, w = route([900 + b])  # routing of all tokens: identical on every rank
        owner = (ids if slot is None else slot[ids]) // epr
        rank_routes.append([int((owner == g).sum()) for g in range(world)])
        mine = owner == rank
        local_routes.append(int(mine.sum()))
        local_experts.append(len(np.unique(ids[mine])))
        x = synthetic.activations(np.random.default_rng([900 + b, rank]), Tr, H_)
        sl = slice(rank * Tr, (rank + 1) * Tr)
        np_batches.append((x, ids[sl], w[sl]))
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
    if not args.no_graph:
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
                log(f"EP graph capture failed: {why}")

    def load(i):
        x, ids, w = batches[i % NB]
        sx.copy_(x)
        sid.copy_(ids)
        sw.copy_(w)

    def timed(n):
        evs = []
        for i in range(n):
            flush.zero_()
            if graph is not None:
                load(i)
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

    timed(warmup)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        evs = timed(steps)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in evs))
    step_s = total_ms / steps / 1e3
    ep.check_status()

    # parity (rank 0's tokens of batch 0, a sample, against the eager loop);
    # every rank runs the step, rank 0 checks
    par = None
    if not args.no_parity:
        # every rank runs the same steps (an fp32-output eager step, then the
        # graph); rank 0 checks its sampled tokens against the eager loop over
        # all experts
        import parity
        f32 = torch.empty(Tr, H_, dtype=torch.float32, device=dev)
        ep(batches[0][0], batches[0][2], batches[0][1], out=f32)
        if graph is not None:
            load(0)
            graph.replay()
        else:
            step(0)
        torch.cuda.synchronize(dev)
        if rank == 0:
            sel = parity.sample_tokens(Tr, 8 if which == "decode" else 4, seed=3)
            blocks = None if which == "decode" else parity.col_blocks(H_, 4, seed=3)
            _xb, idb, wb = np_batches[0]
            xb = batches[0][0].float().cpu().numpy()[sel]
            want = parity.expected_moe(xb, idb[sel], wb[sel], expert_of, E_, blocks)
            idx = torch.from_numpy(sel).to(dev)
            par = parity.compare(f32[idx].cpu().numpy(), want, blocks)
            st_out = parity.compare(out[idx].float().cpu().numpy(), want, blocks)
            par.update(tokens=int(len(sel)), col_blocks=None if blocks is None else len(blocks),
                       graph_output={"dtype": "bfloat16", "max_abs_over_rms": st_out["max_abs_over_rms"],
                                     "cos": st_out["cos"]},
                       note=(f"rank 0: fp32 rows of an eager EP step vs the eager loop over all {E_} experts, "
                             f"{len(sel)} sampled tokens" + ("" if blocks is None else f" x {len(blocks)} "
                             "128-column blocks") + "; graph_output: the timed step's own bf16 rows"))
        if world > 1:
            dist.barrier()

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
            load(i)
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
    if nloc not in (5, 6):
        names = [f"phase{j}" for j in range(nloc)]
    lph = {n: statistics.median(p[j] for p in loc[1:]) * 1e3 for j, n in enumerate(names)}
    # the slowest rank's phases and local forward (the step waits for it)
    eph_max = {n: max_over_ranks(v) for n, v in eph.items()}
    lph_max = {n: max_over_ranks(v) for n, v in lph.items()}

    peak_b, tpk, kind = peaks()
    gu_us = lph.get("gate_up", 0.0) or 1e-9
    gu_s = gu_us / 1e6
    routes = float(np.mean(local_routes))
    if which == "ep":
        flops = routes * 4.0 * H_ * I_
        roof = {"kernel": "tc_gemm_kernel (gate and up) of the local forward, rank %d" % rank,
                "bound": "tensor", "unit": "TFLOP/s", "achieved": flops / gu_s / 1e12, "peak": tpk,
                "peak_kind": kind, "frac": flops / gu_s / 1e12 / tpk, "flops_per_launch": flops,
                "us_per_launch": gu_us, "traffic": None}
    else:
        kb = float(np.mean(kbits))
        per_e = 2 * (H_ // 16) * (I_ // 16) * kb * 32 + 2 * (H_ + I_) * 2
        byts = float(np.mean(local_experts)) * per_e + routes * 2 * H_ * 2
        roof = {"kernel": "gate+up phase of the local forward, rank %d" % rank, "bound": "hbm", "unit": "GB/s",
                "achieved": byts / gu_s / 1e9, "peak": peak_b, "peak_kind": kind,
                "frac": byts / gu_s / 1e9 / peak_b, "bytes_per_launch": byts, "us_per_launch": gu_us,
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

    e2e(max(1, warmup))
    torch.cuda.synchronize(dev)
    evs = e2e(steps)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in evs))
    ep.check_status()
    launches = (2 + nloc + 1) if args.ep_transport == "nccl" else (2 + 1 + nloc + 1 + 1 + 1)
    graph_used = graph is not None
    del graph
    torch.cuda.synchronize(dev)
    ep.close()
    rr = np.asarray(rank_routes, dtype=np.float64).mean(axis=0)
    res = {
        "metric": METRIC if which == "decode" else f"MoE layer prefill tokens/s ({c['name']})",
        "value": Tt * steps / (total_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": total_ms / steps, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None,
        "dtype": "fp16 MMA, fp32 accumulate (int trellis decode); bf16 rows out, fp32 partials back",
        "data": "synthetic",
        "config": {"workload": f"{c['name']}, T={Tt} tokens/step ({Tr} per rank)", "experts": E_,
                   "experts_per_rank": epr, "topk": k, "hidden": H_, "intermediate": I_,
                   "parallelism": f"ep{world}",
                   "placement": ("contiguous: rank g holds experts [g*E/G, (g+1)*E/G)" if slot is None else
                                 "balanced: E/G experts per rank, longest-first by 128-row route tiles of "
                                 "a calibration batch (seed 950, not a timed batch)"),
                   "exchange": ("NVLink peer stores into IPC-mapped windows (library kernels), per-step flags"
                                if args.ep_transport == "nvlink" else "NCCL grouped send/recv")
                   + ", fixed capacity %d rows/rank" % Tr,
                   "l2": "256 MB L2 flush before every step (untimed)",
                   "timing": ("CUDA events per step around one CUDA-graph replay of the EP step" if graph_used
                              else "CUDA events per step around the eager EP step") + ", max over ranks"},
        "us_per_layer": step_s * 1e6,
        "phases_us": {"ep_rank0": eph, "ep_max_over_ranks": eph_max, "local_rank0": lph,
                      "local_max_over_ranks": lph_max},
        "roofline": roof,
        "local_routes_per_rank": {"rank0": routes, "max": float(rr.max()), "min": float(rr.min()),
                                  "max_over_mean": float(rr.max() / rr.mean())},
        "e2e": {"value": Tt * steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": Tr * H_ * 2 + Tr * k * 8 + Tr * k * 4, "d2h_bytes_per_step": Tr * H_ * 2,
                "us_per_step": e2e_ms / steps * 1e3},
        "gpu_launches": launches * steps, "clocks": clk.summary(),
    }
    if par is not None:
        res["parity"] = par
    del layer, ep
    torch.cuda.empty_cache()
    return res


def _ref_line(args, world):
    r = cpu_reference(args.tokens, args.steps, args.warmup, cfg0=True)
    return {"metric": METRIC, "value": r["value"], "unit": "tokens/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (CPU; fp16 weights and activations)",
            "data": "synthetic",
            "config": {"workload": f"configs[1] decode GEMV, T={args.tokens} tokens/step",
                       "experts": E, "topk": TOPK, "hidden": H, "intermediate": I, "K": KBITS,
                       "codebook": "MCG"},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu", "nproc")},
            "equivalent_tokens_per_step": r["equivalent_tokens_per_step"],
            "full_step_seconds_estimate": r["full_step_seconds_estimate"],
            "cfg0_full_layer": r["cfg0_full_layer"],
            "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse()
    rank, local_rank, world = env_rank()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(_ref_line(args, world)), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    # the CPU sample runs first, before CUDA is touched (spawned workers)
    cpu = None
    if rank == 0 and world == 1 and args.workload == "decode" and not args.no_cpu_baseline:
        cpu = cpu_reference(args.tokens, 2, 1)
    if args.workload == "prefill":
        print(json.dumps(run_prefill(args, local_rank, args.steps, args.warmup,
                                     args.tokens if args.tokens != 64 else None)), flush=True)
        return
    if world > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if args.workload == "ep":
        res = run_ep(args, rank, local_rank, world, "ep", args.steps, args.warmup)
    else:
        res = (run_ep(args, rank, local_rank, world, "decode", args.steps, args.warmup) if world > 1
               else run_decode(args, rank, local_rank, world))
        sub_steps, sub_warm = max(3, min(args.steps, 20)), max(3, min(args.warmup, 5))
        if world == 1 and not args.no_prefill:
            res["prefill"] = run_prefill(args, local_rank, sub_steps, sub_warm)
        if world == 1 and not args.no_dense:
            res["dense"] = run_dense(args, local_rank, sub_steps, sub_warm)
        if not args.no_ep_cfg4:
            res["ep_cfg4"] = run_ep(args, rank, local_rank, world, "ep", sub_steps, sub_warm)
    if cpu is not None:
        res["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu", "nproc")}
        res["cpu_baseline"]["ms_per_step"] = cpu["ms_per_step"]
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

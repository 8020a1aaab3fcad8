"""The reference's CPU path for the routed-expert layer, timed as a baseline.

TEST INFRASTRUCTURE ONLY.  ``bench.py`` runs this for its reference arm
(``--impl reference``) and its ``cpu_baseline`` key; the product never
imports it.

What runs is the reference's eager loop ``apply_exl3_python_loop``
(vcruz305/vllm-exl3 src/vllm_exl3/exl3.py:2357-2413), restated with the same
torch operations: per unique local expert, gather its rows, ``h.half()``,
gate and up projections in fp32, ``F.silu(gate) * up``, the down projection
of ``act.half()``, ``out.index_add_`` of ``down * weight``.  Each projection is
the CPU branch of the reference's ``exl3_gemv`` (csrc/bindings.cpp:144-146):
``x.float() @ dequant_trellis(trellis, suh, svh, K, mcg).float()`` with
``dequant_trellis`` the reference's own C++ (csrc/bindings.cpp:15-132)
compiled CPU-only from its sources into ``oracle/_ref`` (kind "reference");
where that build is absent, the C restatement in ``exl3_oracle.c`` stands in
(kind "port").

Two timings:

* :func:`time_layer_serial` -- one whole layer exactly as the reference
  runs it: experts one after another in one process, the dequant
  single-threaded (as the reference's is), torch matmuls on every host core.
* :class:`ExpertPool` -- the loop body of a sample of experts per step, the
  experts spread over one process per host core (the most parallel the
  reference's CPU code can run: its dequant has no threads of its own).  A
  step's time is its measured wall time; its work, as a fraction of the full
  layer step, is the sampled experts over the batch's distinct experts (the
  per-expert dequant is the cost; the matmuls of a few rows are noise).
"""

from __future__ import annotations

import os
import shutil
import sys
import tempfile
import time

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(_HERE)
_MOD = None


def ref_module():
    """("reference", the compiled reference module) or ("port", cpu_oracle)."""
    global _MOD
    if _MOD is None:
        sys.path.insert(0, os.path.join(_HERE, "_ref"))
        try:
            import vllm_exl3_ref_c
            _MOD = ("reference", vllm_exl3_ref_c)
        except Exception:
            import cpu_oracle
            _MOD = ("port", cpu_oracle)
    return _MOD


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def _dequant(trellis, suh, svh, K: int, cb: int):
    """``dequant_trellis`` -> fp16 torch tensor [in, out]."""
    import torch
    kind, mod = ref_module()
    if kind == "reference":
        # np.array copies the memory-mapped (read-only) arrays into writable ones
        return mod.dequant_trellis(torch.from_numpy(np.array(trellis)), torch.from_numpy(np.array(suh)),
                                   torch.from_numpy(np.array(svh)), int(K), cb == 1)
    return torch.from_numpy(mod.dequant(trellis, suh, svh, int(K), cb=cb))


def _forward(proj: dict, inp):
    """LinearEXL3 forward on CPU, out_dtype fp32 (bindings.cpp:144-146)."""
    w = _dequant(proj["trellis"], proj["suh"], proj["svh"], proj["K"], proj["cb"])
    return inp.half().float() @ w.float()


def expert_body(expert: dict, h, weights):
    """The loop body of one expert (exl3.py:2388-2413), SiLU gate, no clamp:
    returns ``down * weight`` rows [n, H] fp32 (the caller index_adds)."""
    import torch.nn.functional as F
    gate = _forward(expert["gate"], h)
    up = _forward(expert["up"], h)
    act = F.silu(gate) * up
    down = _forward(expert["down"], act)
    return down * weights.unsqueeze(-1)


def _as_dict(p) -> dict:
    return {"trellis": p.trellis, "suh": p.suh, "svh": p.svh, "K": int(p.K), "cb": int(p.codebook)}


def time_layer_serial(pack, x: np.ndarray, ids: np.ndarray, w: np.ndarray, reps: int = 3, threads: int = 0):
    """Median seconds of the whole layer, the reference's serial loop.
    Returns (median, all repetition times)."""
    import torch
    if threads > 0:
        torch.set_num_threads(threads)
    experts = [{k: _as_dict(e[k]) for k in ("gate", "up", "down")} for e in pack.experts]
    xt = torch.from_numpy(np.asarray(x, np.float32))
    idt = torch.from_numpy(np.asarray(ids, np.int64))
    wt = torch.from_numpy(np.asarray(w, np.float32))
    times = []
    for r in range(reps + 1):  # the first is a warm-up
        t0 = time.perf_counter()
        out = torch.zeros(xt.shape[0], xt.shape[1], dtype=torch.float32)
        for e in torch.unique(idt).tolist():
            if not 0 <= e < len(experts):
                continue
            tok, kpos = (idt == e).nonzero(as_tuple=True)
            out.index_add_(0, tok, expert_body(experts[e], xt.index_select(0, tok), wt[tok, kpos]))
        if r:
            times.append(time.perf_counter() - t0)
    return float(np.median(times)), times


# ---------------------------------------------------------------------------
# process pool over experts
# ---------------------------------------------------------------------------
_W: dict = {}


def _worker_init(dirpath: str) -> None:
    import torch
    torch.set_num_threads(1)
    for p in (_HERE, os.path.join(_ROOT, "vllm-exl3_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    _W["dir"] = dirpath
    _W["cache"] = {}
    ref_module()


def _worker_expert(e: int) -> dict:
    if e not in _W["cache"]:
        d = {}
        meta = np.load(os.path.join(_W["dir"], "meta.npy"))
        for which in ("gate", "up", "down"):
            base = os.path.join(_W["dir"], f"e{e}_{which}")
            d[which] = {"trellis": np.load(base + "_t.npy", mmap_mode="r"),
                        "suh": np.load(base + "_u.npy", mmap_mode="r"),
                        "svh": np.load(base + "_v.npy", mmap_mode="r"),
                        "K": int(np.load(base + "_k.npy")), "cb": int(meta[0])}
        _W["cache"][e] = d
    return _W["cache"][e]


def _task(args):
    import torch
    e, x_rows, w_rows = args
    ex = _worker_expert(e)
    t0 = time.perf_counter()
    y = expert_body(ex, torch.from_numpy(x_rows), torch.from_numpy(w_rows))
    return y.numpy(), time.perf_counter() - t0


def _touch(e):
    ex = _worker_expert(e)
    return sum(int(np.asarray(ex[k]["trellis"]).sum() & 1) for k in ex)


class ExpertPool:
    """One spawned process per host core; each step runs the loop body of a
    sample of experts (one task each) and index_adds the rows in the parent."""

    def __init__(self, pack, cores: int | None = None):
        import concurrent.futures as cf
        import multiprocessing as mp
        self.cores = max(1, min(os.cpu_count() or 1, 64) if cores is None else cores)
        self.dir = tempfile.mkdtemp(prefix="exl3_refloop_")
        np.save(os.path.join(self.dir, "meta.npy"), np.array([pack.codebook]))
        for e, ex in enumerate(pack.experts):
            for which in ("gate", "up", "down"):
                p = ex[which]
                base = os.path.join(self.dir, f"e{e}_{which}")
                np.save(base + "_t.npy", p.trellis)
                np.save(base + "_u.npy", p.suh)
                np.save(base + "_v.npy", p.svh)
                np.save(base + "_k.npy", np.array(p.K))
        self.n_experts = pack.n_experts
        self.hidden = pack.hidden
        self.pool = cf.ProcessPoolExecutor(self.cores, mp_context=mp.get_context("spawn"),
                                           initializer=_worker_init, initargs=(self.dir,))
        # map every expert's files in every worker before anything is timed
        list(self.pool.map(_touch, range(self.n_experts), chunksize=1))

    def step(self, x: np.ndarray, ids: np.ndarray, w: np.ndarray, experts: list[int]):
        """Wall seconds of the loop over `experts` (their routes in this batch)."""
        import torch
        t0 = time.perf_counter()
        out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32)
        futs = []
        for e in experts:
            tok, kpos = np.nonzero(ids == e)
            futs.append((tok, self.pool.submit(_task, (int(e), np.ascontiguousarray(x[tok], np.float32),
                                                      np.ascontiguousarray(w[tok, kpos], np.float32)))))
        for tok, f in futs:
            y, _ = f.result()
            out.index_add_(0, torch.from_numpy(tok), torch.from_numpy(y))
        return time.perf_counter() - t0

    def close(self) -> None:
        self.pool.shutdown(wait=True, cancel_futures=True)
        shutil.rmtree(self.dir, ignore_errors=True)


def sampled_steps(pool: ExpertPool, batches, steps: int, warmup: int, per_step: int):
    """Time `warmup` + `steps` steps, each the loop over `per_step` of the
    batch's distinct experts (rotating through them).  Returns a dict with
    the measured step seconds and each step's work as a fraction of the
    whole batch's expert work."""
    times, fracs = [], []
    for s in range(warmup + steps):
        x, ids, w = batches[s % len(batches)]
        distinct = np.unique(ids)
        n = min(per_step, distinct.size)
        start = (s * n) % distinct.size
        pick = [int(distinct[(start + j) % distinct.size]) for j in range(n)]
        dt = pool.step(x, ids, w, pick)
        if s >= warmup:
            times.append(dt)
            fracs.append(n / distinct.size)
    return {"seconds": times, "fractions": fracs}

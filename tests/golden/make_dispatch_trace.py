"""Record the native-module call protocol of the REFERENCE's own dispatch.

Run in the build container, where the reference tree exists:

    python tests/golden/make_dispatch_trace.py [--ref-src <reference checkout>/src]

The reference plugin reaches its native module ``vllm_exl3_c`` through
``apply_exl3_experts`` (src/vllm_exl3/exl3.py:3602-3700), which selects
``_apply_native_fused_moe`` (exl3.py:2783-2885) for decode rows, and through
``apply_exl3_batched_fat`` (exl3.py:2981-3159) for experts with more rows than
the batched path's cap.  This script runs those two reference functions
unmodified, on CPU, with a recording stand-in for ``vllm_exl3_c`` (and for
the ExLlamaV3 extension the fat path also calls) installed in
``sys.modules``, and writes down every native call they make: the function,
and for each argument either its value (scalars, routing rows, activation
rows) or which layer / scratch tensor (and which view of it) was passed.

``tests/test_gpu_reference_dispatch.py`` replays these calls, in order and
with the same arguments, through this repository's ``vllm_exl3_c`` on a GPU
and checks the result against the oracle; ``tests/test_reference_dispatch.py``
checks on CPU that every recorded call binds to this module's signatures.
Outputs: ``dispatch_trace.json`` (calls) and ``dispatch_trace.npz`` (inputs,
and the fat cases' EXL3 tensors).

The reference's native dispatch only runs on CUDA inputs
(``_native_moe_dimensions_supported``, exl3.py:2716-2738); the activations are
given to it as a CPU tensor subclass that reports ``is_cuda``.  Nothing of the
dispatch logic itself is changed.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

PTR_KEYS = ("gate_trellis", "gate_suh", "gate_svh", "up_trellis", "up_suh", "up_svh",
            "down_trellis", "down_suh", "down_svh")

# decode cases for _apply_native_fused_moe: hidden is 4096 (the reference's
# native geometry), intermediate 1024 or 2048, K 2..4, up to 8 rows
NATIVE_CASES = [
    dict(name="k4_i1024", seed=11, rows=4, inter=1024, K=4, n_local=4, topk=4, limit=None, n_global=None),
    dict(name="k2_i2048_limit_emap", seed=12, rows=3, inter=2048, K=2, n_local=4, topk=3, limit=0.75,
         n_global=8),
    dict(name="k3_i1024_rows8", seed=13, rows=8, inter=1024, K=3, n_local=4, topk=2, limit=None, n_global=None),
]
# fat cases for apply_exl3_batched_fat: K4 MCG (the reference's kernel condition)
FAT_CASES = [
    dict(name="fat_k4", seed=21, tokens=40, hidden=384, inter=256, n_experts=3, cap=8, limit=None),
    dict(name="fat_k4_limit", seed=22, tokens=24, hidden=256, inter=384, n_experts=2, cap=4, limit=0.5),
]


def main() -> None:
    ap = argparse.ArgumentParser()
    ref_root = os.environ.get("EXL3_REFERENCE_ROOT", os.path.join(os.path.dirname(ROOT), "reference"))
    ap.add_argument("--ref-src", default=os.path.join(ref_root, "src"))
    args = ap.parse_args()
    sys.path.insert(0, args.ref_src)
    os.environ["VLLM_EXL3_MOE_KERNEL"] = "native"
    import torch

    rec = Recorder(torch)
    sys.modules["vllm_exl3_c"] = rec.native_module()
    from vllm_exl3 import exl3 as ref_exl3

    trace = {"source": "vcruz305/vllm-exl3 src/vllm_exl3/exl3.py (apply_exl3_experts -> "
                       "_apply_native_fused_moe; apply_exl3_batched_fat)",
             "native_abi_version": rec.abi, "cases": []}
    arrays = {}
    for case in NATIVE_CASES:
        trace["cases"].append(native_case(torch, ref_exl3, rec, case, arrays))
    for case in FAT_CASES:
        trace["cases"].append(fat_case(torch, ref_exl3, rec, case, arrays))
    with open(os.path.join(HERE, "dispatch_trace.json"), "w") as f:
        json.dump(trace, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "dispatch_trace.npz"), **arrays)
    print(f"wrote {len(trace['cases'])} cases, {sum(len(c['calls']) for c in trace['cases'])} native calls")


class Recorder:
    """Stand-in modules that record calls; tensors are described by role."""

    def __init__(self, torch):
        self.torch = torch
        self.abi = 4  # the newest ABI the reference checks for (clipping, TP2 widths)
        self.calls = []
        self.named = {}  # storage data_ptr -> (name, base tensor)

    def name(self, name, t):
        self.named[t.untyped_storage().data_ptr()] = (name, t)

    def describe(self, a):
        torch = self.torch
        if isinstance(a, torch.Tensor):
            key = a.untyped_storage().data_ptr()
            d = {"kind": "tensor", "dtype": str(a.dtype).replace("torch.", ""), "shape": list(a.shape),
                 "stride": list(a.stride())}
            if key in self.named:
                name, base = self.named[key]
                d["ref"] = name
                d["offset"] = int(a.storage_offset() - base.storage_offset())
                d["base_shape"] = list(base.shape)
            else:
                d["ref"] = None
            if a.numel() <= 64 and a.dtype in (torch.int32, torch.int64, torch.float16, torch.float32):
                d["values"] = a.detach().reshape(-1).to(torch.float64).tolist()
            return d
        if isinstance(a, bool):
            return {"kind": "bool", "value": a}
        if isinstance(a, int):
            return {"kind": "int", "value": a}
        if isinstance(a, float):
            return {"kind": "float", "value": a}
        if a is None:
            return {"kind": "none"}
        raise TypeError(f"unexpected argument {type(a)}")

    def recorder(self, module, fn):
        def call(*args, **kwargs):
            assert not kwargs, "the reference passes native arguments positionally"
            self.calls.append({"module": module, "fn": fn, "args": [self.describe(a) for a in args]})
            return None
        return call

    def native_module(self):
        m = types.ModuleType("vllm_exl3_c")
        m.P2B_MOE_ABI_VERSION = self.abi
        for fn in ("p2b_fused_moe", "exl3_fat_gemm", "exl3_fat_gemm_scatter"):
            setattr(m, fn, self.recorder("vllm_exl3_c", fn))
        return m

    def exllamav3_module(self):
        m = types.SimpleNamespace()
        for fn in ("had_r_128", "reconstruct", "hgemm"):
            setattr(m, fn, self.recorder("exllamav3_ext", fn))
        return m


def fake_cuda(torch):
    class CudaLooking(torch.Tensor):
        """A CPU tensor that answers ``is_cuda`` (the native geometry check)."""

        @property
        def is_cuda(self):
            return True

    return CudaLooking


def native_case(torch, ref_exl3, rec, c, arrays):
    rng = np.random.default_rng(c["seed"])
    n_global = c["n_global"] or c["n_local"]
    x = rng.standard_normal((c["rows"], 4096), dtype=np.float32)
    logits = rng.standard_normal((c["rows"], n_global)).astype(np.float32)
    ids = np.argsort(-logits, axis=1)[:, :c["topk"]].astype(np.int64)
    w = np.exp(np.take_along_axis(logits, ids, 1))
    w = (w / w.sum(1, keepdims=True)).astype(np.float32)
    xt = torch.from_numpy(x).to(torch.bfloat16).as_subclass(fake_cuda(torch))
    layer = types.SimpleNamespace(
        _exl3_inners=[{} for _ in range(c["n_local"])], _exl3_k=c["K"], _exl3_hidden_size=4096,
        _exl3_intermediate_local=c["inter"],
        _exl3_ptrs={k: torch.arange(c["n_local"], dtype=torch.int64) + 1000 * i for i, k in enumerate(PTR_KEYS)})
    for k in PTR_KEYS:
        rec.name(f"ptr:{k}", layer._exl3_ptrs[k])
    if c["n_global"]:
        # global experts 0..n_global-1; this rank holds every other one
        emap = np.full(n_global, -1, np.int64)
        emap[1::2] = np.arange(c["n_local"])
        layer.expert_map = torch.from_numpy(emap)
    rec.calls = []
    out = ref_exl3.apply_exl3_experts(xt, torch.from_numpy(ids), torch.from_numpy(w), layer, limit=c["limit"])
    assert layer._exl3_last_apply == "native", layer._exl3_last_apply
    key = c["name"]
    arrays[f"{key}/x"] = x
    arrays[f"{key}/ids"] = ids
    arrays[f"{key}/w"] = w
    # activation rows and the output rows are fresh fp16 tensors inside the
    # dispatch: record their contents (x rows) and their row positions
    calls = []
    for r, call in enumerate(rec.calls):
        a = call["args"]
        assert call["fn"] == "p2b_fused_moe"
        for j in (0, 1):
            a[j]["role"] = "x_row" if j == 0 else "out_row"
            a[j]["row"] = r
        calls.append(call)
    rec.calls = []
    return {"kind": "native_fused_moe", "name": key, "config": c, "out_dtype": str(out.dtype).replace("torch.", ""),
            "expert_map": layer.expert_map.tolist() if c["n_global"] else None, "calls": calls}


class Proj:
    """What apply_exl3_batched_fat reads from one EXL3 projection."""

    def __init__(self, torch, rng, in_f, out_f, K=4):
        self.trellis = torch.from_numpy(rng.integers(-32768, 32768, (in_f // 16, out_f // 16, 16 * K),
                                                     dtype=np.int16))
        self.suh = torch.from_numpy(rng.choice([-1.0, 1.0], in_f).astype(np.float16))
        # output signs with a per-tensor scale folded in, ~1/sqrt(in) (the
        # magnitudes of real packs: outputs stay O(1) and fp16-safe)
        scale = rng.uniform(0.5, 1.5) / np.sqrt(in_f)
        self.svh = torch.from_numpy((rng.choice([-1.0, 1.0], out_f) * scale).astype(np.float16))
        self.K, self.mcg, self.mul1 = K, True, False
        self.in_features, self.out_features = in_f, out_f


def fat_case(torch, ref_exl3, rec, c, arrays):
    rng = np.random.default_rng(c["seed"])
    ext = rec.exllamav3_module()
    ref_exl3.load_exllamav3_ext = lambda: ext
    inners = []
    for e in range(c["n_experts"]):
        ex = {"gate": Proj(torch, rng, c["hidden"], c["inter"]), "up": Proj(torch, rng, c["hidden"], c["inter"]),
              "down": Proj(torch, rng, c["inter"], c["hidden"])}
        ex["up"].suh = ex["gate"].suh.clone()  # shared gate/up input sign vector: the packed gate|up GEMM
        for p in ("gate", "up", "down"):
            for f in ("trellis", "suh", "svh"):
                rec.name(f"e{e}.{p}.{f}", getattr(ex[p], f))
        inners.append(ex)
    counts = [int(v) for v in rng.integers(c["cap"] + 1, 2 * c["cap"] + 6, c["n_experts"])]
    counts[-1] = min(counts[-1], c["cap"])  # one expert at or under the cap: skipped by the fat path
    token_sorted = np.concatenate([rng.choice(c["tokens"], n, replace=False) for n in counts]).astype(np.int64)
    # fp16 routing weights and int64 token ids, as apply_exl3_fused_moe passes them (exl3.py:3588-3598)
    weight_sorted = rng.uniform(0.05, 1.0, len(token_sorted)).astype(np.float16)
    xh = torch.from_numpy(rng.standard_normal((c["tokens"], c["hidden"]), dtype=np.float32).astype(np.float16))
    out = torch.zeros(c["tokens"], c["hidden"], dtype=torch.float32)
    ts, ws = torch.from_numpy(token_sorted), torch.from_numpy(weight_sorted)
    rec.name("xh", xh)
    rec.name("out", out)
    rec.name("token_sorted", ts)
    rec.name("weight_sorted", ws)
    ref_exl3._FAT_SCRATCH_CACHE.clear()
    real_scratch = ref_exl3._fat_scratch

    def named_scratch(device, n_rows, gate, up):
        s = real_scratch(device, n_rows, gate, up)
        for k, v in s.items():
            rec.name(f"scratch:{k}", v)
        return s

    ref_exl3._fat_scratch = named_scratch
    rec.calls = []
    try:
        ref_exl3.apply_exl3_batched_fat(xh, ts, ws, counts, inners, c["limit"], c["cap"], out)
    finally:
        ref_exl3._fat_scratch = real_scratch
    key = c["name"]
    for e, ex in enumerate(inners):
        for p in ("gate", "up", "down"):
            for f in ("trellis", "suh", "svh"):
                arrays[f"{key}/e{e}.{p}.{f}"] = getattr(ex[p], f).numpy()
    arrays[f"{key}/xh"] = xh.numpy()
    arrays[f"{key}/token_sorted"] = token_sorted
    arrays[f"{key}/weight_sorted"] = weight_sorted
    calls = rec.calls
    rec.calls = []
    return {"kind": "batched_fat", "name": key, "config": c, "counts": counts, "calls": calls}


if __name__ == "__main__":
    main()

"""GPU replay of the reference plugin's own native calls through this module.

``tests/golden/dispatch_trace.json`` records, call by call, what the
reference's dispatch code passed to its native module when run unmodified
(``tests/golden/make_dispatch_trace.py``; the protocol checks are in
``test_reference_dispatch.py``).  Here every recorded call is made again, in
order, with the recorded scalars, routing rows and views, through this
repository's ``vllm_exl3_c`` on real GPU tensors, and the result is compared
with the oracle's eager loop (src/vllm_exl3/exl3.py:2357-2413, restated in
oracle/cpu_oracle.py):

* ``apply_exl3_experts`` -> ``_apply_native_fused_moe`` (exl3.py:2783-2885):
  one ``p2b_fused_moe`` launch per decode row into a preallocated fp16
  output, hidden 4096, intermediate 1024 / 2048, K 2 / 3 / 4, a SwiGLU clamp,
  and an expert map with non-local routes (clamped ids, zero weights);
* ``apply_exl3_batched_fat`` (exl3.py:2981-3159): per expert over the cap,
  ``had_r_128`` (served by this module, as ExLlamaV3's), ``exl3_fat_gemm``
  into the packed gate|up scratch, and ``exl3_fat_gemm_scatter`` into the
  shared fp32 output.  The torch steps the reference runs between those calls
  (row gather, gate|up packing, clamp, SiLU product, fp16 cast) are restated
  here from exl3.py:3010-3130.

Tolerance (north star): max|d| <= 2e-2 * RMS(reference), cosine >= 0.9995.
"""

import json
import os

import numpy as np
import pytest

import cpu_oracle as oracle
import parity
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TRACE = json.load(open(os.path.join(GOLDEN, "dispatch_trace.json")))
NPZ = np.load(os.path.join(GOLDEN, "dispatch_trace.npz"))
NATIVE = [c["name"] for c in TRACE["cases"] if c["kind"] == "native_fused_moe"]
FAT = [c["name"] for c in TRACE["cases"] if c["kind"] == "batched_fat"]
_DT = {"float16": "float16", "float32": "float32", "int32": "int32", "int64": "int64", "int16": "int16"}


def _case(name):
    return next(c for c in TRACE["cases"] if c["name"] == name)


def _small_tensor(a, cuda):
    import torch
    vals = np.asarray(a["values"], np.float64).astype(_DT[a["dtype"]]).reshape(a["shape"])
    return torch.from_numpy(vals).to(cuda)


@pytest.mark.parametrize("name", NATIVE)
def test_reference_native_fused_moe_replay(native, cuda, name):
    import torch
    import vllm_exl3_c
    from exl3_b200 import moe, synthetic
    c = _case(name)
    cfg = c["config"]
    pack = synthetic.make_moe_pack(500 + cfg["seed"], cfg["n_local"], 4096, cfg["inter"], synthetic.CB_MCG,
                                   (cfg["K"],))
    layer = moe.layer_from_pack(pack, cuda)
    # the reference's input: bf16 activations, converted to fp16 for the launch
    x16 = torch.from_numpy(NPZ[f"{name}/x"]).to(torch.bfloat16).to(torch.float16)
    xh = x16.to(cuda)
    out = torch.full_like(xh, float("nan"))
    ids_rows, w_rows = [], []
    for call in c["calls"]:
        assert call["fn"] == "p2b_fused_moe"
        args = []
        for a in call["args"]:
            if a["kind"] != "tensor":
                args.append(a["value"])
            elif a.get("role") == "x_row":
                args.append(xh[a["row"]:a["row"] + 1])
            elif a.get("role") == "out_row":
                args.append(out[a["row"]:a["row"] + 1])
            elif (a.get("ref") or "").startswith("ptr:"):
                args.append(layer._exl3_ptrs[a["ref"][4:]])
            else:
                args.append(_small_tensor(a, cuda))
        ids_rows.append(np.asarray(call["args"][11]["values"], np.int64))
        w_rows.append(np.asarray(call["args"][12]["values"], np.float32))
        vllm_exl3_c.p2b_fused_moe(*args)
    torch.cuda.synchronize(cuda)
    got = out.float().cpu().numpy()
    limit = c["calls"][0]["args"][18]["value"]
    st = parity.check_moe(got, x16.float().numpy(), np.stack(ids_rows), np.stack(w_rows),
                          lambda e: pack.experts[e], cfg["n_local"], limit=limit if limit > 0 else None)
    assert st["pass"], st


@pytest.mark.parametrize("name", FAT)
def test_reference_batched_fat_replay(native, cuda, name):
    import torch
    import vllm_exl3_c
    c = _case(name)
    cfg = c["config"]
    H, I, cap, limit = cfg["hidden"], cfg["inter"], cfg["cap"], cfg["limit"]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    layer = {k.split("/", 1)[1]: dev(NPZ[k]) for k in NPZ.files if k.startswith(name + "/e")}
    xh = dev(NPZ[f"{name}/xh"])
    ts, ws = dev(NPZ[f"{name}/token_sorted"]), dev(NPZ[f"{name}/weight_sorted"])
    out = torch.zeros(xh.shape[0], H, dtype=torch.float32, device=cuda)
    named = {"xh": xh, "out": out, "token_sorted": ts, "weight_sorted": ws}
    named.update(layer)

    def tensor(a):
        ref = a["ref"]
        if ref.startswith("scratch:") and ref not in named:
            named[ref] = torch.empty(a["base_shape"], dtype=getattr(torch, _DT[a["dtype"]]), device=cuda)
        base = named.get(ref)
        assert base is not None, ref
        return base.reshape(-1).as_strided(a["shape"], a["stride"], a["offset"])

    calls = iter(c["calls"])
    offset = 0
    fat_experts = 0
    for e, n in enumerate(c["counts"]):
        start, offset = offset, offset + n
        if n <= cap:
            continue
        fat_experts += 1
        tok = ts[start:offset]
        # 1. gather the expert's rows, rotate by the shared gate/up suh
        call = next(calls)
        assert (call["module"], call["fn"]) == ("exllamav3_ext", "had_r_128")
        h, h13 = tensor(call["args"][0]), tensor(call["args"][1])
        torch.index_select(xh, 0, tok, out=h)
        assert call["args"][2]["ref"] == f"e{e}.gate.suh"
        vllm_exl3_c.had_r_128(h, h13, layer[f"e{e}.gate.suh"], None, call["args"][4]["value"])
        # 2. gate|up in one fat GEMM over the packed trellis and svh
        call = next(calls)
        assert call["fn"] == "exl3_fat_gemm"
        a = call["args"]
        packed13, gate_up, svh13 = tensor(a[1]), tensor(a[2]), tensor(a[3])
        ot = layer[f"e{e}.gate.trellis"].shape[1]
        packed13[:, :ot].copy_(layer[f"e{e}.gate.trellis"])
        packed13[:, ot:].copy_(layer[f"e{e}.up.trellis"])
        svh13[:I].copy_(layer[f"e{e}.gate.svh"])
        svh13[I:].copy_(layer[f"e{e}.up.svh"])
        vllm_exl3_c.exl3_fat_gemm(tensor(a[0]), packed13, gate_up, svh13, a[4]["value"], a[5]["value"],
                                  a[6]["value"])
        g, u = gate_up[:, :I], gate_up[:, I:]
        if limit is not None and limit > 0:
            g.clamp_(max=limit)
            u.clamp_(min=-limit, max=limit)
        act_h = (torch.sigmoid(g) * g * u).to(torch.float16)
        # 3. down input rotation, then the weighted scatter into the output
        call = next(calls)
        assert (call["module"], call["fn"]) == ("exllamav3_ext", "had_r_128")
        ah, h2 = tensor(call["args"][0]), tensor(call["args"][1])
        ah.copy_(act_h)
        vllm_exl3_c.had_r_128(ah, h2, layer[f"e{e}.down.suh"], None, call["args"][4]["value"])
        call = next(calls)
        assert call["fn"] == "exl3_fat_gemm_scatter"
        a = call["args"]
        assert a[4]["ref"] == "token_sorted" and a[4]["offset"] == start and a[4]["shape"] == [n]
        assert a[5]["ref"] == "weight_sorted" and a[5]["offset"] == start
        vllm_exl3_c.exl3_fat_gemm_scatter(tensor(a[0]), layer[f"e{e}.down.trellis"], out,
                                          layer[f"e{e}.down.svh"], tensor(a[4]), tensor(a[5]), a[6]["value"],
                                          a[7]["value"], a[8]["value"])
    assert next(calls, None) is None, "unreplayed reference calls"
    assert fat_experts >= 1
    torch.cuda.synchronize(cuda)

    # oracle: the same experts and rows through the eager loop's arithmetic
    x = NPZ[f"{name}/xh"].astype(np.float32)
    want = np.zeros_like(out.cpu().numpy())
    offset = 0
    for e, n in enumerate(c["counts"]):
        start, offset = offset, offset + n
        if n <= cap:
            continue
        W = {p: oracle.dequant(NPZ[f"{name}/e{e}.{p}.trellis"], NPZ[f"{name}/e{e}.{p}.suh"],
                               NPZ[f"{name}/e{e}.{p}.svh"], 4, cb=oracle.CB_MCG).astype(np.float32)
             for p in ("gate", "up", "down")}
        rows = NPZ[f"{name}/token_sorted"][start:offset]
        hx = x[rows]
        g, u = hx @ W["gate"], hx @ W["up"]
        if limit is not None and limit > 0:
            g, u = np.minimum(g, limit), np.clip(u, -limit, limit)
        act = (oracle.silu(g) * u).astype(np.float16).astype(np.float32)
        wts = NPZ[f"{name}/weight_sorted"][start:offset].astype(np.float32)
        np.add.at(want, rows, (act @ W["down"]) * wts[:, None])
    st = parity.compare(out.cpu().numpy(), want)
    assert st["pass"], st

"""The reference plugin's own calls into its native module bind to this one.

``tests/golden/dispatch_trace.json`` holds every ``vllm_exl3_c`` call (and
the ExLlamaV3 ``had_r_128`` calls of the fat path) that the reference's
dispatch code made when it was run unmodified with a recording stand-in for
the module (``tests/golden/make_dispatch_trace.py``):
``apply_exl3_experts`` -> ``_apply_native_fused_moe``
(src/vllm_exl3/exl3.py:3602-3700, 2783-2885) and ``apply_exl3_batched_fat``
(exl3.py:2981-3159).  On CPU this checks the protocol: each recorded call
binds to the same-named function of this repository's ``vllm_exl3_c`` with
the same positional arguments, the module advertises an ABI at least as new
as the one the reference asked for, and the routing rows the reference handed
over (its ``map_topk_to_local`` + clamp + zero weight) are what this
repository's host mirror of that mapping produces.  The GPU replay of the
same calls is ``test_gpu_reference_dispatch.py``.
"""

import inspect
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

TRACE = json.load(open(os.path.join(GOLDEN, "dispatch_trace.json")))
NPZ = np.load(os.path.join(GOLDEN, "dispatch_trace.npz"))


def _module():
    import vllm_exl3_c
    return vllm_exl3_c


def _placeholder(a):
    return object() if a["kind"] == "tensor" else a.get("value")


def test_trace_covers_both_reference_paths():
    kinds = {c["kind"] for c in TRACE["cases"]}
    assert kinds == {"native_fused_moe", "batched_fat"}
    fns = {(call["module"], call["fn"]) for c in TRACE["cases"] for call in c["calls"]}
    assert ("vllm_exl3_c", "p2b_fused_moe") in fns
    assert ("vllm_exl3_c", "exl3_fat_gemm") in fns
    assert ("vllm_exl3_c", "exl3_fat_gemm_scatter") in fns


def test_module_abi_is_the_one_the_reference_uses():
    m = _module()
    assert m.P2B_MOE_ABI_VERSION >= TRACE["native_abi_version"]
    assert callable(getattr(m, "p2b_fused_moe", None))  # what _load_native_exl3_ext requires


@pytest.mark.parametrize("case", [c["name"] for c in TRACE["cases"]])
def test_recorded_calls_bind_to_this_module(case):
    m = _module()
    c = next(c for c in TRACE["cases"] if c["name"] == case)
    assert c["calls"], "the reference made no native call"
    for call in c["calls"]:
        if call["module"] == "exllamav3_ext":
            # the fat path's ExLlamaV3 rotations are served by this module's had_r_128
            assert call["fn"] == "had_r_128", f"unexpected ExLlamaV3 call {call['fn']}"
            fn = m.had_r_128
        else:
            fn = getattr(m, call["fn"], None)
        assert fn is not None, call["fn"]
        inspect.signature(fn).bind(*[_placeholder(a) for a in call["args"]])


@pytest.mark.parametrize("case", [c["name"] for c in TRACE["cases"] if c["kind"] == "native_fused_moe"])
def test_reference_routing_rows_match_host_mirror(case):
    """The ids / weights rows the reference passed per launch equal this
    repository's map_topk_to_local with the same clamp-and-zero rule."""
    import torch
    from exl3_b200 import moe
    c = next(c for c in TRACE["cases"] if c["name"] == case)
    cfg = c["config"]
    ids = torch.from_numpy(NPZ[f"{case}/ids"])
    w = torch.from_numpy(NPZ[f"{case}/w"])
    emap = None if c["expert_map"] is None else torch.tensor(c["expert_map"], dtype=torch.long)
    local = moe.map_topk_to_local(ids, cfg["n_local"], emap).reshape(ids.shape)
    valid = (local >= 0) & (local < cfg["n_local"])
    safe_ids = local.clamp(0, cfg["n_local"] - 1).to(torch.int32)
    safe_w = (w.to(torch.float16) * valid.to(torch.float16)).numpy()
    assert len(c["calls"]) == cfg["rows"]
    for r, call in enumerate(c["calls"]):
        a_ids, a_w = call["args"][11], call["args"][12]
        assert a_ids["dtype"] == "int32" and a_w["dtype"] == "float16"
        np.testing.assert_array_equal(np.asarray(a_ids["values"], np.int64), safe_ids[r].numpy())
        np.testing.assert_array_equal(np.asarray(a_w["values"], np.float32), safe_w[r].astype(np.float32))
    if c["expert_map"] is not None:
        assert not valid.all(), "the expert-map case must carry non-local routes"

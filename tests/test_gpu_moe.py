"""GPU parity of the routed-expert MoE forward against the CPU eager loop.

Reference semantics: apply_exl3_python_loop (src/vllm_exl3/exl3.py:2357-2413,
restated in oracle/cpu_oracle.py:moe_eager and pinned there against the
reference's own output fixtures).  Tolerance (north star): max|d| <= 2e-2 *
RMS(ref) and cosine >= 0.9995.  Also: the reference's golden MoE fixtures,
mixed-K, SwiGLU clamp, expert_map sentinels, the padded n_valid contract,
the single-row p2b entries, CUDA-graph replay with changed inputs,
bit-identical repeats, and rejection of bad calls before launch.
"""

import json
import math
import os

import numpy as np
import pytest

import cpu_oracle as oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _close(actual, expected):
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    rms = np.sqrt(np.mean(e * e))
    maxd = np.max(np.abs(a - e))
    cos = float(a @ e / (np.linalg.norm(a) * np.linalg.norm(e) + 1e-30))
    assert np.isfinite(a).all()
    assert maxd <= 2e-2 * rms, f"max|d| {maxd:.3e} > 2e-2 * rms {rms:.3e}"
    assert cos >= 0.9995, f"cosine {cos}"


def _dense(pack):
    return [{w: None if e.get(w) is None else oracle.dequant(e[w].trellis, e[w].suh, e[w].svh, e[w].K,
                                                             cb=e[w].codebook)
             for w in ("gate", "up", "down")} for e in pack.experts]


def _setup(cuda, name, seed=0, **over):
    from exl3_b200 import synthetic, moe
    pack, x, ids, w = synthetic.make_config(name, seed=seed, **over)
    layer = moe.layer_from_pack(pack, cuda)
    return pack, layer, x, ids, w


def _run(layer, cuda, x, ids, w, dtype=None, **kw):
    import torch
    xt = torch.from_numpy(x).to(cuda)
    if dtype is not None:
        xt = xt.to(dtype)
    out = layer.apply(xt, torch.from_numpy(w).to(cuda), torch.from_numpy(ids).to(cuda), **kw)
    return out.float().cpu().numpy()


def test_cfg1_layer_matches_eager_loop(native, cuda):
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg1")
    want = oracle.moe_eager(x, ids, w, _dense(pack))
    got = _run(layer, cuda, x, ids, w, dtype=torch.float32)
    _close(got, want)
    got_bf16 = _run(layer, cuda, x, ids, w, dtype=torch.bfloat16)
    _close(got_bf16, want)


@pytest.mark.parametrize("tokens", [1, 8, 33])
def test_decode_config_shape_matches_eager_loop(native, cuda, tokens):
    import torch
    # cfg2 geometry (H 2048, I 768, top-8, K4 MCG) with fewer experts to keep the oracle fast
    pack, layer, x, ids, w = _setup(cuda, "cfg2", seed=tokens, tokens=tokens, n_experts=24)
    want = oracle.moe_eager(x, ids, w, _dense(pack))
    _close(_run(layer, cuda, x, ids, w, dtype=torch.float32), want)


@pytest.mark.parametrize("tokens", [96, 300])
def test_prefill_gemm_path_uniform_k(native, cuda, tokens):
    """>= 32 routes per expert: the tcgen05 grouped GEMM path."""
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg2", seed=40 + tokens, tokens=tokens, n_experts=16,
                                    hidden=512, inter=256)
    want = oracle.moe_eager(x, ids, w, _dense(pack))
    _close(_run(layer, cuda, x, ids, w, dtype=torch.float32), want)


@pytest.mark.parametrize("tokens", [512, 700])
def test_prefill_gemm_256_row_tiles(native, cuda, tokens):
    """>= 192 routes per expert: 256-row work tiles (two TMEM accumulators
    sharing every decoded weight tile), including tiles whose second half is
    partly or wholly empty."""
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg2", seed=90 + tokens, tokens=tokens, n_experts=16,
                                    hidden=512, inter=384, k_choices=(2, 3, 4), k_probs=None)
    want = oracle.moe_eager(x, ids, w, _dense(pack))
    _close(_run(layer, cuda, x, ids, w, dtype=torch.float32), want)
    # bf16 activations in, fp32 rows out (a bf16 output would add half a bf16
    # ulp of rounding, above 2e-2 RMS for the largest outputs of this shape)
    f32 = torch.empty(x.shape[0], x.shape[1], dtype=torch.float32, device=cuda)
    _close(_run(layer, cuda, x, ids, w, dtype=torch.bfloat16, out=f32), want)


@pytest.mark.parametrize("n_valid", [None, 1030])
def test_large_batch_split_prep(native, cuda, n_valid):
    """>= 8192 routes: the routing prep runs as chunk histograms, a one-CTA
    layout pass and a chunked placement; the result must equal the
    eager loop, including the padded n_valid rows."""
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg2", seed=123, tokens=1100, n_experts=16, hidden=256,
                                    inter=256, k_choices=(2, 3), k_probs=None)
    want = oracle.moe_eager(x, ids, w, _dense(pack))
    kw = {}
    if n_valid is not None:
        kw["n_valid"] = torch.tensor([n_valid], dtype=torch.int32, device=cuda)
        want[n_valid:] = 0.0
    f32 = torch.empty(x.shape[0], x.shape[1], dtype=torch.float32, device=cuda)
    got = _run(layer, cuda, x, ids, w, dtype=torch.bfloat16, out=f32, **kw)
    if n_valid is not None:
        assert np.all(got[n_valid:] == 0)
    _close(got, want)


@pytest.mark.parametrize("n_experts", [6, 3])
def test_prefill_gemm_split_k(native, cuda, n_experts):
    """Few (tile, column block) items: each is split over K across up to four
    CTAs whose fp32 partials the last one sums in split order before the
    epilogue (gate rows, the fused up + SwiGLU epilogue and the weighted down
    rows all run split).  Repeats must be bit-identical."""
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg2", seed=55 + n_experts, tokens=16 * n_experts, n_experts=n_experts,
                                    topk=2, hidden=2048, inter=1024, k_choices=(2, 3, 4), k_probs=None)
    want = oracle.moe_eager(x, ids, w, _dense(pack))
    got = _run(layer, cuda, x, ids, w, dtype=torch.float32)
    _close(got, want)
    assert np.array_equal(got, _run(layer, cuda, x, ids, w, dtype=torch.float32))


def test_prefill_gemm_path_mixed_k_mul1_limit(native, cuda):
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg3", seed=77, tokens=256, n_experts=10, hidden=384,
                                    inter=256, k_choices=(2, 3, 4), k_probs=None)
    dense = _dense(pack)
    for limit in (None, 0.75):
        want = oracle.moe_eager(x, ids, w, dense, limit=limit)
        _close(_run(layer, cuda, x, ids, w, dtype=torch.float32, limit=limit), want)


def test_mixed_k_mul1_with_limit(native, cuda):
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg3", seed=5, tokens=24, n_experts=12, hidden=512,
                                    inter=384, k_choices=(2, 3, 4, 5), k_probs=None)
    dense = _dense(pack)
    for limit in (None, 0.75):
        want = oracle.moe_eager(x, ids, w, dense, limit=limit)
        _close(_run(layer, cuda, x, ids, w, dtype=torch.float32, limit=limit), want)


def test_reference_golden_fixtures(native, cuda):
    """The reference eager loop's outputs (tests/golden/moe.npz) directly."""
    import torch
    from exl3_b200 import moe
    data = np.load(os.path.join(GOLDEN, "moe.npz"))
    with open(os.path.join(GOLDEN, "moe_cases.json")) as f:
        metas = json.load(f)
    for meta in metas:
        name = meta["name"]
        cb = 1 if meta["mcg"] else 2
        inners = []
        for e in range(meta["E"]):
            inners.append({wh: moe.Exl3Projection(
                torch.from_numpy(data[f"{name}_e{e}_{wh}_trellis"]).to(cuda),
                torch.from_numpy(data[f"{name}_e{e}_{wh}_suh"]).to(cuda),
                torch.from_numpy(data[f"{name}_e{e}_{wh}_svh"]).to(cuda), cb)
                for wh in ("gate", "up", "down")})
        emap = torch.from_numpy(data[f"{name}_expert_map"]) if meta["expert_map"] else None
        layer = moe.Exl3RoutedExperts(inners, meta["H"], meta["I"], expert_map=emap)
        got = _run(layer, cuda, data[f"{name}_x"], data[f"{name}_ids"], data[f"{name}_w"],
                   dtype=torch.float32, limit=meta["limit"])
        _close(got, data[f"{name}_out"])


def test_expert_map_and_sentinels(native, cuda):
    import torch
    from exl3_b200 import moe
    pack, _, x, ids, w = _setup(cuda, "cfg1", seed=11)
    # this rank owns global experts 8..15 as local 0..7; 0..7 live elsewhere
    emap = np.full(16, -1, dtype=np.int64)
    emap[8:] = np.arange(8)
    layer = moe.layer_from_pack(pack, cuda, expert_map=torch.from_numpy(emap))
    ids2 = ids.copy() + 8
    ids2[0, 0] = 3          # non-local
    ids2[1, 1] = -1         # invalid
    ids2[2, 0] = 99         # out of range
    want = oracle.moe_eager(x, ids2, w, _dense(pack), expert_map=emap)
    _close(_run(layer, cuda, x, ids2, w, dtype=torch.float32), want)


def test_padded_n_valid_rows_are_zero(native, cuda):
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg1", seed=3)
    n_valid = torch.tensor([5], dtype=torch.int32, device=cuda)
    got = _run(layer, cuda, x, ids, w, dtype=torch.float32, n_valid=n_valid)
    want = oracle.moe_eager(x[:5], ids[:5], w[:5], _dense(pack))
    _close(got[:5], want)
    assert np.all(got[5:] == 0.0)


def test_p2b_single_row_entries(native, cuda):
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg1", seed=4)
    dense = _dense(pack)
    p = layer._exl3_ptrs
    tables = [p[k] for k in ("gate_trellis", "gate_suh", "gate_svh", "up_trellis", "up_suh", "up_svh",
                             "down_trellis", "down_suh", "down_svh")]
    row = torch.from_numpy(x[:1]).to(cuda).half()
    ids_r = torch.from_numpy(ids[0]).to(cuda).int()
    w_r = torch.from_numpy(w[0]).to(cuda).half()
    want = oracle.moe_eager(x[:1], ids[:1], w_r.float().cpu().numpy()[None], dense)
    out = torch.empty_like(row)
    native.p2b_fused_moe(row, out, *tables, ids_r, w_r, 4, 4, 4, True, 512, 0.0)
    _close(out.float().cpu().numpy(), want)
    kt = torch.full((8,), 4, dtype=torch.int8, device=cuda)
    out2 = torch.empty_like(row)
    native.p2b_fused_moe_mk(row, out2, *tables, ids_r, w_r, kt, kt, kt, 8, True, 512, 0.0)
    _close(out2.float().cpu().numpy(), want)
    # padded grid: [MAX_T=4, k] with 2 live rows
    xs = torch.from_numpy(x[:4]).to(cuda).half()
    idp = torch.from_numpy(ids[:4]).to(cuda).int()
    wp = torch.from_numpy(w[:4]).to(cuda).half()
    outp = torch.empty_like(xs)
    nv = torch.tensor([2], dtype=torch.int32, device=cuda)
    native.p2b_fused_moe_padded(xs, outp, *tables, idp, wp, nv, kt, kt, kt, 8, 2, True, 512, 0.0)
    wantp = oracle.moe_eager(x[:2], ids[:2], wp.float().cpu().numpy()[:2], dense)
    _close(outp[:2].float().cpu().numpy(), wantp)
    assert torch.all(outp[2:] == 0)


@pytest.mark.parametrize("bad", ["rows", "width", "negative_limit", "nan_limit", "strided_pointers"])
def test_rejects_unsafe_calls_before_launch(native, cuda, bad):
    import torch
    x = torch.zeros(1, 4096, dtype=torch.float16, device=cuda)
    out = torch.empty_like(x)
    ptrs = [torch.zeros(2, dtype=torch.int64, device=cuda) for _ in range(9)]  # null pointees
    ids = torch.zeros(1, dtype=torch.int32, device=cuda)
    weights = torch.ones(1, dtype=torch.float16, device=cuda)
    width, limit = 2048, 0.0
    if bad == "rows":
        x = x.repeat(2, 1)
    elif bad == "width":
        width = 1537
    elif bad == "negative_limit":
        limit = -1.0
    elif bad == "nan_limit":
        limit = math.nan
    else:
        ptrs[0] = torch.zeros(4, dtype=torch.int64, device=cuda)[::2]
    with pytest.raises(RuntimeError, match="fused MoE"):
        native.p2b_fused_moe(x, out, *ptrs, ids, weights, 4, 4, 4, True, width, limit)


def test_null_pointer_tables_flag_status_not_fault(native, cuda):
    """Null pointees inside valid tables: kernels skip and record a status."""
    import torch
    native.device_status(clear=True)
    x = torch.zeros(2, 256, dtype=torch.float16, device=cuda)
    out = torch.empty_like(x)
    ptrs = [torch.zeros(2, dtype=torch.int64, device=cuda) for _ in range(9)]
    ids = torch.zeros(2, 1, dtype=torch.int32, device=cuda)
    w = torch.ones(2, 1, dtype=torch.float16, device=cuda)
    native.exl3_moe(x, out, *ptrs, ids, w, K=4, intermediate_size=128)
    torch.cuda.synchronize()
    assert native.device_status(clear=True) != 0


def test_graph_replay_consumes_new_inputs_and_is_deterministic(native, cuda):
    import torch
    pack, layer, x, ids, w = _setup(cuda, "cfg1", seed=8)
    dense = _dense(pack)
    xt = torch.from_numpy(x).to(cuda)
    wt = torch.from_numpy(w).to(cuda)
    it = torch.from_numpy(ids).to(cuda)
    out = torch.empty_like(xt)
    layer.apply(xt, wt, it, out=out)
    first = out.clone()
    layer.apply(xt, wt, it, out=out)
    assert torch.equal(first, out), "repeat runs must be bit-identical"
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            layer.apply(xt, wt, it, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.apply(xt, wt, it, out=out)
    rng = np.random.default_rng(99)
    for _ in range(2):
        x2 = rng.normal(0, 1, x.shape).astype(np.float32)
        ids2 = np.stack([rng.choice(8, 2, replace=False) for _ in range(x.shape[0])]).astype(np.int64)
        xt.copy_(torch.from_numpy(x2))
        it.copy_(torch.from_numpy(ids2))
        g.replay()
        torch.cuda.synchronize()
        _close(out.cpu().numpy(), oracle.moe_eager(x2, ids2, w, dense))
    del g


def test_graph_survives_workspace_growth(native, cuda):
    """A graph captured with a cached workspace keeps its results after a
    larger eager call on the same stream has grown the workspace, and its
    replay writes into no memory the allocator has since given to other
    tensors (the replaced workspace stays allocated)."""
    import torch
    from exl3_b200 import synthetic
    pack, layer, x, ids, w = _setup(cuda, "cfg1", seed=21, tokens=4)
    dense = _dense(pack)
    s = torch.cuda.Stream(cuda)
    xt, wt, it = (torch.from_numpy(a).to(cuda) for a in (x, w, ids))
    out = torch.empty_like(xt)
    with torch.cuda.stream(s):
        for _ in range(2):  # warm-up: sizes this stream's workspace for the captured shape
            layer.apply(xt, wt, it, out=out)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        layer.apply(xt, wt, it, out=out)
    # 600 tokens (the tensor-core GEMM path) need a far larger workspace
    rng = np.random.default_rng(22)
    xb = synthetic.activations(rng, 600, 1024)
    idb, wb = synthetic.softmax_topk(rng, 600, 8, 2)
    with torch.cuda.stream(s):
        big = layer.apply(torch.from_numpy(xb).to(cuda), torch.from_numpy(wb).to(cuda),
                          torch.from_numpy(idb).to(cuda))
    s.synchronize()
    _close(big.cpu().numpy(), oracle.moe_eager(xb, idb, wb, dense))
    # unrelated tensors take whatever the allocator has free now
    fillers = [torch.full((1 << 18,), 7.0, device=cuda) for _ in range(64)]
    x2 = np.random.default_rng(23).normal(0, 1, x.shape).astype(np.float32)
    xt.copy_(torch.from_numpy(x2))
    with torch.cuda.stream(s):
        g.replay()
    s.synchronize()
    _close(out.cpu().numpy(), oracle.moe_eager(x2, ids, w, dense))
    assert all(bool(torch.all(f == 7.0)) for f in fillers), "graph replay wrote into freed memory"
    del g


@pytest.mark.parametrize("tokens", [6, 160])
@pytest.mark.parametrize("limit", [None, 0.75])
def test_swiglu_oai_activation(native, cuda, tokens, limit):
    """Clamped SwiGLU-OAI (exl3.py:2392-2402: (up + 1) * gate * sigmoid(1.702
    gate), gate clamped from above, up on both sides) on the decode GEMV
    (6 tokens) and the tcgen05 GEMM path (160 tokens: >= 32 rows per expert)."""
    import torch
    from exl3_b200 import _native, moe, synthetic
    pack, x, ids, w = synthetic.make_config("cfg2", seed=300 + tokens, tokens=tokens, n_experts=8, topk=2,
                                            hidden=512, inter=256, k_choices=(2, 3, 4), k_probs=None)
    layer = moe.layer_from_pack(pack, cuda, act=_native.ACT_SWIGLU_OAI)
    want = oracle.moe_eager(x, ids, w, _dense(pack), limit=limit, act="swiglu_oai")
    _close(_run(layer, cuda, x, ids, w, dtype=torch.float32, limit=limit), want)


@pytest.mark.parametrize("tokens", [6, 160])
@pytest.mark.parametrize("cb", [1, 2])
def test_gateless_relu2_layer(native, cuda, tokens, cb):
    """Non-gated relu^2 layer (exl3.py:2386-2391, NemotronH): experts carry no
    gate projection, the fused state aliases the up tables into the gate
    slots, and both paths compute relu(clamp(up))^2 without a gate GEMM."""
    import torch
    from exl3_b200 import _native, moe, synthetic
    pack, x, ids, w = synthetic.make_config("cfg2", seed=400 + tokens + cb, tokens=tokens, n_experts=8, topk=2,
                                            hidden=512, inter=384, codebook=cb, k_choices=(2, 3, 4),
                                            k_probs=None, gateless=True)
    layer = moe.layer_from_pack(pack, cuda)
    assert layer._exl3_gateless and layer._exl3_moe_act == _native.ACT_RELU2
    assert torch.equal(layer._exl3_ptrs["gate_trellis"], layer._exl3_ptrs["up_trellis"])
    dense = _dense(pack)
    for limit in (None, 0.5):
        want = oracle.moe_eager(x, ids, w, dense, limit=limit)
        _close(_run(layer, cuda, x, ids, w, dtype=torch.float32, limit=limit), want)


@pytest.mark.parametrize("gateless", [False, True])
def test_layer_loaded_from_safetensors(native, cuda, tmp_path, gateless):
    """A layer built by the safetensors loader (per-expert keys, markers,
    mixed K per expert) runs on the GPU and matches the eager loop."""
    import torch
    from exl3_b200 import loader, synthetic
    pack, x, ids, w = synthetic.make_config("cfg2", seed=500 + gateless, tokens=12, n_experts=8, topk=2,
                                            hidden=512, inter=256, k_choices=(2, 3, 4), k_probs=None,
                                            gateless=gateless)
    path = str(tmp_path / "pack.safetensors")
    loader.save_routed_experts(path, "model.layers.0.mlp", pack.experts)
    layer = loader.load_routed_experts(path, "model.layers.0.mlp", 8, 512, 256, cuda)
    assert layer._exl3_gateless == gateless
    want = oracle.moe_eager(x, ids, w, _dense(pack))
    _close(_run(layer, cuda, x, ids, w, dtype=torch.float32), want)

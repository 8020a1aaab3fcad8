"""GPU parity at the BASELINE configurations' real shapes.

Every benchmarked configuration is run at full size on the GPU and its
outputs are checked against the CPU eager loop (apply_exl3_python_loop,
src/vllm_exl3/exl3.py:2357-2413, restated in oracle/cpu_oracle.py) with the
reference's own dequant arithmetic (oracle/exl3_oracle.c, pinned to the
reference's compiled csrc/bindings.cpp).  Where the whole output would take
the CPU too long, a seeded subsample of tokens (rows) and of 128-column output
blocks is compared; each row depends only on its own token and each output
block only on its own tiles, so the subsample is exactly that part of the
full result (oracle/parity.py).

* configs[1] decode: 128 experts, top-8, H 2048, I 768, K4 MCG, T in
  {1, 8, 32, 64}, every token and column, eager and as a CUDA-graph replay;
  this also pins the decode GEMV (which multiplies by the unrounded MCG
  codebook sum) against the rounded fp16 weights;
* configs[2] mixed-K prefill: 160 experts, H 5120, I 1536, K2/3 mul1, T in
  {2048, 8192} (128- and 256-row GEMM tiles), 16 sampled tokens;
* configs[3] dense linear: 8192x28672 then 28672x8192, K3 MCG, M in {1, 16,
  256, 4096}, up to 32 sampled rows x 4 column blocks;
* configs[4] expert-parallel layer on one GPU: 256 experts, top-8
  sigmoid+Zipf, H 7168, I 2048, K2/3/4 MCG, T = 8192, 8 sampled tokens x 6
  column blocks; and the NVLink EP step of G in {2, 4, 8} ranks emulated on
  one GPU, against the single-GPU layer on every token and the oracle on a
  sample.

Tolerance (north star): max|d| <= 2e-2 * RMS(reference), cosine >= 0.9995.
"""

import numpy as np
import pytest

import ep_helpers
import parity

pytestmark = pytest.mark.gpu


def _to(cuda, *arrays):
    import torch
    return [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in arrays]


# ---------------------------------------------------------------------------
# decode GEMV layer
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg2_layer(cuda):
    from exl3_b200 import moe, synthetic
    pack = synthetic.make_moe_pack(0, 128, 2048, 768, synthetic.CB_MCG, (4,))
    return pack, moe.layer_from_pack(pack, cuda)


@pytest.mark.parametrize("tokens", [1, 8, 32, 64])
def test_cfg2_decode_full_shape(native, cuda, cfg2_layer, tokens):
    import torch
    from exl3_b200 import synthetic
    pack, layer = cfg2_layer
    rng = np.random.default_rng(7000 + tokens)
    x = synthetic.activations(rng, tokens, 2048)
    ids, w = synthetic.softmax_topk(rng, tokens, 128, 8)
    xt, idt, wt = _to(cuda, x, ids, w)
    xb = xt.to(torch.bfloat16)
    out = torch.empty(tokens, 2048, dtype=torch.float32, device=cuda)
    layer.apply(xb, wt, idt, out=out)
    got = out.cpu().numpy()
    st = parity.check_moe(got, xb.float().cpu().numpy(), ids, w, lambda e: pack.experts[e], 128)
    assert st["pass"], st
    # the same step as a CUDA-graph replay (how the benchmark runs it)
    s = torch.cuda.Stream(cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(s):
        layer.apply(xb, wt, idt, out=out)
    torch.cuda.current_stream(cuda).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.apply(xb, wt, idt, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize(cuda)
    assert np.array_equal(out.cpu().numpy(), got), "graph replay differs from the eager call"
    del g


# ---------------------------------------------------------------------------
# mixed-K prefill (tcgen05 grouped GEMM)
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg3_layer(cuda):
    from exl3_b200 import moe, synthetic
    pack = synthetic.make_moe_pack(0, 160, 5120, 1536, synthetic.CB_MUL1, (2, 3), (0.5, 0.5))
    return pack, moe.layer_from_pack(pack, cuda)


@pytest.mark.parametrize("tokens", [2048, 8192])
def test_cfg3_prefill_full_shape(native, cuda, cfg3_layer, tokens):
    import torch
    from exl3_b200 import synthetic
    pack, layer = cfg3_layer
    rng = np.random.default_rng(8000 + tokens)
    x = synthetic.activations(rng, tokens, 5120)
    ids, w = synthetic.softmax_topk(rng, tokens, 160, 8, 1.5)
    xt, idt, wt = _to(cuda, x, ids, w)
    xb = xt.to(torch.bfloat16)
    out = torch.empty(tokens, 5120, dtype=torch.float32, device=cuda)
    layer.apply(xb, wt, idt, out=out)
    torch.cuda.synchronize(cuda)
    sel = parity.sample_tokens(tokens, 16, seed=tokens)
    got = out[torch.from_numpy(sel).to(cuda)].cpu().numpy()
    st = parity.check_moe(got, xb.float().cpu().numpy()[sel], ids[sel], w[sel], lambda e: pack.experts[e], 160)
    assert st["pass"], st


# ---------------------------------------------------------------------------
# dense EXL3 linear, MLP-sized
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg4_projections(cuda):
    from exl3_b200 import synthetic
    rng = np.random.default_rng(4)
    p1 = synthetic.make_projection(rng, 8192, 28672, 3, synthetic.CB_MCG)
    p2 = synthetic.make_projection(rng, 28672, 8192, 3, synthetic.CB_MCG)
    return [(p, _to(cuda, p.trellis, p.suh, p.svh)) for p in (p1, p2)]


@pytest.mark.parametrize("m", [1, 16, 256, 4096])
def test_cfg4_dense_linear_full_shape(native, cuda, cfg4_projections, m):
    import torch
    for j, (p, (dt, du, dv)) in enumerate(cfg4_projections):
        rng = np.random.default_rng(9000 + 10 * m + j)
        x = rng.normal(0, 1, (m, p.in_features)).astype(np.float32)
        xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
        y = native.exl3_linear(xt, dt, du, dv, 3, 1, out_dtype=torch.float32)
        torch.cuda.synchronize(cuda)
        rows = parity.sample_tokens(m, 32, seed=m + j)
        blocks = parity.col_blocks(p.out_features, 4, seed=m + j)
        w = parity.projection_dense(p, blocks).astype(np.float32)
        want = xt.float().cpu().numpy()[rows].astype(np.float16).astype(np.float32) @ w
        got = y.cpu().numpy()[rows]
        got = np.concatenate([got[:, 128 * b:128 * (b + 1)] for b in blocks], axis=1)
        parity.assert_close(got, want)


# ---------------------------------------------------------------------------
# the expert-parallel layer's shape on one GPU, and its EP step
# ---------------------------------------------------------------------------
CFG5 = dict(E=256, H=7168, I=2048, topk=8, ks=(2, 3, 4), kp=(0.3, 0.5, 0.2), T=8192)


def _cfg5_expert(e):
    from exl3_b200 import synthetic
    c = CFG5
    return synthetic.make_moe_pack_slice(0, c["E"], c["H"], c["I"], synthetic.CB_MCG, c["ks"], c["kp"],
                                         e, e + 1).experts[0]


@pytest.fixture(scope="module")
def cfg5_layer(cuda):
    from exl3_b200 import moe, synthetic
    c = CFG5

    def make(lo, hi):
        return synthetic.make_moe_pack_slice(0, c["E"], c["H"], c["I"], synthetic.CB_MCG, c["ks"], c["kp"], lo, hi)

    return moe.layer_from_slices(make, c["E"], c["H"], c["I"], cuda)


def _cfg5_batch(cuda):
    import torch
    from exl3_b200 import synthetic
    c = CFG5
    rng = np.random.default_rng(900)
    ids, w = synthetic.sigmoid_zipf_topk(rng, c["T"], c["E"], c["topk"])
    x = synthetic.activations(np.random.default_rng(901), c["T"], c["H"])
    xt, idt, wt = _to(cuda, x, ids, w)
    return xt.to(torch.bfloat16), idt, wt, ids, w


def test_cfg5_layer_one_gpu_full_shape(native, cuda, cfg5_layer):
    import torch
    c = CFG5
    xb, idt, wt, ids, w = _cfg5_batch(cuda)
    out = torch.empty(c["T"], c["H"], dtype=torch.float32, device=cuda)
    cfg5_layer.apply(xb, wt, idt, out=out)
    torch.cuda.synchronize(cuda)
    sel = parity.sample_tokens(c["T"], 8, seed=5)
    blocks = parity.col_blocks(c["H"], 6, seed=5)
    got = out[torch.from_numpy(sel).to(cuda)].cpu().numpy()
    st = parity.check_moe(got, xb.float().cpu().numpy()[sel], ids[sel], w[sel], _cfg5_expert, c["E"], blocks)
    assert st["pass"], st


@pytest.mark.parametrize("G", [2, 4, 8])
def test_cfg5_ep_step_emulated_ranks_full_shape(native, cuda, cfg5_layer, G):
    """G ranks' NVLink EP step (window stores, flags, local forward, return,
    combine) emulated on one GPU at the full configs[4] shape: every token
    against the single-GPU layer, a sample against the oracle."""
    import torch
    from exl3_b200.ep import NvlinkEpWindow
    from exl3_b200.moe import Exl3RoutedExperts
    c = CFG5
    xb, idt, wt, ids, w = _cfg5_batch(cuda)
    epr, C = c["E"] // G, c["T"] // G
    inners = cfg5_layer._exl3_inners
    layers = [Exl3RoutedExperts(inners[r * epr:(r + 1) * epr], c["H"], c["I"]) for r in range(G)]
    wins = [NvlinkEpWindow(G, r, C, c["H"], c["topk"], torch.bfloat16, torch.float32, cuda, exchange=False)
            for r in range(G)]
    addrs = [wn.window for wn in wins]
    for wn in wins:
        wn.set_peers(addrs)
    try:
        got = ep_helpers.nvlink_emulated_step(layers, wins, xb, idt, wt, c["E"], G, C, torch.float32)
        single = torch.empty(c["T"], c["H"], dtype=torch.float32, device=cuda)
        cfg5_layer.apply(xb, wt, idt, out=single)
        torch.cuda.synchronize(cuda)
        parity.assert_close(got.cpu().numpy(), single.cpu().numpy())
        sel = parity.sample_tokens(c["T"], 4, seed=G)
        blocks = parity.col_blocks(c["H"], 4, seed=G)
        st = parity.check_moe(got[torch.from_numpy(sel).to(cuda)].cpu().numpy(), xb.float().cpu().numpy()[sel],
                              ids[sel], w[sel], _cfg5_expert, c["E"], blocks)
        assert st["pass"], st
        assert all(wn.status() == 0 for wn in wins)
    finally:
        for wn in wins:
            wn.close()

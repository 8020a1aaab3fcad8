"""Expert parallelism: exchange logic on gloo ranks (CPU) and the native
dispatch / combine kernels plus an emulated multi-rank step (GPU).

The reference has no EP code of its own (it consumes vLLM's expert_map,
src/vllm_exl3/exl3.py:2310-2354); the oracle for an EP layer is the
single-rank eager loop over all experts (exl3.py:2357-2413), so a G-rank
step must reproduce it within the layer tolerance.
"""

import socket

import numpy as np
import pytest

import cpu_oracle as oracle
import ep_helpers


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(worker, world: int, cfg: dict, timeout: float) -> list:
    """Spawn `world` ranks of `worker` and collect their results.  The queue is
    drained before the join: a child whose queued result is larger than the
    pipe buffer cannot exit until the parent reads it."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = mp.start_processes(worker, args=(world, _free_port(), cfg, q), nprocs=world, join=False,
                               start_method="spawn")
    out = [q.get(timeout=timeout) for _ in range(world)]
    while not procs.join(timeout=timeout):
        pass
    return out


def _close(got: np.ndarray, want: np.ndarray, rel: float = 2e-2, cos_min: float = 0.9995) -> None:
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    err = float(np.max(np.abs(got.astype(np.float64) - want)))
    assert err <= rel * rms, (err, rms)
    den = np.linalg.norm(got) * np.linalg.norm(want)
    if den > 0:
        assert float(np.dot(got.ravel(), want.ravel()) / den) >= cos_min


# ---------------------------------------------------------------------------
# CPU: gloo ranks, exchange logic with CPU stand-ins for the kernels
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n_valid,capacity,placement", [
    (None, None, None), (7, None, None), (None, 12, None), (5, 16, None),
    (None, None, [5, 0, 7, 2, 1, 6, 3, 4]), (6, 12, [1, 2, 3, 4, 5, 6, 7, 0])])
def test_ep_gloo_world2_matches_single_rank(n_valid, capacity, placement):
    from exl3_b200 import synthetic

    cfg = dict(seed=11, E=8, H=256, I=128, topk=2, T=12, n_valid=n_valid, capacity=capacity,
               placement=placement)
    world = 2
    got, counts = {}, {}
    for r, y, c in _run_ranks(ep_helpers.gloo_worker, world, cfg, 60):
        got[r] = y
        counts[r] = c
    pack = synthetic.make_moe_pack(cfg["seed"], cfg["E"], cfg["H"], cfg["I"], synthetic.CB_MCG, (4,))
    dense = ep_helpers.dense_experts(pack, 0, cfg["E"])
    rng = np.random.default_rng(cfg["seed"] + 7)
    x = synthetic.activations(rng, cfg["T"] * world, cfg["H"])
    ids, w = synthetic.softmax_topk(rng, cfg["T"] * world, cfg["E"], cfg["topk"])
    ids[::5, 0] = -1
    for r in range(world):
        sl = slice(r * cfg["T"], (r + 1) * cfg["T"])
        want = oracle.moe_eager(x[sl], ids[sl], w[sl], dense)
        if n_valid is not None:
            want[n_valid:] = 0.0
        np.testing.assert_allclose(got[r], want, rtol=1e-5, atol=1e-5 * float(np.abs(want).max() + 1))
    # what rank r sends to q is what q receives from r
    if capacity is None:
        for r in range(world):
            for qq in range(world):
                assert counts[r][0][qq] == counts[qq][1][r]


def test_ep_cpu_dispatch_contract():
    """The stand-in keeps the documented layout: rank-major, token-ascending."""
    import torch
    rng = np.random.default_rng(3)
    T, H, E, topk, G = 20, 128, 12, 3, 3
    x = torch.from_numpy(rng.normal(size=(T, H)).astype(np.float32))
    ids = torch.from_numpy(rng.integers(-2, E + 2, size=(T, topk)))
    w = torch.from_numpy(rng.random((T, topk)).astype(np.float32))
    sx, sid, sw, stok, pidx, counts = ep_helpers.ep_dispatch_cpu(x, ids, w, E, G)
    off = np.concatenate([[0], np.cumsum(counts.numpy())])
    for g in range(G):
        toks = stok[off[g]:off[g + 1]].numpy()
        assert np.all(np.diff(toks) > 0)
        for p in range(off[g], off[g + 1]):
            t = int(stok[p])
            assert int(pidx[t, g]) == p
            assert torch.equal(sx[p], x[t])
            for k in range(topk):
                gid = int(ids[t, k])
                mine = 0 <= gid < E and gid // (E // G) == g
                assert int(sid[p, k]) == (gid - g * (E // G) if mine else -1)
                assert float(sw[p, k]) == (float(w[t, k]) if mine else 0.0)


def test_ep_gloo_world4_balanced_placement():
    """Four gloo ranks with the placement balanced_placement picks for
    skewed counts: every rank's output equals the single-rank eager loop
    over all experts."""
    from exl3_b200 import synthetic
    from exl3_b200.ep import balanced_placement

    E, world = 8, 4
    counts = [90, 3, 40, 7, 200, 1, 12, 60]
    placement = balanced_placement(counts, world, tile_rows=16)
    assert placement != list(range(E))
    cfg = dict(seed=13, E=E, H=256, I=128, topk=2, T=6, n_valid=None, capacity=8, placement=placement)
    got = {r: y for r, y, _c in _run_ranks(ep_helpers.gloo_worker, world, cfg, 120)}
    pack = synthetic.make_moe_pack(cfg["seed"], E, cfg["H"], cfg["I"], synthetic.CB_MCG, (4,))
    dense = ep_helpers.dense_experts(pack, 0, E)
    rng = np.random.default_rng(cfg["seed"] + 7)
    x = synthetic.activations(rng, cfg["T"] * world, cfg["H"])
    ids, w = synthetic.softmax_topk(rng, cfg["T"] * world, E, cfg["topk"])
    ids[::5, 0] = -1
    for r in range(world):
        sl = slice(r * cfg["T"], (r + 1) * cfg["T"])
        want = oracle.moe_eager(x[sl], ids[sl], w[sl], dense)
        np.testing.assert_allclose(got[r], want, rtol=1e-5, atol=1e-5 * float(np.abs(want).max() + 1))


def test_balanced_placement_properties():
    """Every rank keeps E/G experts, the result is a permutation, and the
    most-loaded rank (in 128-row tiles) is no worse than under the
    contiguous split, within the greedy's bound of one expert's cost above
    the mean."""
    from exl3_b200 import synthetic
    from exl3_b200.ep import balanced_placement, experts_of_rank

    E, topk = 256, 8
    ranks = np.random.default_rng(5).permutation(E)
    ids, _ = synthetic.sigmoid_zipf_topk(np.random.default_rng(6), 8192, E, topk, ranks=ranks)
    counts = np.bincount(ids.ravel(), minlength=E)
    tiles = (counts + 127) // 128
    for G in (1, 2, 4, 8):
        slot = balanced_placement(counts, G)
        assert sorted(slot) == list(range(E))
        held = [experts_of_rank(slot, G, g) for g in range(G)]
        assert sorted(e for h in held for e in h) == list(range(E))
        for g in range(G):
            assert all(slot[e] == g * (E // G) + j for j, e in enumerate(held[g]))
        load = [int(tiles[h].sum()) for h in held]
        contiguous = [int(tiles[g * (E // G):(g + 1) * (E // G)].sum()) for g in range(G)]
        assert max(load) <= max(contiguous)
        assert max(load) <= tiles.sum() / G + tiles.max()
    with pytest.raises(ValueError):
        balanced_placement(counts[:255], 4)


def test_ep_rejects_bad_placement():
    from exl3_b200.ep import Exl3ExpertParallel
    layer = ep_helpers.DenseLocalLayer([None] * 8)
    with pytest.raises(ValueError, match="permutation"):
        Exl3ExpertParallel(layer, 8, ops=ep_helpers.CpuEpOps(), placement=[0, 1, 2, 3, 4, 5, 6, 6])


def test_ep_rejects_uneven_split():
    from exl3_b200.ep import Exl3ExpertParallel
    layer = ep_helpers.DenseLocalLayer([{}] * 3)
    with pytest.raises(ValueError):
        Exl3ExpertParallel(layer, 8, ops=ep_helpers.CpuEpOps())  # world 1 holds all 8, not 3


# ---------------------------------------------------------------------------
# GPU: native kernels against the restatement; emulated G-rank step
# ---------------------------------------------------------------------------
@pytest.mark.gpu
@pytest.mark.parametrize("G,dt,ids_dt,nv,cap", [(1, "bf16", "i64", None, 0), (2, "bf16", "i32", None, 0),
                                                (4, "f16", "i64", 13, 0), (8, "f32", "i32", None, 0),
                                                (3, "bf16", "i64", 0, 0), (2, "bf16", "i64", None, 37),
                                                (4, "f32", "i32", 20, 50), (8, "bf16", "i64", None, 64)])
def test_ep_dispatch_combine_match_restatement(native, cuda, G, dt, ids_dt, nv, cap):
    import torch
    from exl3_b200.ep import NativeEpOps
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dt]
    rng = np.random.default_rng(G * 31 + 5)
    T, H, E, topk = 37, 384, 24, 6
    x = torch.from_numpy(rng.normal(size=(T, H)).astype(np.float32)).to(tdt)
    ids = torch.from_numpy(rng.integers(-1, E + 1, size=(T, topk))).to(
        torch.int32 if ids_dt == "i32" else torch.int64)
    w = torch.from_numpy(rng.random((T, topk)).astype(np.float32)).to(torch.bfloat16)
    ops = NativeEpOps()
    nvt = None if nv is None else torch.tensor([nv], dtype=torch.int32, device=cuda)
    sx, sid, sw, pidx, counts = ops.dispatch(x.to(cuda), ids.to(cuda), w.to(cuda), E, G, nvt, capacity=cap)
    wx, wid, ww, wtok, wpidx, wcounts = ep_helpers.ep_dispatch_cpu(x, ids, w, E, G, nv, cap)
    P = int(wcounts.sum()) if not cap else G * cap
    assert torch.equal(counts.cpu(), wcounts)
    assert torch.equal(pidx.cpu()[:T], wpidx)
    assert torch.equal(sid[:P].cpu(), wid)
    assert torch.equal(sw[:P].cpu(), ww)
    used = (wtok >= 0)  # empty capacity slots' rows are not written
    assert torch.equal(sx[:P].cpu()[used], wx[used])
    # combine: fp32 sums in rank order, bit-exact
    for pdt, odt in ((torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16), (torch.float16, torch.float32)):
        part = torch.from_numpy(rng.normal(size=(max(P, 1), H)).astype(np.float32)).to(pdt)
        got = ops.combine(part.to(cuda), pidx, T, G, odt, nvt).cpu()
        want = ep_helpers.ep_combine_cpu(part, wpidx, T, G, nv).to(odt)
        assert torch.equal(got, want)


def _emulated_step(layers, x, ids, w, E, G, combine_dtype):
    """G ranks on one GPU: per-rank dispatch, the all-to-all as slicing,
    per-rank local forward, the return all-to-all, per-rank combine."""
    import torch
    from exl3_b200.ep import NativeEpOps
    ops = NativeEpOps()
    T = x.shape[0] // G
    disp = [ops.dispatch(x[r * T:(r + 1) * T], ids[r * T:(r + 1) * T], w[r * T:(r + 1) * T], E, G) for r in range(G)]
    counts = [d[4].cpu().tolist() for d in disp]
    offs = [np.concatenate([[0], np.cumsum(c)]).astype(int) for c in counts]
    partial_back = [[None] * G for _ in range(G)]
    for q in range(G):  # receiver
        rx = torch.cat([disp[r][0][offs[r][q]:offs[r][q + 1]] for r in range(G)])
        rid = torch.cat([disp[r][1][offs[r][q]:offs[r][q + 1]] for r in range(G)])
        rw = torch.cat([disp[r][2][offs[r][q]:offs[r][q + 1]] for r in range(G)])
        part = ops.local(layers[q], rx, rid, rw, combine_dtype, None)
        o = 0
        for r in range(G):
            n = counts[r][q]
            partial_back[r][q] = part[o:o + n]
            o += n
    outs = []
    for r in range(G):
        back = torch.cat([partial_back[r][q] for q in range(G)])
        outs.append(ops.combine(back, disp[r][3], T, G, torch.float32))
    return torch.cat(outs)


@pytest.mark.gpu
@pytest.mark.parametrize("G,cdt", [(2, "f32"), (4, "f32"), (4, "bf16")])
def test_ep_emulated_ranks_match_single_gpu_and_oracle(native, cuda, G, cdt):
    """fp32 exchange: the layer tolerance (2e-2 RMS, cosine 0.9995).  bf16
    exchange rounds every partial row once (half a bf16 ulp, 2**-9 relative,
    per partial, up to G partials per token): checked against 4e-2 RMS."""
    import torch
    from exl3_b200 import moe, synthetic
    E, H, I, topk, Tr = 16, 512, 256, 4, 24
    pack = synthetic.make_moe_pack(21, E, H, I, synthetic.CB_MCG, (2, 3, 4))
    full = moe.layer_from_pack(pack, cuda)
    epr = E // G
    layers = []
    for r in range(G):
        sub = synthetic.MoEPack(H, I, pack.codebook, pack.experts[r * epr:(r + 1) * epr])
        layers.append(moe.layer_from_pack(sub, cuda))
    rng = np.random.default_rng(99)
    xs = synthetic.activations(rng, Tr * G, H)
    ids, w = synthetic.softmax_topk(rng, Tr * G, E, topk)
    x = torch.from_numpy(xs).to(torch.bfloat16).to(cuda)
    idt = torch.from_numpy(ids).to(cuda)
    wt = torch.from_numpy(w).to(cuda)
    cdt_t = torch.bfloat16 if cdt == "bf16" else torch.float32
    got = _emulated_step(layers, x, idt, wt, E, G, cdt_t).cpu().numpy()
    single = torch.empty(x.shape[0], H, dtype=torch.float32, device=cuda)
    full.apply(x, wt, idt, out=single)
    rel = 2e-2 if cdt == "f32" else 4e-2
    _close(got, single.cpu().numpy(), rel=rel)
    dense = ep_helpers.dense_experts(pack, 0, E)
    want = oracle.moe_eager(x.float().cpu().numpy(), ids, w, dense)
    _close(got, want, rel=rel)


@pytest.mark.gpu
@pytest.mark.parametrize("cap", [None, 48])
def test_ep_world1_module_matches_layer(native, cuda, cap):
    import torch
    from exl3_b200 import moe, synthetic
    from exl3_b200.ep import Exl3ExpertParallel
    pack = synthetic.make_moe_pack(5, 8, 256, 128, synthetic.CB_MCG, (4,))
    layer = moe.layer_from_pack(pack, cuda)
    ep = Exl3ExpertParallel(layer, 8, combine_dtype=torch.float32, capacity=cap)
    rng = np.random.default_rng(4)
    x = torch.from_numpy(synthetic.activations(rng, 40, 256)).to(torch.bfloat16).to(cuda)
    ids, w = synthetic.softmax_topk(rng, 40, 8, 2)
    idt, wt = torch.from_numpy(ids).to(cuda), torch.from_numpy(w).to(cuda)
    f32 = torch.empty(40, 256, dtype=torch.float32, device=cuda)
    got = ep(x, wt, idt, out=f32).cpu().numpy()
    want = torch.empty_like(f32)
    layer.apply(x, wt, idt, out=want)
    want = want.cpu().numpy()
    _close(got, want, rel=1e-3)
    nv = torch.tensor([17], dtype=torch.int32, device=cuda)
    got = ep(x, wt, idt, n_valid=nv, out=f32).cpu().numpy()
    assert np.all(got[17:] == 0)
    _close(got[:17], want[:17], rel=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("G", [2, 4])
def test_ep_nvlink_emulated_ranks(native, cuda, G):
    """The NVLink transport's kernels (window stores, flags, waits, return,
    combine) for G ranks emulated on one GPU, two consecutive steps (the
    flags carry the step number), against the single-GPU layer and the
    oracle."""
    import torch
    from exl3_b200 import moe, synthetic
    from exl3_b200.ep import NvlinkEpWindow
    E, H, I, topk, Tr = 16, 512, 256, 4, 24
    C = Tr
    pack = synthetic.make_moe_pack(31, E, H, I, synthetic.CB_MCG, (2, 3, 4))
    full = moe.layer_from_pack(pack, cuda)
    epr = E // G
    layers = [moe.layer_from_pack(synthetic.MoEPack(H, I, pack.codebook, pack.experts[r * epr:(r + 1) * epr]), cuda)
              for r in range(G)]
    wins = [NvlinkEpWindow(G, r, C, H, topk, torch.bfloat16, torch.float32, cuda, exchange=False) for r in range(G)]
    addrs = [wn.window for wn in wins]
    for wn in wins:
        wn.set_peers(addrs)
    try:
        dense = ep_helpers.dense_experts(pack, 0, E)
        for step in range(2):
            rng = np.random.default_rng(50 + step)
            xs = synthetic.activations(rng, Tr * G, H)
            ids, w = synthetic.softmax_topk(rng, Tr * G, E, topk)
            x = torch.from_numpy(xs).to(torch.bfloat16).to(cuda)
            idt, wt = torch.from_numpy(ids).to(cuda), torch.from_numpy(w).to(cuda)
            got = ep_helpers.nvlink_emulated_step(layers, wins, x, idt, wt, E, G, C, torch.float32).cpu().numpy()
            single = torch.empty(x.shape[0], H, dtype=torch.float32, device=cuda)
            full.apply(x, wt, idt, out=single)
            _close(got, single.cpu().numpy())
            _close(got, oracle.moe_eager(x.float().cpu().numpy(), ids, w, dense))
            assert all(wn.status() == 0 for wn in wins)
    finally:
        for wn in wins:
            wn.close()


@pytest.mark.gpu
def test_ep_nvlink_wait_times_out_with_status(native, cuda):
    """A peer that never signals: the bounded wait gives up (about 2 s) and
    records status 4 in the window instead of spinning on."""
    import time

    import torch
    from exl3_b200 import _native as _n
    from exl3_b200.ep import NvlinkEpWindow
    wins = [NvlinkEpWindow(2, r, 8, 128, 2, torch.float16, torch.float32, cuda, exchange=False) for r in range(2)]
    for wn in wins:
        wn.set_peers([wins[0].window, wins[1].window])
    try:
        lib = _n.load()
        t0 = time.time()
        _n.check(lib.exl3_ep_p2p_wait(wins[0].window, 2, 0, _n.stream_of(wins[0].peers)))
        torch.cuda.synchronize(cuda)
        assert time.time() - t0 < 30
        assert wins[0].status() == 4
        assert wins[0].status() == 0  # cleared
    finally:
        for wn in wins:
            wn.close()


@pytest.mark.gpu
@pytest.mark.parametrize("transport,cap", [("nccl", None), ("nccl", 48), ("nvlink", 48)])
def test_ep_world1_placement_matches_layer(native, cuda, transport, cap):
    """A permuted placement: the rank holds the experts in slot order and
    the layer relabels global ids, so the output equals the unpermuted
    layer's for the same global ids (dropped routes included)."""
    import torch
    from exl3_b200 import moe, synthetic
    from exl3_b200.ep import Exl3ExpertParallel, experts_of_rank
    pack = synthetic.make_moe_pack(7, 8, 256, 128, synthetic.CB_MCG, (3, 4))
    ref = moe.layer_from_pack(pack, cuda)
    slot = [5, 0, 7, 2, 1, 6, 3, 4]
    moved = synthetic.MoEPack(256, 128, synthetic.CB_MCG)
    moved.experts = [pack.experts[e] for e in experts_of_rank(slot, 1, 0)]
    layer = moe.layer_from_pack(moved, cuda)
    ep = Exl3ExpertParallel(layer, 8, combine_dtype=torch.float32, capacity=cap, transport=transport,
                            placement=slot)
    try:
        for step in range(2):
            rng = np.random.default_rng(20 + step)
            x = torch.from_numpy(synthetic.activations(rng, 40, 256)).to(torch.bfloat16).to(cuda)
            ids, w = synthetic.softmax_topk(rng, 40, 8, 2)
            ids[::7, 1] = -1
            idt, wt = torch.from_numpy(ids).to(cuda), torch.from_numpy(w).to(cuda)
            f32 = torch.empty(40, 256, dtype=torch.float32, device=cuda)
            got = ep(x, wt, idt, out=f32).cpu().numpy()
            want = torch.empty_like(f32)
            ref.apply(x, wt, idt, out=want)
            _close(got, want.cpu().numpy(), rel=1e-3)
    finally:
        ep.close()


@pytest.mark.gpu
def test_ep_nvlink_world1_module(native, cuda):
    import torch
    from exl3_b200 import moe, synthetic
    from exl3_b200.ep import Exl3ExpertParallel
    pack = synthetic.make_moe_pack(6, 8, 256, 128, synthetic.CB_MCG, (4,))
    layer = moe.layer_from_pack(pack, cuda)
    ep = Exl3ExpertParallel(layer, 8, combine_dtype=torch.float32, capacity=48, transport="nvlink")
    try:
        for step in range(3):
            rng = np.random.default_rng(10 + step)
            x = torch.from_numpy(synthetic.activations(rng, 40, 256)).to(torch.bfloat16).to(cuda)
            ids, w = synthetic.softmax_topk(rng, 40, 8, 2)
            idt, wt = torch.from_numpy(ids).to(cuda), torch.from_numpy(w).to(cuda)
            f32 = torch.empty(40, 256, dtype=torch.float32, device=cuda)
            got = ep(x, wt, idt, out=f32).cpu().numpy()
            want = torch.empty_like(f32)
            layer.apply(x, wt, idt, out=want)
            _close(got, want.cpu().numpy(), rel=1e-3)
            assert ep.window(x.dtype, 2, 256).status() == 0
    finally:
        ep.close()


@pytest.mark.gpu
@pytest.mark.parametrize("capacity,transport", [(None, "nccl"), (40, "nccl"), (40, "nvlink")])
def test_ep_nccl_two_gpus(native, capacity, transport):
    """Two ranks over NCCL on two GPUs (skipped on a one-GPU box)."""
    import torch
    from exl3_b200 import synthetic
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = dict(seed=17, E=16, H=512, I=256, topk=4, T=40, capacity=capacity, transport=transport)
    world = 2
    got = {r: y for r, y, _c in _run_ranks(ep_helpers.nccl_worker, world, cfg, 120)}
    pack = synthetic.make_moe_pack(cfg["seed"], cfg["E"], cfg["H"], cfg["I"], synthetic.CB_MCG, (2, 3, 4))
    dense = ep_helpers.dense_experts(pack, 0, cfg["E"])
    rng = np.random.default_rng(cfg["seed"] + 7)
    x = synthetic.activations(rng, cfg["T"] * world, cfg["H"])
    ids, w = synthetic.softmax_topk(rng, cfg["T"] * world, cfg["E"], cfg["topk"])
    xh = x.astype(np.float32)
    for r in range(world):
        sl = slice(r * cfg["T"], (r + 1) * cfg["T"])
        _close(got[r], oracle.moe_eager(xh[sl], ids[sl], w[sl], dense))


@pytest.mark.gpu
def test_ep_nvlink_forward_reports_failed_wait(native, cuda):
    """A failure recorded in the window's status word (as a bounded peer wait
    that gave up records it; here written by the host, so no kernel has to
    time out) makes the next forward() raise, and check_status() raises at
    once, instead of steps continuing on stale rows."""
    import torch
    from exl3_b200 import moe, synthetic
    from exl3_b200.ep import Exl3ExpertParallel
    pack = synthetic.make_moe_pack(8, 8, 256, 128, synthetic.CB_MCG, (4,))
    layer = moe.layer_from_pack(pack, cuda)
    ep = Exl3ExpertParallel(layer, 8, combine_dtype=torch.float32, capacity=16, transport="nvlink")
    try:
        rng = np.random.default_rng(3)
        x = torch.from_numpy(synthetic.activations(rng, 16, 256)).to(torch.bfloat16).to(cuda)
        ids, w = synthetic.softmax_topk(rng, 16, 8, 2)
        idt, wt = torch.from_numpy(ids).to(cuda), torch.from_numpy(w).to(cuda)
        ep(x, wt, idt)
        ep.check_status()  # clean
        win = ep.window(x.dtype, 2, 256)
        win.status_tensor().fill_(4)  # what ep_p2p_wait_kernel records on a timeout
        ep(x, wt, idt)                # this step's status copy carries the failure to the host
        torch.cuda.synchronize(cuda)
        with pytest.raises(RuntimeError, match="status 4"):
            ep(x, wt, idt)
        with pytest.raises(RuntimeError, match="status 4"):
            ep.check_status()
        assert win.status(clear=True) == 4
    finally:
        ep.close()

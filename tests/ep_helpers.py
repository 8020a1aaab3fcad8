"""Expert-parallel test helpers: CPU stand-ins for the compute steps and rank workers.

``CpuEpOps`` restates, in torch on the CPU, what ``exl3_ep_dispatch`` and
``exl3_ep_combine`` promise (include/exl3_b200.h) and runs the local expert
forward with the oracle's eager loop, so the exchange logic of
``exl3_b200.ep.Exl3ExpertParallel`` can run on gloo ranks without a GPU.  The
GPU tests check the native dispatch / combine against the same restatement.
"""

from __future__ import annotations

import numpy as np
import torch

import cpu_oracle as oracle


def ep_dispatch_cpu(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, n_global: int, world: int,
                    n_valid: int | None = None, capacity: int = 0):
    """Pairs (token, owning rank), rank-major and token-ascending.

    Returns send_x [P][H], send_ids [P][topk] int32 (local id or -1),
    send_w [P][topk] fp32, send_tok [P] int32, pair_idx [T][world] int32,
    counts [world] int32, where P is the number of pairs -- or, with a
    capacity C, world * C slots with rank g's pairs at [g*C, g*C + count)
    and empty slots of token -1, ids -1, weight 0 and zero rows.
    """
    if capacity:
        px, pid, pw, ptok, pidx, counts = ep_dispatch_cpu(x, ids, weights, n_global, world, n_valid)
        T, H = x.shape
        topk = ids.shape[1]
        sx = x.new_zeros(world * capacity, H)
        sid = torch.full((world * capacity, topk), -1, dtype=torch.int32)
        sw = torch.zeros(world * capacity, topk)
        stok = torch.full((world * capacity,), -1, dtype=torch.int32)
        remap = torch.full((max(1, int(counts.sum())),), -1, dtype=torch.int64)
        o = 0
        for g in range(world):
            n = int(counts[g])
            dst = slice(g * capacity, g * capacity + n)
            sx[dst], sid[dst], sw[dst], stok[dst] = px[o:o + n], pid[o:o + n], pw[o:o + n], ptok[o:o + n]
            remap[o:o + n] = torch.arange(g * capacity, g * capacity + n)
            o += n
        pidx = torch.where(pidx >= 0, remap[pidx.clamp(min=0).long()].to(torch.int32), pidx)
        return sx, sid, sw, stok, pidx, counts
    T, H = x.shape
    topk = ids.shape[1]
    epr = n_global // world
    live = T if n_valid is None else max(0, min(T, int(n_valid)))
    ids64 = ids.to(torch.int64)
    valid = (ids64 >= 0) & (ids64 < n_global)
    owner = torch.where(valid, ids64 // epr, torch.full_like(ids64, -1))
    pair_idx = torch.full((T, world), -1, dtype=torch.int32)
    rows, sid, sw, stok, counts = [], [], [], [], []
    for g in range(world):
        n = 0
        for t in range(live):
            own = owner[t] == g
            if not bool(own.any()):
                continue
            pair_idx[t, g] = len(stok)
            stok.append(t)
            rows.append(x[t])
            sid.append(torch.where(own, ids64[t] - g * epr, torch.full_like(ids64[t], -1)).to(torch.int32))
            sw.append(torch.where(own, weights[t].float(), torch.zeros(topk)))
            n += 1
        counts.append(n)
    P = len(stok)
    send_x = torch.stack(rows) if P else x.new_empty(0, H)
    send_ids = torch.stack(sid) if P else torch.empty(0, topk, dtype=torch.int32)
    send_w = torch.stack(sw) if P else torch.empty(0, topk)
    return (send_x, send_ids, send_w, torch.tensor(stok, dtype=torch.int32), pair_idx,
            torch.tensor(counts, dtype=torch.int32))


def ep_combine_cpu(partial: torch.Tensor, pair_idx: torch.Tensor, tokens: int, world: int,
                   n_valid: int | None = None) -> torch.Tensor:
    """fp32 sum over ranks in rank order; rows past n_valid are zero."""
    H = partial.shape[1]
    out = torch.zeros(tokens, H, dtype=torch.float32)
    live = tokens if n_valid is None else max(0, min(tokens, int(n_valid)))
    pf = partial.float()
    for g in range(world):
        for t in range(live):
            p = int(pair_idx[t, g])
            if p >= 0:
                out[t] += pf[p]
    return out


class DenseLocalLayer:
    """A rank's experts as dequantised fp16 matrices (oracle.dequant)."""

    def __init__(self, dense: list):
        self.dense = dense
        self._exl3_inners = dense
        self.expert_map = None


class CpuEpOps:
    """``ops`` for Exl3ExpertParallel on CPU ranks."""

    def dispatch(self, x, ids, weights, n_global, world, n_valid=None, capacity=0):
        nv = None if n_valid is None else int(n_valid.reshape(-1)[0])
        send_x, send_ids, send_w, _tok, pair_idx, counts = ep_dispatch_cpu(x, ids, weights, n_global, world, nv,
                                                                           capacity)
        return send_x, send_ids, send_w, pair_idx, counts

    def local(self, layer, x, ids, weights, out_dtype, limit):
        if x.shape[0] == 0:
            return torch.empty(0, x.shape[1], dtype=out_dtype)
        y = oracle.moe_eager(x.float().numpy(), ids.numpy(), weights.numpy(), layer.dense, limit=limit)
        return torch.from_numpy(y).to(out_dtype)

    def combine(self, partial, pair_idx, tokens, world, out_dtype, n_valid=None, out=None):
        nv = None if n_valid is None else int(n_valid.reshape(-1)[0])
        y = ep_combine_cpu(partial, pair_idx, tokens, world, nv).to(out_dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y


def dense_experts(pack, lo: int, hi: int) -> list:
    """oracle.dequant of experts [lo, hi) of a synthetic pack."""
    out = []
    for e in pack.experts[lo:hi]:
        d = {}
        for which in ("gate", "up", "down"):
            p = e[which]
            d[which] = oracle.dequant(p.trellis, p.suh, p.svh, p.K, cb=p.codebook)
        out.append(d)
    return out


def gloo_worker(rank: int, world: int, port: int, cfg: dict, result_q) -> None:
    """One gloo rank: run Exl3ExpertParallel with CpuEpOps on this rank's tokens."""
    import os

    import torch.distributed as dist

    from exl3_b200 import synthetic
    from exl3_b200.ep import Exl3ExpertParallel

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        pack = synthetic.make_moe_pack(cfg["seed"], cfg["E"], cfg["H"], cfg["I"], synthetic.CB_MCG, (4,))
        epr = cfg["E"] // world
        placement = cfg.get("placement")
        if placement is None:
            layer = DenseLocalLayer(dense_experts(pack, rank * epr, (rank + 1) * epr))
        else:
            from exl3_b200.ep import experts_of_rank
            dense = dense_experts(pack, 0, cfg["E"])
            layer = DenseLocalLayer([dense[e] for e in experts_of_rank(placement, world, rank)])
        rng = np.random.default_rng(cfg["seed"] + 7)
        x = synthetic.activations(rng, cfg["T"] * world, cfg["H"])
        ids, w = synthetic.softmax_topk(rng, cfg["T"] * world, cfg["E"], cfg["topk"])
        ids[::5, 0] = -1  # dropped routes
        sl = slice(rank * cfg["T"], (rank + 1) * cfg["T"])
        ep = Exl3ExpertParallel(layer, cfg["E"], combine_dtype=torch.float32, ops=CpuEpOps(),
                                capacity=cfg.get("capacity"), placement=placement)
        nv = None
        if cfg.get("n_valid") is not None:
            nv = torch.tensor([cfg["n_valid"]], dtype=torch.int32)
        y = ep(torch.from_numpy(x[sl]), torch.from_numpy(w[sl]), torch.from_numpy(ids[sl]), n_valid=nv)
        result_q.put((rank, y.numpy(), ep.last_counts))
    finally:
        dist.destroy_process_group()


def nccl_worker(rank: int, world: int, port: int, cfg: dict, result_q) -> None:
    """One NCCL rank on its own GPU: the native EP layer on this rank's tokens
    (all ranks build the same synthetic pack and routing; rank r keeps experts
    [r*E/G, (r+1)*E/G) and tokens [r*T, (r+1)*T))."""
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from exl3_b200 import moe, synthetic
    from exl3_b200.ep import Exl3ExpertParallel

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        pack = synthetic.make_moe_pack(cfg["seed"], cfg["E"], cfg["H"], cfg["I"], synthetic.CB_MCG, (2, 3, 4))
        epr = cfg["E"] // world
        sub = synthetic.MoEPack(cfg["H"], cfg["I"], pack.codebook, pack.experts[rank * epr:(rank + 1) * epr])
        layer = moe.layer_from_pack(sub, dev)
        rng = np.random.default_rng(cfg["seed"] + 7)
        x = synthetic.activations(rng, cfg["T"] * world, cfg["H"])
        ids, w = synthetic.softmax_topk(rng, cfg["T"] * world, cfg["E"], cfg["topk"])
        sl = slice(rank * cfg["T"], (rank + 1) * cfg["T"])
        ep = Exl3ExpertParallel(layer, cfg["E"], combine_dtype=torch.float32, capacity=cfg.get("capacity"),
                                transport=cfg.get("transport", "nccl"))
        y = ep(torch.from_numpy(x[sl]).to(torch.bfloat16).to(dev), torch.from_numpy(w[sl]).to(dev),
               torch.from_numpy(ids[sl]).to(dev))
        torch.cuda.synchronize(dev)
        result_q.put((rank, y.float().cpu().numpy(), ep.last_counts))
        ep.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def nvlink_emulated_step(layers, wins, x, ids, w, E, G, C, out_dtype):
    """G ranks' NVLink steps on one GPU, phase by phase across the ranks (all
    dispatches, then every rank's wait + local forward + return, then every
    rank's wait + combine): no wait ever depends on a later launch."""
    from exl3_b200 import _native as _n
    from exl3_b200.moe import moe_forward_ptrs
    lib = _n.load()
    T = x.shape[0] // G
    H = x.shape[1]
    topk = ids.shape[1]
    dev = x.device
    stream = _n.stream_of(x)
    pidx = [torch.empty(C, G, dtype=torch.int32, device=dev) for _ in range(G)]
    part = [torch.empty(G * C, H, dtype=torch.float32, device=dev) for _ in range(G)]
    outs = [torch.empty(T, H, dtype=out_dtype, device=dev) for _ in range(G)]
    for r in range(G):
        xr, ir, wr = x[r * T:(r + 1) * T], ids[r * T:(r + 1) * T], w[r * T:(r + 1) * T]
        _n.check(lib.exl3_ep_p2p_dispatch(xr.data_ptr(), _n.dtype_code(xr), T, H, ir.data_ptr(),
                                          _n.dtype_code(ir), wr.data_ptr(), _n.dtype_code(wr), topk, E, G, r, C,
                                          None, wins[r].window, wins[r].peers.data_ptr(), _n.DT_F32,
                                          pidx[r].data_ptr(), stream))
    for r in range(G):
        _n.check(lib.exl3_ep_p2p_wait(wins[r].window, G, 0, stream))
        moe_forward_ptrs(layers[r], dev, wins[r].recv_x, _n.dtype_code(x), G * C, wins[r].recv_ids, _n.DT_I32,
                         wins[r].recv_w, _n.DT_F32, topk, part[r].data_ptr(), _n.DT_F32)
        _n.check(lib.exl3_ep_p2p_return(part[r].data_ptr(), _n.DT_F32, G, r, C, H, topk, _n.dtype_code(x),
                                        wins[r].window, wins[r].peers.data_ptr(), stream))
    for r in range(G):
        _n.check(lib.exl3_ep_p2p_wait(wins[r].window, G, 1, stream))
        _n.check(lib.exl3_ep_p2p_combine(wins[r].window, G, r, C, H, topk, _n.dtype_code(x), _n.DT_F32,
                                         pidx[r].data_ptr(), T, None, outs[r].data_ptr(), _n.dtype_code(outs[r]),
                                         stream))
    return torch.cat(outs)

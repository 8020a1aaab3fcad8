"""Expert parallelism for the EXL3 routed-expert layer.

One process per GPU.  Rank g of the group owns the global experts
[g*E/G, (g+1)*E/G) -- the contiguous linear expert_map the reference plugin
consumes (src/vllm_exl3/exl3.py:2310-2354); the reference itself leaves the
token exchange to vLLM's all-to-all backends.  One layer step:

1. ``exl3_ep_dispatch`` (native): every token is paired with each rank that
   owns at least one of its routes; pair rows (token row + topk local-id /
   weight slots, -1 / 0 for routes owned elsewhere) are packed rank-major.
2. ``all_to_all_single`` of the per-rank pair counts; the counts come to the
   host (the step's one synchronisation: the row exchange needs its splits).
3. The rows, local ids and weights go to their ranks as one group of
   point-to-point transfers (one NCCL launch over NVLink; gloo on CPU in the
   tests).
4. The local fused forward (``exl3_moe_forward``) over the received pairs,
   which returns one partial row per pair: that token's weighted sum over
   the routes this rank owns.
5. The partial rows go back to their sources (one more group).
6. ``exl3_ep_combine`` (native): per-token sum over ranks in rank order --
   deterministic, no atomics.

A token whose routes fall on one rank crosses the network once, not once per
route.  The compute steps go through an ``ops`` object; the default
:class:`NativeEpOps` calls the C ABI and raises without a GPU.  Tests inject
CPU stand-ins to exercise the exchange logic on gloo ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _native as _n
from .moe import apply_exl3_experts


class NativeEpOps:
    """Dispatch / local forward / combine through ``libexl3_b200.so``."""

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, n_global: int, world: int,
                 n_valid: torch.Tensor | None = None, capacity: int = 0):
        lib = _n.load()
        _n.require_cuda(x, ids, weights, n_valid, who="exl3_ep_dispatch")
        T, H = x.shape
        topk = ids.shape[1]
        P = max(1, world * capacity if capacity else T * min(world, topk))
        dev = x.device
        send_x = torch.empty(P, H, dtype=x.dtype, device=dev)
        send_ids = torch.empty(P, topk, dtype=torch.int32, device=dev)
        send_w = torch.empty(P, topk, dtype=torch.float32, device=dev)
        send_tok = torch.empty(P, dtype=torch.int32, device=dev)
        pair_idx = torch.empty(max(1, T), world, dtype=torch.int32, device=dev)
        counts = torch.empty(world, dtype=torch.int32, device=dev)
        _n.check(lib.exl3_ep_dispatch(
            x.data_ptr(), _n.dtype_code(x), T, H, ids.data_ptr(), _n.dtype_code(ids), weights.data_ptr(),
            _n.dtype_code(weights), topk, n_global, world, _n.ptr(n_valid), send_x.data_ptr(),
            send_ids.data_ptr(), send_w.data_ptr(), send_tok.data_ptr(), pair_idx.data_ptr(),
            counts.data_ptr(), int(capacity), _n.stream_of(x)), "exl3_ep_dispatch")
        return send_x, send_ids, send_w, pair_idx, counts

    def local(self, layer, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, out_dtype: torch.dtype,
              limit: float | None) -> torch.Tensor:
        out = torch.empty(x.shape[0], x.shape[1], dtype=out_dtype, device=x.device)
        if x.shape[0]:
            apply_exl3_experts(x, ids, weights, layer, limit=limit, out=out)
        return out

    def combine(self, partial: torch.Tensor, pair_idx: torch.Tensor, tokens: int, world: int,
                out_dtype: torch.dtype, n_valid: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        lib = _n.load()
        H = partial.shape[1]
        if out is None:
            out = torch.empty(tokens, H, dtype=out_dtype, device=partial.device)
        if tokens == 0:
            return out
        _n.require_cuda(partial, pair_idx, out, n_valid, who="exl3_ep_combine")
        _n.check(lib.exl3_ep_combine(
            partial.data_ptr(), _n.dtype_code(partial), pair_idx.data_ptr(), tokens, world, H, _n.ptr(n_valid),
            out.data_ptr(), _n.dtype_code(out), _n.stream_of(partial)), "exl3_ep_combine")
        return out


class Exl3ExpertParallel(torch.nn.Module):
    """Routed-expert layer sharded by experts over a process group.

    ``local_layer`` holds this rank's ``n_global // world`` experts (an
    :class:`exl3_b200.moe.Exl3RoutedExperts`, no expert_map); ``forward``
    takes this rank's tokens with GLOBAL expert ids and returns their full
    routed output, like the single-GPU layer.  ``combine_dtype`` is the dtype
    partial rows travel in: fp32 (default) keeps each rank's partial sum
    exact; bf16 halves the return traffic at the cost of one bf16 rounding
    per partial (about one bf16 ulp of the output).

    ``capacity`` (rows, >= the tokens any rank passes in one call, the same
    on every rank) switches to fixed per-rank blocks: the exchanges become
    equal-split all-to-alls of ``capacity`` rows per rank, no count reaches
    the host, and a step can be captured in a CUDA graph; the cost is moving
    the empty slots.  Without it (None) the exchanges carry exactly the
    pairs, with one host synchronisation per step for the split sizes.
    """

    def __init__(self, local_layer, n_global: int, group=None, combine_dtype: torch.dtype = torch.float32,
                 ops=None, capacity: int | None = None):
        super().__init__()
        self.layer = local_layer
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if n_global % self.world:
            raise ValueError(f"{n_global} experts do not split evenly over {self.world} ranks")
        n_local = len(local_layer._exl3_inners)
        if n_local != n_global // self.world:
            raise ValueError(f"rank holds {n_local} experts, expected {n_global // self.world}")
        if getattr(local_layer, "expert_map", None) is not None:
            raise ValueError("the local layer of an expert-parallel group takes local ids (no expert_map)")
        self.n_global = int(n_global)
        self.combine_dtype = combine_dtype
        self.ops = ops if ops is not None else NativeEpOps()
        if capacity is not None and capacity < 1:
            raise ValueError("capacity must be a positive row count")
        self.capacity = None if capacity is None else int(capacity)
        self.last_counts: tuple[list[int], list[int]] | None = None
        self.profile = False  # record CUDA events between the step's phases (benchmarks)
        self._events: list = []

    PHASES = ("dispatch", "counts", "exchange", "local", "return", "combine")

    def _mark(self) -> None:
        if self.profile:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._events.append(ev)

    def phase_ms(self) -> dict:
        """Milliseconds of each phase of the last profiled step (synchronises)."""
        ev = self._events
        if len(ev) != len(self.PHASES) + 1:
            return {}
        ev[-1].synchronize()
        return {n: ev[i].elapsed_time(ev[i + 1]) for i, n in enumerate(self.PHASES)}

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_split: list[int], in_split: list[int]) -> None:
        if self.world == 1:
            out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, out_split, in_split, group=self.group)

    def _exchange(self, pairs: list, s_split: list[int], r_split: list[int]) -> None:
        """All-to-all of several (recv, send) tensor pairs as ONE group of
        point-to-point transfers (one NCCL launch): rank q's block of each
        send tensor goes to q, whose block of the recv tensor receives it.
        The block to this rank itself is a local copy."""
        so = [0] * (self.world + 1)
        ro = [0] * (self.world + 1)
        for g in range(self.world):
            so[g + 1] = so[g] + s_split[g]
            ro[g + 1] = ro[g] + r_split[g]
        ops = []
        for q in range(self.world):
            peer = q if self.group is None else dist.get_global_rank(self.group, q)
            for recv, send in pairs:
                if q == self.rank:
                    if s_split[q]:
                        recv[ro[q]:ro[q + 1]].copy_(send[so[q]:so[q + 1]])
                    continue
                if s_split[q]:
                    ops.append(dist.P2POp(dist.isend, send[so[q]:so[q + 1]], peer, group=self.group))
                if r_split[q]:
                    ops.append(dist.P2POp(dist.irecv, recv[ro[q]:ro[q + 1]], peer, group=self.group))
        if ops:
            for work in dist.batch_isend_irecv(ops):
                work.wait()

    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                limit: float | None = None, n_valid: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        T, H = x.shape
        G = self.world
        ids = topk_ids.reshape(T, -1)
        if ids.dtype not in (torch.int32, torch.int64):
            ids = ids.long()
        w = topk_weights.reshape(T, -1)
        if w.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            w = w.float()
        topk = ids.shape[1]
        self._events = []
        if self.capacity is not None:
            return self._forward_fixed(x, ids, w, limit, n_valid, out)
        self._mark()
        send_x, send_ids, send_w, pair_idx, send_counts = self.ops.dispatch(x, ids, w, self.n_global, G, n_valid)
        self._mark()
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, [1] * G, [1] * G)
        both = torch.cat([send_counts, recv_counts]).cpu().tolist()
        self._mark()
        s_split, r_split = both[:G], both[G:]
        S, R = sum(s_split), sum(r_split)
        self.last_counts = (s_split, r_split)
        if G == 1:  # nothing crosses a link: the pairs are already local
            recv_x, recv_ids, recv_w = send_x[:S], send_ids[:S], send_w[:S]
        else:
            recv_x = x.new_empty(R, H)
            recv_ids = send_ids.new_empty(R, topk)
            recv_w = send_w.new_empty(R, topk)
            self._exchange([(recv_x, send_x), (recv_ids, send_ids), (recv_w, send_w)], s_split, r_split)
        self._mark()
        partial = self.ops.local(self.layer, recv_x, recv_ids, recv_w, self.combine_dtype, limit)
        self._mark()
        if G == 1:
            back = partial
        else:
            back = partial.new_empty(max(S, 1), H)
            self._exchange([(back, partial)], r_split, s_split)
        self._mark()
        y = self.ops.combine(back, pair_idx, T, G, x.dtype, n_valid, out=out)
        self._mark()
        return y

    def _forward_fixed(self, x, ids, w, limit, n_valid, out):
        T, H = x.shape
        G, C = self.world, self.capacity
        if T > C:
            raise ValueError(f"{T} tokens exceed the exchange capacity {C}")
        topk = ids.shape[1]
        self._mark()
        send_x, send_ids, send_w, pair_idx, _counts = self.ops.dispatch(x, ids, w, self.n_global, G, n_valid,
                                                                        capacity=C)
        self._mark()
        self._mark()  # no count exchange in this mode
        if G == 1:
            recv_x, recv_ids, recv_w = send_x, send_ids, send_w
        else:
            recv_x = torch.empty_like(send_x)
            recv_ids = torch.empty_like(send_ids)
            recv_w = torch.empty_like(send_w)
            self._exchange([(recv_x, send_x), (recv_ids, send_ids), (recv_w, send_w)], [C] * G, [C] * G)
        self._mark()
        partial = self.ops.local(self.layer, recv_x, recv_ids, recv_w, self.combine_dtype, limit)
        self._mark()
        if G == 1:
            back = partial
        else:
            back = torch.empty_like(partial)
            self._exchange([(back, partial)], [C] * G, [C] * G)
        self._mark()
        y = self.ops.combine(back, pair_idx, T, G, x.dtype, n_valid, out=out)
        self._mark()
        return y

    apply = forward

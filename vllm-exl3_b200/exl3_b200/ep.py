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

``placement`` (optional) is a permutation of expert ids: expert e sits in
slot ``placement[e]`` and rank g owns slots [g*E/G, (g+1)*E/G), so skewed
expert popularity can be spread evenly over the ranks
(:func:`balanced_placement`).  The layer relabels the step's ids through it
before the dispatch; the kernels keep the contiguous slot ownership.

A token whose routes fall on one rank crosses the network once, not once per
route.  ``transport="nvlink"`` replaces the NCCL transfers with the library's
own kernels storing straight into the peers' memory (CUDA IPC windows,
per-step flags; see include/exl3_b200.h).  The compute steps go through an ``ops`` object; the default
:class:`NativeEpOps` calls the C ABI and raises without a GPU.  Tests inject
CPU stand-ins to exercise the exchange logic on gloo ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

import ctypes

from . import _native as _n
from .moe import apply_exl3_experts, moe_forward_ptrs


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


class NvlinkEpWindow:
    """This rank's NVLink exchange window and its peers' windows.

    The window (``exl3_ep_window_size`` bytes, allocated by the library so
    it can be exported) receives the rows other ranks route here and the
    partial rows they return; ``peers`` is a device int64 array of every
    rank's window address as mapped on this GPU (CUDA IPC).  With
    ``peer_windows`` given (single-process emulation of several ranks on
    one GPU) no IPC is done and those addresses are used directly.
    """

    def __init__(self, world: int, rank: int, capacity: int, hidden: int, topk: int, x_dtype: torch.dtype,
                 partial_dtype: torch.dtype, device: torch.device, group=None, exchange: bool = True):
        self.lib = _n.load()
        self.world, self.rank, self.capacity, self.hidden, self.topk = world, rank, capacity, hidden, topk
        self.x_code = _n._DTYPE_CODE[x_dtype]
        self.p_code = _n._DTYPE_CODE[partial_dtype]
        self.device = device
        geom = (world, capacity, hidden, topk, self.x_code, self.p_code)
        self.nbytes = int(self.lib.exl3_ep_window_size(*geom))
        if self.nbytes == 0:
            raise ValueError("unsupported expert-parallel window geometry")
        ptr = _n.P()
        with torch.cuda.device(device):
            _n.check(self.lib.exl3_ep_window_alloc(self.nbytes, ctypes.byref(ptr)), "exl3_ep_window_alloc")
        self.window = int(ptr.value)
        xo, io, wo = _n.SZ(), _n.SZ(), _n.SZ()
        _n.check(self.lib.exl3_ep_window_recv(*geom, ctypes.byref(xo), ctypes.byref(io), ctypes.byref(wo)),
                 "exl3_ep_window_recv")
        self.recv_x, self.recv_ids, self.recv_w = self.window + xo.value, self.window + io.value, self.window + wo.value
        self.mapped: list[int] = []
        self.peers = None
        if exchange:
            self._exchange(group)

    def _exchange(self, group) -> None:
        handle = (ctypes.c_char * 64)()
        _n.check(self.lib.exl3_ep_ipc_handle(self.window, handle), "exl3_ep_ipc_handle")
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        addrs = []
        with torch.cuda.device(self.device):
            for g in range(self.world):
                if g == self.rank:
                    addrs.append(self.window)
                    continue
                m = _n.P()
                buf = (ctypes.c_char * 64).from_buffer_copy(handles[g])
                _n.check(self.lib.exl3_ep_ipc_open(buf, ctypes.byref(m)), "exl3_ep_ipc_open")
                self.mapped.append(int(m.value))
                addrs.append(int(m.value))
        self.set_peers(addrs)

    def set_peers(self, addrs: list[int]) -> None:
        self.peers = torch.tensor(addrs, dtype=torch.int64, device=self.device)

    def status_tensor(self) -> torch.Tensor:
        """The window's device status word as a one-element int32 tensor
        (a view of the library-owned window, not a copy)."""
        addr, dev = self.window + 4, self.device

        class _View:
            __cuda_array_interface__ = {"shape": (1,), "typestr": "<i4", "data": (addr, False), "version": 3}

        with torch.cuda.device(dev):
            return torch.as_tensor(_View(), device=dev)

    def status(self, clear: bool = True) -> int:
        """The window's device status word (4 = a peer wait timed out)."""
        v = _n.I32(0)
        _n.check(self.lib.exl3_device_status(self.window + 4, int(clear), _n.stream_of(self.peers),
                                             ctypes.byref(v)), "exl3_device_status")
        return int(v.value)

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for m in self.mapped:
                self.lib.exl3_ep_ipc_close(m)
            self.mapped = []
            if self.window:
                self.lib.exl3_ep_window_free(self.window)
                self.window = 0


def balanced_placement(route_counts, world: int, tile_rows: int = 128) -> list[int]:
    """A permutation of expert ids that evens out the ranks' local forward.

    ``route_counts[e]`` is expert e's number of routes over a calibration
    batch.  Every rank keeps ``E/world`` experts (the slots
    [g*E/world, (g+1)*E/world)).  An expert's cost is its count of
    ``tile_rows``-row tiles, because the grouped GEMM decodes an expert's
    weights once per 128-row tile of its routes; ties go by route count.
    Experts are placed longest first, each onto the least-loaded rank that
    still has a free slot (longest-processing-time greedy).  Returns
    ``slot[e]``, the slot expert e occupies.
    """
    counts = [int(c) for c in route_counts]
    E = len(counts)
    if world < 1 or E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    epr = E // world
    cost = [((c + tile_rows - 1) // tile_rows, c) for c in counts]
    order = sorted(range(E), key=lambda e: (cost[e][0], cost[e][1], -e), reverse=True)
    load = [(0, 0)] * world
    held = [[] for _ in range(world)]
    for e in order:
        g = min((q for q in range(world) if len(held[q]) < epr), key=lambda q: (load[q], q))
        held[g].append(e)
        load[g] = (load[g][0] + cost[e][0], load[g][1] + cost[e][1])
    slot = [0] * E
    for g in range(world):
        for j, e in enumerate(sorted(held[g])):
            slot[e] = g * epr + j
    return slot


def _layer_device(layer):
    """The device of a routed-expert layer's weights, or None when its
    experts are not torch tensors."""
    try:
        t = layer._exl3_inners[0]["down"].trellis
    except (AttributeError, IndexError, KeyError, TypeError):
        return None
    return t.device if isinstance(t, torch.Tensor) else None


def experts_of_rank(placement, world: int, rank: int) -> list[int]:
    """The global expert ids rank ``rank`` holds, in its local-id order
    (local id j is slot rank*E/world + j)."""
    E = len(placement)
    epr = E // world
    inv = [0] * E
    for e, s in enumerate(placement):
        inv[int(s)] = e
    return inv[rank * epr:(rank + 1) * epr]


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

    ``placement`` (``n_global`` ints, a permutation, the same on every rank):
    expert e sits in slot ``placement[e]``; this rank's local expert j is
    the one in slot ``rank*n_global/world + j`` (:func:`experts_of_rank`).
    None keeps expert e in slot e.
    """

    def __init__(self, local_layer, n_global: int, group=None, combine_dtype: torch.dtype = torch.float32,
                 ops=None, capacity: int | None = None, transport: str = "nccl", placement=None):
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
        self._slot = None
        self._slot_dev: dict = {}
        if placement is not None:
            slot = [int(v) for v in placement]
            if sorted(slot) != list(range(self.n_global)):
                raise ValueError(f"placement must be a permutation of the {self.n_global} expert ids")
            self._slot = torch.tensor(slot, dtype=torch.int64)
            # the slot table goes to the layer's GPU now, so a first step
            # inside a CUDA-graph capture needs no host copy
            dev = _layer_device(local_layer)
            if dev is not None and dev.type == "cuda":
                for dt in (torch.int64, torch.int32):
                    self._slot_dev[(dev, dt)] = self._slot.to(device=dev, dtype=dt)
        self.combine_dtype = combine_dtype
        self.ops = ops if ops is not None else NativeEpOps()
        if capacity is not None and capacity < 1:
            raise ValueError("capacity must be a positive row count")
        self.capacity = None if capacity is None else int(capacity)
        if transport not in ("nccl", "nvlink"):
            raise ValueError("transport must be 'nccl' or 'nvlink'")
        if transport == "nvlink" and (self.capacity is None or ops is not None):
            raise ValueError("the NVLink transport needs a capacity and the native kernels")
        self.transport = transport
        self._win: NvlinkEpWindow | None = None
        self._pair_idx = None
        self._partial = None
        self.last_counts: tuple[list[int], list[int]] | None = None
        self.profile = False  # record CUDA events between the step's phases (benchmarks)
        self._events: list = []
        # NVLink transport: the window's status word, copied to pinned host
        # memory at the end of every step (asynchronously, so it also works
        # inside a captured graph); a nonzero value means a bounded peer wait
        # gave up in that step, whose output and every later step's are then
        # invalid, so the next forward() raises
        self._status_host: torch.Tensor | None = None
        self._status_dev: torch.Tensor | None = None

    PHASES = ("dispatch", "counts", "exchange", "local", "return", "combine")
    # NVLink transport: dispatch stores rows into the owners' windows,
    # "arrive" waits for every peer's rows, "return" stores the partial rows
    # back and waits for the peers' partial rows
    NVLINK_PHASES = ("dispatch", "arrive", "local", "return", "combine")

    @property
    def phases(self) -> tuple:
        return self.NVLINK_PHASES if self.transport == "nvlink" else self.PHASES

    def _mark(self) -> None:
        if self.profile:
            # inside a CUDA-graph capture the marks become event-record nodes,
            # so a replay of the captured step times its own phases
            ev = torch.cuda.Event(enable_timing=True, external=torch.cuda.is_current_stream_capturing())
            ev.record()
            self._events.append(ev)

    def phase_ms(self) -> dict:
        """Milliseconds of each phase of the last profiled step (synchronises)."""
        ev = self._events
        names = self.phases
        if len(ev) != len(names) + 1:
            return {}
        ev[-1].synchronize()
        return {n: ev[i].elapsed_time(ev[i + 1]) for i, n in enumerate(names)}

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
        if self._slot is not None:
            ids = self._relabel(ids)
        if self.transport == "nvlink":
            return self._forward_nvlink(x, ids, w, limit, n_valid, out)
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

    def _relabel(self, ids: torch.Tensor) -> torch.Tensor:
        """Global expert ids -> slots; ids outside [0, n_global) pass
        through, so the dispatch treats them as before."""
        key = (ids.device, ids.dtype)
        slot = self._slot_dev.get(key)
        if slot is None:
            if ids.is_cuda and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("the expert placement table is not on this device yet: "
                                   "run one step outside the CUDA-graph capture first")
            slot = self._slot.to(device=ids.device, dtype=ids.dtype)
            self._slot_dev[key] = slot
        n = self.n_global
        valid = (ids >= 0) & (ids < n)
        return torch.where(valid, slot[ids.clamp(0, n - 1)], ids)

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

    def _raise_on_status(self, status: int) -> None:
        if status:
            raise RuntimeError(
                f"expert-parallel NVLink exchange failed on rank {self.rank}: device status {status} "
                "(4 = a peer's rows or partial rows did not arrive within the wait budget); this step's "
                "output and every later step's are invalid -- close this group and build a new one")

    def check_status(self) -> None:
        """Synchronise this rank's stream and raise if any step so far
        recorded a failure in the window's status word (the word is kept, so
        every later call raises too)."""
        if self._win is not None:
            self._raise_on_status(self._win.status(clear=False))

    def window(self, x_dtype: torch.dtype, topk: int, hidden: int) -> NvlinkEpWindow:
        """The NVLink window, created on first use (every rank must call it
        at the same point: the IPC handles are exchanged collectively)."""
        if self._win is None:
            dev = torch.device("cuda", torch.cuda.current_device())
            self._win = NvlinkEpWindow(self.world, self.rank, self.capacity, hidden, topk, x_dtype,
                                       self.combine_dtype, dev, group=self.group)
            self._pair_idx = torch.empty(self.capacity, self.world, dtype=torch.int32, device=dev)
            self._partial = torch.empty(self.world * self.capacity, hidden, dtype=self.combine_dtype, device=dev)
            self._status_dev = self._win.status_tensor()
            self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        return self._win

    def _forward_nvlink(self, x, ids, w, limit, n_valid, out):
        T, H = x.shape
        G, C = self.world, self.capacity
        if T > C:
            raise ValueError(f"{T} tokens exceed the exchange capacity {C}")
        topk = ids.shape[1]
        win = self.window(x.dtype, topk, H)
        # an earlier step (its status copy has landed by the time the host
        # gets here again in all but the last few steps in flight) failed
        self._raise_on_status(int(self._status_host[0]))
        lib = win.lib
        stream = _n.stream_of(x)
        if out is None:
            out = torch.empty(T, H, dtype=x.dtype, device=x.device)
        _n.require_cuda(x, ids, w, n_valid, out, who="expert-parallel NVLink step")
        pc, xc = win.p_code, win.x_code
        self._mark()
        _n.check(lib.exl3_ep_p2p_dispatch(
            x.data_ptr(), xc, T, H, ids.data_ptr(), _n.dtype_code(ids), w.data_ptr(), _n.dtype_code(w), topk,
            self.n_global, G, self.rank, C, _n.ptr(n_valid), win.window, win.peers.data_ptr(), pc,
            self._pair_idx.data_ptr(), stream), "exl3_ep_p2p_dispatch")
        self._mark()
        _n.check(lib.exl3_ep_p2p_wait(win.window, G, 0, stream), "exl3_ep_p2p_wait")
        self._mark()
        moe_forward_ptrs(self.layer, x.device, win.recv_x, xc, G * C, win.recv_ids, _n.DT_I32, win.recv_w,
                         _n.DT_F32, topk, self._partial.data_ptr(), pc, limit)
        self._mark()
        _n.check(lib.exl3_ep_p2p_return(self._partial.data_ptr(), pc, G, self.rank, C, H, topk, xc, win.window,
                                        win.peers.data_ptr(), stream), "exl3_ep_p2p_return")
        _n.check(lib.exl3_ep_p2p_wait(win.window, G, 1, stream), "exl3_ep_p2p_wait")
        self._mark()
        _n.check(lib.exl3_ep_p2p_combine(win.window, G, self.rank, C, H, topk, xc, pc, self._pair_idx.data_ptr(),
                                         T, _n.ptr(n_valid), out.data_ptr(), _n.dtype_code(out), stream),
                 "exl3_ep_p2p_combine")
        self._status_host.copy_(self._status_dev, non_blocking=True)
        self._mark()
        return out

    def close(self) -> None:
        """Unmap the peers' windows and free this rank's (call on every rank,
        after the last step; ranks synchronise first so no peer is still
        writing)."""
        if self._win is not None:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            self._win.close()
            self._win = None

    apply = forward

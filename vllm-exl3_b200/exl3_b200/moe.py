"""Host-side mirror of the reference's routed-expert dispatch for this path.

Same names, argument meaning and error behaviour as the reference
(vcruz305/vllm-exl3 src/vllm_exl3/exl3.py):

* :func:`map_topk_to_local` / :func:`pin_exl3_expert_map` -- exl3.py:2310-2354;
* :func:`build_exl3_fused_state` -- the nine int64 pointer tables and the
  per-expert K arrays (exl3.py:2443-2682), here int8 as the native mixed-K
  entry takes them;
* :func:`apply_exl3_experts` -- exl3.py:3602-3703, except that every backend
  choice resolves to ONE native call over all tokens (no per-row host loop,
  no fallback: a failure raises);
* :class:`Exl3Projection` -- the attributes of ExLlamaV3's ``LinearEXL3`` the
  path reads (trellis, suh, svh, K, in/out features) and ``forward``;
* :class:`Exl3RoutedExperts` -- a minimal layer holding ``_exl3_inners`` and
  the fused state, with ``apply(x, topk_weights, topk_ids)`` as
  ``Exl3MoEMethod.apply`` (exl3.py:5120-5144).
"""

from __future__ import annotations

import math

import torch

from . import _native as _n

EXL3_MCG_MARKER = -877912083   # exl3.py:113-116
EXL3_MUL1_MARKER = -2082680531


def map_topk_to_local(ids: torch.Tensor, n_local: int, expert_map: torch.Tensor | None) -> torch.Tensor:
    """ids (T, K) global expert ids -> local ids; invalid/non-local -> n_local."""
    flat = ids.reshape(-1)
    if expert_map is None:
        invalid = (flat < 0) | (flat >= n_local)
        return torch.where(invalid, flat.new_full(flat.shape, n_local), flat)
    if expert_map.device != flat.device or expert_map.dtype != torch.long:
        raise RuntimeError(
            "EXL3 expert_map is not pinned to the hidden-state device; "
            "call pin_exl3_expert_map before fused apply (CUDA graphs forbid the copy)")
    n_global = int(expert_map.numel())
    safe = flat.clamp(min=0, max=max(n_global - 1, 0))
    mapped = expert_map[safe] if n_global else flat.new_full(flat.shape, n_local)
    invalid = (flat < 0) | (flat >= n_global) | (mapped < 0) | (mapped >= n_local)
    return torch.where(invalid, flat.new_full(flat.shape, n_local), mapped)


def pin_exl3_expert_map(layer, device: torch.device) -> torch.Tensor | None:
    """Move expert_map onto `device` once (int64, as the reference) and keep an
    int32 twin for the native entry."""
    emap = getattr(layer, "expert_map", None)
    if emap is None:
        return None
    cached = getattr(layer, "_exl3_pinned_expert_map", None)
    if (getattr(layer, "_exl3_raw_expert_map_id", None) == id(emap) and cached is not None
            and cached.device == device and cached.dtype == torch.long):
        return cached
    pinned = emap.to(device=device, dtype=torch.long)
    layer._exl3_pinned_expert_map = pinned
    layer._exl3_pinned_expert_map_i32 = pinned.to(torch.int32).contiguous()
    layer._exl3_raw_expert_map_id = id(emap)
    return pinned


class Exl3Projection:
    """One EXL3 projection resident on the GPU."""

    def __init__(self, trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor,
                 codebook: int = _n.CB_MCG):
        if trellis.dim() != 3 or trellis.dtype != torch.int16 or trellis.shape[-1] % 16:
            raise ValueError("EXL3 trellis must be int16 [in/16, out/16, 16*K]")
        self.trellis = trellis.contiguous()
        self.suh = suh.to(torch.float16).contiguous()
        self.svh = svh.to(torch.float16).contiguous()
        self.K = int(trellis.shape[-1]) // 16   # exl3.py:2554
        self.codebook = int(codebook)
        self.in_features = int(trellis.shape[0]) * 16
        self.out_features = int(trellis.shape[1]) * 16

    def forward(self, x: torch.Tensor, params: dict | None = None, out_dtype=None) -> torch.Tensor:
        import vllm_exl3_c
        return vllm_exl3_c.exl3_linear(x, self.trellis, self.suh, self.svh, self.K, self.codebook,
                                       out_dtype=out_dtype or x.dtype)


def build_exl3_fused_state(layer, inners: list[dict]) -> None:
    """Pointer tables + per-expert K tables, once after load (no per-token alloc).

    Gateless layers (every expert's "gate" is None: non-gated relu^2,
    exl3.py:2455-2491) alias the up tables into the gate slots, as the
    reference does, and select the relu^2 activation; the kernels never read
    the gate tables then."""
    if not inners:
        raise ValueError("EXL3 experts were not built after weight load")
    device = inners[0]["up"].trellis.device
    gateless = all(pack.get("gate") is None for pack in inners)
    if not gateless and any(pack.get("gate") is None for pack in inners):
        raise ValueError("EXL3 gateless layer must not carry gate projections")
    projs = ("up", "down") if gateless else ("gate", "up", "down")
    cbs = {pack[p].codebook for pack in inners for p in projs}
    if len(cbs) != 1:
        raise ValueError("EXL3 layer mixes codebooks across experts")

    def _ptrs(which: str, attr: str) -> torch.Tensor:
        return torch.tensor([int(getattr(pack[which], attr).data_ptr()) for pack in inners],
                            dtype=torch.int64, device=device)

    src = {"gate": "up" if gateless else "gate", "up": "up", "down": "down"}
    layer._exl3_ptrs = {
        f"{p}_{a}": _ptrs(src[p], a) for p in ("gate", "up", "down") for a in ("trellis", "suh", "svh")
    }
    layer._exl3_ptrs.update({
        f"{p}_{'t' if a == 'trellis' else a}_ptrs": layer._exl3_ptrs[f"{p}_{a}"]
        for p in ("gate", "up", "down") for a in ("trellis", "suh", "svh")
    })

    def _k(which: str) -> torch.Tensor:
        return torch.tensor([int(pack[src[which]].trellis.shape[-1]) // 16 for pack in inners],
                            dtype=torch.int8, device=device)

    kg, ku, kd = _k("gate"), _k("up"), _k("down")
    ks = {int(pack[p].K) for pack in inners for p in projs}
    if min(ks) < 2 or max(ks) > 8:
        raise ValueError(f"EXL3 K outside 2..8: {sorted(ks)}")
    layer._exl3_k_tables = (kg, ku, kd)
    layer._exl3_k_max_launch = max(ks)
    layer._exl3_mixed_k = len(ks) > 1
    layer._exl3_k = None if layer._exl3_mixed_k else next(iter(ks))
    layer._exl3_codebook = next(iter(cbs))
    layer._exl3_gateless = gateless
    if gateless:
        layer._exl3_moe_act = _n.ACT_RELU2
    elif getattr(layer, "_exl3_moe_act", _n.ACT_SILU) == _n.ACT_RELU2:
        raise ValueError("EXL3 relu^2 (non-gated) activation on a layer with gate projections")


def apply_exl3_experts(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, layer,
                       *, limit: float | None = None, fused: bool | None = None,
                       n_valid: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed-expert apply: all tokens of the step in one native call.

    ``limit`` > 0 clamps gate from above and up on both sides before the
    activation (exl3.py:2404-2409); None or <= 0 disables it.  Returns the
    routed contribution in ``x.dtype`` (exl3.py:3703).
    """
    import vllm_exl3_c

    del fused  # every backend resolves to the single native path
    inners = getattr(layer, "_exl3_inners", None)
    if not inners:
        raise RuntimeError("EXL3 experts were not built after weight load")
    if getattr(layer, "_exl3_ptrs", None) is None:
        build_exl3_fused_state(layer, inners)
    tokens, hidden = x.shape[-2], x.shape[-1]
    x2d = x.reshape(tokens, hidden)
    ids = topk_ids.reshape(tokens, -1)
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.long)
    weights = topk_weights.reshape(tokens, -1)
    if weights.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        weights = weights.float()
    pin_exl3_expert_map(layer, x2d.device)
    emap = getattr(layer, "_exl3_pinned_expert_map_i32", None) if getattr(layer, "expert_map", None) is not None else None
    if out is None:
        out = torch.empty((tokens, hidden), dtype=x.dtype, device=x.device)
    lim = 0.0 if limit is None or not (limit > 0) else float(limit)
    if not math.isfinite(lim):
        raise RuntimeError("EXL3 SwiGLU limit must be finite")
    p = layer._exl3_ptrs
    kg, ku, kd = layer._exl3_k_tables
    vllm_exl3_c.exl3_moe(
        x2d, out, p["gate_trellis"], p["gate_suh"], p["gate_svh"], p["up_trellis"], p["up_suh"],
        p["up_svh"], p["down_trellis"], p["down_suh"], p["down_svh"], ids, weights,
        k_gate_tbl=kg, k_up_tbl=ku, k_down_tbl=kd, n_local=len(inners),
        intermediate_size=int(layer._exl3_intermediate_local), swiglu_limit=lim,
        expert_map=emap, n_valid=n_valid, kmax=int(layer._exl3_k_max_launch),
        codebook=int(layer._exl3_codebook), activation=int(getattr(layer, "_exl3_moe_act", 0)))
    layer._exl3_last_apply = "b200"
    return out.view(*x.shape[:-1], hidden)


def moe_forward_ptrs(layer, device: torch.device, x_ptr: int, x_dtype: int, tokens: int, ids_ptr: int,
                     ids_dtype: int, w_ptr: int, w_dtype: int, topk: int, out_ptr: int, out_dtype: int,
                     limit: float | None = None) -> None:
    """The layer's fused forward on raw device buffers (dtype codes of the C
    ABI): rows that live outside torch, e.g. an expert-parallel window."""
    lib = _n.load()
    inners = getattr(layer, "_exl3_inners", None)
    if not inners:
        raise RuntimeError("EXL3 experts were not built after weight load")
    if getattr(layer, "_exl3_ptrs", None) is None:
        build_exl3_fused_state(layer, inners)
    lim = 0.0 if limit is None or not (limit > 0) else float(limit)
    hidden = int(layer._exl3_hidden_size)
    inter = int(layer._exl3_intermediate_local)
    kmax = int(layer._exl3_k_max_launch)
    with torch.cuda.device(device):
        need = lib.exl3_moe_workspace_size(tokens, topk, hidden, inter, len(inners), kmax)
        if need == 0:
            raise RuntimeError("fused MoE: unsupported geometry")
        ws = _n.workspace(device, need)
        p = layer._exl3_ptrs
        kg, ku, kd = layer._exl3_k_tables
        tables = [p[k] for k in ("gate_trellis", "gate_suh", "gate_svh", "up_trellis", "up_suh", "up_svh",
                                 "down_trellis", "down_suh", "down_svh")]
        _n.check(lib.exl3_moe_forward(
            x_ptr, x_dtype, tokens, hidden, inter, *[t.data_ptr() for t in tables], ids_ptr, ids_dtype, w_ptr,
            w_dtype, topk, None, 0, _n.ptr(kg), _n.ptr(ku), _n.ptr(kd), 0, kmax, len(inners),
            int(layer._exl3_codebook), int(getattr(layer, "_exl3_moe_act", 0)), lim, None, out_ptr, out_dtype,
            ws.data_ptr(), ws.numel(), torch.cuda.current_stream(device).cuda_stream), "fused MoE")


class Exl3RoutedExperts(torch.nn.Module):
    """Minimal routed-expert layer: EXL3 experts + fused state + apply."""

    def __init__(self, inners: list[dict], hidden: int, intermediate: int,
                 expert_map: torch.Tensor | None = None, act: int = _n.ACT_SILU):
        super().__init__()
        self._exl3_inners = inners
        self._exl3_hidden_size = int(hidden)
        self._exl3_intermediate_local = int(intermediate)
        self._exl3_moe_act = int(act)
        self.expert_map = expert_map
        self._exl3_ptrs = None
        build_exl3_fused_state(self, inners)

    def apply(self, x, topk_weights, topk_ids, limit: float | None = None, **kw):
        return apply_exl3_experts(x, topk_ids, topk_weights, self, limit=limit, **kw)

    forward = apply


def upload_experts(experts, device) -> list[dict]:
    """GPU projections of synthetic experts ({"gate", "up", "down"} dicts of
    :class:`exl3_b200.synthetic.Projection`; "gate" may be None)."""
    inners = []
    for e in experts:
        d = {}
        for which in ("gate", "up", "down"):
            p = e.get(which)
            d[which] = None if p is None else Exl3Projection(
                torch.from_numpy(p.trellis).to(device), torch.from_numpy(p.suh).to(device),
                torch.from_numpy(p.svh).to(device), p.codebook)
        inners.append(d)
    return inners


def layer_from_pack(pack, device, expert_map: torch.Tensor | None = None, act: int = _n.ACT_SILU
                    ) -> Exl3RoutedExperts:
    """Upload a :class:`exl3_b200.synthetic.MoEPack` and build its layer."""
    return Exl3RoutedExperts(upload_experts(pack.experts, device), pack.hidden, pack.inter,
                             expert_map=expert_map, act=act)


def layer_from_slices(make_slice, n_experts: int, hidden: int, inter: int, device, chunk: int = 32,
                      act: int = _n.ACT_SILU) -> Exl3RoutedExperts:
    """A layer built ``chunk`` experts at a time from ``make_slice(lo, hi)``
    (a :class:`exl3_b200.synthetic.MoEPack` of experts [lo, hi)), so the host
    never holds every expert of a large layer at once."""
    inners = []
    for lo in range(0, n_experts, chunk):
        inners += upload_experts(make_slice(lo, min(n_experts, lo + chunk)).experts, device)
    return Exl3RoutedExperts(inners, hidden, inter, act=act)

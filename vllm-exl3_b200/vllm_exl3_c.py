"""Drop-in replacement for the reference's native module ``vllm_exl3_c``.

The reference plugin locates its extension with
``importlib.import_module("vllm_exl3_c")`` and accepts it when
``p2b_fused_moe`` is callable (vcruz305/vllm-exl3 src/vllm_exl3/exl3.py:2147-2153).
This module keeps the reference's pybind names, argument order, defaults,
error texts and capability attributes (csrc/bindings.cpp:197-266) and runs
every entry on the B200 kernels of ``libexl3_b200.so`` through its C ABI
(``include/exl3_b200.h``).  Put ``vllm-exl3_b200/`` on ``sys.path`` (or
install it) ahead of any other ``vllm_exl3_c``.

Differences from the reference, all supersets:
* every entry accepts both codebooks (the reference's p2b kernels are built
  for one, selected at compile time by ``-DP2B_CB``);
* ``exl3_gemv`` runs any K in 2..8; ``exl3_gemm`` any row count in one launch;
* ``exl3_moe`` (new) runs all tokens of a step in one call.
There is no CPU path: CUDA tensors are required (``dequant_trellis`` on CPU
tensors raises), because the product has no CPU fallback.
"""

from __future__ import annotations

import math

import torch

from exl3_b200 import _native as _n

# capability attributes read by the plugin (bindings.cpp:243-257, exl3.py:2813-2823)
P2B_MOE_ABI_VERSION = 4
P2B_MOE_MIXED_K = True
P2B_MOE_PADDED = True
# new capabilities of this implementation
EXL3_B200 = True
EXL3_MOE_BATCHED = True


def _cb(mcg: bool) -> int:
    return _n.CB_MCG if bool(mcg) else _n.CB_MUL1


def _packed_dims(trellis: torch.Tensor, K: int) -> tuple[int, int]:
    if trellis.dim() != 3 or trellis.dtype != torch.int16:
        raise RuntimeError("trellis must be int16 [rows/16, cols/16, 16*K]")
    if trellis.size(2) != 16 * int(K):
        raise RuntimeError("trellis last dimension must be 16*K")
    if trellis.size(0) <= 0 or trellis.size(1) <= 0:
        raise RuntimeError("trellis dimensions must be positive")
    return int(trellis.size(0)) * 16, int(trellis.size(1)) * 16


def dequant_trellis(trellis, suh, svh, K, mcg):
    """Decode an EXL3 trellis tensor into an fp16 weight matrix (bit-exact with
    the reference's CPU dequant, csrc/bindings.cpp:117-132)."""
    K = int(K)
    if K not in (2, 3, 4, 8):
        raise RuntimeError("K must be one of 2, 3, 4, or 8")
    return exl3_reconstruct(trellis, suh, svh, K, _cb(mcg))


def exl3_reconstruct(trellis, suh, svh, K, codebook=_n.CB_MCG):
    """W = diag(suh) H W~ H diag(svh) / 128 as fp16 [in, out]; K in 2..8."""
    rows, cols = _packed_dims(trellis, K)
    if suh.dtype != torch.float16 or svh.dtype != torch.float16:
        raise RuntimeError("suh and svh must be float16")
    if suh.numel() < rows or svh.numel() < cols:
        raise RuntimeError("suh/svh are too short")
    _n.require_cuda(trellis, suh, svh, who="dequant_trellis")
    t, u, v = trellis.contiguous(), suh.contiguous(), svh.contiguous()
    out = torch.empty((rows, cols), dtype=torch.float16, device=t.device)
    with torch.cuda.device(t.device):
        _n.check(_n.load().exl3_reconstruct(t.data_ptr(), u.data_ptr(), v.data_ptr(), rows, cols,
                                            int(K), int(codebook), out.data_ptr(), _n.stream_of(t)))
    return out


def exl3_decode_raw(trellis, K, codebook=_n.CB_MCG):
    """The decoded, un-rotated W~ as fp16 [in, out] (ExLlamaV3 ``reconstruct``)."""
    rows, cols = _packed_dims(trellis, K)
    _n.require_cuda(trellis, who="exl3_decode_raw")
    t = trellis.contiguous()
    out = torch.empty((rows, cols), dtype=torch.float16, device=t.device)
    with torch.cuda.device(t.device):
        _n.check(_n.load().exl3_decode_raw(t.data_ptr(), rows, cols, int(K), int(codebook),
                                           out.data_ptr(), _n.stream_of(t)))
    return out


def had_r_128(input, output, pre_scale, post_scale, scale=1.0):
    """ExLlamaV3 ``had_r_128`` semantics: output = fp16(H128(input o pre) /
    sqrt(128) o post * scale) per 128-column block; output may alias input."""
    _n.require_cuda(input, output, pre_scale, post_scale, who="had_r_128")
    if input.dtype != torch.float16 or output.dtype != torch.float16:
        raise RuntimeError("had_r_128 requires fp16 tensors")
    if not (input.is_contiguous() and output.is_contiguous()) or input.shape != output.shape:
        raise RuntimeError("had_r_128 input/output must be contiguous and the same shape")
    n = int(input.shape[-1])
    rows = input.numel() // max(n, 1)
    pre = pre_scale.contiguous() if pre_scale is not None else None
    post = post_scale.contiguous() if post_scale is not None else None
    with torch.cuda.device(input.device):
        _n.check(_n.load().exl3_had128(input.data_ptr(), output.data_ptr(), rows, n, _n.ptr(pre),
                                       _n.ptr(post), float(scale), _n.stream_of(input)))
    return output


exl3_had128 = had_r_128


def exl3_linear(x, trellis, suh, svh, K, codebook=_n.CB_MCG, out_dtype=None):
    """y[m, out] = x[m, in] W for any m (one launch), x cast to fp16 first."""
    rows_in, cols = _packed_dims(trellis, K)
    _n.require_cuda(x, trellis, suh, svh, who="exl3_linear")
    if x.size(-1) != rows_in:
        raise RuntimeError("x feature dimension does not match trellis")
    x2 = x.contiguous().view(-1, rows_in)
    m = int(x2.size(0))
    y = torch.empty((m, cols), dtype=out_dtype or x.dtype, device=x.device)
    lib = _n.load()
    with torch.cuda.device(x.device):
        need = lib.exl3_linear_workspace_size(m, rows_in, cols, int(K))
        ws = _n.workspace(x.device, need)
        t, u, v = trellis.contiguous(), suh.contiguous(), svh.contiguous()
        _n.check(lib.exl3_linear(x2.data_ptr(), _n.dtype_code(x2), m, t.data_ptr(), u.data_ptr(),
                                 v.data_ptr(), rows_in, cols, int(K), int(codebook), y.data_ptr(),
                                 _n.dtype_code(y), ws.data_ptr(), ws.numel(), _n.stream_of(x)))
    return y.view(*x.shape[:-1], cols)


def exl3_gemv(x, trellis, suh, svh, K, mcg, mmode=1):
    """Native small-m EXL3 GEMV (csrc/bindings.cpp:134-147): 1 <= m <= 8."""
    if x.dim() < 2:
        raise RuntimeError("x must have shape [..., in_features]")
    m = x.numel() // x.size(-1)
    if not (1 <= m <= 8):
        raise RuntimeError("native GEMV supports 1 <= m <= 8")
    if x.size(-1) != trellis.size(0) * 16:
        raise RuntimeError("x feature dimension does not match trellis")
    if int(mmode) not in (0, 1):
        raise RuntimeError("mmode must be 0 or 1")
    if not x.is_cuda or x.dtype != torch.float16:
        raise RuntimeError("CUDA GEMV requires fp16 input")
    return exl3_linear(x.contiguous().view(m, x.size(-1)), trellis, suh, svh, K, _cb(mcg))


def exl3_gemm(x, trellis, suh, svh, K, mcg):
    """Native tiled EXL3 GEMM (csrc/exl3_gemm.cu:9-31), any row count."""
    if not x.is_cuda or x.dtype != torch.float16:
        raise RuntimeError("GEMM requires CUDA fp16 input")
    x2 = x.contiguous().view(x.numel() // x.size(-1), x.size(-1))
    return exl3_linear(x2, trellis, suh, svh, K, _cb(mcg))


def p2b_gemv_batched(x, trellis_ptrs, suh_ptrs, svh_ptrs, expert_indices, K, mcg, mmode=1,
                     out_features=2048):
    """Batched MoE EXL3 GEMV (csrc/bindings.cpp:149-156): one shared input
    x [m, in] against each listed expert; returns [n_active, m, out_features]
    (the reference fixes out_features = 2048)."""
    if not x.is_cuda or x.dtype != torch.float16:
        raise RuntimeError("batched GEMV requires CUDA fp16")
    for t in (trellis_ptrs, suh_ptrs, svh_ptrs, expert_indices):
        if not t.is_cuda:
            raise RuntimeError("batched GEMV requires CUDA tensors")
    if int(K) not in range(2, 9):
        raise RuntimeError("batched GEMV supports K in 2..8")
    if int(mmode) not in (0, 1):
        raise RuntimeError("mmode must be 0 or 1")
    x2 = x.contiguous().view(-1, x.size(-1))
    m, in_f = int(x2.size(0)), int(x2.size(1))
    idx = expert_indices.to(torch.int32).contiguous().view(-1)
    n_active = int(idx.numel())
    tabs = [t.contiguous() for t in (trellis_ptrs, suh_ptrs, svh_ptrs)]
    y = torch.zeros((n_active, m, int(out_features)), dtype=torch.float16, device=x.device)
    if n_active == 0:
        return y
    lib = _n.load()
    with torch.cuda.device(x.device):
        need = lib.exl3_batched_linear_workspace_size(m, n_active, in_f, int(out_features),
                                                      int(tabs[0].numel()), int(K))
        if need == 0:
            raise RuntimeError("batched GEMV: unsupported geometry")
        ws = _n.workspace(x.device, need)
        _n.check(lib.exl3_batched_linear(
            x2.data_ptr(), _n.DT_F16, m, tabs[0].data_ptr(), tabs[1].data_ptr(), tabs[2].data_ptr(),
            int(tabs[0].numel()), idx.data_ptr(), n_active, in_f, int(out_features), int(K), _cb(mcg),
            y.data_ptr(), _n.DT_F16, ws.data_ptr(), ws.numel(), _n.stream_of(x)), "batched GEMV")
    return y


def _fat_checks(a, packed, out, svh, K, mcg, mul1):
    if not (a.is_cuda and packed.is_cuda and out.is_cuda and svh.is_cuda):
        raise RuntimeError("exl3_fat_gemm tensors must be CUDA tensors")
    if not (a.is_contiguous() and packed.is_contiguous() and out.is_contiguous() and svh.is_contiguous()):
        raise RuntimeError("exl3_fat_gemm tensors must be contiguous")
    if a.dtype != torch.float16:
        raise RuntimeError("a must be float16")
    if packed.dtype != torch.int16:
        raise RuntimeError("packed must be int16")
    if out.dtype != torch.float32:
        raise RuntimeError("out must be float32")
    if svh.dtype != torch.float16:
        raise RuntimeError("svh must be float16")
    if a.dim() != 2 or packed.dim() != 3 or out.dim() != 2 or svh.dim() != 1:
        raise RuntimeError("exl3_fat_gemm expects rank-2/rank-3 tensors")
    if bool(mcg) and bool(mul1):
        raise RuntimeError("exl3_fat_gemm: mcg and mul1 are exclusive")
    if a.size(1) != packed.size(0) * 16:
        raise RuntimeError("a K dimension does not match packed tensor")
    if svh.numel() != packed.size(1) * 16:
        raise RuntimeError("svh N dimension does not match packed tensor")
    if svh.numel() % 128:
        raise RuntimeError("output dimension must be divisible by 128")
    if packed.size(2) != 16 * int(K):
        raise RuntimeError("packed block width must be 16*K int16 words")
    if len({a.device, packed.device, out.device, svh.device}) != 1:
        raise RuntimeError("exl3_fat_gemm tensors must share a device")
    return _n.CB_MCG if mcg else (_n.CB_MUL1 if mul1 else _n.CB_3INST)


def _fat_call(a, packed, out, svh, K, cb, token_idx=None, route_weight=None):
    m, in_f, n = int(a.size(0)), int(a.size(1)), int(svh.numel())
    lib = _n.load()
    with torch.cuda.device(a.device):
        need = lib.exl3_linear_workspace_size(max(m, 1), in_f, n, int(K))
        ws = _n.workspace(a.device, need)
        _n.check(lib.exl3_fat_gemm(a.data_ptr(), m, packed.data_ptr(), svh.data_ptr(), in_f, n, int(K),
                                   int(cb), out.data_ptr(), _n.ptr(token_idx), _n.ptr(route_weight),
                                   ws.data_ptr(), ws.numel(), _n.stream_of(a)), "exl3_fat_gemm")


def exl3_fat_gemm(a, packed, out, svh, K, mcg, mul1):
    """Prefill GEMM on a pre-rotated input (csrc/exl3_fat_gemm.cu:266-278):
    out [M, N] fp32 = (a W~) H/sqrt(128) o svh."""
    cb = _fat_checks(a, packed, out, svh, K, mcg, mul1)
    if out.size(0) != a.size(0) or out.size(1) != svh.numel():
        raise RuntimeError("out shape must be [M, N]")
    _fat_call(a, packed, out, svh, K, cb)


def exl3_fat_gemm_scatter(a, packed, out, svh, token_idx, route_weight, K, mcg, mul1):
    """Scatter variant (csrc/exl3_fat_gemm.cu:281-305): out[token_idx[r]] +=
    route_weight[r] * row r; rows of one call must target distinct tokens."""
    cb = _fat_checks(a, packed, out, svh, K, mcg, mul1)
    if out.size(1) != svh.numel():
        raise RuntimeError("out N dimension mismatch")
    if not (token_idx.is_cuda and route_weight.is_cuda):
        raise RuntimeError("routing tensors must be CUDA tensors")
    if not (token_idx.is_contiguous() and route_weight.is_contiguous()):
        raise RuntimeError("routing tensors must be contiguous")
    if token_idx.dtype != torch.int64:
        raise RuntimeError("token_idx must be int64")
    if route_weight.dtype != torch.float16:
        raise RuntimeError("route_weight must be float16")
    if token_idx.numel() != a.size(0) or route_weight.numel() != a.size(0):
        raise RuntimeError("routing tensors must have M elements")
    if token_idx.device != a.device or route_weight.device != a.device:
        raise RuntimeError("routing tensors must share a device with a")
    _fat_call(a, packed, out, svh, K, cb, token_idx, route_weight)


# ---------------------------------------------------------------------------
# routed-expert MoE
# ---------------------------------------------------------------------------
def _check_tables(who: str, x, tables, k_tables=None):
    gt = tables[0]
    for t in tables:
        if not isinstance(t, torch.Tensor) or t.dim() != 1 or t.dtype != torch.int64 \
                or t.numel() != gt.numel() or t.numel() == 0:
            raise RuntimeError(f"{who} pointer tables must be equally sized nonempty int64 vectors")
    for t in tables + list(k_tables or []):
        if t.device != x.device or not t.is_contiguous():
            raise RuntimeError(f"{who} tensors must be contiguous and on the input CUDA device")
    for t in k_tables or []:
        if t.dim() != 1 or t.dtype != torch.int8 or t.numel() != gt.numel():
            raise RuntimeError(
                f"{who} requires int8 CUDA K tables with one entry per pointer-table slot")


def _moe_call(who, x, out, tables, ids, rw, *, k_tables=None, k_uniform=0, kmax=8, n_local,
              codebook, intermediate, limit, expert_map=None, n_valid=None, act=_n.ACT_SILU):
    lib = _n.load()
    tokens, hidden = int(x.size(0)), int(x.size(1))
    topk = int(ids.size(-1)) if ids.dim() > 1 else int(ids.numel())
    with torch.cuda.device(x.device):
        need = lib.exl3_moe_workspace_size(tokens, topk, hidden, int(intermediate), int(n_local), int(kmax))
        if need == 0:
            raise RuntimeError(f"{who}: unsupported geometry")
        ws = _n.workspace(x.device, need)
        kg, ku, kd = (k_tables if k_tables is not None else (None, None, None))
        emap = expert_map
        if emap is not None:
            emap = emap.to(device=x.device, dtype=torch.int32).contiguous()
        rc = lib.exl3_moe_forward(
            x.data_ptr(), _n.dtype_code(x), tokens, hidden, int(intermediate),
            *[t.data_ptr() for t in tables],
            ids.data_ptr(), _n.dtype_code(ids), rw.data_ptr(), _n.dtype_code(rw), topk,
            _n.ptr(emap), int(emap.numel()) if emap is not None else 0,
            _n.ptr(kg), _n.ptr(ku), _n.ptr(kd), int(k_uniform), int(kmax), int(n_local),
            int(codebook), int(act), float(limit), _n.ptr(n_valid),
            out.data_ptr(), _n.dtype_code(out), ws.data_ptr(), ws.numel(), _n.stream_of(x))
        _n.check(rc, who)
    return out


def _limit(swiglu_limit: float, who: str) -> float:
    lim = float(swiglu_limit)
    if not math.isfinite(lim) or lim < 0:
        raise RuntimeError(f"{who} SwiGLU limit must be finite and nonnegative (0 disables clipping)")
    return lim


def _moe_common_checks(who, x, out, intermediate_size):
    if not x.is_cuda or x.dtype != torch.float16:
        raise RuntimeError(f"{who} requires CUDA fp16 input")
    if not out.is_cuda or out.dtype != torch.float16:
        raise RuntimeError(f"{who} output must be CUDA fp16")
    if out.shape != x.shape:
        raise RuntimeError(f"{who} output shape must match input")
    if x.size(-1) <= 0 or x.size(-1) % 128:
        raise RuntimeError(f"{who} hidden width must be a positive multiple of 128")
    if int(intermediate_size) <= 0 or int(intermediate_size) % 128:
        raise RuntimeError(f"{who} local intermediate width must be a positive multiple of 128")


def p2b_fused_moe(x, out, gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs,
                  up_suh_ptrs, up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs,
                  expert_indices, routing_weights, K_gate, K_up, K_down, mcg,
                  intermediate_size=2048, swiglu_limit=0.0):
    """Fused MoE decode for one token row (csrc/p2b_moe.cu:2431-2488)."""
    who = "fused MoE"
    _moe_common_checks(who, x, out, intermediate_size)
    if x.dim() != 2 or x.size(0) != 1:
        raise RuntimeError("fused MoE requires exactly one input row")
    lim = _limit(swiglu_limit, who)
    if not (int(K_gate) == int(K_up) == int(K_down) and int(K_gate) in (2, 3, 4)):
        raise RuntimeError("unsupported fused MoE K, or codebook mismatch")
    if expert_indices.dim() != 1 or expert_indices.dtype != torch.int32 or expert_indices.numel() == 0:
        raise RuntimeError("fused MoE expert indices must be a nonempty int32 routing vector")
    if routing_weights.dtype != torch.float16 or routing_weights.numel() != expert_indices.numel():
        raise RuntimeError("fused MoE requires one fp16 routing weight per expert index")
    tables = [gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs, up_suh_ptrs,
              up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs]
    _check_tables(who, x, tables)
    for t in (x, out, expert_indices, routing_weights):
        if t.device != x.device or not t.is_contiguous():
            raise RuntimeError("fused MoE tensors must be contiguous and on the input CUDA device")
    return _moe_call(who, x, out, tables, expert_indices.view(1, -1), routing_weights.view(1, -1),
                     k_uniform=int(K_gate), kmax=int(K_gate), n_local=tables[0].numel(),
                     codebook=_cb(mcg), intermediate=int(intermediate_size), limit=lim)


def p2b_fused_moe_mk(x, out, gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs,
                     up_suh_ptrs, up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs,
                     expert_indices, routing_weights, k_gate_tbl, k_up_tbl, k_down_tbl, n_local,
                     mcg, intermediate_size=2048, swiglu_limit=0.0):
    """Mixed-K fused MoE for one token row with int8 per-expert K tables and
    the n_local sentinel (csrc/p2b_moe.cu:1201-1265)."""
    who = "mixed-K fused MoE"
    _moe_common_checks(who, x, out, intermediate_size)
    if x.dim() != 2 or x.size(0) != 1:
        raise RuntimeError("mixed-K fused MoE requires exactly one input row")
    lim = _limit(swiglu_limit, who)
    if expert_indices.dim() != 1 or expert_indices.dtype != torch.int32 or expert_indices.numel() == 0:
        raise RuntimeError("mixed-K fused MoE expert indices must be a nonempty int32 routing vector")
    if routing_weights.dtype != torch.float16 or routing_weights.numel() != expert_indices.numel():
        raise RuntimeError("mixed-K fused MoE requires one fp16 routing weight per expert index")
    tables = [gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs, up_suh_ptrs,
              up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs]
    ktabs = [k_gate_tbl, k_up_tbl, k_down_tbl]
    _check_tables(who, x, tables, ktabs)
    if not (1 <= int(n_local) <= tables[0].numel()):
        raise RuntimeError(
            "mixed-K fused MoE n_local must bound the pointer tables (1 <= n_local <= table length)")
    return _moe_call(who, x, out, tables, expert_indices.view(1, -1), routing_weights.view(1, -1),
                     k_tables=ktabs, kmax=8, n_local=int(n_local), codebook=_cb(mcg),
                     intermediate=int(intermediate_size), limit=lim)


def p2b_fused_moe_padded(x, out, gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs,
                         up_suh_ptrs, up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs,
                         expert_indices_padded, routing_weights_padded, n_valid, k_gate_tbl,
                         k_up_tbl, k_down_tbl, n_local, max_k, mcg, intermediate_size=2048,
                         swiglu_limit=0.0):
    """Fixed-shape padded MoE: [MAX_T, MAX_K] routing grid, live rows counted
    on the device by ``n_valid`` (never read on the host); padded rows are
    written as zeros (csrc/p2b_moe.cu:2330-2428)."""
    who = "padded fused MoE"
    if not x.is_cuda or x.dtype != torch.float16:
        raise RuntimeError("padded fused MoE requires CUDA fp16 input")
    if not out.is_cuda or out.dtype != torch.float16:
        raise RuntimeError("padded fused MoE output must be CUDA fp16")
    if x.dim() != 2 or x.size(0) < 1:
        raise RuntimeError("padded fused MoE input must be a [MAX_T, hidden] matrix")
    _moe_common_checks(who, x, out, intermediate_size)
    lim = _limit(swiglu_limit, who)
    ids = expert_indices_padded
    if ids.dim() != 2 or ids.dtype != torch.int32 or ids.size(0) != x.size(0) or ids.size(1) < 1:
        raise RuntimeError(
            "padded fused MoE requires an int32 [MAX_T, MAX_K] routing grid whose rows match x")
    rw = routing_weights_padded
    if rw.dtype != torch.float16 or rw.shape != ids.shape:
        raise RuntimeError("padded fused MoE requires one fp16 routing weight per routing-grid slot")
    if not (n_valid.is_cuda and n_valid.dim() == 1 and n_valid.numel() == 1
            and n_valid.dtype == torch.int32 and n_valid.is_contiguous()
            and n_valid.device == x.device):
        raise RuntimeError(
            "padded fused MoE requires a contiguous int32 CUDA n_valid scalar tensor on x.device()")
    tables = [gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs, up_suh_ptrs,
              up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs]
    ktabs = [k_gate_tbl, k_up_tbl, k_down_tbl]
    _check_tables(who, x, tables, ktabs)
    if not (1 <= int(n_local) <= tables[0].numel()):
        raise RuntimeError(
            "padded fused MoE n_local must bound the pointer tables (1 <= n_local <= table length)")
    if int(max_k) != ids.size(1):
        raise RuntimeError("padded fused MoE max_k must equal the routing grid's column count")
    return _moe_call(who, x, out, tables, ids.contiguous(), rw.contiguous(), k_tables=ktabs,
                     kmax=8, n_local=int(n_local), codebook=_cb(mcg),
                     intermediate=int(intermediate_size), limit=lim, n_valid=n_valid)


def exl3_moe(x, out, gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs, up_suh_ptrs,
             up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs, topk_ids, topk_weights,
             k_gate_tbl=None, k_up_tbl=None, k_down_tbl=None, K=None, n_local=None, mcg=True,
             intermediate_size=2048, swiglu_limit=0.0, expert_map=None, n_valid=None, kmax=8,
             codebook=None, activation=_n.ACT_SILU):
    """All tokens of a step in one call (new).  x [T, hidden] fp16/bf16/fp32;
    out [T, hidden] any float dtype, written in place; topk_ids [T, k]
    int32/int64 global ids; topk_weights [T, k] float.  Per-expert int8 K
    tables (mixed-K) or a uniform ``K``."""
    who = "fused MoE"
    _n.require_cuda(x, out, topk_ids, topk_weights, who=who)
    if x.dim() != 2 or out.shape != x.shape:
        raise RuntimeError(f"{who} x/out must be matching [T, hidden] matrices")
    if topk_ids.shape != topk_weights.shape or topk_ids.dim() != 2 or topk_ids.size(0) != x.size(0):
        raise RuntimeError(f"{who} requires [T, k] routing ids and weights matching x")
    lim = _limit(swiglu_limit, who)
    tables = [gate_trellis_ptrs, gate_suh_ptrs, gate_svh_ptrs, up_trellis_ptrs, up_suh_ptrs,
              up_svh_ptrs, down_trellis_ptrs, down_suh_ptrs, down_svh_ptrs]
    ktabs = None if k_gate_tbl is None else [k_gate_tbl, k_up_tbl, k_down_tbl]
    _check_tables(who, x, tables, ktabs)
    if ktabs is None and K is None:
        raise RuntimeError(f"{who} needs per-expert K tables or a uniform K")
    nl = tables[0].numel() if n_local is None else int(n_local)
    if not (1 <= nl <= tables[0].numel()):
        raise RuntimeError(f"{who} n_local must bound the pointer tables")
    cb = _cb(mcg) if codebook is None else int(codebook)
    return _moe_call(who, x.contiguous(), out, tables, topk_ids.contiguous(),
                     topk_weights.contiguous(), k_tables=ktabs,
                     k_uniform=int(K) if K is not None else 0,
                     kmax=int(kmax) if ktabs is not None else int(K), n_local=nl, codebook=cb,
                     intermediate=int(intermediate_size), limit=lim, expert_map=expert_map,
                     n_valid=n_valid, act=int(activation))


def ngram_dequant(packed, bits, heads, head_bias, out):
    """ExLlamaV3 ``ngram_dequant`` semantics (the reference's call site
    src/vllm_exl3/exl3.py:5536-5544; pure-torch twin exl3.py:5213-5239):
    packed int16 [N, 1 + 10 * bits] rows, heads int [N], head_bias fp16
    [heads, 160] -> out [N, 160] (fp16, bf16 or fp32), written in place."""
    _n.require_cuda(packed, heads, head_bias, out, who="ngram_dequant")
    bits = int(bits)
    if not 1 <= bits <= 8:
        raise RuntimeError("ngram_dequant: bits must be in 1..8")
    if packed.dtype != torch.int16 or packed.dim() != 2 or packed.size(1) != 1 + 10 * bits:
        raise RuntimeError("ngram_dequant: packed must be int16 [N, 1 + 160 * bits / 16]")
    if head_bias.dtype != torch.float16 or head_bias.dim() != 2 or head_bias.size(1) != 160:
        raise RuntimeError("ngram_dequant: head_bias must be fp16 [heads, 160]")
    if out.shape != (packed.size(0), 160) or not out.is_contiguous():
        raise RuntimeError("ngram_dequant: out must be a contiguous [N, 160] tensor")
    h = heads.to(torch.int32).contiguous().view(-1)
    if h.numel() != packed.size(0):
        raise RuntimeError("ngram_dequant: one head per row")
    p, b = packed.contiguous(), head_bias.contiguous()
    with torch.cuda.device(packed.device):
        _n.check(_n.load().exl3_ngram_dequant(p.data_ptr(), int(p.size(0)), bits, h.data_ptr(), b.data_ptr(),
                                              int(b.size(0)), out.data_ptr(), _n.dtype_code(out),
                                              _n.stream_of(p)), "ngram_dequant")
    return out


def device_status(workspace=None, clear=True) -> int:
    """Device-side status word of a workspace (0 = clean).  Without one: the
    first nonzero word among every workspace of the current device (all
    streams; synchronises the device first)."""
    import ctypes

    lib = _n.load()
    if workspace is not None:
        spaces = [workspace]
    else:
        dev = torch.device("cuda", torch.cuda.current_device())
        torch.cuda.synchronize(dev)
        spaces = _n.device_workspaces(dev) or [_n.workspace(dev, 1 << 20)]
    first = 0
    for ws in spaces:
        v = ctypes.c_int(0)
        _n.check(lib.exl3_device_status(ws.data_ptr(), int(bool(clear)), _n.stream_of(ws), ctypes.byref(v)))
        if v.value and not first:
            first = int(v.value)
    return first

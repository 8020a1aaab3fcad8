"""Dense (non-routed) EXL3 linear layers on the B200 kernels.

Mirrors the reference's ``Exl3LinearMethod`` (src/vllm_exl3/exl3.py) for
the part on this path:

* :meth:`Exl3LinearMethod.apply` -- exl3.py:6656-6669: through the opaque
  custom op ``torch.ops.exl3_b200.exl3_linear_forward(x, layer_name)`` when
  the layer is registered (the reference's ``torch.ops.vllm.exl3_linear_forward``,
  exl3.py:5670-5752: torch.compile sees one opaque call with a shape-only fake
  implementation), else eagerly; bias added after;
* :meth:`Exl3LinearMethod._apply_impl` -- exl3.py:6671-6739: flatten to rows,
  cast to fp16, optional input padding, every shard in declared order (EXL3
  shards through :func:`dense_forward`, bf16 shards through ``F.linear``),
  concatenate along the output, trim padded columns, cast back to the input
  dtype, restore the leading shape;
* :func:`dense_forward` -- ``_dense_forward`` (exl3.py:5797-5819).  The
  reference picks between a small-row GEMV, a cooperative GEMM and
  reconstruct + hgemm by row count; here one library call serves every row
  count (the decode GEMV below 32 rows, the tcgen05 GEMM from 32), so the
  row ranges collapse into one path.  Each shard's fp32 result is rounded
  once to the output dtype, exactly as the reference's fp32 concatenation
  followed by ``.to(x.dtype)``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .moe import Exl3Projection

_LAYERS: dict[str, torch.nn.Module] = {}
_OPS_READY = False


def dense_forward(linear: Exl3Projection, x_fp16: torch.Tensor, out_dtype: torch.dtype = torch.float32
                  ) -> torch.Tensor:
    """One EXL3 shard: y [rows, out] = x W in ``out_dtype`` (one launch)."""
    import vllm_exl3_c
    return vllm_exl3_c.exl3_linear(x_fp16, linear.trellis, linear.suh, linear.svh, linear.K, linear.codebook,
                                   out_dtype=out_dtype)


def _forward_op(x: torch.Tensor, layer_name: str) -> torch.Tensor:
    layer = _LAYERS[layer_name]
    return layer.quant_method._apply_impl(layer, x)


def _forward_fake(x: torch.Tensor, layer_name: str) -> torch.Tensor:
    layer = _LAYERS[layer_name]
    out = int(sum(getattr(layer, "_exl3_linear_true_out", layer._exl3_linear_output_partition_sizes)))
    return x.new_empty(*x.shape[:-1], out)


def register_custom_ops() -> bool:
    """Register ``torch.ops.exl3_b200.exl3_linear_forward`` once."""
    global _OPS_READY
    if _OPS_READY:
        return True
    try:
        if not hasattr(torch.ops.exl3_b200, "exl3_linear_forward"):
            lib = torch.library.Library("exl3_b200", "FRAGMENT")
            lib.define("exl3_linear_forward(Tensor x, str layer_name) -> Tensor")
            lib.impl("exl3_linear_forward", _forward_op, "CUDA")
            lib.impl("exl3_linear_forward", _forward_fake, "Meta")
            register_custom_ops._lib = lib  # keep the library alive
    except Exception:  # pragma: no cover - registration is best effort, eager path stays
        return False
    _OPS_READY = True
    return True


class Exl3LinearMethod:
    """The dense linear method: per-shard EXL3 projections of one layer."""

    def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        name = getattr(layer, "_exl3_opaque_name", None)
        if name is not None and _OPS_READY and x.is_cuda:
            y = torch.ops.exl3_b200.exl3_linear_forward(x, name)
        else:
            y = self._apply_impl(layer, x)
        if bias is not None:
            y = y + bias
        return y

    def _apply_impl(self, layer, x: torch.Tensor) -> torch.Tensor:
        linears = getattr(layer, "_exl3_linears", None)
        if not linears:
            raise RuntimeError("EXL3 linear layers were not built after weight load")
        orig_shape = x.shape
        x_2d = x.reshape(-1, orig_shape[-1])
        x_fp16 = x_2d.to(torch.float16).contiguous()
        if getattr(layer, "_exl3_linear_padded", False):
            pad_in = int(layer._exl3_linear_input_size_per_partition) - int(x_fp16.shape[1])
            if pad_in > 0:
                x_fp16 = F.pad(x_fp16, (0, pad_in))
        bf16_shards = list(getattr(layer, "_exl3_linear_bf16_shards", []))
        bf16_weight = getattr(layer, "_exl3_bf16_weight", None)
        output_sizes = layer._exl3_linear_output_partition_sizes
        padded = getattr(layer, "_exl3_linear_padded", False)
        # each shard's fp32 result rounded once to the output dtype (= the
        # reference's fp32 concatenation then .to(x.dtype)); padded layers
        # keep fp32 until the trim, like the reference
        shard_dtype = torch.float32 if padded else x.dtype
        outputs = []
        for i, linear in enumerate(linears):
            if i in bf16_shards:
                if bf16_weight is None:
                    raise RuntimeError(f"EXL3 bf16 shard {i} but _exl3_bf16_weight is missing")
                j = bf16_shards.index(i)
                start = sum(output_sizes[s] for s in bf16_shards[:j])
                w = bf16_weight[start:start + output_sizes[i]]
                outputs.append(F.linear(x_2d, w).to(torch.float32).to(shard_dtype))
                continue
            if linear is None:
                raise RuntimeError(f"EXL3 linear shard {i} is None")
            outputs.append(dense_forward(linear, x_fp16, shard_dtype))
        y = torch.cat(outputs, dim=1) if len(outputs) > 1 else outputs[0]
        if padded:
            y = y[:, : sum(layer._exl3_linear_true_out)]
        y = y.to(dtype=x.dtype)
        return y.reshape(*orig_shape[:-1], y.shape[-1])


class Exl3Linear(torch.nn.Module):
    """A dense EXL3 layer: shards (Exl3Projection, or None for a bf16 shard
    held in ``bf16_weight``) concatenated along the output."""

    def __init__(self, shards: list[Exl3Projection | None], name: str | None = None,
                 bf16_weight: torch.Tensor | None = None, bf16_shards: list[int] | None = None,
                 output_sizes: list[int] | None = None, bias: torch.Tensor | None = None):
        super().__init__()
        self.quant_method = Exl3LinearMethod()
        self._exl3_linears = list(shards)
        self._exl3_linear_output_partition_sizes = list(
            output_sizes if output_sizes is not None else [s.out_features for s in shards])
        self._exl3_linear_bf16_shards = list(bf16_shards or [])
        self._exl3_bf16_weight = bf16_weight
        self.bias = bias
        if name is not None:
            _LAYERS[name] = self
            self._exl3_opaque_name = name
            register_custom_ops()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.quant_method.apply(self, x, self.bias)


def linear_from_projections(projs, device, name: str | None = None) -> Exl3Linear:
    """Upload synthetic projections (:class:`exl3_b200.synthetic.Projection`)
    as the shards of one dense layer."""
    shards = [Exl3Projection(torch.from_numpy(p.trellis).to(device), torch.from_numpy(p.suh).to(device),
                             torch.from_numpy(p.svh).to(device), p.codebook) for p in projs]
    return Exl3Linear(shards, name=name)


__all__ = ["Exl3Linear", "Exl3LinearMethod", "dense_forward", "linear_from_projections", "register_custom_ops"]

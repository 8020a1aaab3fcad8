"""Row-wise EXL3 embedding tables (the n-gram format) on the B200 kernel.

Mirrors the lookup of the reference's ``Exl3EmbeddingMethod``
(src/vllm_exl3/exl3.py:5300-5587) with the table resident on the device:
``embedding(ids)`` gathers the packed rows of the ids, finds each id's head
(the last ``head_offsets`` entry <= id, as ``searchsorted(..., right=True) -
1`` clamped), decodes the 160 values of each row (mul1 codebook x the row's
fp16 scale + the head's bias) and casts to the table's dtype -- one kernel
launch (``exl3_ngram_lookup``) instead of the reference's index_select,
searchsorted and decode.  Ids outside the table give zero rows and record
status 7 in the module's status word (``status()``).
"""

from __future__ import annotations


import torch

from . import _native as _n

NGRAM_ROW_DIM = 160


def ngram_words_per_row(bits: int) -> int:
    """int16 words per packed row: one fp16 scale plus the K-bit ring (exl3.py:5174-5176)."""
    return 1 + NGRAM_ROW_DIM * int(bits) // 16


class Exl3NgramEmbedding(torch.nn.Module):
    """A device-resident n-gram table: ``rows`` int16 [n_rows, words],
    ``head_offsets`` int64 [heads] (ascending first ids), ``head_bias`` fp16
    [heads, 160]."""

    def __init__(self, rows: torch.Tensor, bits: int, head_offsets: torch.Tensor, head_bias: torch.Tensor,
                 dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        bits = int(bits)
        if not 1 <= bits <= 8:
            raise ValueError(f"unsupported ngram_embedding bits={bits}")
        if rows.dtype != torch.int16 or rows.dim() != 2 or rows.size(1) != ngram_words_per_row(bits):
            raise ValueError(f"n-gram rows must be int16 [n, {ngram_words_per_row(bits)}]")
        if head_bias.shape != (head_offsets.numel(), NGRAM_ROW_DIM):
            raise ValueError("head_bias must be [heads, 160] with one row per head offset")
        self.bits = bits
        self.rows = rows.contiguous()
        self.head_offsets = head_offsets.to(device=rows.device, dtype=torch.int64).contiguous()
        self.head_bias = head_bias.to(device=rows.device, dtype=torch.float16).contiguous()
        self.dtype = dtype
        self._status = torch.zeros(1, dtype=torch.int32, device=rows.device)

    def embedding(self, ids: torch.Tensor) -> torch.Tensor:
        _n.require_cuda(ids, self.rows, who="n-gram lookup")
        flat = ids.reshape(-1)
        if flat.dtype not in (torch.int32, torch.int64):
            flat = flat.to(torch.int64)
        flat = flat.contiguous()
        out = torch.empty(flat.numel(), NGRAM_ROW_DIM, dtype=self.dtype, device=self.rows.device)
        with torch.cuda.device(self.rows.device):
            _n.check(_n.load().exl3_ngram_lookup(
                self.rows.data_ptr(), int(self.rows.size(0)), self.bits, flat.data_ptr(), _n.dtype_code(flat),
                int(flat.numel()), self.head_offsets.data_ptr(), int(self.head_offsets.numel()),
                self.head_bias.data_ptr(), out.data_ptr(), _n.dtype_code(out), self._status.data_ptr(),
                _n.stream_of(self.rows)), "n-gram lookup")
        return out.view(*ids.shape, NGRAM_ROW_DIM)

    forward = embedding

    def status(self, clear: bool = True) -> int:
        """The lookup status word (7 = an id outside the table); synchronises."""
        v = int(self._status.item())
        if clear and v:
            self._status.zero_()
        return v


__all__ = ["Exl3NgramEmbedding", "NGRAM_ROW_DIM", "ngram_words_per_row"]

"""Loading routed-expert EXL3 packs into the fused B200 layer.

Mirrors the reference's routed-expert weight path for whole experts (expert
parallel, no tensor-parallel slicing of an expert):

* :class:`Exl3ExpertStore` -- the parameters ``Exl3MoEMethod.create_weights``
  registers (src/vllm_exl3/exl3.py:4351-4481): stacked ``w13_suh`` [E, 2, H],
  ``w13_svh`` [E, 2, I], ``w2_suh`` [E, I], ``w2_svh`` [E, H], int32 codebook
  markers ``w13_mcg`` / ``w13_mul1`` [E, 2, 1] and ``w2_mcg`` / ``w2_mul1``
  [E, 1], and ragged per-expert trellis lists (each expert may have its own
  K per projection);
* :meth:`Exl3ExpertStore.load` -- ``_load_exl3`` (exl3.py:4559-4818): global
  to local expert ids (non-local experts are skipped), the w1 -> w3 remap of
  non-gated layers, marker scalars, trellis tile-prefix and word-count checks
  (exl3.py:4650-4667), exact-shape scale copies;
* :meth:`Exl3ExpertStore.finalize` -- ``process_weights_after_loading``
  (exl3.py:4819-5000): the codebook-marker checks
  (``_check_moe_codebook_markers``, exl3.py:4282-4303, and the gateless
  lane rules), completeness of every expert, then the projections and the
  fused state (:func:`exl3_b200.moe.build_exl3_fused_state`);
* :func:`load_routed_experts` -- reads the per-expert tensors
  ``<prefix>.experts.<e>.<proj>.<trellis|suh|svh|mcg|mul1>`` of one layer
  from safetensors files (``proj`` as the checkpoint names it, ``gate_proj`` /
  ``up_proj`` / ``down_proj``, or as vLLM maps it, ``w1`` / ``w3`` / ``w2``).

Failures raise before anything reaches the GPU kernels, with the
reference's messages where it has one.
"""

from __future__ import annotations

import json
import os
import re
import struct
from typing import Callable, Iterable

import numpy as np
import torch

from . import _native as _n
from .moe import EXL3_MCG_MARKER, EXL3_MUL1_MARKER, Exl3Projection, Exl3RoutedExperts

# checkpoint projection names -> vLLM's shard ids (gate = w1, down = w2, up = w3)
SHARD_OF = {"gate_proj": "w1", "w1": "w1", "down_proj": "w2", "w2": "w2", "up_proj": "w3", "w3": "w3"}
SUFFIXES = ("trellis", "suh", "svh", "mcg", "mul1")


def _suffix(weight_name: str) -> str:
    return weight_name.rsplit(".", 1)[-1]


def check_codebook_markers(mcg: torch.Tensor, mul1: torch.Tensor, what: str) -> None:
    """Every expert tensor carries exactly one codebook marker with the known
    value (exl3.py:4282-4303)."""
    mcg_v, mul1_v = mcg.reshape(-1), mul1.reshape(-1)
    mcg_set, mul1_set = mcg_v != 0, mul1_v != 0
    if bool((mcg_set & mul1_set).any()):
        raise RuntimeError(f"EXL3 {what}: an expert tensor has both mcg and mul1 markers")
    if bool((~mcg_set & ~mul1_set).any()):
        raise RuntimeError(f"EXL3 {what}: an expert tensor has no codebook marker (mcg or mul1 never loaded)")
    if bool((mcg_v[mcg_set] != EXL3_MCG_MARKER).any()):
        raise RuntimeError(f"EXL3 {what}: mcg marker is not the MCG int32 {EXL3_MCG_MARKER}; packed ABI mismatch")
    if bool((mul1_v[mul1_set] != EXL3_MUL1_MARKER).any()):
        raise RuntimeError(
            f"EXL3 {what}: mul1 marker is not the mul1 int32 {EXL3_MUL1_MARKER}; packed ABI mismatch")


class Exl3ExpertStore:
    """Staging for one routed-expert layer's EXL3 tensors, then the layer.

    ``num_experts`` local experts; ``global_to_local`` maps a checkpoint
    expert id to the local id or -1 (default: identity over
    [start, start + num_experts) with ``start = starting_expert_offset``, the
    reference's linear expert-parallel placement).  Tensors are kept on
    ``device`` as they load."""

    def __init__(self, num_experts: int, hidden_size: int, intermediate_size: int, *, gateless: bool = False,
                 device: torch.device | str = "cpu", starting_expert_offset: int = 0,
                 global_to_local: Callable[[int], int] | None = None, act: int = _n.ACT_SILU):
        if hidden_size % 128 or intermediate_size % 128 or hidden_size <= 0 or intermediate_size <= 0:
            raise ValueError(
                "EXL3 routed transforms require 128-aligned local dimensions; "
                f"hidden={hidden_size} intermediate_local={intermediate_size}. "
                "Use whole-expert EP or an aligned TP partition; no padding/truncation is safe.")
        E, H, I = int(num_experts), int(hidden_size), int(intermediate_size)
        self.num_experts, self.hidden, self.inter = E, H, I
        self.gateless = bool(gateless)
        self.device = torch.device(device)
        self.act = _n.ACT_RELU2 if self.gateless else int(act)
        self.in_tiles, self.out_tiles = H // 16, I // 16
        dev = self.device
        self.w13_suh = torch.zeros(E, 2, H, dtype=torch.float16, device=dev)
        self.w13_svh = torch.zeros(E, 2, I, dtype=torch.float16, device=dev)
        self.w13_mcg = torch.zeros(E, 2, 1, dtype=torch.int32)
        self.w13_mul1 = torch.zeros(E, 2, 1, dtype=torch.int32)
        self.w2_suh = torch.zeros(E, I, dtype=torch.float16, device=dev)
        self.w2_svh = torch.zeros(E, H, dtype=torch.float16, device=dev)
        self.w2_mcg = torch.zeros(E, 1, dtype=torch.int32)
        self.w2_mul1 = torch.zeros(E, 1, dtype=torch.int32)
        self.gate_trellis: list[torch.Tensor | None] = [None] * E
        self.up_trellis: list[torch.Tensor | None] = [None] * E
        self.down_trellis: list[torch.Tensor | None] = [None] * E
        self.start = int(starting_expert_offset)
        self._g2l = global_to_local

    def local_id(self, expert_id: int) -> int:
        if self._g2l is not None:
            return int(self._g2l(int(expert_id)))
        e = int(expert_id) - self.start
        return e if 0 <= e < self.num_experts else -1

    def load(self, loaded: torch.Tensor, weight_name: str, shard_id: str, expert_id: int) -> bool:
        """One checkpoint tensor of one expert (``_load_exl3``).  Returns False
        for experts this store does not hold."""
        e = self.local_id(expert_id)
        if e < 0:
            return False
        if shard_id == "w1" and self.gateless:
            shard_id = "w3"  # non-gated: the up payload lands in the up slot
        if shard_id not in ("w1", "w2", "w3"):
            raise ValueError(f"unknown EXL3 shard_id={shard_id}")
        suffix = _suffix(weight_name)
        t = loaded.detach()
        if suffix in ("mcg", "mul1"):
            v = int(t.reshape(-1)[0].item()) if t.numel() else 0
            if shard_id == "w2":
                getattr(self, "w2_" + suffix)[e].fill_(v)
            else:
                getattr(self, "w13_" + suffix)[e, 0 if shard_id == "w1" else 1].fill_(v)
            return True
        if suffix == "trellis":
            expect = (self.in_tiles, self.out_tiles) if shard_id in ("w1", "w3") else (self.out_tiles, self.in_tiles)
            if t.dim() != 3 or tuple(t.shape[:2]) != expect:
                raise RuntimeError(
                    f"EXL3 trellis tile mismatch {weight_name} shard={shard_id} expert={expert_id}: "
                    f"got {tuple(t.shape)} expected prefix {expect}+K_words")
            if int(t.shape[-1]) % 16 != 0:
                raise RuntimeError(f"EXL3 trellis K_words not multiple of 16: {tuple(t.shape)}")
            K = int(t.shape[-1]) // 16
            if not 2 <= K <= 8:
                raise RuntimeError(f"EXL3 trellis {weight_name}: K={K} outside 2..8")
            if t.dtype != torch.int16:
                if not t.is_floating_point() and t.element_size() == 2:
                    t = t.view(torch.int16)
                else:
                    raise RuntimeError(f"EXL3 trellis {weight_name} must be 16-bit words, got {t.dtype}")
            plist = {"w1": self.gate_trellis, "w3": self.up_trellis, "w2": self.down_trellis}[shard_id]
            plist[e] = t.to(device=self.device).contiguous()
            return True
        if suffix in ("suh", "svh"):
            if shard_id == "w2":
                dest = getattr(self, "w2_" + suffix)[e]
            else:
                dest = getattr(self, "w13_" + suffix)[e, 0 if shard_id == "w1" else 1]
            if tuple(dest.shape) != tuple(t.shape):
                raise RuntimeError(
                    f"EXL3 load shape mismatch {weight_name} shard={shard_id} expert={expert_id}: "
                    f"dest {tuple(dest.shape)} != loaded {tuple(t.shape)}")
            dest.copy_(t.to(torch.float16))
            return True
        raise ValueError(f"unknown EXL3 tensor suffix {suffix!r} in {weight_name}")

    def _check_markers(self) -> None:
        check_codebook_markers(self.w2_mcg, self.w2_mul1, "w2")
        if not self.gateless:
            check_codebook_markers(self.w13_mcg, self.w13_mul1, "w13")
            return
        mcg_v, mul1_v = self.w13_mcg.reshape(-1), self.w13_mul1.reshape(-1)
        gate_mcg, gate_mul1, up_mcg, up_mul1 = mcg_v[0::2], mul1_v[0::2], mcg_v[1::2], mul1_v[1::2]
        if bool((gate_mcg != 0).any()) or bool((gate_mul1 != 0).any()):
            raise RuntimeError("EXL3 gateless w13: gate lane must stay empty (no gate projection)")
        if bool(((up_mcg != 0) & (up_mul1 != 0)).any()) or bool(((up_mcg == 0) & (up_mul1 == 0)).any()):
            raise RuntimeError("EXL3 gateless w13: every up lane must carry exactly one codebook marker")
        if bool((up_mcg[up_mcg != 0] != EXL3_MCG_MARKER).any()) or bool(
                (up_mul1[up_mul1 != 0] != EXL3_MUL1_MARKER).any()):
            raise RuntimeError("EXL3 gateless w13: up-lane marker ABI mismatch")

    @staticmethod
    def _codebook(mcg: int, mul1: int) -> int:
        return _n.CB_MCG if mcg else _n.CB_MUL1

    def finalize(self, expert_map: torch.Tensor | None = None) -> Exl3RoutedExperts:
        """Checks (markers, completeness) and the fused layer on ``device``."""
        self._check_markers()
        inners = []
        for e in range(self.num_experts):
            gt, ut, dt = self.gate_trellis[e], self.up_trellis[e], self.down_trellis[e]
            if ut is None or dt is None or (not self.gateless and gt is None):
                shape = lambda t: None if t is None else tuple(t.shape)  # noqa: E731
                raise RuntimeError(f"EXL3 mixed-K load incomplete for local expert {e}: "
                                   f"gate={shape(gt)} up={shape(ut)} down={shape(dt)}")
            d = {"gate": None}
            if not self.gateless:
                d["gate"] = Exl3Projection(gt, self.w13_suh[e, 0], self.w13_svh[e, 0],
                                           self._codebook(int(self.w13_mcg[e, 0]), int(self.w13_mul1[e, 0])))
            d["up"] = Exl3Projection(ut, self.w13_suh[e, 1], self.w13_svh[e, 1],
                                     self._codebook(int(self.w13_mcg[e, 1]), int(self.w13_mul1[e, 1])))
            d["down"] = Exl3Projection(dt, self.w2_suh[e], self.w2_svh[e],
                                       self._codebook(int(self.w2_mcg[e]), int(self.w2_mul1[e])))
            inners.append(d)
        return Exl3RoutedExperts(inners, self.hidden, self.inter, expert_map=expert_map, act=self.act)


# ---------------------------------------------------------------------------
# safetensors
# ---------------------------------------------------------------------------
_ST_DTYPES = {"I16": np.int16, "U16": np.uint16, "F16": np.float16, "I32": np.int32, "F32": np.float32,
              "I64": np.int64, "U8": np.uint8, "I8": np.int8}


def read_safetensors(path: str, names: Iterable[str] | None = None) -> dict[str, torch.Tensor]:
    """Tensors of a safetensors file (all, or `names`), read through a memory
    map (8-byte little-endian header length, JSON header, raw data)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    want = None if names is None else set(names)
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    base = 8 + n
    out = {}
    for name, meta in header.items():
        if name == "__metadata__" or (want is not None and name not in want):
            continue
        dt = _ST_DTYPES.get(meta["dtype"])
        if dt is None:
            raise RuntimeError(f"{path}: tensor {name} has unsupported dtype {meta['dtype']}")
        b, e = meta["data_offsets"]
        arr = np.frombuffer(mm[base + b: base + e], dtype=dt).reshape(meta["shape"])
        out[name] = torch.from_numpy(arr.copy())
    return out


def safetensors_keys(path: str) -> list[str]:
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    return [k for k in header if k != "__metadata__"]


def write_safetensors(path: str, tensors: dict[str, np.ndarray | torch.Tensor]) -> None:
    """Write a safetensors file (used to build test packs)."""
    rev = {v: k for k, v in _ST_DTYPES.items()}
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        a = t.numpy() if isinstance(t, torch.Tensor) else np.asarray(t)
        a = np.ascontiguousarray(a)
        header[name] = {"dtype": rev[a.dtype.type], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


_KEY = re.compile(r"^(?P<prefix>.*)\.experts\.(?P<e>\d+)\.(?P<proj>gate_proj|up_proj|down_proj|w1|w2|w3)\."
                  r"(?P<suffix>trellis|suh|svh|mcg|mul1)$")


def load_routed_experts(paths: str | list[str], prefix: str, num_experts: int, hidden_size: int,
                        intermediate_size: int, device: torch.device | str, *, gateless: bool | None = None,
                        starting_expert_offset: int = 0, expert_map: torch.Tensor | None = None,
                        act: int = _n.ACT_SILU) -> Exl3RoutedExperts:
    """One routed-expert layer from safetensors files: every
    ``<prefix>.experts.<e>.<proj>.<suffix>`` tensor of the experts this rank
    holds goes through :meth:`Exl3ExpertStore.load`, then
    :meth:`Exl3ExpertStore.finalize`.  ``gateless`` None: decided from the
    files (no gate tensors at all)."""
    files = [paths] if isinstance(paths, str) else list(paths)
    entries = []
    for path in files:
        for k in safetensors_keys(path):
            m = _KEY.match(k)
            if m and m.group("prefix") == prefix:
                entries.append((path, k, SHARD_OF[m.group("proj")], int(m.group("e"))))
    if not entries:
        raise RuntimeError(f"no EXL3 expert tensors under {prefix!r}.experts in {files}")
    if gateless is None:
        gateless = not any(sid == "w1" for _p, _k, sid, _e in entries)
    store = Exl3ExpertStore(num_experts, hidden_size, intermediate_size, gateless=gateless, device=device,
                            starting_expert_offset=starting_expert_offset, act=act)
    by_file: dict[str, list] = {}
    for path, k, sid, e in entries:
        if store.local_id(e) >= 0:
            by_file.setdefault(path, []).append((k, sid, e))
    for path, items in by_file.items():
        tensors = read_safetensors(path, [k for k, _s, _e in items])
        for k, sid, e in items:
            store.load(tensors.pop(k), k, sid, e)
    return store.finalize(expert_map=expert_map)


def save_routed_experts(path: str, prefix: str, experts: list[dict], names: str = "hf",
                        expert_offset: int = 0) -> None:
    """Write synthetic experts ({"gate", "up", "down"} of
    :class:`exl3_b200.synthetic.Projection`) as an EXL3 pack file, one marker
    per projection (``mcg`` or ``mul1``, exl3.py:113-116).  ``names`` "hf":
    gate_proj/up_proj/down_proj; "vllm": w1/w3/w2."""
    pn = {"gate": "gate_proj", "up": "up_proj", "down": "down_proj"} if names == "hf" else \
        {"gate": "w1", "up": "w3", "down": "w2"}
    out = {}
    for i, ex in enumerate(experts):
        for which, p in ex.items():
            if p is None:
                continue
            key = f"{prefix}.experts.{expert_offset + i}.{pn[which]}"
            out[key + ".trellis"] = p.trellis
            out[key + ".suh"] = p.suh
            out[key + ".svh"] = p.svh
            if p.codebook == _n.CB_MCG:
                out[key + ".mcg"] = np.array([EXL3_MCG_MARKER], dtype=np.int32)
            else:
                out[key + ".mul1"] = np.array([EXL3_MUL1_MARKER], dtype=np.int32)
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    write_safetensors(path, out)

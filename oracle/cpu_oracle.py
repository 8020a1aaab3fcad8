"""CPU oracle for the EXL3 routed-expert MoE path.

TEST INFRASTRUCTURE ONLY.  This module (oracle/cpu_oracle.py) is the parity checker for the CUDA
kernels of ``vllm-exl3_b200``; only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU legs import it.  The product path never calls it.

Contents, each restating the reference (vcruz305/vllm-exl3) function cited:

* ``dequant`` / ``decode_raw`` / ``decode_codebook`` -- the C restatement in
  ``exl3_oracle.c`` of ``csrc/bindings.cpp:15-100`` and
  ``csrc/exl3_dequant.cuh:12-179`` (bit-exact, pinned against the reference
  compiled from its own sources and its test vectors).
* ``map_topk_to_local`` -- ``src/vllm_exl3/exl3.py:2332-2354``.
* ``moe_eager`` -- ``apply_exl3_python_loop`` (``exl3.py:2357-2413``) with each
  projection realised as ``x.half().float() @ dequant(...).float()``, the CPU
  branch of ``exl3_gemv`` (``bindings.cpp:144-146``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None
_lock = threading.Lock()

CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2


def _load():
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(_LIB_PATH):
            subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
        lib = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        lib.oracle_dequant.argtypes = [P, P, P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, P]
        lib.oracle_dequant.restype = ctypes.c_int
        lib.oracle_dequant_cols.argtypes = [P, P, P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int64, ctypes.c_int64, P]
        lib.oracle_dequant_cols.restype = ctypes.c_int
        lib.oracle_decode_raw.argtypes = [P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, P]
        lib.oracle_decode_raw.restype = None
        lib.oracle_decode_codebook_many.argtypes = [P, ctypes.c_int64, ctypes.c_int, P]
        lib.oracle_decode_codebook_many.restype = None
        lib.oracle_float_to_half_many.argtypes = [P, ctypes.c_int64, P]
        lib.oracle_float_to_half_many.restype = None
        lib.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        lib.oracle_half_to_float.restype = ctypes.c_float
        lib.oracle_float_to_half.argtypes = [ctypes.c_float]
        lib.oracle_float_to_half.restype = ctypes.c_uint16
        lib.oracle_read_window.argtypes = [P, ctypes.c_size_t, ctypes.c_size_t]
        lib.oracle_read_window.restype = ctypes.c_uint16
        _lib = lib
        return lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def float_to_half_bits(value: float) -> int:
    """RTNE float32 -> binary16 bits (``exl3_dequant.cuh:40-86``)."""
    return int(_load().oracle_float_to_half(ctypes.c_float(value)))


def half_bits_to_float(bits: int) -> float:
    """binary16 bits -> float (``exl3_dequant.cuh:25-38``)."""
    return float(_load().oracle_half_to_float(int(bits) & 0xFFFF))


def decode_codebook(windows, cb: int) -> np.ndarray:
    """16-bit trellis states -> fp16 bit patterns (``exl3_dequant.cuh:105-124``)."""
    w = np.ascontiguousarray(np.asarray(windows, dtype=np.uint16).reshape(-1))
    out = np.empty_like(w)
    _load().oracle_decode_codebook_many(_ptr(w), w.size, int(cb), _ptr(out))
    return out


def read_window(tile_words, bit: int) -> int:
    """Window at ``bit`` of one tile (``exl3_dequant.cuh:141-159``)."""
    t = np.ascontiguousarray(np.asarray(tile_words).view(np.uint16).reshape(-1))
    return int(_load().oracle_read_window(_ptr(t), t.size, int(bit)))


def _check_trellis(trellis: np.ndarray, K: int) -> np.ndarray:
    t = np.ascontiguousarray(trellis)
    if t.dtype != np.int16 or t.ndim != 3 or t.shape[2] != 16 * K:
        raise ValueError("trellis must be int16 [in/16, out/16, 16*K]")
    return t


def decode_raw(trellis: np.ndarray, K: int, cb: int) -> np.ndarray:
    """Trellis -> un-rotated fp16 W~ [in, out] (tile permutation of
    ``bindings.cpp:37-77``), returned as float16."""
    t = _check_trellis(trellis, K)
    rows, cols = t.shape[0] * 16, t.shape[1] * 16
    out = np.empty((rows, cols), dtype=np.uint16)
    _load().oracle_decode_raw(_ptr(t), rows, cols, int(K), int(cb), _ptr(out))
    return out.view(np.float16)


def dequant(trellis: np.ndarray, suh: np.ndarray, svh: np.ndarray, K: int, mcg: bool = True,
            cb: int | None = None) -> np.ndarray:
    """``dequant_trellis`` (``bindings.cpp:117-132`` -> ``dequant_cpu`` :15-100):
    W = diag(suh) H W~ H diag(svh) / 128 as float16 [in, out]."""
    t = _check_trellis(trellis, K)
    if cb is None:
        cb = CB_MCG if mcg else CB_MUL1
    rows, cols = t.shape[0] * 16, t.shape[1] * 16
    su = np.ascontiguousarray(np.asarray(suh, dtype=np.float16).reshape(-1)[:rows]).view(np.uint16)
    sv = np.ascontiguousarray(np.asarray(svh, dtype=np.float16).reshape(-1)[:cols]).view(np.uint16)
    out = np.empty((rows, cols), dtype=np.uint16)
    rc = _load().oracle_dequant(_ptr(t), _ptr(su), _ptr(sv), rows, cols, int(K), int(cb), _ptr(out))
    if rc != 0:
        raise ValueError("trellis dimensions must reconstruct whole 128-element Hadamard blocks")
    return out.view(np.float16)


def dequant_cols(trellis: np.ndarray, suh: np.ndarray, svh: np.ndarray, K: int, cb: int, c0: int,
                 c1: int) -> np.ndarray:
    """Columns [c0, c1) (multiples of 128) of ``dequant``'s result as float16
    [in, c1 - c0].  Each 128x128 block of the reconstruction depends only on
    its own tiles and scales, so this equals ``dequant(...)[:, c0:c1]`` bit
    for bit without decoding the other columns."""
    t = _check_trellis(trellis, K)
    rows, cols = t.shape[0] * 16, t.shape[1] * 16
    su = np.ascontiguousarray(np.asarray(suh, dtype=np.float16).reshape(-1)[:rows]).view(np.uint16)
    sv = np.ascontiguousarray(np.asarray(svh, dtype=np.float16).reshape(-1)[:cols]).view(np.uint16)
    out = np.empty((rows, c1 - c0), dtype=np.uint16)
    rc = _load().oracle_dequant_cols(_ptr(t), _ptr(su), _ptr(sv), rows, cols, int(K), int(cb), int(c0), int(c1),
                                     _ptr(out))
    if rc != 0:
        raise ValueError("column range and dimensions must be whole 128-element Hadamard blocks")
    return out.view(np.float16)


def map_topk_to_local(ids: np.ndarray, n_local: int, expert_map: np.ndarray | None) -> np.ndarray:
    """Global expert ids -> local ids; invalid or non-local routes -> the
    ``n_local`` sentinel (``exl3.py:2332-2354``)."""
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    if expert_map is None:
        bad = (flat < 0) | (flat >= n_local)
        return np.where(bad, n_local, flat).reshape(np.shape(ids))
    emap = np.asarray(expert_map, dtype=np.int64).reshape(-1)
    n_global = emap.size
    safe = np.clip(flat, 0, max(n_global - 1, 0))
    mapped = emap[safe] if n_global else np.full_like(flat, n_local)
    bad = (flat < 0) | (flat >= n_global) | (mapped < 0) | (mapped >= n_local)
    return np.where(bad, n_local, mapped).reshape(np.shape(ids))


def silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x.astype(np.float64))).astype(np.float32)


def moe_eager(x: np.ndarray, ids: np.ndarray, weights: np.ndarray, dense,
              expert_map: np.ndarray | None = None, limit: float | None = None,
              act: str = "silu", n_local: int | None = None) -> np.ndarray:
    """``apply_exl3_python_loop`` (``exl3.py:2357-2413``).

    ``dense[e]`` maps ``"gate"``, ``"up"``, ``"down"`` to the float16 weights
    ``dequant`` produced for local expert e (``"gate"`` may be None for a
    gateless layer).  ``dense`` may also be a callable ``dense(e)`` returning
    that dict (then ``n_local`` is required): experts are then decoded one at
    a time, only those the routes touch, and dropped after use, so
    full-size layers fit in host memory.  ``"down"`` may hold a subset of the
    output columns; the result then has those columns only.

    Per unique local expert, ascending: gather its routes, ``h.half()``,
    gate/up in fp32, clamp (gate from above, up both sides) when
    ``limit > 0``, ``act = silu(g) * u`` (or the OAI / relu^2 variants),
    ``down = act.half() @ W_down`` in fp32, and ``out.index_add_`` of
    ``down * w``.  Returns fp32 [T, H].
    """
    x = np.asarray(x)
    T, H = x.shape
    if callable(dense):
        if n_local is None:
            raise ValueError("n_local is required with a callable dense")
        get = dense
    else:
        n_local = len(dense)
        get = dense.__getitem__
    out = None
    local = map_topk_to_local(ids, n_local, expert_map).reshape(np.shape(ids))
    w = np.asarray(weights, dtype=np.float32).reshape(local.shape)
    xh = x.astype(np.float16).astype(np.float32)
    for e in np.unique(local).tolist():
        if e >= n_local:
            continue
        tok, kpos = np.nonzero(local == e)
        h = xh[tok]
        pack = get(e)
        if out is None:
            out = np.zeros((T, pack["down"].shape[1]), dtype=np.float32)
        up = h @ pack["up"].astype(np.float32)
        if pack.get("gate") is None:
            if limit is not None and limit > 0:
                up = np.clip(up, -limit, limit)
            a = np.square(np.maximum(up, 0.0))
        else:
            g = h @ pack["gate"].astype(np.float32)
            if limit is not None and limit > 0:
                g = np.minimum(g, limit)
                up = np.clip(up, -limit, limit)
            if act == "swiglu_oai":
                a = (up + 1.0) * g * (1.0 / (1.0 + np.exp(-1.702 * g.astype(np.float64)))).astype(np.float32)
            else:
                a = silu(g) * up
        a = a.astype(np.float32).astype(np.float16).astype(np.float32)
        d = a @ pack["down"].astype(np.float32)
        np.add.at(out, tok, d * w[tok, kpos][:, None])
    if out is None:
        out = np.zeros((T, H), dtype=np.float32)
    return out


NGRAM_ROW_DIM = 160


def ngram_dequant(packed: np.ndarray, bits: int, heads: np.ndarray, head_bias: np.ndarray) -> np.ndarray:
    """Row-wise EXL3 embedding decode (``ngram_dequant_rows_torch``,
    ``exl3.py:5213-5239``; ring layout ``_ngram_bit_tables`` :5198-5208;
    codebook ``ngram_mul1_codebook`` :5186-5195).  packed int16 [N, 1 + 10K];
    element i's state takes bit m from stream bit ((i - m // K) mod 160) * K +
    m % K (LSB-first words after the scale word); value =
    fp16(codebook[state] * scale + head_bias[head]) in fp32 arithmetic."""
    K = int(bits)
    p = np.asarray(packed, dtype=np.int16)
    words = p.astype(np.int64) & 0xFFFF
    i = np.arange(NGRAM_ROW_DIM)[:, None]
    m = np.arange(16)[None, :]
    sb = ((i - m // K) % NGRAM_ROW_DIM) * K + m % K
    widx, bidx = 1 + (sb >> 4), sb & 15
    state = (((words[:, widx] >> bidx) & 1) << m).sum(-1)               # [N, 160]
    prod = (np.arange(65536, dtype=np.int64) * 0x83DCD12D) & 0xFFFFFFFF
    h = (1024 + (prod & 0xFF) + ((prod >> 8) & 0xFF) + ((prod >> 16) & 0xFF) + (prod >> 24)).astype(np.float32)
    kinv = np.float32(np.array([0x1EEE], np.uint16).view(np.float16)[0])
    kbias = np.float32(np.array([0xC931], np.uint16).view(np.float16)[0])
    codebook = ((h * kinv).astype(np.float32) + kbias).astype(np.float16)
    scale = p[:, 0].view(np.float16).astype(np.float32)
    vals = codebook[state].astype(np.float32)
    bias = np.asarray(head_bias, np.float16)[np.asarray(heads, np.int64)].astype(np.float32)
    return ((vals * scale[:, None]).astype(np.float32) + bias).astype(np.float16)

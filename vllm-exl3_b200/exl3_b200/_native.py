"""ctypes binding of ``libexl3_b200.so`` (the C ABI in ``include/exl3_b200.h``).

There is no CPU fallback: if the library is missing or cannot load, every
entry raises.  Tensors are passed as raw device pointers; the stream is
torch's current stream of the tensors' device.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import build as _build

_lock = threading.Lock()
_lib = None

EXL3_OK, EXL3_ERR_ARG, EXL3_ERR_CUDA, EXL3_ERR_WORKSPACE = 0, 1, 2, 3
DT_F32, DT_F16, DT_BF16, DT_I32, DT_I64 = 0, 1, 2, 3, 4
CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2
ACT_SILU, ACT_RELU2, ACT_SWIGLU_OAI = 0, 2, 3

_DTYPE_CODE = {
    torch.float32: DT_F32,
    torch.float16: DT_F16,
    torch.bfloat16: DT_BF16,
    torch.int32: DT_I32,
    torch.int64: DT_I64,
}

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t
F32 = ctypes.c_float

# name -> (restype, argtypes); must cover every function in include/exl3_b200.h
SIGNATURES = {
    "exl3_abi_version": (I32, []),
    "exl3_last_error": (ctypes.c_char_p, []),
    "exl3_device_status": (I32, [P, I32, P, ctypes.POINTER(I32)]),
    "exl3_reconstruct": (I32, [P, P, P, I64, I64, I32, I32, P, P]),
    "exl3_decode_raw": (I32, [P, I64, I64, I32, I32, P, P]),
    "exl3_had128": (I32, [P, P, I64, I64, P, P, F32, P]),
    "exl3_linear_workspace_size": (SZ, [I64, I64, I64, I32]),
    "exl3_linear": (I32, [P, I32, I64, P, P, P, I64, I64, I32, I32, P, I32, P, SZ, P]),
    "exl3_moe_workspace_size": (SZ, [I64, I32, I64, I64, I32, I32]),
    "exl3_moe_forward": (
        I32,
        [P, I32, I64, I64, I64, P, P, P, P, P, P, P, P, P, P, I32, P, I32, I32, P, I64,
         P, P, P, I32, I32, I32, I32, I32, F32, P, P, I32, P, SZ, P],
    ),
    "exl3_batched_linear_workspace_size": (SZ, [I64, I32, I64, I64, I32, I32]),
    "exl3_batched_linear": (I32, [P, I32, I64, P, P, P, I32, P, I32, I64, I64, I32, I32, P, I32, P, SZ, P]),
    "exl3_fat_gemm": (I32, [P, I64, P, P, I64, I64, I32, I32, P, P, P, P, SZ, P]),
    "exl3_linear_noalloc": (I32, [P, I32, I64, P, P, P, I64, I64, I32, I32, P, I32, P]),
    "exl3_ep_dispatch": (I32, [P, I32, I64, I64, P, I32, P, I32, I32, I64, I32, P, P, P, P, P, P, P, I64, P]),
    "exl3_ep_combine": (I32, [P, I32, P, I64, I32, I64, P, P, I32, P]),
    "exl3_ep_window_size": (SZ, [I32, I64, I64, I32, I32, I32]),
    "exl3_ep_window_alloc": (I32, [SZ, ctypes.POINTER(P)]),
    "exl3_ep_window_free": (I32, [P]),
    "exl3_ep_ipc_handle": (I32, [P, P]),
    "exl3_ep_ipc_open": (I32, [P, ctypes.POINTER(P)]),
    "exl3_ep_ipc_close": (I32, [P]),
    "exl3_ep_p2p_dispatch": (I32, [P, I32, I64, I64, P, I32, P, I32, I32, I64, I32, I32, I64, P, P, P, I32, P, P]),
    "exl3_ep_p2p_wait": (I32, [P, I32, I32, P]),
    "exl3_ep_p2p_return": (I32, [P, I32, I32, I32, I64, I64, I32, I32, P, P, P]),
    "exl3_ep_p2p_combine": (I32, [P, I32, I32, I64, I64, I32, I32, I32, P, I64, P, P, I32, P]),
    "exl3_ep_window_recv": (I32, [I32, I64, I64, I32, I32, I32, ctypes.POINTER(SZ), ctypes.POINTER(SZ),
                                  ctypes.POINTER(SZ)]),
    "exl3_ngram_dequant": (I32, [P, I64, I32, P, P, I32, P, I32, P]),
    "exl3_ngram_lookup": (I32, [P, I64, I32, P, I32, I64, P, I32, P, P, I32, P, P]),
    "exl3_profile_enable": (I32, [I32, ctypes.c_longlong]),
    "exl3_profile_read": (I32, [ctypes.POINTER(F32), I32, ctypes.POINTER(I32)]),
}


def lib_path() -> str:
    return _build.LIB_PATH


def load():
    """Load (building first if the sources are newer) and bind the library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if not _build.up_to_date():
            try:
                _build.build()
            except Exception as exc:  # no nvcc on this machine: use the shipped binary
                if not os.path.exists(path):
                    raise RuntimeError(f"EXL3 CUDA library unavailable: {exc}") from exc
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return load().exl3_last_error().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    if rc != EXL3_OK:
        raise RuntimeError(last_error() or f"{what} failed with status {rc}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {t.dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None, who: str) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{who} requires CUDA tensors (the B200 path has no CPU fallback)")


def profile_enable(on: bool, delay_cycles: int = 0) -> None:
    check(load().exl3_profile_enable(int(bool(on)), int(delay_cycles)))


def profile_read(max_phases: int = 8) -> list[float]:
    """Milliseconds of each kernel phase of the last profiled call."""
    buf = (F32 * max_phases)()
    n = I32(0)
    check(load().exl3_profile_read(buf, max_phases, ctypes.byref(n)))
    return [float(buf[i]) for i in range(n.value)]


_ws_cache: dict[tuple, torch.Tensor] = {}
# Every workspace ever handed out stays referenced for the life of the
# process: a CUDA graph captured with one keeps its address, so freeing it
# when a larger call replaces it would let the next replay write into memory
# that other tensors own.  Growth is geometric, so what is retained is bounded
# by about twice the largest workspace of each (device, stream).
_ws_retired: list[torch.Tensor] = []


def workspace(device: torch.device, nbytes: int, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """A cached uint8 workspace of at least ``nbytes`` for ``stream`` (torch's
    current stream of ``device`` when None).

    One workspace per (device, stream): calls on one stream run in order, so
    they may share it; calls on different streams never do.  A workspace that
    is too small is replaced by one at least twice as large, and the old one
    is kept alive (see ``_ws_retired``), so graphs captured earlier stay
    valid.  Sizes come from the library's ``*_workspace_size`` queries; call
    each shape once outside capture (a warm-up) so capture finds the
    workspace already large enough.
    """
    if stream is None:
        stream = torch.cuda.current_stream(device)
    key = (device.type, device.index, int(stream.cuda_stream))
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(int(nbytes), 1 << 20)
        if buf is not None:
            size = max(size, 2 * buf.numel())
            _ws_retired.append(buf)
        with torch.cuda.stream(stream):
            buf = torch.empty(size, dtype=torch.uint8, device=device)
            buf[:256].zero_()  # the device status word starts clean
        _ws_cache[key] = buf
    return buf


def device_workspaces(device: torch.device) -> list[torch.Tensor]:
    """Every workspace handed out on ``device`` (current and retained)."""
    out = [b for k, b in _ws_cache.items() if k[0] == device.type and k[1] == device.index]
    return out + [b for b in _ws_retired if b.device == device]

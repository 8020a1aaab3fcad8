"""GPU: exl3_linear_noalloc, the dense linear for callers that cannot allocate
device memory when they run a projection (an engine that has handed all free
HBM to its KV cache, a C/FFI host without a caching allocator).  It must give
the same result as exl3_linear -- the workspace entry -- on consecutive calls
that reuse its built-in scratch (through both the decode GEMV and the
tensor-core GEMM path), and reject a call that would not fit.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest

import cpu_oracle as oracle

pytestmark = pytest.mark.gpu


def _close(actual, expected):
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    rms = np.sqrt(np.mean(e * e))
    cos = float(a @ e / (np.linalg.norm(a) * np.linalg.norm(e) + 1e-30))
    assert np.isfinite(a).all()
    assert np.max(np.abs(a - e)) <= 2e-2 * rms
    assert cos >= 0.9995


def test_noalloc_matches_workspace_linear_on_consecutive_calls(native, cuda):
    import torch
    from exl3_b200 import _native
    lib = _native.load()
    rng = np.random.default_rng(2024)
    in_f, out_f, K, cb = 1024, 768, 3, 1
    t = rng.integers(-32768, 32768, (in_f // 16, out_f // 16, 16 * K), dtype=np.int16)
    u = (rng.integers(0, 2, in_f) * 2 - 1).astype(np.float16)
    v = ((rng.integers(0, 2, out_f) * 2 - 1) * np.float16(1 / 32)).astype(np.float16)
    dt, du, dv = (torch.from_numpy(a).to(cuda) for a in (t, u, v))
    stream = torch.cuda.current_stream(cuda).cuda_stream
    # calls in a row on one scratch: m = 5 and 19 take the decode GEMV, m = 64
    # the tcgen05 GEMM path (>= 32 rows), each reusing what the last one left
    for call, m in enumerate((5, 19, 64)):
        x = torch.from_numpy(rng.normal(0, 1, (m, in_f)).astype(np.float32)).to(cuda)
        want = native.exl3_linear(x, dt, du, dv, K, cb, out_dtype=torch.float32)
        y = torch.full((m, out_f), float("nan"), dtype=torch.float32, device=cuda)
        rc = lib.exl3_linear_noalloc(x.data_ptr(), _native.DT_F32, m, dt.data_ptr(), du.data_ptr(),
                                     dv.data_ptr(), in_f, out_f, K, cb, y.data_ptr(), _native.DT_F32,
                                     stream)
        assert rc == _native.EXL3_OK, _native.last_error()
        torch.cuda.synchronize(cuda)
        _close(y.cpu().numpy(), want.cpu().numpy())
        if call == 0:
            dense = oracle.dequant(t, u, v, K, cb=cb).astype(np.float32)
            _close(y.cpu().numpy(), x.cpu().numpy().astype(np.float16).astype(np.float32) @ dense)


def test_noalloc_rejects_calls_beyond_its_scratch(native, cuda):
    import torch
    from exl3_b200 import _native
    lib = _native.load()
    m, in_f, out_f, K = 8192, 2048, 128, 4
    t = torch.zeros((in_f // 16, out_f // 16, 16 * K), dtype=torch.int16, device=cuda)
    s = torch.ones(in_f, dtype=torch.float16, device=cuda)
    x = torch.zeros((m, in_f), dtype=torch.float16, device=cuda)
    y = torch.zeros((m, out_f), dtype=torch.float16, device=cuda)
    rc = lib.exl3_linear_noalloc(x.data_ptr(), _native.DT_F16, m, t.data_ptr(), s.data_ptr(), s.data_ptr(),
                                 in_f, out_f, K, 1, y.data_ptr(), _native.DT_F16,
                                 torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _native.EXL3_ERR_ARG
    assert "scratch" in _native.last_error()

"""CPU: the C ABI library loads and exports every symbol include/exl3_b200.h
declares; the host wrappers mirror the reference's interface.  No GPU calls."""

import ctypes
import os
import re

import pytest

from conftest import ROOT


def _header_functions():
    with open(os.path.join(ROOT, "include", "exl3_b200.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(exl3_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from exl3_b200 import _native
    lib = _native.load()
    names = _header_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), f"missing export {name}"
    assert set(names) == set(_native.SIGNATURES), "ctypes signatures must cover the header exactly"
    assert lib.exl3_abi_version() == 1


def test_workspace_queries_without_gpu():
    from exl3_b200 import _native
    lib = _native.load()
    assert lib.exl3_moe_workspace_size(64, 8, 2048, 768, 128, 4) > 0
    assert lib.exl3_moe_workspace_size(64, 8, 2000, 768, 128, 4) == 0  # not a multiple of 128
    assert lib.exl3_linear_workspace_size(16, 8192, 28672, 3) > 0


def test_arg_validation_happens_on_host():
    from exl3_b200 import _native
    lib = _native.load()
    rc = lib.exl3_reconstruct(None, None, None, 128, 128, 4, 1, None, None)
    assert rc == _native.EXL3_ERR_ARG
    assert "null" in _native.last_error()
    rc = lib.exl3_had128(1, 1, 1, 100, None, None, 1.0, None)
    assert rc == _native.EXL3_ERR_ARG and "128" in _native.last_error()


def test_dropin_module_surface():
    import vllm_exl3_c as m
    for name in ("dequant_trellis", "exl3_gemv", "exl3_gemm", "p2b_fused_moe", "p2b_fused_moe_mk",
                 "p2b_fused_moe_padded", "had_r_128", "exl3_reconstruct", "exl3_linear", "exl3_moe",
                 "p2b_gemv_batched", "exl3_fat_gemm", "exl3_fat_gemm_scatter"):
        assert callable(getattr(m, name)), name
    assert m.P2B_MOE_ABI_VERSION >= 4 and m.P2B_MOE_MIXED_K and m.P2B_MOE_PADDED


def test_cpu_tensors_fail_loudly():
    import torch
    import vllm_exl3_c as m
    t = torch.zeros((8, 8, 64), dtype=torch.int16)
    ones = torch.ones(128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        m.dequant_trellis(t, ones, ones, 4, True)


def test_host_map_topk_to_local_matches_oracle():
    import numpy as np
    import torch
    import cpu_oracle as oracle
    from exl3_b200.moe import map_topk_to_local
    rng = np.random.default_rng(0)
    ids = rng.integers(-3, 20, (9, 4))
    emap = rng.integers(-1, 6, 16)
    for em in (None, emap):
        got = map_topk_to_local(torch.from_numpy(ids), 6, None if em is None else torch.from_numpy(em))
        np.testing.assert_array_equal(got.reshape(ids.shape).numpy(), oracle.map_topk_to_local(ids, 6, em))

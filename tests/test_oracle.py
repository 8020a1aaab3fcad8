"""CPU: pin the oracle against the reference's golden vectors and its own code.

* half conversion and codebook known-answer vectors: the reference test's
  values (tests/test_dequant_parity.py:18-104 of the reference) and seeded
  windows, all computed by the reference's src/vllm_exl3/dequant.py
  (fixtures made by tests/golden/make_golden.py);
* dequant_trellis: the reference's csrc/bindings.cpp compiled CPU-only,
  stored as fixtures, and -- when the compiled reference is present
  (oracle/_ref) -- compared live on fresh seeds;
* the eager MoE loop: apply_exl3_python_loop outputs stored as fixtures.
"""

import hashlib
import json
import math
import os

import numpy as np
import pytest

import cpu_oracle as oracle
from conftest import GOLDEN, ROOT


def _load_json(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


@pytest.mark.parametrize("value,expected", [
    (2**-15, 0x0200), (1.00075, 0x3C01), (-1.00075, 0xBC01), (2**-24, 0x0001), (2**-25, 0x0000),
    (1.0 + 2**-11, 0x3C00), (1.0 + 3 * 2**-11, 0x3C02), (65504.0, 0x7BFF), (65520.0, 0x7C00),
    (0.0, 0x0000), (-0.0, 0x8000), (math.inf, 0x7C00), (-math.inf, 0xFC00),
])
def test_half_edge_vectors(value, expected):
    assert oracle.float_to_half_bits(value) == expected


def test_half_conversion_fixture():
    for case in _load_json("half_kat.json"):
        assert oracle.float_to_half_bits(case["value"]) == case["bits"], case


def test_nan_conversion():
    bits = oracle.float_to_half_bits(float("nan"))
    assert (bits & 0x7C00) == 0x7C00 and bits & 0x3FF
    assert math.isnan(oracle.half_bits_to_float(bits))
    assert math.copysign(1.0, oracle.half_bits_to_float(0x8000)) < 0


@pytest.mark.parametrize("window,mcg_bits,mul1_bits,mcg_value,mul1_value", [
    (0x0000, 0x3F60, 0xC2E8, 1.84375, -3.453125),
    (0x0001, 0x304E, 0x3921, 0.134521484375, 0.6410751342773438),
    (0x1234, 0x3E0F, 0xB89E, 1.5142822265625, -0.5770339965820312),
    (0x7FFF, 0x4172, 0x3FCA, 2.72216796875, 1.9471588134765625),
    (0xFFFF, 0x3ACD, 0xB936, 0.85009765625, -0.6514739990234375),
])
def test_codebook_reference_vectors(window, mcg_bits, mul1_bits, mcg_value, mul1_value):
    assert int(oracle.decode_codebook([window], 1)[0]) == mcg_bits
    assert int(oracle.decode_codebook([window], 2)[0]) == mul1_bits
    assert oracle.half_bits_to_float(mcg_bits) == pytest.approx(mcg_value, abs=1e-3)
    assert oracle.half_bits_to_float(mul1_bits) == pytest.approx(mul1_value, abs=2e-3)


def test_codebook_fixture_all_codebooks():
    cases = _load_json("codebook_kat.json")["bits"]
    for cb in (0, 1, 2):
        sel = [c for c in cases if c["cb"] == cb]
        got = oracle.decode_codebook([c["window"] for c in sel], cb)
        assert [int(v) for v in got] == [c["bits"] for c in sel]


def test_read_window_wraps_tail_biting():
    # the window at the last bit of a tile continues at its first word
    tile = np.arange(1, 33, dtype=np.uint16)  # K=2: 32 int16
    total = 32 * 16
    for bit in (0, 15, 16, 31, total - 8, total - 1):
        w = oracle.read_window(tile, bit)
        u32 = [int(tile[2 * i]) | (int(tile[2 * i + 1]) << 16) for i in range(16)]
        stream = "".join(format(x, "032b") for x in u32)
        s2 = stream + stream
        assert w == int(s2[bit:bit + 16], 2)


def test_dequant_fixtures_bit_exact():
    data = np.load(os.path.join(GOLDEN, "dequant.npz"))
    for case in _load_json("dequant_cases.json"):
        tag = case["tag"]
        w = oracle.dequant(data[tag + "_trellis"], data[tag + "_suh"], data[tag + "_svh"], case["K"],
                           case["mcg"])
        assert hashlib.sha256(w.view(np.uint16).tobytes()).hexdigest() == case["sha256"], tag
        if tag + "_w" in data:
            assert np.array_equal(w.view(np.uint16), data[tag + "_w"].view(np.uint16)), tag


def test_dequant_rejects_partial_hadamard_blocks():
    t = np.zeros((4, 8, 64), dtype=np.int16)  # 64 x 128
    with pytest.raises(ValueError, match="128-element Hadamard"):
        oracle.dequant(t, np.ones(64, np.float16), np.ones(128, np.float16), 4)


def _ref_module():
    import sys
    d = os.path.join(ROOT, "oracle", "_ref")
    if not os.path.isdir(d):
        return None
    sys.path.insert(0, d)
    try:
        import torch  # noqa: F401  (the extension needs torch initialised first)
        import vllm_exl3_ref_c
        return vllm_exl3_ref_c
    except Exception:
        return None


@pytest.mark.parametrize("K", [2, 3, 4, 8])
@pytest.mark.parametrize("mcg", [True, False])
def test_dequant_matches_compiled_reference_live(K, mcg):
    ref = _ref_module()
    if ref is None:
        pytest.skip("compiled reference (oracle/_ref) not built here")
    import torch
    rng = np.random.default_rng(1000 + K * 2 + int(mcg))
    t = rng.integers(-32768, 32768, (16, 8, 16 * K), dtype=np.int16)
    u = (rng.integers(0, 2, 256) * 2 - 1).astype(np.float16)
    v = ((rng.integers(0, 2, 128) * 2 - 1) * 0.6875).astype(np.float16)
    a = oracle.dequant(t, u, v, K, mcg)
    b = ref.dequant_trellis(torch.from_numpy(t), torch.from_numpy(u), torch.from_numpy(v), K, mcg).numpy()
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


def _moe_layer(data, meta):
    name = meta["name"]
    dense = []
    for e in range(meta["E"]):
        d = {}
        for which in ("gate", "up", "down"):
            t = data[f"{name}_e{e}_{which}_trellis"]
            d[which] = oracle.dequant(t, data[f"{name}_e{e}_{which}_suh"], data[f"{name}_e{e}_{which}_svh"],
                                      t.shape[-1] // 16, meta["mcg"])
        dense.append(d)
    return dense


def test_eager_moe_matches_reference_loop_fixture():
    data = np.load(os.path.join(GOLDEN, "moe.npz"))
    for meta in _load_json("moe_cases.json"):
        name = meta["name"]
        dense = _moe_layer(data, meta)
        emap = data[f"{name}_expert_map"] if meta["expert_map"] else None
        out = oracle.moe_eager(data[f"{name}_x"], data[f"{name}_ids"], data[f"{name}_w"], dense,
                               expert_map=emap, limit=meta["limit"])
        ref = data[f"{name}_out"]
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5 * float(np.abs(ref).max()))


def test_map_topk_to_local_semantics():
    ids = np.array([[0, 3, -1], [5, 2, 7]])
    np.testing.assert_array_equal(oracle.map_topk_to_local(ids, 4, None), [[0, 3, 4], [4, 2, 4]])
    emap = np.array([-1, -1, 0, 1, -1, 2])
    np.testing.assert_array_equal(oracle.map_topk_to_local(ids, 3, emap), [[3, 1, 3], [2, 0, 3]])


def test_activation_reference_values():
    # the reference's tests/test_activation_parity.py:46-53 values, through the eager loop
    class P:
        pass
    one = np.ones((1, 1), np.float16)
    dense = [{"gate": one * 20, "up": one * 20, "down": one}]
    x = np.ones((1, 1), np.float32)
    out = oracle.moe_eager(x, np.array([[0]]), np.array([[1.0]]), dense)
    assert out[0, 0] == pytest.approx(400.0, abs=1e-4)
    out = oracle.moe_eager(x, np.array([[0]]), np.array([[1.0]]), dense, limit=10.0)
    assert out[0, 0] == pytest.approx(99.9954605, abs=0.01)


def test_ngram_decode_matches_reference_fixtures():
    """The n-gram row decode restatement against the reference's own
    ngram_dequant_rows_torch outputs (tests/golden/ngram.npz), bit for bit."""
    data = np.load(os.path.join(GOLDEN, "ngram.npz"))
    for K in range(1, 9):
        got = oracle.ngram_dequant(data[f"K{K}_packed"], K, data[f"K{K}_heads"], data[f"K{K}_bias"])
        assert np.array_equal(got.view(np.uint16), data[f"K{K}_out"].view(np.uint16)), K

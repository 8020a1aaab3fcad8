"""CPU tests of the routed-expert EXL3 loader (exl3_b200.loader).

The reference behaviour it mirrors: Exl3MoEMethod.create_weights /
_load_exl3 / process_weights_after_loading (src/vllm_exl3/exl3.py:4351-4481,
4559-4818, 4819-5000) and _check_moe_codebook_markers (exl3.py:4282-4303):
per-expert ragged trellis of any K, stacked scales with exact-shape checks,
one codebook marker per projection, tile-prefix and word-count checks,
non-local experts skipped, non-gated layers with an empty gate lane.  Every
failure is raised before a tensor reaches the kernels.
"""

import os

import numpy as np
import pytest
import torch

from exl3_b200 import loader, synthetic
from exl3_b200.moe import EXL3_MCG_MARKER, EXL3_MUL1_MARKER


def _pack(seed=1, E=4, H=256, I=128, cb=synthetic.CB_MCG, ks=(2, 3, 4), gateless=False):
    return synthetic.make_moe_pack(seed, E, H, I, cb, ks, None, gateless)


def _file(tmp_path, pack, names="hf", prefix="model.layers.3.mlp", offset=0):
    path = os.path.join(tmp_path, f"pack_{names}.safetensors")
    loader.save_routed_experts(path, prefix, pack.experts, names=names, expert_offset=offset)
    return path


@pytest.mark.parametrize("names", ["hf", "vllm"])
def test_roundtrip_mixed_k(tmp_path, names):
    pack = _pack()
    path = _file(tmp_path, pack, names)
    layer = loader.load_routed_experts(path, "model.layers.3.mlp", 4, 256, 128, "cpu")
    assert not layer._exl3_gateless
    for e, ex in enumerate(pack.experts):
        for which in ("gate", "up", "down"):
            got = layer._exl3_inners[e][which]
            want = ex[which]
            assert np.array_equal(got.trellis.numpy(), want.trellis)
            assert np.array_equal(got.suh.numpy(), want.suh) and np.array_equal(got.svh.numpy(), want.svh)
            assert got.K == want.K and got.codebook == synthetic.CB_MCG
    kg, ku, kd = layer._exl3_k_tables
    assert kg.tolist() == [e["gate"].K for e in pack.experts]
    assert kd.tolist() == [e["down"].K for e in pack.experts]
    assert layer._exl3_ptrs["up_trellis"].tolist() == [
        inn["up"].trellis.data_ptr() for inn in layer._exl3_inners]


def test_mul1_markers_select_mul1(tmp_path):
    pack = _pack(cb=synthetic.CB_MUL1)
    layer = loader.load_routed_experts(_file(tmp_path, pack), "model.layers.3.mlp", 4, 256, 128, "cpu")
    assert layer._exl3_codebook == synthetic.CB_MUL1


def test_expert_parallel_rank_loads_only_its_experts(tmp_path):
    pack = _pack(E=8)
    path = _file(tmp_path, pack)
    layer = loader.load_routed_experts(path, "model.layers.3.mlp", 4, 256, 128, "cpu", starting_expert_offset=4)
    for e in range(4):
        assert np.array_equal(layer._exl3_inners[e]["down"].trellis.numpy(), pack.experts[4 + e]["down"].trellis)


def test_gateless_layer(tmp_path):
    pack = _pack(gateless=True)
    layer = loader.load_routed_experts(_file(tmp_path, pack), "model.layers.3.mlp", 4, 256, 128, "cpu")
    assert layer._exl3_gateless and layer._exl3_moe_act == 2
    assert all(inn["gate"] is None for inn in layer._exl3_inners)
    assert torch.equal(layer._exl3_ptrs["gate_trellis"], layer._exl3_ptrs["up_trellis"])


def test_gateless_w1_payload_lands_in_up_slot():
    """Non-gated checkpoints mapped onto shard w1 (exl3.py:4580-4590)."""
    pack = _pack(E=1, gateless=True)
    st = loader.Exl3ExpertStore(1, 256, 128, gateless=True)
    up = pack.experts[0]["up"]
    st.load(torch.from_numpy(up.trellis), "x.experts.0.w1.trellis", "w1", 0)
    assert st.gate_trellis[0] is None and torch.equal(st.up_trellis[0], torch.from_numpy(up.trellis))


def _store_with(pack, skip=None, marker_override=None):
    st = loader.Exl3ExpertStore(len(pack.experts), pack.hidden, pack.inter)
    for e, ex in enumerate(pack.experts):
        for which, sid in (("gate", "w1"), ("up", "w3"), ("down", "w2")):
            p = ex[which]
            for suffix, t in (("trellis", p.trellis), ("suh", p.suh), ("svh", p.svh)):
                if skip == (e, which, suffix):
                    continue
                st.load(torch.from_numpy(t), f"l.experts.{e}.{sid}.{suffix}", sid, e)
            m = np.array([EXL3_MCG_MARKER], np.int32)
            if marker_override and marker_override[0] == (e, which):
                for suffix, v in marker_override[1].items():
                    st.load(torch.tensor([v], dtype=torch.int32), f"l.experts.{e}.{sid}.{suffix}", sid, e)
                continue
            if skip != (e, which, "mcg"):
                st.load(torch.from_numpy(m), f"l.experts.{e}.{sid}.mcg", sid, e)
    return st


def test_fail_both_markers():
    st = _store_with(_pack(E=2), marker_override=((1, "down"), {"mcg": EXL3_MCG_MARKER, "mul1": EXL3_MUL1_MARKER}))
    with pytest.raises(RuntimeError, match="both mcg and mul1"):
        st.finalize()


def test_fail_missing_marker():
    st = _store_with(_pack(E=2), skip=(0, "up", "mcg"))
    with pytest.raises(RuntimeError, match="no codebook marker"):
        st.finalize()


def test_fail_wrong_marker_value():
    st = _store_with(_pack(E=2), marker_override=((0, "gate"), {"mcg": 12345}))
    with pytest.raises(RuntimeError, match="packed ABI mismatch"):
        st.finalize()


def test_fail_incomplete_expert():
    st = _store_with(_pack(E=2), skip=(1, "down", "trellis"))
    with pytest.raises(RuntimeError, match="load incomplete for local expert 1"):
        st.finalize()


def test_fail_trellis_tile_mismatch():
    st = loader.Exl3ExpertStore(1, 256, 128)
    with pytest.raises(RuntimeError, match="tile mismatch"):
        st.load(torch.zeros(8, 16, 48, dtype=torch.int16), "l.experts.0.w1.trellis", "w1", 0)  # transposed
    with pytest.raises(RuntimeError, match="tile mismatch"):
        st.load(torch.zeros(16, 8, 48, dtype=torch.int16), "l.experts.0.w2.trellis", "w2", 0)


def test_fail_trellis_words_not_multiple_of_16():
    st = loader.Exl3ExpertStore(1, 256, 128)
    with pytest.raises(RuntimeError, match="K_words not multiple of 16"):
        st.load(torch.zeros(16, 8, 40, dtype=torch.int16), "l.experts.0.w1.trellis", "w1", 0)


def test_fail_scale_shape_mismatch():
    st = loader.Exl3ExpertStore(1, 256, 128)
    with pytest.raises(RuntimeError, match="shape mismatch"):
        st.load(torch.zeros(128, dtype=torch.float16), "l.experts.0.w1.suh", "w1", 0)


def test_fail_unaligned_geometry():
    with pytest.raises(ValueError, match="128-aligned"):
        loader.Exl3ExpertStore(4, 256, 144)


def test_fail_gateless_gate_marker():
    pack = _pack(E=1, gateless=True)
    st = loader.Exl3ExpertStore(1, 256, 128, gateless=True)
    for which, sid in (("up", "w3"), ("down", "w2")):
        p = pack.experts[0][which]
        for suffix, t in (("trellis", p.trellis), ("suh", p.suh), ("svh", p.svh)):
            st.load(torch.from_numpy(t), f"l.experts.0.{sid}.{suffix}", sid, 0)
        st.load(torch.tensor([EXL3_MCG_MARKER], dtype=torch.int32), f"l.experts.0.{sid}.mcg", sid, 0)
    st.w13_mcg[0, 0] = EXL3_MCG_MARKER  # a gate-lane marker a gateless layer must not carry
    with pytest.raises(RuntimeError, match="gate lane must stay empty"):
        st.finalize()


def test_fail_no_tensors(tmp_path):
    path = _file(tmp_path, _pack(E=1))
    with pytest.raises(RuntimeError, match="no EXL3 expert tensors"):
        loader.load_routed_experts(path, "model.layers.9.mlp", 1, 256, 128, "cpu")


def test_safetensors_roundtrip_matches_library(tmp_path):
    """The reader/writer against the safetensors package's own format."""
    from safetensors.numpy import load_file, save_file
    a = {"t": np.arange(48, dtype=np.int16).reshape(1, 3, 16), "s": np.ones(5, np.float16),
         "m": np.array([EXL3_MUL1_MARKER], np.int32)}
    p1 = os.path.join(tmp_path, "a.safetensors")
    loader.write_safetensors(p1, a)
    got = load_file(p1)
    assert all(np.array_equal(got[k], a[k]) for k in a)
    p2 = os.path.join(tmp_path, "b.safetensors")
    save_file(a, p2)
    got2 = loader.read_safetensors(p2)
    assert all(np.array_equal(got2[k].numpy(), a[k]) for k in a)

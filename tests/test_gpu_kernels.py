"""GPU parity of the decode kernels against the CPU oracle, through the C ABI.

Rows >= 32 per projection take the tcgen05 grouped-GEMM path, fewer the
decode GEMV; both are covered.

* exl3_reconstruct (dequant_trellis): bit-exact with the oracle and with the
  reference fixtures, K 2..8 x codebooks 3INST/MCG/mul1;
* exl3_decode_raw: bit-exact W~;
* had_r_128: fp32 FWHT reference;
* exl3_linear / exl3_gemv / exl3_gemm: dense fp32 matmul with the oracle's
  fp16 weights; tolerance max|d| <= 2e-2 * RMS(ref) and cosine >= 0.9995.
"""

import json
import os

import numpy as np
import pytest

import cpu_oracle as oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _rand_packed(rng, in_f, out_f, K):
    t = rng.integers(-32768, 32768, (in_f // 16, out_f // 16, 16 * K), dtype=np.int16)
    u = (rng.integers(0, 2, in_f) * 2 - 1).astype(np.float16)
    v = ((rng.integers(0, 2, out_f) * 2 - 1) * np.float16(0.75 / np.sqrt(in_f))).astype(np.float16)
    return t, u, v


def _close(actual, expected):
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    rms = np.sqrt(np.mean(e * e))
    maxd = np.max(np.abs(a - e))
    cos = float(a @ e / (np.linalg.norm(a) * np.linalg.norm(e) + 1e-30))
    assert np.isfinite(a).all()
    assert maxd <= 2e-2 * rms, f"max|d| {maxd:.3e} > 2e-2 * rms {rms:.3e}"
    assert cos >= 0.9995, f"cosine {cos}"
    return maxd / rms, cos


@pytest.mark.parametrize("K", [2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("cb", [0, 1, 2])
def test_reconstruct_bit_exact(native, cuda, K, cb):
    import torch
    rng = np.random.default_rng(100 + 10 * K + cb)
    t, u, v = _rand_packed(rng, 256, 384, K)
    want = oracle.dequant(t, u, v, K, cb=cb)
    got = native.exl3_reconstruct(torch.from_numpy(t).to(cuda), torch.from_numpy(u).to(cuda),
                                  torch.from_numpy(v).to(cuda), K, cb).cpu().numpy()
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
    raw = native.exl3_decode_raw(torch.from_numpy(t).to(cuda), K, cb).cpu().numpy()
    assert np.array_equal(raw.view(np.uint16), oracle.decode_raw(t, K, cb).view(np.uint16))


def test_dequant_trellis_matches_reference_fixtures(native, cuda):
    import torch
    data = np.load(os.path.join(GOLDEN, "dequant.npz"))
    with open(os.path.join(GOLDEN, "dequant_cases.json")) as f:
        cases = json.load(f)
    import hashlib
    for c in cases:
        tag = c["tag"]
        w = native.dequant_trellis(torch.from_numpy(data[tag + "_trellis"]).to(cuda),
                                   torch.from_numpy(data[tag + "_suh"]).to(cuda),
                                   torch.from_numpy(data[tag + "_svh"]).to(cuda), c["K"], c["mcg"])
        w = w.cpu().numpy()
        assert hashlib.sha256(w.view(np.uint16).tobytes()).hexdigest() == c["sha256"], tag


def test_dequant_trellis_rejects_bad_arguments(native, cuda):
    import torch
    t = torch.zeros((8, 8, 64), dtype=torch.int16, device=cuda)
    ones = torch.ones(128, dtype=torch.float16, device=cuda)
    with pytest.raises(RuntimeError, match="K must be one of"):
        native.dequant_trellis(torch.zeros((8, 8, 80), dtype=torch.int16, device=cuda), ones, ones, 5, True)
    with pytest.raises(RuntimeError, match="16\\*K"):
        native.dequant_trellis(t, ones, ones, 3, True)
    with pytest.raises(RuntimeError, match="float16"):
        native.dequant_trellis(t, ones.float(), ones, 4, True)
    with pytest.raises(RuntimeError, match="Hadamard"):
        native.dequant_trellis(torch.zeros((4, 8, 64), dtype=torch.int16, device=cuda), ones, ones, 4, True)
    with pytest.raises(RuntimeError, match="CUDA"):
        native.dequant_trellis(t.cpu(), ones.cpu(), ones.cpu(), 4, True)


def test_had_r_128(native, cuda):
    import torch
    rng = np.random.default_rng(7)
    x = rng.normal(0, 1, (5, 384)).astype(np.float16)
    pre = (rng.integers(0, 2, 384) * 2 - 1).astype(np.float16)
    post = rng.uniform(0.5, 1.5, 384).astype(np.float16)
    H = np.array([[1.0]])
    for _ in range(7):
        H = np.block([[H, H], [H, -H]])
    xf = x.astype(np.float64) * pre.astype(np.float64)
    want = np.concatenate([xf[:, b * 128:(b + 1) * 128] @ H for b in range(3)], axis=1) / np.sqrt(128)
    want = want * post.astype(np.float64) * 0.5
    xt = torch.from_numpy(x).to(cuda)
    y = torch.empty_like(xt)
    native.had_r_128(xt, y, torch.from_numpy(pre).to(cuda), torch.from_numpy(post).to(cuda), 0.5)
    np.testing.assert_allclose(y.cpu().numpy().astype(np.float64), want, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("m", [1, 5, 8, 16, 17, 40, 128, 300])
@pytest.mark.parametrize("K,cb", [(2, 1), (3, 1), (4, 1), (3, 2), (4, 2), (8, 1)])
def test_linear_matches_dense(native, cuda, m, K, cb):
    import torch
    rng = np.random.default_rng(1000 * m + 10 * K + cb)
    in_f, out_f = 512, 384
    t, u, v = _rand_packed(rng, in_f, out_f, K)
    w = oracle.dequant(t, u, v, K, cb=cb).astype(np.float32)
    x = rng.normal(0, 1, (m, in_f)).astype(np.float32)
    want = x.astype(np.float16).astype(np.float32) @ w
    y = native.exl3_linear(torch.from_numpy(x).to(cuda), torch.from_numpy(t).to(cuda),
                           torch.from_numpy(u).to(cuda), torch.from_numpy(v).to(cuda), K, cb,
                           out_dtype=torch.float32)
    _close(y.cpu().numpy(), want)


@pytest.mark.parametrize("m", [1, 7, 16, 40])
@pytest.mark.parametrize("out_f", [256, 768])
@pytest.mark.parametrize("K,cb", [(4, 1), (3, 2), (3, 0)])
def test_linear_paired_column_blocks(native, cuda, m, out_f, K, cb):
    """An even number of 128-column blocks: the GEMV takes two blocks per work
    item on one shared input slice (m < 32), every codebook including 3INST;
    m = 40 takes the tensor-core GEMM on the same shapes."""
    import torch
    rng = np.random.default_rng(7 * m + out_f + 10 * K + cb)
    in_f = 384
    t, u, v = _rand_packed(rng, in_f, out_f, K)
    w = oracle.dequant(t, u, v, K, cb=cb).astype(np.float32)
    x = rng.normal(0, 1, (m, in_f)).astype(np.float32)
    want = x.astype(np.float16).astype(np.float32) @ w
    y = native.exl3_linear(torch.from_numpy(x).to(cuda), torch.from_numpy(t).to(cuda),
                           torch.from_numpy(u).to(cuda), torch.from_numpy(v).to(cuda), K, cb,
                           out_dtype=torch.float32)
    _close(y.cpu().numpy(), want)


def test_gemv_and_gemm_entries(native, cuda):
    import torch
    rng = np.random.default_rng(3)
    t, u, v = _rand_packed(rng, 256, 256, 4)
    w = oracle.dequant(t, u, v, 4, True).astype(np.float32)
    dev = lambda a: torch.from_numpy(a).to(cuda)
    x = rng.normal(0, 1, (6, 256)).astype(np.float16)
    y = native.exl3_gemv(dev(x), dev(t), dev(u), dev(v), 4, True)
    assert y.dtype == torch.float16 and y.shape == (6, 256)
    _close(y.float().cpu().numpy(), x.astype(np.float32) @ w)
    with pytest.raises(RuntimeError, match="1 <= m <= 8"):
        native.exl3_gemv(dev(np.zeros((9, 256), np.float16)), dev(t), dev(u), dev(v), 4, True)
    x2 = rng.normal(0, 1, (2, 33, 256)).astype(np.float16)
    y2 = native.exl3_gemm(dev(x2), dev(t), dev(u), dev(v), 4, True)
    _close(y2.float().cpu().numpy().reshape(-1, 256), x2.reshape(-1, 256).astype(np.float32) @ w)


def test_p2b_gemv_batched(native, cuda):
    import torch
    rng = np.random.default_rng(21)
    E_tab, in_f, out_f, K = 5, 256, 2048, 3
    packs = [_rand_packed(rng, in_f, out_f, K) for _ in range(E_tab)]
    dev = [tuple(torch.from_numpy(a).to(cuda) for a in p) for p in packs]
    tabs = [torch.tensor([d[i].data_ptr() for d in dev], dtype=torch.int64, device=cuda) for i in range(3)]
    idx = torch.tensor([3, 0, 3, 4], dtype=torch.int32, device=cuda)
    x = rng.normal(0, 1, (3, in_f)).astype(np.float16)
    y = native.p2b_gemv_batched(torch.from_numpy(x).to(cuda), *tabs, idx, K, True)
    assert y.shape == (4, 3, out_f) and y.dtype == torch.float16
    for j, e in enumerate([3, 0, 3, 4]):
        w = oracle.dequant(*packs[e], K, True).astype(np.float32)
        _close(y[j].float().cpu().numpy(), x.astype(np.float32) @ w)


@pytest.mark.parametrize("K,mcg,mul1", [(4, True, False), (2, False, True), (3, True, False)])
def test_fat_gemm_and_scatter(native, cuda, K, mcg, mul1):
    import torch
    rng = np.random.default_rng(31 + K)
    in_f, out_f, M, T = 384, 256, 70, 90
    t, u, v = _rand_packed(rng, in_f, out_f, K)
    cb = 1 if mcg else 2
    h = rng.normal(0, 1, (M, in_f)).astype(np.float16)
    ht = torch.from_numpy(h).to(cuda)
    a = torch.empty_like(ht)
    native.had_r_128(ht, a, torch.from_numpy(u).to(cuda), None, 1.0)  # the reference's input rotation
    w = oracle.dequant(t, u, v, K, cb=cb).astype(np.float32)
    want = h.astype(np.float32) @ w
    out = torch.empty((M, out_f), dtype=torch.float32, device=cuda)
    native.exl3_fat_gemm(a, torch.from_numpy(t).to(cuda), out, torch.from_numpy(v).to(cuda), K, mcg, mul1)
    _close(out.cpu().numpy(), want)
    tok = torch.from_numpy(rng.permutation(T)[:M].astype(np.int64)).to(cuda)
    rw = torch.from_numpy(rng.uniform(0.1, 1, M).astype(np.float16)).to(cuda)
    acc0 = rng.normal(0, 1, (T, out_f)).astype(np.float32)
    acc = torch.from_numpy(acc0).to(cuda)
    native.exl3_fat_gemm_scatter(a, torch.from_numpy(t).to(cuda), acc, torch.from_numpy(v).to(cuda),
                                 tok, rw, K, mcg, mul1)
    exp = acc0.copy()
    exp[tok.cpu().numpy()] += want * rw.float().cpu().numpy()[:, None]
    _close(acc.cpu().numpy(), exp)


@pytest.mark.parametrize("rows", [1, 5, 40, 300])
def test_dense_linear_method_shards(native, cuda, rows):
    """Exl3LinearMethod mirror (exl3.py:6656-6739) on the GPU: three EXL3
    shards (QKV-like, K 2/3/4) through the opaque custom op, fp32 per shard
    rounded once to bf16, concatenated, 3-D input shape restored; the decode
    GEMV (< 32 rows) and the tcgen05 GEMM path (>= 32)."""
    import torch
    from exl3_b200 import linear as lin
    from exl3_b200 import synthetic
    rng = np.random.default_rng(600 + rows)
    projs = [synthetic.make_projection(rng, 512, o, K, synthetic.CB_MCG) for o, K in ((512, 4), (256, 2), (256, 3))]
    layer = lin.linear_from_projections(projs, cuda, name=f"test.dense.{rows}")
    x = torch.from_numpy(rng.normal(0, 1, (rows, 1, 512)).astype(np.float32)).to(cuda).to(torch.bfloat16)
    y = layer(x)
    assert y.shape == (rows, 1, 1024) and y.dtype == torch.bfloat16
    xh = x.reshape(rows, 512).float().cpu().numpy().astype(np.float16).astype(np.float32)
    want = np.concatenate([xh @ oracle.dequant(p.trellis, p.suh, p.svh, p.K, cb=1).astype(np.float32)
                           for p in projs], axis=1)
    # fp32 kernel output (the pass/fail comparison), then the bf16 layer output
    # equals that fp32 result rounded once
    f32 = torch.cat([native.exl3_linear(x.reshape(rows, 512), s.trellis, s.suh, s.svh, s.K, 1,
                                        out_dtype=torch.float32) for s in layer._exl3_linears], dim=1)
    _close(f32.cpu().numpy(), want)
    assert torch.equal(y.reshape(rows, 1024), f32.to(torch.bfloat16))


def test_ngram_dequant_bit_exact_with_reference_fixtures(native, cuda):
    """exl3_ngram_dequant (ExLlamaV3 ngram_dequant, exl3.py:5536-5544) against
    the reference's ngram_dequant_rows_torch outputs, K = 1..8, bit for bit."""
    import torch
    data = np.load(os.path.join(GOLDEN, "ngram.npz"))
    for K in range(1, 9):
        packed = torch.from_numpy(data[f"K{K}_packed"]).to(cuda)
        heads = torch.from_numpy(data[f"K{K}_heads"]).to(cuda)
        bias = torch.from_numpy(data[f"K{K}_bias"]).to(cuda)
        out = torch.empty(packed.shape[0], 160, dtype=torch.float16, device=cuda)
        native.ngram_dequant(packed, K, heads, bias, out)
        assert np.array_equal(out.cpu().numpy().view(np.uint16), data[f"K{K}_out"].view(np.uint16)), K


@pytest.mark.parametrize("K", [2, 3, 4, 8])
def test_ngram_embedding_lookup(native, cuda, K):
    """The fused lookup (gather, head search, decode, cast; exl3.py:5576-5587)
    against the oracle; an id outside the table gives a zero row and status 7."""
    import torch
    from exl3_b200.ngram import Exl3NgramEmbedding, ngram_words_per_row
    rng = np.random.default_rng(700 + K)
    n_rows, words = 5000, ngram_words_per_row(K)
    table = rng.integers(-32768, 32768, (n_rows, words), dtype=np.int16)
    table[:, 0] = rng.normal(0, 0.05, n_rows).astype(np.float16).view(np.int16)
    offsets = np.array([0, 1000, 1700, 4000], dtype=np.int64)
    bias = rng.normal(0, 0.02, (4, 160)).astype(np.float16)
    emb = Exl3NgramEmbedding(torch.from_numpy(table).to(cuda), K, torch.from_numpy(offsets),
                             torch.from_numpy(bias).to(cuda), dtype=torch.bfloat16)
    ids = rng.integers(0, n_rows, (3, 37)).astype(np.int64)
    ids[0, :4] = [0, 999, 1000, 4999]
    got = emb(torch.from_numpy(ids).to(cuda))
    assert got.shape == (3, 37, 160) and got.dtype == torch.bfloat16
    flat = ids.reshape(-1)
    heads = np.clip(np.searchsorted(offsets, flat, side="right") - 1, 0, 3)
    want = oracle.ngram_dequant(table[flat], K, heads, bias)
    want_bf16 = torch.from_numpy(want.astype(np.float32)).to(torch.bfloat16)
    assert torch.equal(got.reshape(-1, 160).cpu(), want_bf16)
    assert emb.status() == 0
    bad = torch.tensor([[5, n_rows, -1]], dtype=torch.int32, device=cuda)
    got_bad = emb(bad)
    assert emb.status() == 7
    assert torch.all(got_bad[0, 1:] == 0)
    want5 = oracle.ngram_dequant(table[[5]], K, np.array([0]), bias).astype(np.float32)
    assert torch.equal(got_bad[0, 0].cpu(), torch.from_numpy(want5[0]).to(torch.bfloat16))

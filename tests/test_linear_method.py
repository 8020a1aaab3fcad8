"""CPU tests of the dense linear method's host logic (exl3_b200.linear),
the mirror of Exl3LinearMethod.apply / _apply_impl (src/vllm_exl3/exl3.py:
6656-6739): shard order, fp32 concatenation and the cast back, bf16 shards,
input padding and output trimming, leading-shape restore, bias, and the
opaque custom op's shape-only fake implementation.  The EXL3 shard kernel
is replaced by the oracle's dense matmul here (no GPU); the GPU tests run the
real kernel.
"""

import numpy as np
import pytest
import torch

import cpu_oracle as oracle
from exl3_b200 import linear as lin
from exl3_b200 import synthetic
from exl3_b200.moe import Exl3Projection


def _proj(rng, i, o, K):
    p = synthetic.make_projection(rng, i, o, K, synthetic.CB_MCG)
    return p, Exl3Projection(torch.from_numpy(p.trellis), torch.from_numpy(p.suh), torch.from_numpy(p.svh), 1)


@pytest.fixture
def oracle_shards(monkeypatch):
    dense = {}

    def fake(linear, x_fp16, out_dtype=torch.float32):
        w = dense[id(linear)]
        return torch.from_numpy(x_fp16.float().numpy() @ w).to(out_dtype)

    monkeypatch.setattr(lin, "dense_forward", fake)
    return dense


def test_shards_concatenate_in_order_and_cast_back(oracle_shards):
    rng = np.random.default_rng(0)
    ps = [_proj(rng, 256, o, K) for o, K in ((256, 3), (128, 2), (128, 4))]
    for p, proj in ps:
        oracle_shards[id(proj)] = oracle.dequant(p.trellis, p.suh, p.svh, p.K, cb=1).astype(np.float32)
    layer = lin.Exl3Linear([proj for _p, proj in ps])
    x = torch.randn(2, 3, 256, dtype=torch.bfloat16)
    y = layer(x)
    assert y.shape == (2, 3, 512) and y.dtype == torch.bfloat16
    xh = x.reshape(6, 256).to(torch.float16).float().numpy()
    want = np.concatenate([xh @ oracle_shards[id(proj)] for _p, proj in ps], axis=1)
    assert torch.equal(y.reshape(6, 512), torch.from_numpy(want).to(torch.bfloat16))


def test_bf16_shard_bias_and_padding(oracle_shards):
    rng = np.random.default_rng(1)
    p, proj = _proj(rng, 256, 128, 3)
    oracle_shards[id(proj)] = oracle.dequant(p.trellis, p.suh, p.svh, p.K, cb=1).astype(np.float32)
    wb = torch.randn(64, 200, dtype=torch.bfloat16)
    layer = lin.Exl3Linear([proj, None], bf16_weight=wb, bf16_shards=[1], output_sizes=[128, 64],
                           bias=torch.ones(192, dtype=torch.bfloat16))
    layer._exl3_linear_padded = True
    layer._exl3_linear_input_size_per_partition = 256
    layer._exl3_linear_true_out = [128, 60]
    # the bf16 shard sees the unpadded input (F.linear on x itself)
    x = torch.randn(4, 200, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        layer(x)  # bias of the untrimmed width no longer matches: the trim happened
    layer.bias = torch.ones(188, dtype=torch.bfloat16)
    y = layer(x)
    assert y.shape == (4, 188)
    xp = torch.nn.functional.pad(x.to(torch.float16), (0, 56)).float().numpy()
    want = np.concatenate([xp @ oracle_shards[id(proj)], torch.nn.functional.linear(x, wb).float().numpy()], 1)
    want = torch.from_numpy(want[:, :188]).to(torch.bfloat16) + 1
    assert torch.allclose(y.float(), want.float(), atol=0.02 * float(want.float().abs().max()))


def test_missing_linears_raise():
    layer = lin.Exl3Linear([])
    with pytest.raises(RuntimeError, match="not built after weight load"):
        layer(torch.zeros(1, 128))


def test_custom_op_fake_shape():
    rng = np.random.default_rng(2)
    _p, proj = _proj(rng, 128, 256, 2)
    layer = lin.Exl3Linear([proj], name="test.layers.0.mlp.down_proj")
    assert lin.register_custom_ops()
    x = torch.empty(5, 7, 128, device="meta", dtype=torch.bfloat16)
    y = torch.ops.exl3_b200.exl3_linear_forward(x, "test.layers.0.mlp.down_proj")
    assert y.shape == (5, 7, 256) and y.dtype == torch.bfloat16 and y.device.type == "meta"
    del layer

"""Seeded synthetic EXL3 packs and routings for the benchmark configurations.

No real EXL3 checkpoint is available offline, so every weight and input is
drawn from a fixed numpy PCG64 seed (identical on every machine):

* trellis words: uniform int16 (every 16-bit state equally likely);
* SUH: random +-1 fp16;
* SVH: random +-1 times an fp16 per-tensor scale.  The reference format has
  no separate per-tensor scale field (src/vllm_exl3/exl3.py:117), so the scale
  s ~ U(0.5, 1.5) is folded into SVH together with 1/sqrt(in_features):
  svh = +-fp16(fp16(s) / sqrt(in)).  The extra 1/sqrt(in) keeps gate/up
  outputs O(1); without it the fp16 activation cast (act.half(),
  exl3.py:2410) overflows at hidden 7168.  Oracle and kernels consume the
  identical tensors;
* activations: N(0, 1) as bf16;
* routing: softmax(N(0, sigma) logits) -> top-k, weights not renormalised
  (configs 1-3), or sigmoid(N(0,1) logits + Zipf(1.1) expert bias) for
  selection with the selected sigmoids normalised to sum 1 (config 5).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

CB_MCG, CB_MUL1 = 1, 2


@dataclass
class Projection:
    trellis: np.ndarray  # int16 [in/16, out/16, 16K]
    suh: np.ndarray      # fp16 [in]
    svh: np.ndarray      # fp16 [out]
    K: int
    codebook: int

    @property
    def in_features(self) -> int:
        return self.trellis.shape[0] * 16

    @property
    def out_features(self) -> int:
        return self.trellis.shape[1] * 16


@dataclass
class MoEPack:
    hidden: int
    inter: int
    codebook: int
    experts: list = field(default_factory=list)  # [{"gate": P, "up": P, "down": P}]

    @property
    def n_experts(self) -> int:
        return len(self.experts)

    def k_table(self, which: str) -> np.ndarray:
        return np.array([e[which].K for e in self.experts], dtype=np.int8)

    @property
    def gateless(self) -> bool:
        return bool(self.experts) and all(e.get("gate") is None for e in self.experts)


def make_projection(rng: np.random.Generator, in_f: int, out_f: int, K: int, codebook: int,
                    scale: bool = True) -> Projection:
    trellis = rng.integers(-32768, 32768, size=(in_f // 16, out_f // 16, 16 * K), dtype=np.int16)
    suh = (rng.integers(0, 2, size=in_f) * 2 - 1).astype(np.float16)
    sign = (rng.integers(0, 2, size=out_f) * 2 - 1).astype(np.float32)
    s = np.float32(np.float16(rng.uniform(0.5, 1.5))) if scale else np.float32(1.0)
    mag = np.float16(s / np.sqrt(np.float32(in_f)))
    svh = (sign * np.float32(mag)).astype(np.float16)
    return Projection(trellis, suh, svh, int(K), int(codebook))


def make_moe_pack(seed: int, n_experts: int, hidden: int, inter: int, codebook: int,
                  k_choices=(4,), k_probs=None, gateless: bool = False) -> MoEPack:
    """Experts drawn from one generator in order; ``gateless`` packs have no
    gate projection (non-gated relu^2 layers)."""
    rng = np.random.default_rng(seed)
    ks = rng.choice(np.asarray(k_choices), size=n_experts, p=k_probs)
    pack = MoEPack(hidden, inter, codebook)
    for e in range(n_experts):
        K = int(ks[e])
        pack.experts.append({
            "gate": None if gateless else make_projection(rng, hidden, inter, K, codebook),
            "up": make_projection(rng, hidden, inter, K, codebook),
            "down": make_projection(rng, inter, hidden, K, codebook),
        })
    return pack


def make_moe_pack_slice(seed: int, n_experts: int, hidden: int, inter: int, codebook: int,
                        k_choices=(4,), k_probs=None, lo: int = 0, hi: int | None = None) -> MoEPack:
    """Experts [lo, hi) of an n_experts pack whose expert e is drawn from its
    own generator (seed, e): any rank of an expert-parallel group builds its
    shard without generating the others.  Per-expert K comes from one draw
    over all experts, so every rank agrees on it."""
    hi = n_experts if hi is None else hi
    ks = np.random.default_rng(seed).choice(np.asarray(k_choices), size=n_experts, p=k_probs)
    pack = MoEPack(hidden, inter, codebook)
    for e in range(lo, hi):
        rng = np.random.default_rng([seed, e])
        K = int(ks[e])
        pack.experts.append({
            "gate": make_projection(rng, hidden, inter, K, codebook),
            "up": make_projection(rng, hidden, inter, K, codebook),
            "down": make_projection(rng, inter, hidden, K, codebook),
        })
    return pack


def softmax_topk(rng: np.random.Generator, tokens: int, n_experts: int, topk: int,
                 sigma: float = 1.0):
    logits = rng.normal(0.0, sigma, size=(tokens, n_experts)).astype(np.float32)
    z = np.exp(logits - logits.max(axis=1, keepdims=True))
    p = z / z.sum(axis=1, keepdims=True)
    ids = np.argsort(-p, axis=1, kind="stable")[:, :topk]
    w = np.take_along_axis(p, ids, axis=1).astype(np.float32)
    return ids.astype(np.int64), w


def sigmoid_zipf_topk(rng: np.random.Generator, tokens: int, n_experts: int, topk: int,
                      s: float = 1.1, ranks: np.ndarray | None = None):
    """Top-k of sigmoid(N(0,1) logits + a per-expert Zipf(s) bias).  Expert e
    has popularity rank ``ranks[e]`` (0 = most popular).  A layer's router
    bias is a property of the layer, so batches of one layer pass the same
    ``ranks``; without it a permutation is drawn from ``rng``."""
    rank = rng.permutation(n_experts) if ranks is None else np.asarray(ranks)
    pz = 1.0 / np.power(rank + 1.0, s)
    pz /= pz.sum()
    bias = np.log(pz * n_experts).astype(np.float32)
    logits = rng.normal(0.0, 1.0, size=(tokens, n_experts)).astype(np.float32) + bias
    sig = 1.0 / (1.0 + np.exp(-logits))
    ids = np.argsort(-sig, axis=1, kind="stable")[:, :topk]
    w = np.take_along_axis(sig, ids, axis=1)
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids.astype(np.int64), w


def activations(rng: np.random.Generator, tokens: int, hidden: int) -> np.ndarray:
    """N(0,1) activations rounded to bf16, returned as float32."""
    x = rng.normal(0.0, 1.0, size=(tokens, hidden)).astype(np.float32)
    u = x.view(np.uint32)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)  # RNE to bf16
    return u.view(np.float32)


# --- the BASELINE configurations -------------------------------------------
CONFIGS = {
    # 1: CPU reference case
    "cfg1": dict(n_experts=8, topk=2, hidden=1024, inter=512, codebook=CB_MCG, k_choices=(4,),
                 tokens=16, routing="softmax", sigma=1.0),
    # 2: decode GEMV
    "cfg2": dict(n_experts=128, topk=8, hidden=2048, inter=768, codebook=CB_MCG, k_choices=(4,),
                 tokens=64, routing="softmax", sigma=1.0),
    # 3: mixed-K prefill (GLM-class)
    "cfg3": dict(n_experts=160, topk=8, hidden=5120, inter=1536, codebook=CB_MUL1,
                 k_choices=(2, 3), k_probs=(0.5, 0.5), tokens=2048, routing="softmax", sigma=1.5),
    # 5: expert-parallel layer
    "cfg5": dict(n_experts=256, topk=8, hidden=7168, inter=2048, codebook=CB_MCG,
                 k_choices=(2, 3, 4), k_probs=(0.3, 0.5, 0.2), tokens=8192, routing="sigmoid_zipf"),
}


def make_config(name: str, seed: int = 0, tokens: int | None = None, **over):
    """Return (pack, x [T,H] float32 holding bf16 values, ids [T,k] int64, w [T,k] float32)."""
    c = dict(CONFIGS[name])
    c.update(over)
    T = int(tokens if tokens is not None else c["tokens"])
    pack = make_moe_pack(seed, c["n_experts"], c["hidden"], c["inter"], c["codebook"],
                         c["k_choices"], c.get("k_probs"), c.get("gateless", False))
    rng = np.random.default_rng(seed + 1_000_003)
    x = activations(rng, T, c["hidden"])
    if c["routing"] == "sigmoid_zipf":
        ids, w = sigmoid_zipf_topk(rng, T, c["n_experts"], c["topk"])
    else:
        ids, w = softmax_topk(rng, T, c["n_experts"], c["topk"], c.get("sigma", 1.0))
    return pack, x, ids, w

"""Generate the golden fixtures in tests/golden/ from the REFERENCE itself.

Run in the build container, where the reference tree exists and its CPU
dequant is compiled (``make -C oracle ref``):

    python tests/golden/make_golden.py [--ref-src <reference checkout>/src]

Every expected value comes from reference code, never from this repository:

* ``half_kat.json`` / ``codebook_kat.json`` -- vllm_exl3.dequant
  (src/vllm_exl3/dequant.py:20-126) on the edge values of the reference's
  tests/test_dequant_parity.py plus seeded random windows for all three
  codebooks;
* ``dequant.npz`` -- ``dequant_trellis`` of the reference's own
  csrc/bindings.cpp (compiled CPU-only, oracle/_ref) on seeded trellises for
  K in {2,3,4,8} x {MCG, mul1}; the inputs are stored with the outputs;
* ``moe.npz`` -- the reference's eager loop ``apply_exl3_python_loop``
  (src/vllm_exl3/exl3.py:2357-2413) with projections realised as
  ``x.float() @ dequant_trellis(...).float()`` (the CPU branch of exl3_gemv,
  csrc/bindings.cpp:144-146), on small seeded layers: uniform-K MCG,
  mixed-K mul1 with a SwiGLU limit, and an expert_map with non-local routes;
* ``ngram.npz`` -- the reference's n-gram row decode ngram_dequant_rows_torch
  (src/vllm_exl3/exl3.py:5213-5239) for K in 1..8.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def main() -> None:
    ap = argparse.ArgumentParser()
    # the reference checkout: EXL3_REFERENCE_ROOT, else a sibling of this repository
    ref_root = os.environ.get("EXL3_REFERENCE_ROOT", os.path.join(os.path.dirname(ROOT), "reference"))
    ap.add_argument("--ref-src", default=os.path.join(ref_root, "src"))
    ap.add_argument("--only", choices=["all", "ngram"], default="all",
                    help="ngram: write only ngram.npz (the other fixtures stay as they are)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref_src)
    sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))
    import torch
    import vllm_exl3_ref_c as ref_c  # the reference's bindings.cpp, CPU-only build
    from vllm_exl3 import dequant as ref_dq
    from vllm_exl3 import exl3 as ref_exl3

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if args.only == "ngram":
        make_ngram(ref_exl3)
        return

    # ---- half conversion and codebook KATs
    values = [2.0**-15, 1.00075, -1.00075, 2.0**-24, 2.0**-25, 1.0 + 2.0**-11, 1.0 + 3 * 2.0**-11,
              65504.0, 65520.0, 0.0, -0.0, -70000.0, -32.125, -(2.0**-14), 0.333251953125,
              32.125, 70000.0, 1e-8, -1e-8, 6.1e-5, 3.14159265]
    rng = np.random.default_rng(20261201)
    values += [float(v) for v in rng.normal(0, 100, 32).astype(np.float32)]
    half = [{"value": v, "bits": int(ref_dq.float_to_half_bits_py(v))} for v in values]
    windows = [0x0000, 0x0001, 0x1234, 0x7FFF, 0xFFFF] + [int(w) for w in rng.integers(0, 65536, 123)]
    cbk = [{"window": w, "cb": cb, "bits": int(ref_dq.decode_codebook_bits_py(w, cb))}
           for w in windows for cb in (0, 1, 2)]
    cbk_float = [{"window": w, "mcg": ref_dq.decode_mcg_py(w), "mul1": ref_dq.decode_mul1_py(w)}
                 for w in windows[:5]]
    with open(os.path.join(HERE, "half_kat.json"), "w") as f:
        json.dump(half, f, indent=0)
    with open(os.path.join(HERE, "codebook_kat.json"), "w") as f:
        json.dump({"bits": cbk, "float": cbk_float}, f, indent=0)

    # ---- dequant_trellis
    deq = {}
    cases = []
    for K in (2, 3, 4, 8):
        for mcg in (True, False):
            for (rows, cols) in ((128, 128), (256, 384)):
                tag = f"K{K}_{'mcg' if mcg else 'mul1'}_{rows}x{cols}"
                t = rng.integers(-32768, 32768, (rows // 16, cols // 16, 16 * K), dtype=np.int16)
                u = (rng.integers(0, 2, rows) * 2 - 1).astype(np.float16)
                v = ((rng.integers(0, 2, cols) * 2 - 1) * np.float16(rng.uniform(0.5, 1.5))).astype(np.float16)
                w = ref_c.dequant_trellis(torch.from_numpy(t), torch.from_numpy(u), torch.from_numpy(v),
                                          K, mcg).numpy()
                deq[tag + "_trellis"] = t
                deq[tag + "_suh"] = u
                deq[tag + "_svh"] = v
                if rows == 128:
                    deq[tag + "_w"] = w
                cases.append({"tag": tag, "K": K, "mcg": mcg, "rows": rows, "cols": cols,
                              "sha256": hashlib.sha256(w.view(np.uint16).tobytes()).hexdigest()})
    np.savez_compressed(os.path.join(HERE, "dequant.npz"), **deq)
    with open(os.path.join(HERE, "dequant_cases.json"), "w") as f:
        json.dump(cases, f, indent=1)

    # ---- eager MoE loop
    class RefProj:
        def __init__(self, t, u, v, K, mcg):
            self.w = ref_c.dequant_trellis(torch.from_numpy(t), torch.from_numpy(u), torch.from_numpy(v),
                                           K, mcg).float()

        def forward(self, x, params, out_dtype=torch.float32):
            return (x.float() @ self.w).to(out_dtype)

    moe = {}
    meta = []
    layer_specs = [
        ("uniform_mcg", dict(E=4, topk=2, H=256, I=128, ks=(3,), mcg=True, T=8, limit=None, emap=False)),
        ("mixed_mul1_limit", dict(E=5, topk=3, H=256, I=256, ks=(2, 3, 4), mcg=False, T=7, limit=0.5,
                                  emap=False)),
        ("expert_map", dict(E=4, topk=2, H=128, I=128, ks=(4,), mcg=True, T=6, limit=None, emap=True)),
    ]
    for name, s in layer_specs:
        E, H, I = s["E"], s["H"], s["I"]
        inners = []
        for e in range(E):
            K = int(rng.choice(s["ks"]))
            proj = {}
            for which, (i_f, o_f) in (("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
                t = rng.integers(-32768, 32768, (i_f // 16, o_f // 16, 16 * K), dtype=np.int16)
                u = (rng.integers(0, 2, i_f) * 2 - 1).astype(np.float16)
                v = ((rng.integers(0, 2, o_f) * 2 - 1) * np.float16(1.0 / np.sqrt(i_f))).astype(np.float16)
                moe[f"{name}_e{e}_{which}_trellis"] = t
                moe[f"{name}_e{e}_{which}_suh"] = u
                moe[f"{name}_e{e}_{which}_svh"] = v
                proj[which] = RefProj(t, u, v, K, s["mcg"])
            inners.append(proj)
        T, topk = s["T"], s["topk"]
        x = rng.normal(0, 1, (T, H)).astype(np.float32)
        n_global = E * 2 if s["emap"] else E
        ids = np.stack([rng.choice(n_global, topk, replace=False) for _ in range(T)]).astype(np.int64)
        if s["emap"]:
            ids[0, 0] = -1          # invalid id -> sentinel
            ids[1, 1] = n_global + 3
        w = rng.uniform(0.05, 1.0, (T, topk)).astype(np.float32)
        emap = None
        if s["emap"]:
            # experts E..2E-1 are local 0..E-1; 0..E-1 belong to another rank
            emap_np = np.full(n_global, -1, dtype=np.int64)
            emap_np[E:] = np.arange(E)
            emap = torch.from_numpy(emap_np)
            moe[f"{name}_expert_map"] = emap_np
        out = ref_exl3.apply_exl3_python_loop(torch.from_numpy(x), torch.from_numpy(ids),
                                              torch.from_numpy(w), inners, emap, s["limit"]).numpy()
        moe[f"{name}_x"] = x
        moe[f"{name}_ids"] = ids
        moe[f"{name}_w"] = w
        moe[f"{name}_out"] = out
        meta.append({"name": name, "E": E, "topk": topk, "H": H, "I": I, "T": T,
                     "mcg": s["mcg"], "limit": s["limit"], "expert_map": s["emap"],
                     "K": [int(inners and moe[f"{name}_e{e}_gate_trellis"].shape[-1] // 16)
                           for e in range(E)]})
    np.savez_compressed(os.path.join(HERE, "moe.npz"), **moe)
    with open(os.path.join(HERE, "moe_cases.json"), "w") as f:
        json.dump(meta, f, indent=1)
    make_ngram(ref_exl3)
    print("golden fixtures written to", HERE)


def make_ngram(ref_exl3) -> None:
    """``ngram.npz``: the reference's own n-gram row decode,
    ``ngram_dequant_rows_torch`` (src/vllm_exl3/exl3.py:5213-5239), on seeded
    packed rows for every K in 1..8 with edge scale words and 3 heads."""
    import torch
    rng = np.random.default_rng(20261202)
    out = {}
    for K in range(1, 9):
        n = 12
        words = ref_exl3.ngram_words_per_row(K)
        packed = rng.integers(-32768, 32768, (n, words), dtype=np.int16)
        scales = rng.normal(0, 0.05, n).astype(np.float16)
        scales[0] = np.float16(0.0)
        scales[1] = np.float16(-1.5)
        packed[:, 0] = scales.view(np.int16)
        heads = rng.integers(0, 3, n).astype(np.int32)
        bias = rng.normal(0, 0.02, (3, ref_exl3.NGRAM_ROW_DIM)).astype(np.float16)
        got = ref_exl3.ngram_dequant_rows_torch(torch.from_numpy(packed), K, torch.from_numpy(heads),
                                                torch.from_numpy(bias)).numpy()
        out[f"K{K}_packed"] = packed
        out[f"K{K}_heads"] = heads
        out[f"K{K}_bias"] = bias
        out[f"K{K}_out"] = got
    np.savez_compressed(os.path.join(HERE, "ngram.npz"), **out)


if __name__ == "__main__":
    main()

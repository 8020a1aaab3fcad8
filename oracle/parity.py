"""Parity checks of device outputs against the CPU eager loop.

TEST INFRASTRUCTURE ONLY.  Used by ``tests/`` and by ``bench.py`` (which
checks each benchmarked line's outputs outside its timed region); the
product path never imports it.

The reference's eager loop (``apply_exl3_python_loop``,
src/vllm_exl3/exl3.py:2357-2413, restated in ``cpu_oracle.moe_eager``) is
evaluated on a subsample of tokens and, optionally, a subset of output
column blocks: each output row depends only on its own token's routes, and
each 128-column block of the down projection's reconstruction depends only on
its own tiles (``cpu_oracle.dequant_cols``), so a subsample is exactly the
corresponding part of the full result.  Tolerance (north star): max|d| <=
2e-2 * RMS(reference) and cosine >= 0.9995.
"""

from __future__ import annotations

import numpy as np

import cpu_oracle as oracle

TOL_MAX_OVER_RMS = 2e-2
TOL_COS = 0.9995


def stats(actual, expected) -> dict:
    """max|d| / RMS(expected) and the cosine similarity, in float64."""
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    rms = float(np.sqrt(np.mean(e * e)))
    maxd = float(np.max(np.abs(a - e))) if a.size else 0.0
    cos = float(a @ e / (np.linalg.norm(a) * np.linalg.norm(e) + 1e-30))
    return {"max_abs_over_rms": maxd / (rms + 1e-30), "cos": cos, "finite": bool(np.isfinite(a).all()),
            "n": int(a.size)}


def passes(st: dict) -> bool:
    return st["finite"] and st["max_abs_over_rms"] <= TOL_MAX_OVER_RMS and st["cos"] >= TOL_COS


def assert_close(actual, expected) -> dict:
    st = stats(actual, expected)
    assert st["finite"], "non-finite output"
    assert st["max_abs_over_rms"] <= TOL_MAX_OVER_RMS, f"max|d|/rms {st['max_abs_over_rms']:.3e} > {TOL_MAX_OVER_RMS}"
    assert st["cos"] >= TOL_COS, f"cosine {st['cos']}"
    return st


def col_blocks(hidden: int, nblocks: int, seed: int = 0) -> list[int]:
    """`nblocks` distinct 128-column block indices of a hidden width, sorted."""
    n = hidden // 128
    if nblocks >= n:
        return list(range(n))
    return sorted(np.random.default_rng(seed).choice(n, nblocks, replace=False).tolist())


def projection_dense(p, blocks: list[int] | None = None) -> np.ndarray:
    """fp16 weights of one synthetic projection (``exl3_b200.synthetic``
    Projection): every column, or the listed 128-column blocks in order."""
    if blocks is None:
        return oracle.dequant(p.trellis, p.suh, p.svh, p.K, cb=p.codebook)
    parts = [oracle.dequant_cols(p.trellis, p.suh, p.svh, p.K, p.codebook, 128 * b, 128 * (b + 1))
             for b in blocks]
    return np.concatenate(parts, axis=1)


def expert_dense_fn(expert_of, blocks: list[int] | None = None):
    """A callable for ``moe_eager``: local expert e -> dense gate/up (all
    columns) and down (the listed output blocks).  ``expert_of(e)`` returns
    the synthetic expert dict {"gate", "up", "down"}."""

    def get(e: int) -> dict:
        ex = expert_of(e)
        gate = ex.get("gate")
        return {"gate": None if gate is None else projection_dense(gate),
                "up": projection_dense(ex["up"]),
                "down": projection_dense(ex["down"], blocks)}

    return get


def expected_moe(x_rows, ids_rows, w_rows, expert_of, n_local: int, blocks: list[int] | None = None,
                 limit: float | None = None, act: str = "silu", expert_map=None) -> np.ndarray:
    """The eager loop's fp32 output on these rows (the listed column blocks,
    concatenated, when `blocks` is given)."""
    return oracle.moe_eager(np.asarray(x_rows), np.asarray(ids_rows), np.asarray(w_rows),
                            expert_dense_fn(expert_of, blocks), expert_map=expert_map, limit=limit, act=act,
                            n_local=n_local)


def compare(got_rows, want: np.ndarray, blocks: list[int] | None = None) -> dict:
    """Statistics and verdict of device rows (full width, or already the
    listed blocks) against :func:`expected_moe`'s result."""
    got = np.asarray(got_rows, np.float32)
    if blocks is not None and got.shape[1] != want.shape[1]:
        got = np.concatenate([got[:, 128 * b:128 * (b + 1)] for b in blocks], axis=1)
    st = stats(got, want)
    st["pass"] = passes(st)
    return st


def check_moe(got_rows, x_rows, ids_rows, w_rows, expert_of, n_local: int, blocks: list[int] | None = None,
              limit: float | None = None, act: str = "silu", expert_map=None) -> dict:
    """Compare device output rows (fp32 [t, H], or [t, 128 * len(blocks)]
    already restricted to `blocks`) with the eager loop on the same rows."""
    want = expected_moe(x_rows, ids_rows, w_rows, expert_of, n_local, blocks, limit, act, expert_map)
    st = compare(got_rows, want, blocks)
    st["tokens"] = int(np.asarray(x_rows).shape[0])
    st["col_blocks"] = None if blocks is None else len(blocks)
    return st


def sample_tokens(tokens: int, n: int, seed: int = 0) -> np.ndarray:
    """`n` distinct token indices of a batch (all when n >= tokens), sorted."""
    if n >= tokens:
        return np.arange(tokens)
    return np.sort(np.random.default_rng(seed).choice(tokens, n, replace=False))

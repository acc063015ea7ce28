"""numpy restatement of lorafusion's CPU reference op (TEST INFRASTRUCTURE ONLY).

Follows ``lorafusion/ops/mock_ops.py`` step by step, in the dtype of the
inputs (float32 for every comparison in this repository; bf16 problems are
compared by running this oracle in float32 on the bf16-rounded values):

* :func:`fused_lora_forward` — ``mock_ops.py:15-48``: ``out = x @ W.T`` then,
  route by route, ``out[rows] += scaling * ((x[rows] @ A.T) @ B.T)``.
* :func:`fused_lora_backward` — ``mock_ops.py:51-95``: ``grad_x = g @ W``;
  per route ``xa = x_s @ A.T``, ``dB = s * (g_s.T @ xa)``, ``gxa = s * (g_s @ B)``,
  ``dA = gxa.T @ x_s``, ``grad_x[rows] += gxa @ A``; gradients of an adapter
  that owns several routes are summed in route order, and the dicts hold only
  adapters that appear in the routes, in order of first appearance.

Routes are ``(row_start, row_end, adapter_id)`` triples; ``scaling`` maps
adapter id to ``alpha / rank``.  Validation mirrors
``lorafusion/ops/config.py:55-69``.
"""

from __future__ import annotations

import numpy as np


def validate_routes(routes, total_rows: int) -> None:
    """Raise ValueError on a gap/overlap or a coverage mismatch (config.py:55-69)."""
    expect = 0
    covered = 0
    for rs, re_, _ in routes:
        if rs != expect:
            raise ValueError(f"Routing gap/overlap at row {rs}, expected {expect}")
        covered += re_ - rs
        expect = re_
    if covered != total_rows:
        raise ValueError(f"Routing covers {covered} rows, expected {total_rows}")


def fused_lora_forward(x, w, lora_a, lora_b, scaling, routes):
    """``y = x W^T + s_i (x A_i^T) B_i^T`` per routed row range (mock_ops.py:15-48)."""
    validate_routes(routes, x.shape[0])
    out = x @ w.T
    for rs, re_, aid in routes:
        xs = x[rs:re_]
        delta = (xs @ lora_a[aid].T) @ lora_b[aid].T
        out[rs:re_] += np.asarray(scaling[aid], dtype=out.dtype) * delta
    return out


def fused_lora_backward(g, x, w, lora_a, lora_b, scaling, routes):
    """Return ``(grad_x, grad_a, grad_b)`` exactly as mock_ops.py:51-95 defines them."""
    validate_routes(routes, x.shape[0])
    grad_x = g @ w
    grad_a: dict[int, np.ndarray] = {}
    grad_b: dict[int, np.ndarray] = {}
    for rs, re_, aid in routes:
        s = np.asarray(scaling[aid], dtype=grad_x.dtype)
        xs = x[rs:re_]
        gs = g[rs:re_]
        a = lora_a[aid]
        b = lora_b[aid]
        xa = xs @ a.T
        gb = s * (gs.T @ xa)
        gxa = s * (gs @ b)
        ga = gxa.T @ xs
        grad_x[rs:re_] += gxa @ a
        grad_a[aid] = ga if aid not in grad_a else grad_a[aid] + ga
        grad_b[aid] = gb if aid not in grad_b else grad_b[aid] + gb
    return grad_x, grad_a, grad_b


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32).reshape(a.shape)
    return np.where(nan, np.float32(np.nan), out)


def allclose_report(got: np.ndarray, ref: np.ndarray, rtol: float, atol: float) -> tuple[bool, str]:
    """Elementwise ``|got-ref| <= rtol*|ref| + atol*max(1, max|ref|)``; returns (ok, summary).

    The absolute term is scaled by the tensor's largest magnitude: the gradient
    sums reach |ref| ~ 1e2 and cancel, so any implementation that sums in
    another order (another BLAS included) differs from the reference by about
    eps * sum|terms| in near-zero entries, which a fixed atol cannot absorb.
    """
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if got.shape != ref.shape:
        return False, f"shape {got.shape} != {ref.shape}"
    if not np.all(np.isfinite(got)):
        return False, f"{int((~np.isfinite(got)).sum())} non-finite values"
    err = np.abs(got - ref)
    scale = max(1.0, float(np.abs(ref).max())) if ref.size else 1.0
    bad = err > atol * scale + rtol * np.abs(ref)
    n_bad = int(bad.sum())
    worst = float(err.max()) if err.size else 0.0
    return n_bad == 0, f"{n_bad}/{err.size} outside tol, max abs err {worst:.3e}"

"""numpy restatement of lorafusion's CPU reference op (TEST INFRASTRUCTURE ONLY).

Follows ``lorafusion/ops/mock_ops.py`` step by step, in the dtype of the
inputs.  The parity tests run it in float64 on the very values the GPU gets
(bf16/f16 problems: the bf16/f16-rounded values), i.e. as the exact math of
the reference's formula, and compare with the plain elementwise rule of
:func:`allclose_report`:

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


def as_f64(d):
    """A dict of arrays (or one array) as float64 copies."""
    if isinstance(d, dict):
        return {k: np.asarray(v, dtype=np.float64) for k, v in d.items()}
    return np.asarray(d, dtype=np.float64)


def allclose_report(got: np.ndarray, ref: np.ndarray, rtol: float, atol: float,
                    bound: np.ndarray | None = None) -> tuple[bool, str]:
    """Elementwise ``|got - ref| <= atol + rtol * |ref|`` (plus ``bound`` when given); returns
    (ok, summary).  The summary gives the worst ratio ``|got - ref| / (atol + rtol |ref|)``: at
    most 1 means every element is within tolerance."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if got.shape != ref.shape:
        return False, f"shape {got.shape} != {ref.shape}"
    if not np.all(np.isfinite(got)):
        return False, f"{int((~np.isfinite(got)).sum())} non-finite values"
    err = np.abs(got - ref)
    lim = atol + rtol * np.abs(ref)
    if bound is not None:
        lim = lim + np.asarray(bound, dtype=np.float64)
    n_bad = int((err > lim).sum())
    worst = float((err / lim).max()) if err.size else 0.0
    return n_bad == 0, f"{n_bad}/{err.size} outside tol, worst |err|/tol {worst:.3f}, max abs err " \
                       f"{float(err.max()) if err.size else 0.0:.3e}"


_U32 = 2.0 ** -24  # unit roundoff of float32


def fp32_forward_error_bounds(x, w, lora_a, lora_b, scaling, routes, g=None):
    """Elementwise bounds on how far a float32 evaluation of the reference's formula (any
    summation order) can be from the exact value: gamma_L * M, where M is the same computation on
    absolute values (the sum of |terms| of every dot product on the path) and
    gamma_L = L u / (1 - L u) with L the longest chain of roundings on any path (at most
    K + N + T + max rank + routes + 4), u = 2^-24 (the classic forward error bound of summation
    and dot products).  Used only to pin this oracle against the reference's own float32
    outputs.  Returns (y_bound,) or, with ``g``, (y_bound, gx_bound, ga_bounds, gb_bounds)."""
    T, K = np.shape(x)
    N = np.shape(w)[0]
    max_rank = max((np.shape(a)[0] for a in lora_a.values()), default=0)
    L = K + N + T + max_rank + len(routes) + 4
    gamma = L * _U32 / (1.0 - L * _U32)
    ab = lambda d: {k: np.abs(np.asarray(v, dtype=np.float64)) for k, v in d.items()}  # noqa: E731
    sc = {k: abs(float(v)) for k, v in scaling.items()}
    xa, wa = np.abs(np.asarray(x, dtype=np.float64)), np.abs(np.asarray(w, dtype=np.float64))
    my = fused_lora_forward(xa, wa, ab(lora_a), ab(lora_b), sc, routes)
    if g is None:
        return (gamma * my,)
    mgx, mga, mgb = fused_lora_backward(np.abs(np.asarray(g, dtype=np.float64)), xa, wa, ab(lora_a), ab(lora_b), sc,
                                        routes)
    return (gamma * my, gamma * mgx, {k: gamma * v for k, v in mga.items()}, {k: gamma * v for k, v in mgb.items()})

"""Pin the CPU oracle against outputs of the reference itself (golden fixtures)."""

import numpy as np
import pytest

from conftest import op_case
from oracle import mock_oracle, scheduler_oracle

FP32_TOL = dict(rtol=1e-5, atol=1e-5)


def _names(z):
    return [str(n) for n in z["names"]]


def test_fixtures_present(ops_golden, layout_golden):
    assert len(_names(ops_golden)) >= 6
    assert len(_names(layout_golden)) >= 13


@pytest.mark.parametrize("name", ["cfg1", "single_route", "split_adapter", "rank1_one_row_routes",
                                  "unused_adapter", "bf16_mixed_ranks"])
def test_oracle_forward_backward_matches_reference(ops_golden, name):
    """The oracle, evaluated in float64 (the exact math of the formula), against the reference's
    own float32 outputs.  The reference rounds in float32, so an element may differ from the exact
    value by its float32 forward-error bound on top of rtol = atol = 1e-5; every element must be
    within that, and all but a handful within the plain 1e-5 rule."""
    c = op_case(ops_golden, name)
    f = mock_oracle.as_f64
    x, w, g, a, b = f(c["x"]), f(c["w"]), f(c["g"]), f(c["a"]), f(c["b"])
    by, bgx, bga, bgb = mock_oracle.fp32_forward_error_bounds(x, w, a, b, c["scaling"], c["routes"], g=g)
    plain_misses = 0

    def check(got, ref, bound, what):
        nonlocal plain_misses
        ok, msg = mock_oracle.allclose_report(got, ref, **FP32_TOL, bound=bound)
        assert ok, f"{what}: {msg}"
        plain_misses += int(not mock_oracle.allclose_report(got, ref, **FP32_TOL)[0])

    y = mock_oracle.fused_lora_forward(x, w, a, b, c["scaling"], c["routes"])
    check(y, c["y"], by, "forward")
    gx, ga, gb = mock_oracle.fused_lora_backward(g, x, w, a, b, c["scaling"], c["routes"])
    check(gx, c["gx"], bgx, "grad_x")
    assert list(ga.keys()) == c["grad_keys"] and list(gb.keys()) == c["grad_keys"]
    for k in c["grad_keys"]:
        check(ga[k], c["ga"][k], bga[k], f"grad_a[{k}]")
        check(gb[k], c["gb"][k], bgb[k], f"grad_b[{k}]")
    assert plain_misses <= 1, f"{plain_misses} tensors outside the plain 1e-5 rule"


def test_fp32_bound_is_not_vacuous(ops_golden):
    """The float32 bound is a small fraction of the values it bounds, and a wrong oracle (one
    adapter's scaling off by 1e-3) falls outside it."""
    c = op_case(ops_golden, "cfg1")
    f = mock_oracle.as_f64
    x, w, g, a, b = f(c["x"]), f(c["w"]), f(c["g"]), f(c["a"]), f(c["b"])
    by, bgx, bga, bgb = mock_oracle.fp32_forward_error_bounds(x, w, a, b, c["scaling"], c["routes"], g=g)
    assert float(np.max(by / np.maximum(np.abs(c["y"]), 1.0))) < 1e-3
    wrong = dict(c["scaling"])
    k0 = c["grad_keys"][0]
    wrong[k0] *= 1.001
    _, ga, _ = mock_oracle.fused_lora_backward(g, x, w, a, b, wrong, c["routes"])
    ok, _ = mock_oracle.allclose_report(ga[k0], c["ga"][k0], **FP32_TOL, bound=bga[k0])
    assert not ok


def test_oracle_validate_errors():
    with pytest.raises(ValueError, match="gap/overlap"):
        mock_oracle.validate_routes([(0, 10, 0), (15, 20, 1)], 20)
    with pytest.raises(ValueError, match="covers 10 rows"):
        mock_oracle.validate_routes([(0, 10, 0)], 20)


def test_bf16_round_matches_torch():
    import torch
    a = np.random.default_rng(0).standard_normal(4096).astype(np.float32) * 37.0
    a[:4] = [0.0, -0.0, 1e-40, 3.4e38]
    ref = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(mock_oracle.bf16_round(a), ref)


def test_scheduler_oracle_matches_reference(layout_golden):
    z = layout_golden
    for name in _names(z):
        reqs = [tuple(int(v) for v in r) for r in z[f"{name}/requests"]]
        cap = int(z[f"{name}/cap"])
        rows = scheduler_oracle.bucket_rows(reqs)
        bins = scheduler_oracle.greedy_bins(rows, cap)
        flat = [(b, a, n) for b, entries in enumerate(bins) for a, n in entries]
        assert flat == [tuple(int(v) for v in r) for r in z[f"{name}/bins"]], name
        routes, row_order, source = scheduler_oracle.microbatch_layout(reqs, bins)
        assert routes == [tuple(int(v) for v in r) for r in z[f"{name}/routes"]], name
        assert row_order == [int(v) for v in z[f"{name}/row_order"]], name
        assert source == [tuple(int(v) for v in r) for r in z[f"{name}/source"]], name

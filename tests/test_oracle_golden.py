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
    c = op_case(ops_golden, name)
    y = mock_oracle.fused_lora_forward(c["x"], c["w"], c["a"], c["b"], c["scaling"], c["routes"])
    ok, msg = mock_oracle.allclose_report(y, c["y"], **FP32_TOL)
    assert ok, "forward " + msg
    gx, ga, gb = mock_oracle.fused_lora_backward(c["g"], c["x"], c["w"], c["a"], c["b"], c["scaling"], c["routes"])
    ok, msg = mock_oracle.allclose_report(gx, c["gx"], **FP32_TOL)
    assert ok, "grad_x " + msg
    assert list(ga.keys()) == c["grad_keys"] and list(gb.keys()) == c["grad_keys"]
    for k in c["grad_keys"]:
        ok, msg = mock_oracle.allclose_report(ga[k], c["ga"][k], **FP32_TOL)
        assert ok, f"grad_a[{k}] " + msg
        ok, msg = mock_oracle.allclose_report(gb[k], c["gb"][k], **FP32_TOL)
        assert ok, f"grad_b[{k}] " + msg


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

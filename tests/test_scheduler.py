"""The shipped scheduler reproduces the reference's layout bit-exactly, plus the
reference's own property tests (lorafusion tests/test_scheduler.py:14-98)."""

import numpy as np
import pytest
import torch

from lorafusion_b200.config import TileRoute, TileRoutingConfig
from lorafusion_b200.scheduler import (AdapterGroup, Request, bucket_by_adapter, build_microbatch,
                                       check_bubble_lemma, greedy_pack, group_by_adapter, milp_pack,
                                       scatter_outputs)


def _names(z):
    return [str(n) for n in z["names"]]


def test_layout_bit_exact_against_reference(layout_golden):
    z = layout_golden
    for name in _names(z):
        reqs = [Request(*(int(v) for v in r)) for r in z[f"{name}/requests"]]
        cap = int(z[f"{name}/cap"])
        groups = bucket_by_adapter(reqs)
        assert check_bubble_lemma(groups, reqs)
        packing = greedy_pack({g.adapter_id: g.total_rows for g in groups}, cap)
        flat = [(b, a, n) for b, entries in enumerate(packing.bins) for a, n in entries]
        assert flat == [tuple(int(v) for v in r) for r in z[f"{name}/bins"]], name
        tensors = {r.request_id: torch.stack([torch.full((r.num_rows,), float(r.request_id), dtype=torch.float64),
                                              torch.arange(r.num_rows, dtype=torch.float64)], 1) for r in reqs}
        fused, routing, row_order = build_microbatch(reqs, tensors, packing)
        routes = [(rt.row_start, rt.row_end, rt.adapter_id) for rt in routing.routes]
        assert routes == [tuple(int(v) for v in r) for r in z[f"{name}/routes"]], name
        assert routing.num_tiles() == int(z[f"{name}/num_tiles"])
        assert row_order == [int(v) for v in z[f"{name}/row_order"]], name
        np.testing.assert_array_equal(fused.numpy().astype(np.int64), z[f"{name}/source"])
        routing.validate(fused.shape[0])
        out = scatter_outputs(fused, row_order)
        assert list(out.keys()) == [int(k) for k in z[f"{name}/scatter_keys"]]
        rows = np.concatenate([v[:, 1].numpy() for v in out.values()]).astype(np.int64)
        np.testing.assert_array_equal(rows, z[f"{name}/scatter_rows"])


def test_greedy_pack_respects_capacity():
    result = greedy_pack({0: 100, 1: 50, 2: 30}, tile_capacity=64)
    assert all(sum(r for _, r in b) <= 64 for b in result.bins)
    assert sum(r for b in result.bins for _, r in b) == 180
    assert result.method == "greedy"


def test_greedy_pack_splits_oversized_adapter():
    result = greedy_pack({0: 150}, tile_capacity=64)
    rows = [sum(r for _, r in b) for b in result.bins]
    assert all(r <= 64 for r in rows) and sum(rows) == 150


def test_pack_rejects_bad_capacity():
    with pytest.raises(ValueError):
        greedy_pack({0: 3}, 0)


def test_milp_pack_no_worse_than_greedy_and_falls_back():
    rows = {0: 40, 1: 40, 2: 40, 3: 40}
    assert milp_pack(rows, 64, time_limit_s=5.0).num_bins <= greedy_pack(rows, 64).num_bins
    res = milp_pack({0: 10, 1: 200}, tile_capacity=64, time_limit_s=1.0)
    assert sum(r for b in res.bins for _, r in b) == 210
    assert all(sum(r for _, r in b) <= 64 for b in res.bins)


def test_grouping_semantics():
    reqs = [Request(0, 1, 4), Request(1, 1, 6), Request(2, 2, 3), Request(3, 1, 2)]
    g = group_by_adapter(reqs)
    assert [(x.adapter_id, x.total_rows) for x in g] == [(1, 10), (2, 3), (1, 2)]
    b = bucket_by_adapter([Request(0, 1, 4), Request(1, 2, 6), Request(2, 1, 3)])
    assert {x.adapter_id: x.total_rows for x in b} == {1: 7, 2: 6}
    assert [x.adapter_id for x in b] == [1, 2]


def test_bubble_lemma():
    reqs = [Request(0, 1, 4), Request(1, 1, 6), Request(2, 2, 3)]
    assert check_bubble_lemma(group_by_adapter(reqs), reqs)
    bad = [AdapterGroup(1, [0], 6), AdapterGroup(1, [0], 4)]
    assert not check_bubble_lemma(bad, [Request(0, 1, 10)])


def test_routing_validate_errors():
    with pytest.raises(ValueError, match="gap/overlap"):
        TileRoutingConfig(64, [TileRoute(0, 10, 0), TileRoute(15, 20, 1)]).validate(20)
    with pytest.raises(ValueError, match="covers 10 rows"):
        TileRoutingConfig(64, [TileRoute(0, 10, 0)]).validate(20)
    TileRoutingConfig(64, []).validate(0)


def _random_rows(rng, n, cap):
    rows = {}
    for _ in range(n):
        aid = int(rng.integers(-50, 10_000))
        rows[aid] = int(rng.choice([0, -3, 1, cap - 1, cap, cap + 1, 3 * cap + 7, int(rng.integers(1, 4 * cap))]))
    return rows


@pytest.mark.parametrize("seed", range(12))
def test_native_greedy_pack_equals_oracle_first_fit(seed):
    """lf_greedy_pack (segment-tree first fit) gives the reference's bins exactly, ties included."""
    from oracle.scheduler_oracle import greedy_bins
    rng = np.random.default_rng(seed)
    cap = int(rng.choice([1, 16, 64, 128, 1000]))
    rows = _random_rows(rng, int(rng.integers(0, 300)), cap)
    assert greedy_pack(rows, cap).bins == greedy_bins(rows, cap)


def test_native_greedy_pack_at_config_sizes():
    from oracle.scheduler_oracle import greedy_bins
    from lorafusion_b200.workloads import WORKLOADS, row_counts
    for wl in WORKLOADS.values():
        rows = dict(enumerate(row_counts(wl, wl.total_rows)))
        assert greedy_pack(rows, wl.tile_capacity).bins == greedy_bins(rows, wl.tile_capacity), wl.name


def test_native_greedy_pack_argument_errors():
    import ctypes
    from lorafusion_b200 import _native as nat
    with pytest.raises(ValueError):
        greedy_pack({0: 3}, -1)
    with pytest.raises(ValueError):
        greedy_pack({1 << 40: 3}, 8)
    assert greedy_pack({}, 8).bins == []
    assert greedy_pack({3: 0, 4: -2}, 8).bins == []
    P = ctypes.POINTER(ctypes.c_int32)
    ids = (ctypes.c_int32 * 1)(7)
    rows = (ctypes.c_int32 * 1)(100)
    n_ent, n_bins = ctypes.c_int32(0), ctypes.c_int32(0)
    out = (ctypes.c_int32 * 8)()
    rc = nat.lib().lf_greedy_pack(ids, rows, 1, 16, 2, out, out, out, ctypes.byref(n_ent), ctypes.byref(n_bins))
    assert rc == nat.LF_ERR_CAPACITY and n_ent.value == 7  # ceil(100 / 16) chunks needed

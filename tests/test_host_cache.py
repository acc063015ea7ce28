"""Host-side caches of the op (no GPU needed): route validation is redone exactly when the routes
or the row count change, adapter records follow tensor identity, storage and version counters,
and the gradient dicts are views of the packed gradient buffers in slot order."""

import pytest
import torch

from lorafusion_b200 import b200_ops as ops
from lorafusion_b200.config import AdapterSpec, TileRoute, TileRoutingConfig


def _routing():
    return TileRoutingConfig(16, [TileRoute(0, 5, 2), TileRoute(5, 9, 0), TileRoute(9, 12, 2)])


def test_routes_are_revalidated_only_when_they_change():
    ops.clear_weight_cache()
    rt = _routing()
    r1 = ops._routes(rt, 12)
    assert ops._routes(rt, 12) is r1
    assert r1.slots == (2, 0) and list(r1.route_slot) == [0, 1, 0]
    with pytest.raises(ValueError, match="covers"):
        ops._routes(rt, 13)  # another row count is validated again
    rt.routes[1] = TileRoute(5, 8, 0)  # routes edited in place: no longer tile [0, 12)
    with pytest.raises(ValueError, match="gap/overlap"):
        ops._routes(rt, 12)
    rt.routes[1] = TileRoute(5, 9, 1)
    r2 = ops._routes(rt, 12)
    assert r2 is not r1 and r2.slots == (2, 1)


def test_adapter_records_follow_identity_storage_and_version():
    ops.clear_weight_cache()
    rt = ops._routes(_routing(), 12)
    a = {0: torch.randn(4, 8), 2: torch.randn(8, 8)}
    b = {0: torch.randn(6, 4), 2: torch.randn(6, 8)}
    ad = {0: AdapterSpec(0, 4, 8.0, 8, 6), 2: AdapterSpec(2, 8, 4.0, 8, 6)}
    rec = ops._adapters(rt, a, b, ad)
    assert rec.ranks == (8, 4) and rec.scales == (0.5, 2.0)  # slot order: adapter 2, then 0
    assert ops._adapters(rt, dict(a), dict(b), dict(ad)) is rec  # new dicts, same tensors
    a[0].add_(1.0)  # in-place update bumps the version counter
    rec2 = ops._adapters(rt, a, b, ad)
    assert rec2 is not rec and ops._adapters(rt, a, b, ad) is rec2
    b[2] = torch.randn(6, 8)  # another tensor object
    rec3 = ops._adapters(rt, a, b, ad)
    assert rec3 is not rec2
    ad2 = {0: AdapterSpec(0, 4, 16.0, 8, 6), 2: ad[2]}  # new scaling, same tensors: same slabs
    rec4 = ops._adapters(rt, a, b, ad2)
    assert rec4 is rec3 and rec4.scales == (0.5, 4.0)
    with pytest.raises(KeyError):
        ops._adapters(rt, {0: a[0]}, b, ad)


class _Info:
    def __init__(self, rank_total):
        self.rank_total = rank_total


class _PlanStub:
    def __init__(self, slots, ranks):
        self.slots, self.ranks, self.info = tuple(slots), tuple(ranks), _Info(sum(ranks))
        self.vslots = ops._virtual_slots(ranks)


@pytest.mark.parametrize("ranks", [[16] * 5, [16, 16, 8, 32, 32, 4, 4, 64], [1], []])
def test_grad_dicts_are_views_in_slot_order(ranks):
    K, N = 24, 40
    slots = [10 + 3 * i for i in range(len(ranks))]
    plan = _PlanStub(slots, ranks)
    rtot = sum(ranks)
    ga = torch.arange(max(rtot * K, 1), dtype=torch.float32)
    gb = torch.arange(max(rtot * N, 1), dtype=torch.float32) + 0.5
    da, db = ops._grad_dicts(plan, ga, gb, K, N)
    assert list(da) == slots and list(db) == slots
    off = 0
    for aid, r in zip(slots, ranks):
        assert da[aid].shape == (r, K) and db[aid].shape == (N, r)
        assert da[aid].is_contiguous() and db[aid].is_contiguous()
        assert torch.equal(da[aid], ga[off * K:(off + r) * K].view(r, K))
        assert torch.equal(db[aid], gb[off * N:(off + r) * N].view(N, r))
        assert da[aid].data_ptr() == ga[off * K:].data_ptr()  # views, no copies
        off += r


def test_grad_dicts_of_ranks_above_64_join_virtual_slot_blocks():
    """An adapter of rank 130 has three virtual slots (64, 64, 2): its dA rows are one view, its dB
    is the three [N, r_v] blocks joined along the rank dimension."""
    K, N = 8, 6
    ranks = [16, 130, 8]
    slots = [4, 9, 2]
    plan = _PlanStub(slots, ranks)
    assert plan.vslots == ((0, 0, 16), (1, 0, 64), (1, 64, 64), (1, 128, 2), (2, 0, 8))
    rtot = sum(ranks)
    ga = torch.arange(rtot * K, dtype=torch.float32)
    gb = torch.arange(rtot * N, dtype=torch.float32)
    da, db = ops._grad_dicts(plan, ga, gb, K, N)
    assert da[9].shape == (130, K) and torch.equal(da[9], ga[16 * K:146 * K].view(130, K))
    blocks = [gb[(16 + c0) * N:(16 + c0 + r) * N].view(N, r) for c0, r in ((0, 64), (64, 64), (128, 2))]
    assert db[9].shape == (N, 130) and db[9].is_contiguous() and torch.equal(db[9], torch.cat(blocks, dim=1))
    assert torch.equal(db[2], gb[146 * N:154 * N].view(N, 8)) and torch.equal(db[4], gb[:16 * N].view(N, 16))


def test_many_adapter_sets_on_one_routing_all_stay_cached():
    """A model calls the op with one routing and many adapter sets (layers x projections): every
    set keeps its record (and so its packed slabs) instead of being evicted in a cycle."""
    ops.clear_weight_cache()
    rt = ops._routes(_routing(), 12)
    sets = []
    for _ in range(40):
        a = {0: torch.randn(4, 8), 2: torch.randn(8, 8)}
        b = {0: torch.randn(6, 4), 2: torch.randn(6, 8)}
        ad = {0: AdapterSpec(0, 4, 8.0, 8, 6), 2: AdapterSpec(2, 8, 4.0, 8, 6)}
        sets.append((a, b, ad, ops._adapters(rt, a, b, ad)))
    for a, b, ad, rec in sets:  # second pass, same order: every lookup hits
        assert ops._adapters(rt, a, b, ad) is rec


def test_saved_sf_is_kept_per_input_and_adapter_set():
    """Forwards of several projections on the same x (q, k, v) each keep their own S_f; an entry
    whose x has died is dropped."""
    ops.clear_weight_cache()
    rt = ops._routes(_routing(), 12)
    x = torch.randn(12, 8)
    recs = []
    for _ in range(3):
        a = {0: torch.randn(4, 8), 2: torch.randn(8, 8)}
        b = {0: torch.randn(6, 4), 2: torch.randn(6, 8)}
        ad = {0: AdapterSpec(0, 4, 8.0, 8, 6), 2: AdapterSpec(2, 8, 4.0, 8, 6)}
        aset = ops._adapters(rt, a, b, ad)
        ws = torch.empty(16, dtype=torch.uint8)
        ops._save_sf(x, rt, "plan", aset, ws, 1)
        recs.append((aset, ws))
    for aset, ws in recs:
        assert ops._saved_sf(x, rt, "plan", aset) == (ws, 1)
    y = torch.randn(12, 8)
    ops._save_sf(y, rt, "plan", recs[0][0], recs[0][1], 2)
    del y
    ops._save_sf(x, rt, "plan", recs[1][0], recs[1][1], 1)  # insertion drops the dead entry
    assert len(ops._SAVED_SF) == 3

"""Row sharding across ranks: bin assignment, local layouts and the gradient all-reduce of
adapters that span ranks, checked on CPU with world-size-2 gloo process groups."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from lorafusion_b200.scheduler import Request, bucket_by_adapter, build_microbatch, greedy_pack
from lorafusion_b200.sharding import allreduce_spanning_grads, assign_bins, local_layout
from lorafusion_b200.workloads import WORKLOADS, row_counts


def _packing(counts, cap):
    reqs = [Request(i, i, c) for i, c in enumerate(counts)]
    groups = bucket_by_adapter(reqs)
    return reqs, greedy_pack({g.adapter_id: g.total_rows for g in groups}, cap)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("name", ["cfg2_h4096_a16_r16", "cfg4_decode_skew_a512", "cfg5_70b_a256_r64"])
def test_assignment_covers_every_bin_and_balances(name, world):
    wl = WORKLOADS[name]
    _, packing = _packing(row_counts(wl, wl.total_rows * world), wl.tile_capacity)
    plan = assign_bins(packing.bins, world)
    assert plan == assign_bins(packing.bins, world)  # deterministic
    assert len(plan.bin_rank) == len(packing.bins) and set(plan.bin_rank) <= set(range(world))
    loads = [plan.rank_rows(r) for r in range(world)]
    assert sum(loads) == sum(sum(n for _, n in b) for b in packing.bins)
    total = sum(loads)
    cap = -(-(-(-total // world)) // 256) * 256  # even share rounded up to 256-row tile pairs
    assert max(loads) <= cap  # no rank needs an extra pair of row tiles
    if total % (256 * world) == 0:
        assert loads == [total // world] * world
    # the ranges partition the global rows
    flat = sorted(x for rr in plan.rank_ranges for x in rr)
    assert flat[0][0] == 0 and flat[-1][1] == total and all(a[1] == b[0] for a, b in zip(flat, flat[1:]))
    owners, cur = {}, 0
    for entries in packing.bins:
        for a, n in entries:
            for r, rr in enumerate(plan.rank_ranges):
                if any(s0 < cur + n and e0 > cur for s0, e0 in rr):
                    owners.setdefault(a, set()).add(r)
            cur += n
    assert plan.spanning == sorted(a for a, r in owners.items() if len(r) > 1)
    if world == 1:
        assert plan.spanning == []


def test_local_layouts_partition_the_global_batch():
    wl = WORKLOADS["cfg2_h4096_a16_r16"]
    world = 3
    reqs, packing = _packing(row_counts(wl, 4096 * world), wl.tile_capacity)
    tensors = {r.request_id: torch.arange(r.num_rows, dtype=torch.float64)[:, None] + 1e6 * r.request_id
               for r in reqs}
    fused, routing, _ = build_microbatch(reqs, tensors, packing)
    plan = assign_bins(packing.bins, world)
    seen = []
    for rank in range(world):
        rows, local = local_layout(plan, packing.bins, rank, wl.tile_capacity)
        local.validate(len(rows))
        seen.extend(rows)
        # every local route is a global route shifted to local row numbers
        # every local route is a piece of one global route of the same adapter, rows contiguous
        for lr in local.routes:
            g0 = rows[lr.row_start]
            assert rows[lr.row_end - 1] == g0 + lr.num_rows - 1
            assert any(r.adapter_id == lr.adapter_id and r.row_start <= g0 and g0 + lr.num_rows <= r.row_end
                       for r in routing.routes)
    assert sorted(seen) == list(range(fused.shape[0]))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import torch.distributed as dist
    from oracle import mock_oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        K, N = 48, 40
        counts = [300, 90, 60, 33, 20, 9]
        reqs, packing = _packing(counts, 64)
        plan = assign_bins(packing.bins, world)
        rng = np.random.default_rng(0)
        ranks = {i: [4, 8, 4, 16, 8, 4][i] for i in range(len(counts))}
        x_g = rng.standard_normal((sum(counts), K)).astype(np.float32)
        g_g = rng.standard_normal((sum(counts), N)).astype(np.float32)
        w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
        a = {i: (rng.standard_normal((r, K)) / np.sqrt(K)).astype(np.float32) for i, r in ranks.items()}
        b = {i: (0.02 * rng.standard_normal((N, r))).astype(np.float32) for i, r in ranks.items()}
        sc = {i: 2.0 for i in ranks}
        rows, local = local_layout(plan, packing.bins, rank, 64)
        lroutes = [(r.row_start, r.row_end, r.adapter_id) for r in local.routes]
        _, ga, gb = mock_oracle.fused_lora_backward(g_g[rows], x_g[rows], w, a, b, sc, lroutes)
        ga_t = {k: torch.from_numpy(v.copy()) for k, v in ga.items()}
        gb_t = {k: torch.from_numpy(v.copy()) for k, v in gb.items()}
        allreduce_spanning_grads(plan, ga_t, gb_t, ranks, K, N, torch.device("cpu"))
        # full-batch reference
        groutes, cur = [], 0
        for entries in packing.bins:
            for aid, n in entries:
                groutes.append((cur, cur + n, aid))
                cur += n
        _, ga_ref, gb_ref = mock_oracle.fused_lora_backward(g_g, x_g, w, a, b, sc, groutes)
        ok = bool(plan.spanning)
        for aid in plan.spanning:
            ok &= np.allclose(ga_t[aid].numpy(), ga_ref[aid], rtol=1e-4, atol=1e-4)
            ok &= np.allclose(gb_t[aid].numpy(), gb_ref[aid], rtol=1e-4, atol=1e-4)
        for aid in ga_t:
            if aid not in plan.spanning:  # whole on this rank already
                ok &= np.allclose(ga_t[aid].numpy(), ga_ref[aid], rtol=1e-4, atol=1e-4)
        result_q.put((rank, ok, list(plan.spanning)))
    finally:
        dist.destroy_process_group()


def test_spanning_gradients_allreduce_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results), results
    assert results[0][2] and results[0][2] == results[1][2]


@pytest.mark.parametrize("seed", range(10))
def test_native_assignment_equals_oracle(seed):
    """lf_assign_rows matches the plain-Python restatement on random packings and world sizes."""
    from oracle.scheduler_oracle import assign_rows
    rng = np.random.default_rng(100 + seed)
    cap = int(rng.choice([16, 64, 128]))
    counts = [int(v) for v in rng.integers(1, 6 * cap, size=int(rng.integers(1, 80)))]
    _, packing = _packing(counts, cap)
    for world in (1, 2, 3, 5, 8):
        plan = assign_bins(packing.bins, world)
        got = sorted((s0, e0, k) for k, rr in enumerate(plan.rank_ranges) for s0, e0 in rr)
        assert got == assign_rows(packing.bins, world), (seed, world)
    bins = [[], [(3, 5), (4, 2)], [(3, 7)], [(3, 9)], []]  # empty and mixed bins
    for world in (1, 2, 4):
        plan = assign_bins(bins, world)
        assert sorted((s0, e0, k) for k, rr in enumerate(plan.rank_ranges) for s0, e0 in rr) == assign_rows(bins, world)
    with pytest.raises(ValueError):
        assign_bins(packing.bins, 0)


def test_only_adapters_larger_than_a_share_span():
    """cfg2 at 8 ranks: adapters that fit in a rank's capacity stay whole on one rank."""
    wl = WORKLOADS["cfg2_h4096_a16_r16"]
    counts = row_counts(wl, wl.total_rows * 8)
    _, packing = _packing(counts, wl.tile_capacity)
    plan = assign_bins(packing.bins, 8)
    assert len(plan.spanning) <= 8 + sum(c > 4096 for c in counts)


def _failing_worker(rank, world, port, result_q):
    """Rank 1 raises before the gradient all-reduce (a failed step); rank 0 must get an error from
    its collective, bounded by the group's short timeout, not hang."""
    import datetime
    import time

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    counts = [300, 90, 60, 33, 20, 9]
    _, packing = _packing(counts, 64)
    plan = assign_bins(packing.bins, world)
    ranks = {i: 4 for i in range(len(counts))}
    K, N = 16, 8
    ga = {a: torch.ones(4, K) for a in plan.spanning}
    gb = {a: torch.ones(N, 4) for a in plan.spanning}
    dist.barrier()
    if rank == 1:
        result_q.put((rank, "raised", 0.0))
        raise SystemExit(3)  # the failing rank leaves between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        allreduce_spanning_grads(plan, ga, gb, ranks, K, N, torch.device("cpu"))
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - the collective's error type depends on the backend
        outcome = f"error: {type(e).__name__}"
    result_q.put((rank, outcome, time.monotonic() - t0))


def test_rank_failure_before_allreduce_is_reported_not_hung():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, outcome, dt = q.get(timeout=120)
        results[r] = (outcome, dt)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1][0] == "raised"
    assert results[0][0].startswith("error"), results
    assert results[0][1] < 60.0, results
    assert procs[1].exitcode == 3

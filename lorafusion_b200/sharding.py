"""Row sharding of a packed fused batch across the GPUs of one node.

The reference has no multi-GPU code; this module adds the data-parallel layer
the op needs to run one process per GPU:

* The global layout is untouched: every rank runs the same scheduler
  (``bucket_by_adapter -> greedy_pack -> build_microbatch``) and gets the same
  bins and routes, bit for bit.
* :func:`assign_bins` gives each rank whole bins (``lf_assign_bins``, C++).  Runs of consecutive
  single-adapter bins form bundles so an adapter's rows stay on one rank where
  possible; bundles larger than a rank's share are cut.  Every rank gets a
  capacity of its even share rounded up to whole 256-row tile pairs; bundles,
  largest first, go to the rank they fit best (a bundle that fits nowhere is
  placed bin by bin, and a bin that fits nowhere goes to the least-loaded
  rank).  Deterministic, so every rank computes the same assignment without
  communicating.
* :func:`local_layout` turns a rank's bins into its own fused row ranges and a
  rebased :class:`TileRoutingConfig`.
* The forward needs no communication (base weight replicated, adapters
  resident on every rank).  In the backward, :func:`allreduce_spanning_grads`
  sums dA/dB of adapters whose routes land on more than one rank with a
  single ``all_reduce(SUM)`` over one packed float32 buffer.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from lorafusion_b200.config import TileRoute, TileRoutingConfig

TILE_PAIR_ROWS = 256  # rows of one CTA-pair tile of the fused GEMM


@dataclass(frozen=True)
class ShardPlan:
    world_size: int
    bin_rank: list[int]                 # rank of every global bin
    bin_rows: list[tuple[int, int]]     # [start, end) of every bin in the global fused rows
    spanning: list[int]                 # adapters whose routes land on more than one rank, ascending

    def rank_bins(self, rank: int) -> list[int]:
        return [b for b, r in enumerate(self.bin_rank) if r == rank]

    def rank_rows(self, rank: int) -> int:
        return sum(e - s for (s, e), r in zip(self.bin_rows, self.bin_rank) if r == rank)


def assign_bins(bins: list[list[tuple[int, int]]], world_size: int) -> ShardPlan:
    """Deterministic bin -> rank assignment (see module docstring), computed by
    ``lf_assign_bins`` in the native library."""
    from lorafusion_b200 import _native as nat

    if world_size <= 0:
        raise ValueError("world_size must be positive")
    rows = [sum(n for _, n in entries) for entries in bins]
    starts, cur = [], 0
    for r in rows:
        starts.append((cur, cur + r))
        cur += r
    counts = np.fromiter((len(e) for e in bins), dtype=np.int64, count=len(bins))
    bin_start = np.concatenate(([0], np.cumsum(counts))).astype(np.int32)
    flat = [x for entries in bins for x in entries]
    ent_a = np.array([a for a, _ in flat] or [0], dtype=np.int32)
    ent_r = np.array([n for _, n in flat] or [0], dtype=np.int32)
    bin_rank = np.zeros(max(len(bins), 1), dtype=np.int32)
    P = ctypes.POINTER(ctypes.c_int32)
    rc = nat.lib().lf_assign_bins(bin_start.ctypes.data_as(P), ent_a.ctypes.data_as(P), ent_r.ctypes.data_as(P),
                                  len(bins), world_size, TILE_PAIR_ROWS, bin_rank.ctypes.data_as(P))
    nat.check(rc, "lf_assign_bins")
    ranks = bin_rank[:len(bins)].tolist()
    owners: dict[int, set[int]] = {}
    for b, entries in enumerate(bins):
        for a, _ in entries:
            owners.setdefault(a, set()).add(ranks[b])
    spanning = sorted(a for a, rk in owners.items() if len(rk) > 1)
    return ShardPlan(world_size=world_size, bin_rank=ranks, bin_rows=starts, spanning=spanning)


def local_layout(plan: ShardPlan, bins: list[list[tuple[int, int]]], rank: int, tile_size: int):
    """(global row index of each local row, local routing) for one rank's bins.

    Local rows are the rank's bins in global order; routes are the global
    routes of those bins shifted to local row numbers.
    """
    rows: list[int] = []
    routes: list[TileRoute] = []
    cur = 0
    for b in plan.rank_bins(rank):
        g0, g1 = plan.bin_rows[b]
        rows.extend(range(g0, g1))
        for a, n in bins[b]:
            routes.append(TileRoute(cur, cur + n, a))
            cur += n
    return rows, TileRoutingConfig(tile_size=tile_size, routes=routes)


def allreduce_spanning_grads(plan: ShardPlan, grad_a: dict[int, torch.Tensor], grad_b: dict[int, torch.Tensor],
                             ranks: dict[int, int], in_features: int, out_features: int, device,
                             group=None) -> None:
    """Sum dA/dB of the spanning adapters over all ranks, in place in the dicts.

    Every rank packs the spanning adapters in ascending id order into one
    float32 buffer (zeros for adapters it does not hold), runs one
    ``all_reduce(SUM)`` and unpacks; afterwards every rank holds the full
    gradient of each spanning adapter (inserted if it had none).
    """
    import torch.distributed as dist

    if not plan.spanning or plan.world_size == 1:
        return
    K, N = in_features, out_features
    sizes = [ranks[a] * (K + N) for a in plan.spanning]
    buf = torch.zeros(sum(sizes), dtype=torch.float32, device=device)
    off = 0
    for a, sz in zip(plan.spanning, sizes):
        r = ranks[a]
        if a in grad_a:
            buf[off:off + r * K].copy_(grad_a[a].reshape(-1))
            buf[off + r * K:off + sz].copy_(grad_b[a].reshape(-1))
        off += sz
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    off = 0
    for a, sz in zip(plan.spanning, sizes):
        r = ranks[a]
        dtype = grad_a[a].dtype if a in grad_a else torch.float32
        ga = buf[off:off + r * K].view(r, K).to(dtype)
        gb = buf[off + r * K:off + sz].view(N, r).to(dtype)
        if a in grad_a:
            grad_a[a].copy_(ga)
            grad_b[a].copy_(gb)
        else:
            grad_a[a] = ga.clone()
            grad_b[a] = gb.clone()
        off += sz

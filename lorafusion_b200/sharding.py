"""Row sharding of a packed fused batch across the GPUs of one node.

The reference has no multi-GPU code; this module adds the data-parallel layer
the op needs to run one process per GPU:

* The global layout is untouched: every rank runs the same scheduler
  (``bucket_by_adapter -> greedy_pack -> build_microbatch``) and gets the same
  bins and routes, bit for bit.
* :func:`assign_bins` (``lf_assign_rows``, C++) gives each rank row ranges of
  that global layout: adapters, largest first, go whole to the rank they fit
  best, where every rank's capacity is its even share rounded up to 256-row
  tile pairs (so no rank needs an extra, mostly empty pair of row tiles); an
  adapter that fits nowhere is cut over the ranks with most room.  Only the cut
  adapters span ranks.  Deterministic, so every rank computes the same
  assignment without communicating.
* :func:`local_layout` turns a rank's row ranges into its own fused rows and a
  rebased :class:`TileRoutingConfig`.
* The forward needs no communication (base weight replicated, adapters
  resident on every rank).  In the backward, the gradients of adapters whose
  routes land on more than one rank are summed over the ranks: inside the
  dA/dB kernel over NVLink peer mappings (:class:`PeerExchange`, passed as
  ``fused_lora_backward(..., peer=...)``), or by
  :func:`allreduce_spanning_grads` with a single ``all_reduce(SUM)`` over one
  packed float32 buffer.
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
    bin_rank: list[int]                 # rank holding the first row of every global bin
    bin_rows: list[tuple[int, int]]     # [start, end) of every bin in the global fused rows
    spanning: list[int]                 # adapters whose routes land on more than one rank, ascending
    rank_ranges: tuple = ()             # per rank: its global row ranges [start, end), ascending
    holders: tuple = ()                 # (adapter, ranks holding its rows) of every spanning adapter

    def rank_bins(self, rank: int) -> list[int]:
        return [b for b, r in enumerate(self.bin_rank) if r == rank]

    def rank_rows(self, rank: int) -> int:
        return sum(e - s for s, e in self.rank_ranges[rank])


def _global_routes(bins: list[list[tuple[int, int]]]) -> list[tuple[int, int, int]]:
    out, cur = [], 0
    for entries in bins:
        for a, n in entries:
            out.append((cur, cur + n, a))
            cur += n
    return out


def assign_bins(bins: list[list[tuple[int, int]]], world_size: int) -> ShardPlan:
    """Deterministic row -> rank assignment of a packing (see module docstring), computed by
    ``lf_assign_rows`` in the native library."""
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
    P = ctypes.POINTER(ctypes.c_int32)
    P64 = ctypes.POINTER(ctypes.c_int64)
    cap = max(2 * len(flat) + world_size, 16)
    while True:
        r_s = np.zeros(cap, dtype=np.int64)
        r_e = np.zeros(cap, dtype=np.int64)
        r_k = np.zeros(cap, dtype=np.int32)
        n_ranges = ctypes.c_int32(0)
        rc = nat.lib().lf_assign_rows(bin_start.ctypes.data_as(P), ent_a.ctypes.data_as(P), ent_r.ctypes.data_as(P),
                                      len(bins), world_size, TILE_PAIR_ROWS, cap, r_s.ctypes.data_as(P64),
                                      r_e.ctypes.data_as(P64), r_k.ctypes.data_as(P), ctypes.byref(n_ranges))
        if rc == nat.LF_ERR_CAPACITY and n_ranges.value > cap:
            cap = n_ranges.value
            continue
        nat.check(rc, "lf_assign_rows")
        break
    n = n_ranges.value
    ranges: list[list[tuple[int, int]]] = [[] for _ in range(world_size)]
    for s0, e0, k in zip(r_s[:n].tolist(), r_e[:n].tolist(), r_k[:n].tolist()):
        ranges[k].append((s0, e0))
    rank_ranges = tuple(tuple(rr) for rr in ranges)
    owner = []  # rank of each bin's first row
    bounds = sorted((s0, e0, k) for k, rr in enumerate(ranges) for s0, e0 in rr)
    j = 0
    for g0, g1 in starts:
        while j + 1 < len(bounds) and bounds[j][1] <= g0:
            j += 1
        owner.append(bounds[j][2] if bounds and g1 > g0 else 0)
    owners: dict[int, set[int]] = {}
    groutes = _global_routes(bins)
    for s0, e0, k in bounds:
        for g0, g1, a in groutes:
            if g0 < e0 and g1 > s0:
                owners.setdefault(a, set()).add(k)
    spanning = sorted(a for a, rk in owners.items() if len(rk) > 1)
    return ShardPlan(world_size=world_size, bin_rank=owner, bin_rows=starts, spanning=spanning,
                     rank_ranges=rank_ranges, holders=tuple((a, tuple(sorted(owners[a]))) for a in spanning))


def local_layout(plan: ShardPlan, bins: list[list[tuple[int, int]]], rank: int, tile_size: int):
    """(global row index of each local row, local routing) for one rank's rows.

    Local rows are the rank's global row ranges in ascending order; routes are
    the global routes cut to those ranges and shifted to local row numbers.
    """
    groutes = _global_routes(bins)
    rows: list[int] = []
    routes: list[TileRoute] = []
    cur = 0
    for s0, e0 in plan.rank_ranges[rank]:
        rows.extend(range(s0, e0))
        for g0, g1, a in groutes:
            lo, hi = max(g0, s0), min(g1, e0)
            if lo < hi:
                routes.append(TileRoute(cur + lo - s0, cur + hi - s0, a))
        cur += e0 - s0
    return rows, TileRoutingConfig(tile_size=tile_size, routes=routes)


def allreduce_spanning_grads(plan: ShardPlan, grad_a: dict[int, torch.Tensor], grad_b: dict[int, torch.Tensor],
                             ranks: dict[int, int], in_features: int, out_features: int, device,
                             group=None) -> None:
    """Sum dA/dB of the spanning adapters over all ranks, in place in the dicts.

    Every rank packs the spanning adapters in ascending id order into one
    float32 buffer (zeros for adapters it does not hold), runs one
    ``all_reduce(SUM)`` and unpacks; afterwards every rank holds the full
    gradient of each spanning adapter (inserted if it had none).  Pass the
    gradients of ``fused_lora_backward(..., grad_dtype=torch.float32)`` to sum
    unrounded partials; bf16 ones are widened first.  With a gloo group the
    buffer lives in host memory.
    """
    import torch.distributed as dist

    if not plan.spanning or plan.world_size == 1:
        return
    K, N = in_features, out_features
    if dist.get_backend(group) == "gloo":
        device = torch.device("cpu")
    sizes = [ranks[a] * (K + N) for a in plan.spanning]
    buf = torch.zeros(sum(sizes), dtype=torch.float32, device=device)
    dst, src, off = [], [], 0
    views = []
    for a, sz in zip(plan.spanning, sizes):
        r = ranks[a]
        va, vb = buf[off:off + r * K].view(r, K), buf[off + r * K:off + sz].view(N, r)
        views.append((a, va, vb))
        if a in grad_a:
            dst += [va, vb]
            src += [grad_a[a], grad_b[a]]
        off += sz
    if dst:  # one multi-tensor launch packs (and converts) every held gradient
        torch._foreach_copy_(dst, src)
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    back_dst, back_src = [], []
    for a, va, vb in views:
        if a in grad_a:
            back_dst += [grad_a[a], grad_b[a]]
            back_src += [va, vb]
        else:
            grad_a[a] = va.clone()
            grad_b[a] = vb.clone()
    if back_dst:
        torch._foreach_copy_(back_dst, back_src)


class PeerExchange:
    """The exchange buffers ``fused_lora_backward(..., peer=...)`` needs, one set per process.

    Every rank holds one buffer (device memory of its own GPU) and maps every other rank's through
    CUDA IPC handles exchanged over ``group`` (processes of one node).  The dA/dB kernel of each
    rank pushes the blocks it computes for spanning adapters into all of them over NVLink and sums,
    in rank order, what the adapters' holders pushed: every rank ends with the same sums, and no
    separate all-reduce runs.  Creation and growth are collective: every rank makes the same calls
    in the same order.  The buffer grows to the largest projection it has served.
    """

    def __init__(self, plan: ShardPlan, ranks: dict[int, int], device, group=None):
        import torch.distributed as dist

        if any(plan.rank_rows(r) == 0 for r in range(plan.world_size)):
            raise ValueError("every rank needs rows of its own for the in-kernel exchange")
        self.plan, self.group = plan, group
        self.device = torch.device(device)
        self.world = plan.world_size
        self.rank = dist.get_rank(group)
        holders = dict(plan.holders)
        # spanning virtual slots (a slot of rank > 64 is several), numbered alike on every rank
        self.vslots: list[tuple[int, int, int]] = []
        for a in plan.spanning:
            r = int(ranks[a])
            self.vslots += [(a, c0, min(64, r - c0)) for c0 in range(0, r, 64)]
        self.index = {(a, c0): i for i, (a, c0, _) in enumerate(self.vslots)}
        self.masks = [sum(1 << k for k in holders.get(a, ())) for a, _, _ in self.vslots]
        rmax = max((r for _, _, r in self.vslots), default=16)
        self.r_pad_x = 16 if rmax <= 16 else 32 if rmax <= 32 else 64
        self.gen = 0
        self.bytes = 0
        self.local = None
        self.ptrs: list[int] = []
        self.opened: list[int] = []

    def ensure(self, n_blocks: int) -> None:
        """Collective: buffers of at least the bytes `n_blocks` exchanged blocks need."""
        import torch.distributed as dist

        from lorafusion_b200 import _native as nat

        need = int(nat.lib().lf_peer_exchange_bytes(self.world, n_blocks, self.r_pad_x))
        if need <= self.bytes:
            return
        L = nat.lib()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still uses the old buffers
        self._release()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            nat.check(L.lf_peer_alloc(need, ctypes.byref(ptr)), "lf_peer_alloc")
        self.local, self.bytes = ptr.value, need
        handle = (ctypes.c_char * nat.IPC_HANDLE_BYTES)()
        nat.check(L.lf_ipc_handle(ctypes.c_void_p(self.local), handle), "lf_ipc_handle")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        self.ptrs = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self.local)
                    continue
                peer = ctypes.c_void_p()
                buf = (ctypes.c_char * nat.IPC_HANDLE_BYTES).from_buffer_copy(h)
                nat.check(L.lf_ipc_open(buf, ctypes.byref(peer)), "lf_ipc_open")
                self.ptrs.append(peer.value)
                self.opened.append(peer.value)
        dist.barrier(group=self.group)

    def next_gen(self) -> int:
        self.gen += 1
        return self.gen

    def _release(self) -> None:
        from lorafusion_b200 import _native as nat
        L = nat.lib()
        for p in self.opened:
            L.lf_ipc_close(ctypes.c_void_p(p))
        self.opened = []
        if self.local is not None:
            L.lf_peer_free(ctypes.c_void_p(self.local))
        self.local, self.bytes, self.ptrs = None, 0, []

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._release()

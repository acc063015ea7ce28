"""Plain-Python restatement of lorafusion's layout logic (TEST INFRASTRUCTURE ONLY).

Integer-only: no tensors.  Used to check the shipped scheduler and routing
tables bit-exactly.

* :func:`bucket_rows` — ``lorafusion/scheduler/adapter_grouper.py:67-88`` as
  used by ``lorafusion/runtime/coordinator.py:48-49`` (adapter -> total rows,
  adapters ascending).
* :func:`greedy_bins` — ``lorafusion/scheduler/milp_packer.py:36-72``.
* :func:`microbatch_layout` — ``lorafusion/scheduler/data_batcher.py:18-87``,
  returning routes, ``row_order`` and, per fused row, the source
  ``(request_id, row_in_request)``.
* :func:`assign_bins` — the bin -> rank assignment of the multi-GPU layer (no
  counterpart in the reference, which runs on one device), restated in plain
  Python to check ``lf_assign_bins``.
"""

from __future__ import annotations


def bucket_rows(requests):
    """``requests``: iterable of (request_id, adapter_id, num_rows)."""
    totals: dict[int, int] = {}
    for _, aid, n in requests:
        totals[aid] = totals.get(aid, 0) + n
    return {aid: totals[aid] for aid in sorted(totals)}


def greedy_bins(adapter_rows: dict[int, int], cap: int):
    if cap <= 0:
        raise ValueError("tile_capacity must be positive")
    items = []
    for aid, rows in adapter_rows.items():
        left = rows
        while left > 0:
            take = cap if left > cap else left
            items.append((aid, take))
            left -= take
    # stable descending sort by chunk size
    items = [it for _, it in sorted(enumerate(items), key=lambda p: (-p[1][1], p[0]))]
    bins: list[list[tuple[int, int]]] = []
    free: list[int] = []
    for aid, n in items:
        target = next((b for b in range(len(bins)) if free[b] >= n), None)
        if target is None:
            bins.append([(aid, n)])
            free.append(cap - n)
        else:
            bins[target].append((aid, n))
            free[target] -= n
    return bins


def microbatch_layout(requests, bins):
    """``requests``: list of (request_id, adapter_id, num_rows) in arrival order."""
    per_adapter: dict[int, list[tuple[int, int]]] = {}
    for rid, aid, n in requests:
        per_adapter.setdefault(aid, []).append((rid, n))
    used: dict[int, int] = {}
    routes = []
    row_order: list[int] = []
    source: list[tuple[int, int]] = []
    cursor = 0
    for entries in bins:
        for aid, n in entries:
            need = n
            for rid, size in per_adapter.get(aid, []):
                if need <= 0:
                    break
                start = used.get(rid, 0)
                if size - start <= 0:
                    continue
                k = min(need, size - start)
                for j in range(k):
                    row_order.append(rid)
                    source.append((rid, start + j))
                used[rid] = start + k
                need -= k
            routes.append((cursor, cursor + n, aid))
            cursor += n
    return routes, row_order, source


def assign_bins(bins, world_size: int, granule_rows: int = 256):
    """Rank of every bin: bundles of consecutive single-adapter bins (at most the
    even share of rows), capacity = share rounded up to ``granule_rows``,
    largest bundle first into the best-fitting rank; bundles that fit nowhere
    are placed bin by bin, and bins that fit nowhere go to the least-loaded rank."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    rows = [sum(n for _, n in entries) for entries in bins]
    total = sum(rows)
    share = max(1, -(-total // world_size))
    cap = -(-share // granule_rows) * granule_rows
    bundles, cur, cur_adapter, cur_rows = [], [], None, 0
    for b, entries in enumerate(bins):
        adapters = {a for a, _ in entries}
        solo = next(iter(adapters)) if len(adapters) == 1 else None
        if cur and (solo is None or solo != cur_adapter or cur_rows + rows[b] > share):
            bundles.append(cur)
            cur, cur_rows, cur_adapter = [], 0, None
        cur.append(b)
        cur_rows += rows[b]
        cur_adapter = solo
        if solo is None:
            bundles.append(cur)
            cur, cur_rows, cur_adapter = [], 0, None
    if cur:
        bundles.append(cur)
    order = sorted(range(len(bundles)), key=lambda i: -sum(rows[b] for b in bundles[i]))
    load = [0] * world_size
    rank = [0] * len(bins)

    def place(members):
        n = sum(rows[b] for b in members)
        fits = [k for k in range(world_size) if load[k] + n <= cap]
        if not fits:
            return False
        r = min(fits, key=lambda k: (cap - load[k] - n, k))
        for b in members:
            rank[b] = r
        load[r] += n
        return True

    for i in order:
        if place(bundles[i]):
            continue
        for b in sorted(bundles[i], key=lambda b: (-rows[b], b)):
            if not place([b]):
                r = min(range(world_size), key=lambda k: (load[k], k))
                rank[b] = r
                load[r] += rows[b]
    return rank

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
* :func:`assign_rows` — the row -> rank assignment of the multi-GPU layer (no
  counterpart in the reference, which runs on one device), restated in plain
  Python to check ``lf_assign_rows``.
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


def assign_rows(bins, world_size: int, granule_rows: int = 256):
    """Global row ranges (start, end, rank), ascending, adjacent ranges of one rank merged:
    adapters, most rows first (ties: first appearance), whole into the best-fitting rank (least
    room left, then lowest); an adapter that fits nowhere is cut over the ranks with most room
    (then lowest), each taking what it has room for; its rows go to its parts in row order."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    entries = [(a, n) for b in bins for a, n in b]
    total = sum(n for _, n in entries)
    share = max(1, -(-total // world_size))
    cap = -(-share // granule_rows) * granule_rows
    totals: dict[int, int] = {}
    for a, n in entries:
        totals[a] = totals.get(a, 0) + n  # dict keeps first appearance
    order = sorted(totals, key=lambda a: -totals[a])  # stable
    load = [0] * world_size
    parts: dict[int, list[list[int]]] = {}
    for a in order:
        left = totals[a]
        fits = [k for k in range(world_size) if load[k] + left <= cap]
        if fits:
            k = min(fits, key=lambda k: (cap - load[k] - left, k))
            parts[a] = [[k, left]]
            load[k] += left
            continue
        parts[a] = []
        while left > 0:
            k = min(range(world_size), key=lambda k: (load[k], k))
            room = cap - load[k]
            take = min(room, left) if room > 0 else left
            parts[a].append([k, take])
            load[k] += take
            left -= take
    out, cur = [], 0
    for a, n in entries:
        while n > 0:
            k, rem = parts[a][0]
            take = min(n, rem)
            if out and out[-1][2] == k and out[-1][1] == cur:
                out[-1][1] = cur + take
            else:
                out.append([cur, cur + take, k])
            cur += take
            n -= take
            if take == rem:
                parts[a].pop(0)
            else:
                parts[a][0][1] = rem - take
    return [tuple(x) for x in out]

"""Host-side layout producer: request grouping, tile bin-packing, fused batch assembly.

This module produces the fused row layout and the route table that the fused
op consumes.  Its outputs are bit-identical to lorafusion's scheduler on the
same inputs (same bins, same route order, same ``row_order``):

* ``Request``/``AdapterGroup``/``group_by_adapter``/``bucket_by_adapter``/
  ``check_bubble_lemma`` follow ``lorafusion/scheduler/adapter_grouper.py:17-114``;
* ``PackingResult``/``greedy_pack``/``milp_pack`` follow
  ``lorafusion/scheduler/milp_packer.py:23-143``;
* ``build_microbatch``/``scatter_outputs`` follow
  ``lorafusion/scheduler/data_batcher.py:18-103``.

``scatter_outputs`` gathers each request's rows with one indexed copy instead
of stacking single rows; the result holds the same values in the same order.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from lorafusion_b200.config import TileRoute, TileRoutingConfig

try:  # the exact packer is optional, exactly as in the reference
    import pulp  # type: ignore

    PULP_AVAILABLE = True
except ImportError:  # pragma: no cover - pulp is absent in this image
    PULP_AVAILABLE = False


# --------------------------------------------------------------------------
# Request grouping (adapter_grouper.py)
# --------------------------------------------------------------------------


@dataclass(frozen=True)
class Request:
    """One request: ``num_rows`` activation rows that all use ``adapter_id``."""

    request_id: int
    adapter_id: int
    num_rows: int


@dataclass(frozen=True)
class AdapterGroup:
    """A run of requests that share one adapter."""

    adapter_id: int
    request_ids: list[int]
    total_rows: int


def group_by_adapter(requests: list[Request]) -> list[AdapterGroup]:
    """Merge only *consecutive* requests of the same adapter (arrival order kept).

    lorafusion/scheduler/adapter_grouper.py:35-64.
    """
    out: list[AdapterGroup] = []
    run_adapter = None
    run_ids: list[int] = []
    run_rows = 0
    for req in requests:
        if run_ids and req.adapter_id != run_adapter:
            out.append(AdapterGroup(run_adapter, run_ids, run_rows))
            run_ids, run_rows = [], 0
        run_adapter = req.adapter_id
        run_ids.append(req.request_id)
        run_rows += req.num_rows
    if run_ids:
        out.append(AdapterGroup(run_adapter, run_ids, run_rows))
    return out


def bucket_by_adapter(requests: list[Request]) -> list[AdapterGroup]:
    """One group per adapter holding all its requests, groups sorted by adapter id.

    lorafusion/scheduler/adapter_grouper.py:67-88.
    """
    members: dict[int, list[Request]] = {}
    for req in requests:
        members.setdefault(req.adapter_id, []).append(req)
    return [
        AdapterGroup(
            adapter_id=aid,
            request_ids=[r.request_id for r in members[aid]],
            total_rows=sum(r.num_rows for r in members[aid]),
        )
        for aid in sorted(members)
    ]


def check_bubble_lemma(groups: list[AdapterGroup], requests: list[Request]) -> bool:
    """True iff every request sits in exactly one group of its own adapter and
    each group's ``total_rows`` equals the rows of its members.

    lorafusion/scheduler/adapter_grouper.py:91-114.
    """
    by_id = {r.request_id: r for r in requests}
    placed: set[int] = set()
    for g in groups:
        ids = g.request_ids
        if len(set(ids)) != len(ids):
            return False
        if sum(by_id[i].num_rows for i in ids) != g.total_rows:
            return False
        for i in ids:
            if i in placed or by_id[i].adapter_id != g.adapter_id:
                return False
            placed.add(i)
    return placed == set(by_id)


# --------------------------------------------------------------------------
# Bin packing (milp_packer.py)
# --------------------------------------------------------------------------


@dataclass(frozen=True)
class PackingResult:
    """Bins of ``(adapter_id, rows)`` entries, in bin order; ``method`` is
    ``"greedy"`` or ``"milp"``."""

    bins: list[list[tuple[int, int]]]
    tile_capacity: int
    method: str

    @property
    def num_bins(self) -> int:
        return len(self.bins)


def _split_into_chunks(adapter_rows: dict[int, int], cap: int) -> list[tuple[int, int]]:
    """Cut every adapter's rows into ``cap``-row chunks plus one remainder chunk,
    adapters in dict order (milp_packer.py:47-53)."""
    chunks: list[tuple[int, int]] = []
    for aid, rows in adapter_rows.items():
        full, rest = divmod(rows, cap) if rows > 0 else (0, 0)
        chunks.extend([(aid, cap)] * full)
        if rest:
            chunks.append((aid, rest))
    return chunks


def greedy_pack(adapter_rows: dict[int, int], tile_capacity: int) -> PackingResult:
    """First-fit-decreasing packing of per-adapter row counts into bins of
    ``tile_capacity`` rows (milp_packer.py:36-72).

    Chunks are ordered by size, largest first, keeping dict order among equal
    sizes (a stable sort); each goes into the first bin with room, else a new
    bin at the end.
    """
    if tile_capacity <= 0:
        raise ValueError("tile_capacity must be positive")
    order = sorted(_split_into_chunks(adapter_rows, tile_capacity), key=lambda c: -c[1])
    bins: list[list[tuple[int, int]]] = []
    room: list[int] = []
    for aid, n in order:
        for b, free in enumerate(room):
            if free >= n:
                bins[b].append((aid, n))
                room[b] = free - n
                break
        else:
            bins.append([(aid, n)])
            room.append(tile_capacity - n)
    return PackingResult(bins=bins, tile_capacity=tile_capacity, method="greedy")


def milp_pack(
    adapter_rows: dict[int, int],
    tile_capacity: int,
    max_bins: int | None = None,
    time_limit_s: float = 10.0,
) -> PackingResult:
    """Exact bin count via a 0/1 program when PuLP is importable, else
    :func:`greedy_pack` (milp_packer.py:75-143).

    The program has one binary ``use[j]`` per candidate bin and one binary
    ``x[i][j]`` per (chunk, bin): minimise ``sum(use)`` subject to every chunk
    placed once and each bin's rows ``<= tile_capacity * use[j]``.  Any
    solver status other than Optimal falls back to the greedy packing.
    """
    if not PULP_AVAILABLE:
        return greedy_pack(adapter_rows, tile_capacity)
    if tile_capacity <= 0:
        raise ValueError("tile_capacity must be positive")
    chunks = _split_into_chunks(adapter_rows, tile_capacity)
    if not chunks:
        return PackingResult(bins=[], tile_capacity=tile_capacity, method="milp")
    nb = max_bins or len(chunks)
    prob = pulp.LpProblem("lorafusion_b200_bins", pulp.LpMinimize)
    use = [pulp.LpVariable(f"use_{j}", cat="Binary") for j in range(nb)]
    put = [[pulp.LpVariable(f"x_{i}_{j}", cat="Binary") for j in range(nb)] for i in range(len(chunks))]
    prob += pulp.lpSum(use)
    for i in range(len(chunks)):
        prob += pulp.lpSum(put[i]) == 1
    for j in range(nb):
        prob += pulp.lpSum(chunks[i][1] * put[i][j] for i in range(len(chunks))) <= tile_capacity * use[j]
    status = prob.solve(pulp.PULP_CBC_CMD(msg=False, timeLimit=time_limit_s))
    if pulp.LpStatus[status] != "Optimal":
        return greedy_pack(adapter_rows, tile_capacity)
    bins = []
    for j in range(nb):
        if pulp.value(use[j]) < 0.5:
            continue
        members = [chunks[i] for i in range(len(chunks)) if pulp.value(put[i][j]) > 0.5]
        if members:
            bins.append(members)
    return PackingResult(bins=bins, tile_capacity=tile_capacity, method="milp")


# --------------------------------------------------------------------------
# Fused batch assembly (data_batcher.py)
# --------------------------------------------------------------------------


def build_microbatch(
    requests: list[Request],
    request_tensors: dict[int, torch.Tensor],
    packing: PackingResult,
) -> tuple[torch.Tensor, TileRoutingConfig, list[int]]:
    """Lay the requests' rows out bin by bin and emit one route per bin entry.

    lorafusion/scheduler/data_batcher.py:18-87.  For a bin entry
    ``(adapter, n)`` the adapter's requests are drained in arrival order,
    each remembering how many of its rows earlier entries already took; the
    entry's route always spans ``n`` rows from the running cursor.
    Returns ``(fused_x, routing, row_order)`` where ``row_order[i]`` is the
    request id of fused row ``i``.
    """
    in_features = next(iter(request_tensors.values())).shape[1]
    queue: dict[int, list[Request]] = {}
    for req in requests:
        queue.setdefault(req.adapter_id, []).append(req)
    taken: dict[int, int] = {}
    pieces: list[torch.Tensor] = []
    routes: list[TileRoute] = []
    row_order: list[int] = []
    cursor = 0
    for bin_entries in packing.bins:
        for aid, n in bin_entries:
            want = n
            for req in queue.get(aid, ()):
                if want <= 0:
                    break
                src = request_tensors[req.request_id]
                start = taken.get(req.request_id, 0)
                avail = src.shape[0] - start
                if avail <= 0:
                    continue
                k = want if want < avail else avail
                pieces.append(src[start : start + k])
                row_order.extend([req.request_id] * k)
                taken[req.request_id] = start + k
                want -= k
            routes.append(TileRoute(row_start=cursor, row_end=cursor + n, adapter_id=aid))
            cursor += n
    fused_x = torch.cat(pieces, dim=0) if pieces else torch.empty((0, in_features))
    return fused_x, TileRoutingConfig(tile_size=packing.tile_capacity, routes=routes), row_order


def scatter_outputs(fused_out: torch.Tensor, row_order: list[int]) -> dict[int, torch.Tensor]:
    """Split fused output rows back per request (data_batcher.py:90-103).

    Requests appear in order of their first fused row; each request's rows
    keep their fused order.
    """
    rows_of: dict[int, list[int]] = {}
    for i, rid in enumerate(row_order):
        rows_of.setdefault(rid, []).append(i)
    out: dict[int, torch.Tensor] = {}
    for rid, idx in rows_of.items():
        index = torch.tensor(idx, dtype=torch.long, device=fused_out.device)
        out[rid] = fused_out.index_select(0, index)
    return out

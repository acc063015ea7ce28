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

Where the reference loops in Python, this module hands the work to the native
library: ``greedy_pack`` runs ``lf_greedy_pack`` (C++, same bins bit for bit),
and for CUDA tensors ``build_microbatch`` gathers and ``scatter_outputs``
splits rows with one ``lf_copy_rows`` launch (byte-exact copies) instead of
``torch.cat`` over slices and a per-row Python loop.  CPU tensors keep the
reference's torch semantics.  ``scatter_outputs`` returns, for CUDA input,
disjoint contiguous views of one freshly allocated buffer.
"""

from __future__ import annotations

import ctypes
import functools
from dataclasses import dataclass

import numpy as np
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
    ``tile_capacity`` rows (milp_packer.py:36-72), computed by ``lf_greedy_pack``.

    Chunks are ordered by size, largest first, keeping dict order among equal
    sizes (a stable sort); each goes into the first bin with room, else a new
    bin at the end.
    """
    from lorafusion_b200 import _native as nat

    if tile_capacity <= 0:
        raise ValueError("tile_capacity must be positive")
    ids = np.fromiter(adapter_rows.keys(), dtype=np.int64, count=len(adapter_rows))
    rows = np.fromiter(adapter_rows.values(), dtype=np.int64, count=len(adapter_rows))
    lim = np.iinfo(np.int32)
    if tile_capacity > lim.max or ids.size and (ids.min() < lim.min or ids.max() > lim.max or rows.max() > lim.max):
        raise ValueError("adapter ids and row counts must fit in 32 bits")
    ids32, rows32 = ids.astype(np.int32), rows.astype(np.int32)
    n_chunks = int(np.sum((rows32[rows32 > 0].astype(np.int64) + tile_capacity - 1) // tile_capacity))
    bin_start = np.zeros(n_chunks + 1, dtype=np.int32)
    ent_a = np.zeros(max(n_chunks, 1), dtype=np.int32)
    ent_r = np.zeros(max(n_chunks, 1), dtype=np.int32)
    n_ent, n_bins = ctypes.c_int32(0), ctypes.c_int32(0)
    P = ctypes.POINTER(ctypes.c_int32)
    rc = nat.lib().lf_greedy_pack(ids32.ctypes.data_as(P), rows32.ctypes.data_as(P), ids32.size, tile_capacity,
                                  n_chunks, bin_start.ctypes.data_as(P), ent_a.ctypes.data_as(P),
                                  ent_r.ctypes.data_as(P), ctypes.byref(n_ent), ctypes.byref(n_bins))
    nat.check(rc, "lf_greedy_pack")
    a_list, r_list, starts = ent_a.tolist(), ent_r.tolist(), bin_start.tolist()
    bins = [list(zip(a_list[starts[b]:starts[b + 1]], r_list[starts[b]:starts[b + 1]]))
            for b in range(n_bins.value)]
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


_RUN_DTYPE = np.dtype([("src", "<u8"), ("dst", "<u8"), ("src_stride", "<i8"), ("dst_stride", "<i8"),
                       ("rows", "<i8"), ("row0", "<i8")])
_RUN_STAGING: dict[int, list] = {}  # device index -> [pinned host table, device table, copy-done event]


def _copy_runs(runs: list[tuple[int, int, int, int, int]], row_bytes: int, device: torch.device) -> None:
    """One ``lf_copy_rows`` launch over ``(src, dst, src_stride, dst_stride, rows)`` runs.

    The run table goes through a per-device pinned staging buffer that is reused once the copy
    that last read it has finished (else a fresh one is taken)."""
    from lorafusion_b200 import _native as nat

    if not runs or row_bytes == 0:
        return
    n = len(runs)
    nbytes = n * _RUN_DTYPE.itemsize
    idx = device.index if device.index is not None else torch.cuda.current_device()
    stage = _RUN_STAGING.get(idx)
    if stage is None or stage[0].numel() < nbytes or not stage[2].query():
        cap = max(nbytes, 64 * _RUN_DTYPE.itemsize)
        stage = [torch.empty(cap, dtype=torch.uint8, pin_memory=True), torch.empty(cap, dtype=torch.uint8, device=device),
                 torch.cuda.Event()]
        _RUN_STAGING[idx] = stage
    host, dev, done = stage
    table = host.numpy()[:nbytes].view(_RUN_DTYPE)
    cols = np.array(runs, dtype=np.int64).reshape(n, 5)
    table["src"], table["dst"] = cols[:, 0].astype(np.uint64), cols[:, 1].astype(np.uint64)
    table["src_stride"], table["dst_stride"], table["rows"] = cols[:, 2], cols[:, 3], cols[:, 4]
    row0 = np.cumsum(cols[:, 4])
    table["row0"][1:] = row0[:-1]
    table["row0"][0] = 0
    stream = torch.cuda.current_stream(device)
    dev[:nbytes].copy_(host[:nbytes], non_blocking=True)
    nat.check(nat.lib().lf_copy_rows(dev.data_ptr(), n, row_bytes, int(row0[-1]), stream.cuda_stream), "lf_copy_rows")
    done.record(stream)  # both tables are free again once the launch that reads them has finished


class _RowOrder(list):
    """``row_order`` as returned by :func:`build_microbatch`: a plain list of request ids that also
    carries the row runs it was built from, so :func:`scatter_outputs` can skip re-encoding it
    (used only while the list still equals the copy taken at build time)."""

    __slots__ = ("_lf_pieces", "_lf_copy")


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
    request id of fused row ``i``.  With CUDA request tensors the rows are
    gathered by one ``lf_copy_rows`` launch; ``fused_x`` equals the
    reference's ``torch.cat`` of the same slices byte for byte.
    """
    in_features = next(iter(request_tensors.values())).shape[1]
    queue: dict[int, list[Request]] = {}
    for req in requests:
        queue.setdefault(req.adapter_id, []).append(req)
    taken: dict[int, int] = {}
    pieces: list[tuple[int, int, int]] = []  # (request id, first row, rows)
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
                pieces.append((req.request_id, start, k))
                row_order.extend([req.request_id] * k)
                taken[req.request_id] = start + k
                want -= k
            routes.append(TileRoute(row_start=cursor, row_end=cursor + n, adapter_id=aid))
            cursor += n
    routing = TileRoutingConfig(tile_size=packing.tile_capacity, routes=routes)
    order = _RowOrder(row_order)
    order._lf_pieces = pieces
    order._lf_copy = row_order
    row_order = order
    if not pieces:
        return torch.empty((0, in_features)), routing, row_order
    srcs = [request_tensors[rid] for rid, _, _ in pieces]
    if not all(t.is_cuda for t in srcs):
        fused_x = torch.cat([request_tensors[rid][a:a + k] for rid, a, k in pieces], dim=0)
        return fused_x, routing, row_order
    device = srcs[0].device
    if any(t.device != device or t.dim() != 2 for t in srcs):
        raise ValueError("request tensors must be 2-D and on one device")
    dtype = functools.reduce(torch.promote_types, {t.dtype for t in srcs})
    ready: dict[int, torch.Tensor] = {}
    for rid, _, _ in pieces:  # rows as contiguous lines of the result dtype
        if rid not in ready:
            t = request_tensors[rid]
            if t.dtype != dtype:
                t = t.to(dtype)
            if t.shape[1] > 0 and t.stride(1) != 1:
                t = t.contiguous()
            ready[rid] = t
    fused_x = torch.empty((len(row_order), in_features), dtype=dtype, device=device)
    es = fused_x.element_size()
    runs, at = [], 0
    for rid, a, k in pieces:
        t = ready[rid]
        runs.append((t.data_ptr() + a * t.stride(0) * es, fused_x.data_ptr() + at * in_features * es,
                     t.stride(0) * es, in_features * es, k))
        at += k
    _copy_runs(runs, in_features * es, device)
    return fused_x, routing, row_order


def scatter_outputs(fused_out: torch.Tensor, row_order: list[int]) -> dict[int, torch.Tensor]:
    """Split fused output rows back per request (data_batcher.py:90-103).

    Requests appear in order of their first fused row; each request's rows
    keep their fused order.  CUDA input: one ``lf_copy_rows`` launch over the
    runs of equal ids in ``row_order``; the values are views of one new
    buffer, request after request.
    """
    if len(row_order) > fused_out.shape[0]:
        raise IndexError(f"row_order has {len(row_order)} rows, fused output only {fused_out.shape[0]}")
    if not row_order:
        return {}
    if not fused_out.is_cuda:
        rows_of: dict[int, list[int]] = {}
        for i, rid in enumerate(row_order):
            rows_of.setdefault(rid, []).append(i)
        out: dict[int, torch.Tensor] = {}
        for rid, idx in rows_of.items():
            index = torch.tensor(idx, dtype=torch.long, device=fused_out.device)
            out[rid] = fused_out.index_select(0, index)
        return out
    src = fused_out.contiguous()
    pieces = getattr(row_order, "_lf_pieces", None)
    if pieces is not None and list.__eq__(row_order, row_order._lf_copy):
        run_id = np.fromiter((p[0] for p in pieces), dtype=np.int64, count=len(pieces))
        run_len = np.fromiter((p[2] for p in pieces), dtype=np.int64, count=len(pieces))
        run_start = np.concatenate(([0], np.cumsum(run_len)[:-1])).astype(np.int64)
        ids_size = int(run_len.sum())
    else:  # runs of equal ids
        ids = np.fromiter(row_order, dtype=np.int64, count=len(row_order))
        cut = np.flatnonzero(ids[1:] != ids[:-1]) + 1
        run_start = np.concatenate(([0], cut))
        run_len = np.diff(np.concatenate((run_start, [ids.size])))
        run_id = ids[run_start]
        ids_size = ids.size
    first = {}
    count: dict[int, int] = {}
    for rid, n in zip(run_id.tolist(), run_len.tolist()):
        if rid not in first:
            first[rid] = len(first)
        count[rid] = count.get(rid, 0) + n
    order = list(first.keys())
    row_shape = tuple(src.shape[1:])
    row_elems = int(np.prod(row_shape)) if row_shape else 1
    buf = torch.empty((ids_size,) + row_shape, dtype=src.dtype, device=src.device)
    base, off = {}, 0
    for rid in order:
        base[rid] = off
        off += count[rid]
    es = src.element_size()
    row_bytes = row_elems * es
    runs, filled = [], dict.fromkeys(order, 0)
    for rid, a, n in zip(run_id.tolist(), run_start.tolist(), run_len.tolist()):
        runs.append((src.data_ptr() + a * row_bytes, buf.data_ptr() + (base[rid] + filled[rid]) * row_bytes,
                     row_bytes, row_bytes, n))
        filled[rid] += n
    _copy_runs(runs, row_bytes, src.device)
    parts = torch.split(buf, [count[rid] for rid in order], dim=0)
    return dict(zip(order, parts))

"""The C-ABI library loads on a CPU-only host, exports every entry point the
header declares, and its host-side table builder is bit-exact (no GPU needed)."""

import ctypes

import numpy as np
import pytest

from lorafusion_b200 import _native as nat


def _tables(routes, total_rows, ranks, scales):
    L = nat.lib()
    starts = np.array([r[0] for r in routes], dtype=np.int32)
    ends = np.array([r[1] for r in routes], dtype=np.int32)
    slots = np.array([r[2] for r in routes], dtype=np.int32)
    rk = np.array(ranks, dtype=np.int32)
    sc = np.array(scales, dtype=np.float32)
    cap = L.lf_plan_table_words(len(routes), total_rows, len(ranks))
    i32p = ctypes.POINTER(ctypes.c_int32)
    for _ in range(2):  # ranks above 64 may need more than the bound: the call reports the need
        table = np.zeros(max(cap, 1), dtype=np.int32)
        info = nat.PlanInfo()
        rc = L.lf_plan_tables(starts.ctypes.data_as(i32p), ends.ctypes.data_as(i32p), slots.ctypes.data_as(i32p),
                              len(routes), total_rows, rk.ctypes.data_as(i32p),
                              sc.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), len(ranks),
                              table.ctypes.data_as(i32p), cap, ctypes.byref(info))
        if rc != nat.LF_ERR_CAPACITY or info.table_words <= cap:
            break
        cap = info.table_words
    return rc, info, table


def _sec(info, table, name, n):
    off = getattr(info, "off_" + name)
    return table[off:off + n]


def test_library_loads_and_exports_header_symbols():
    L = nat.lib()
    declared = nat.header_symbols()
    assert len(declared) >= 10
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/lorafusion_b200.h but not exported"
    assert L.lf_version().decode().startswith("lorafusion_b200")
    assert nat.status_text(nat.LF_ERR_ROUTING).startswith("routes")


def test_plan_info_struct_matches_header():
    text = open(nat.HEADER_PATH).read()
    body = text.split("typedef struct lf_plan_info {")[1].split("} lf_plan_info;")[0]
    names = [ln.split(";")[0].split()[-1] for ln in body.splitlines() if ln.strip().startswith("int32_t")]
    assert names == [f[0] for f in nat.PlanInfo._fields_]
    body = text.split("typedef struct lf_problem {")[1].split("} lf_problem;")[0]
    fields = []
    for ln in body.splitlines():
        ln = ln.split("/*")[0].strip()
        if not ln:
            continue
        decl = ln.rstrip(";")
        for part in decl.split(","):
            fields.append(part.strip().split()[-1].lstrip("*"))
    assert fields == [f[0] for f in nat.Problem._fields_]
    body = text.split("typedef struct lf_row_run {")[1].split("} lf_row_run;")[0]
    names = [ln.split("/*")[0].strip().rstrip(";").split()[-1] for ln in body.splitlines() if ln.split("/*")[0].strip()]
    assert names == [f[0] for f in nat.RowRun._fields_]
    assert ctypes.sizeof(nat.RowRun) == 48


def _reconstruct(info, table):
    n_st = info.n_segtiles
    tile = _sec(info, table, "st_tile", n_st)
    lo = _sec(info, table, "st_lo", n_st)
    hi = _sec(info, table, "st_hi", n_st)
    slot = _sec(info, table, "st_slot", n_st)
    route = _sec(info, table, "st_route", n_st)
    out = {}
    for j in range(n_st):
        r0 = int(tile[j]) * nat.TILE_ROWS + int(lo[j])
        r1 = int(tile[j]) * nat.TILE_ROWS + int(hi[j])
        cur = out.setdefault(int(route[j]), [r0, r1, int(slot[j])])
        assert cur[2] == slot[j]
        if cur[1] < r1:
            assert cur[1] == r0
            cur[1] = r1
        if cur[0] > r0:
            cur[0] = r0
    return out


def test_tables_round_trip_reference_routes(layout_golden):
    """Every golden route layout survives the tile cut bit-exactly."""
    z = layout_golden
    for name in [str(n) for n in z["names"]]:
        routes = [tuple(int(v) for v in r) for r in z[f"{name}/routes"]]
        T = routes[-1][1] if routes else 0
        slot_of = {}
        sroutes = [(s, e, slot_of.setdefault(a, len(slot_of))) for s, e, a in routes]
        rc, info, table = _tables(sroutes, T, [16] * len(slot_of), [2.0] * len(slot_of))
        assert rc == 0, name
        rec = _reconstruct(info, table)
        nonempty = [(i, r) for i, r in enumerate(sroutes) if r[1] > r[0]]
        assert sorted(rec) == [i for i, _ in nonempty]
        for i, r in nonempty:
            assert tuple(rec[i]) == r, (name, i)
        # CSR over tiles covers every segment tile once, in row order
        tile_st = _sec(info, table, "tile_st", info.n_tiles + 1)
        assert tile_st[0] == 0 and tile_st[-1] == info.n_segtiles and np.all(np.diff(tile_st) >= 0)
        # per-slot lists are in route order and partition the segment tiles
        slot_st = _sec(info, table, "slot_st", info.n_slots + 1)
        lst = _sec(info, table, "slot_list", info.n_segtiles)
        assert sorted(lst.tolist()) == list(range(info.n_segtiles))
        for s in range(info.n_slots):
            part = lst[slot_st[s]:slot_st[s + 1]]
            assert np.all(np.diff(part) > 0)
        # shrink units cover each tile's segment tiles in runs of <= 64 / r_pad
        nst = _sec(info, table, "unit_nst", info.n_shrink_units)
        assert nst.sum() == info.n_segtiles and nst.max(initial=1) <= 64 // info.r_pad


def test_tables_errors_and_padding():
    assert _tables([(0, 10, 0), (12, 20, 0)], 20, [8], [2.0])[0] == nat.LF_ERR_ROUTING
    assert _tables([(0, 10, 0)], 20, [8], [2.0])[0] == nat.LF_ERR_ROUTING
    assert _tables([(0, 10, 1)], 10, [8], [2.0])[0] == nat.LF_ERR_ROUTING
    for r, pad in [(1, 16), (16, 16), (17, 32), (32, 32), (33, 64), (64, 64)]:
        rc, info, _ = _tables([(0, 300, 0)], 300, [r], [1.0])
        assert rc == 0 and info.r_pad == pad and info.rank_total == r
    rc, info, _ = _tables([], 0, [], [])
    assert rc == 0 and info.n_segtiles == 0 and info.n_tiles == 0
    rc, info, table = _tables([(0, 0, 0), (0, 5, 1)], 5, [4, 8], [2.0, 1.0])
    assert rc == 0 and info.n_slots == 2 and info.n_segtiles == 1
    slot_st = _sec(info, table, "slot_st", 3)
    assert slot_st.tolist() == [0, 0, 1]


def test_workspace_sizes():
    rc, info, _ = _tables([(0, 1000, 0), (1000, 1300, 1)], 1300, [16, 64], [2.0, 2.0])
    assert rc == 0
    L = nat.lib()
    fw = L.lf_forward_workspace_bytes(ctypes.byref(info), nat.LF_BF16)
    bw = L.lf_backward_workspace_bytes(ctypes.byref(info), nat.LF_BF16)
    sext = (info.n_segtiles + 1) * 128 * info.r_pad * 4
    assert fw >= sext + info.n_shrink_units * 8 and fw % 256 == 0
    assert bw >= fw + sext and bw % 256 == 0


def test_ops_raise_without_gpu_inputs():
    import torch
    from lorafusion_b200 import b200_ops
    from lorafusion_b200.config import AdapterSpec, TileRoute, TileRoutingConfig
    x = torch.zeros(4, 8)
    rt = TileRoutingConfig(16, [TileRoute(0, 4, 0)])
    ad = {0: AdapterSpec(0, 2, 4.0, 8, 8)}
    with pytest.raises(ValueError, match="CUDA"):
        b200_ops.fused_lora_forward(x, torch.zeros(8, 8), {0: torch.zeros(2, 8)}, {0: torch.zeros(8, 2)}, ad, rt)
    with pytest.raises(ValueError, match="covers"):
        b200_ops.fused_lora_forward(torch.zeros(5, 8), torch.zeros(8, 8), {}, {}, ad, rt)


def test_co_scheduling_switch_rejects_unknown_modes():
    L = nat.lib()
    assert L.lf_set_co_scheduling(3) == nat.LF_ERR_INVALID_ARG
    assert L.lf_set_co_scheduling(-1) == nat.LF_ERR_INVALID_ARG
    for mode in (0, 2, 1):  # ends on the default
        assert L.lf_set_co_scheduling(mode) == 0


def test_release_holds_nothing_without_gpu_work():
    from lorafusion_b200 import b200_ops
    assert nat.lib().lf_release() == 0
    b200_ops.release()  # host caches and library state; safe to repeat
    assert nat.lib().lf_release() == 0


def test_host_streamed_forward_rejects_bad_chunk_lists():
    """lf_forward_host checks its chunk list before touching the GPU: chunks must follow each other
    from row 0, match their tables' row counts and cover the batch exactly."""
    L = nat.lib()
    rc0, info_a, _ = _tables([(0, 256, 0)], 256, [16], [2.0])
    rc1, info_b, _ = _tables([(0, 44, 0)], 44, [16], [2.0])
    assert rc0 == 0 and rc1 == 0
    prob = nat.Problem()
    prob.dtype, prob.T, prob.K, prob.N = nat.LF_BF16, 300, 64, 64
    chunks = (nat.HostChunk * 2)()
    chunks[0].row0, chunks[0].rows, chunks[0].info = 0, 256, ctypes.pointer(info_a)
    chunks[1].row0, chunks[1].rows, chunks[1].info = 256, 44, ctypes.pointer(info_b)
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)

    def call(n, T=300):
        prob.T = T
        return L.lf_forward_host(ctypes.byref(prob), chunks, n, p, p, p, p, p, 64, None, None, None)

    assert call(2, T=301) == nat.LF_ERR_INVALID_ARG  # rows do not add up to T
    assert call(1) == nat.LF_ERR_INVALID_ARG          # batch not covered
    chunks[1].row0 = 200
    assert call(2) == nat.LF_ERR_INVALID_ARG          # overlapping chunks
    chunks[1].row0, chunks[1].rows = 256, 45
    assert call(2) == nat.LF_ERR_INVALID_ARG          # chunk rows differ from its tables'
    assert call(0, T=0) == 0                          # nothing to do
    assert L.lf_forward_host(None, chunks, 0, p, p, p, p, p, 64, None, None, None) == nat.LF_ERR_INVALID_ARG


def test_ranks_above_64_become_virtual_slots():
    """A slot of rank r > 64 is carried as ceil(r/64) consecutive virtual slots (64, ..., remainder)
    over the same rows; the other slots keep their order; a too-small table buffer reports the need."""
    routes = [(0, 100, 0), (100, 300, 1), (300, 310, 2)]
    rc, info, table = _tables(routes, 310, [16, 130, 64], [2.0, 0.5, 1.0])
    assert rc == 0
    assert info.n_slots == 1 + 3 + 1 and info.r_pad == 64 and info.max_rank == 130 and info.rank_total == 210
    assert _sec(info, table, "slot_rank", info.n_slots).tolist() == [16, 64, 64, 2, 64]
    assert _sec(info, table, "rank_prefix", info.n_slots + 1).tolist() == [0, 16, 80, 144, 146, 210]
    lo, hi = _sec(info, table, "st_lo", info.n_segtiles), _sec(info, table, "st_hi", info.n_segtiles)
    tile, slot = _sec(info, table, "st_tile", info.n_segtiles), _sec(info, table, "st_slot", info.n_segtiles)
    scale = _sec(info, table, "st_scale", info.n_segtiles).view(np.float32)
    rows = {}
    for j in range(info.n_segtiles):
        rows.setdefault(int(slot[j]), []).append((int(tile[j]) * 128 + int(lo[j]), int(tile[j]) * 128 + int(hi[j])))
    assert rows[0] == [(0, 100)]
    for v in (1, 2, 3):  # the rank-130 slot: three virtual slots over rows 100..300, scaling 0.5
        assert rows[v] == [(100, 128), (128, 256), (256, 300)]
        assert np.all(scale[slot == v] == 0.5)
    assert rows[4] == [(300, 310)]
    # within a tile, the virtual slots of one route follow each other
    t1 = [int(v) for v, t in zip(slot, tile) if t == 1]
    assert t1 == [1, 2, 3]
    # a buffer that is too small: LF_ERR_CAPACITY and the words needed
    i32p = ctypes.POINTER(ctypes.c_int32)
    starts = np.array([s for s, _, _ in routes], np.int32)
    ends = np.array([e for _, e, _ in routes], np.int32)
    slots = np.array([a for _, _, a in routes], np.int32)
    rk = np.array([16, 700, 64], np.int32)
    sc = np.array([2.0, 0.5, 1.0], np.float32)
    cap = nat.lib().lf_plan_table_words(3, 310, 3)
    buf = np.zeros(cap, np.int32)
    inf = nat.PlanInfo()
    rc = nat.lib().lf_plan_tables(starts.ctypes.data_as(i32p), ends.ctypes.data_as(i32p), slots.ctypes.data_as(i32p),
                                  3, 310, rk.ctypes.data_as(i32p), sc.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                  3, buf.ctypes.data_as(i32p), cap, ctypes.byref(inf))
    assert rc == nat.LF_ERR_CAPACITY and inf.table_words > cap


def test_peer_exchange_sizes():
    """lf_peer_exchange_bytes: two halves (alternate calls), each one 16-byte entry of two
    generation-tagged 64-bit words per (source rank, block, rank-column pair, column), rounded up
    to 256 bytes; unsupported arguments give 0."""
    L = nat.lib()

    def half(world, n_blocks, r_pad):
        return (world * n_blocks * 128 * r_pad * 8 + 255) // 256 * 256

    for world, n_blocks, r_pad in ((2, 1, 16), (4, 3 * 64, 16), (8, 7, 64), (2, 5, 32), (3, 1, 16)):
        assert L.lf_peer_exchange_bytes(world, n_blocks, r_pad) == 2 * half(world, n_blocks, r_pad)
    assert L.lf_peer_exchange_bytes(1, 0, 16) == 0  # nothing to exchange
    for world, n_blocks, r_pad in ((0, 1, 16), (nat.MAX_PEERS + 1, 1, 16), (2, -1, 16), (2, 1, 24), (2, 1, 128)):
        assert L.lf_peer_exchange_bytes(world, n_blocks, r_pad) == 0

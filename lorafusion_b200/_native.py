"""ctypes binding of the C ABI declared in ``include/lorafusion_b200.h``.

The shared library is built in-tree (``python -m lorafusion_b200.csrc.build``)
into ``lorafusion_b200/_lib/liblorafusion_b200.so``.  :func:`lib` loads it once
and raises ``RuntimeError`` when it is missing: the operator has no fallback.
"""

from __future__ import annotations

import ctypes
import os
import re
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "liblorafusion_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "lorafusion_b200.h")

LF_OK = 0
LF_ERR_INVALID_ARG = 1
LF_ERR_ROUTING = 2
LF_ERR_UNSUPPORTED = 3
LF_ERR_CUDA = 4
LF_ERR_CAPACITY = 5
LF_ERR_DEVICE = 6

LF_F32, LF_BF16, LF_F16 = 0, 1, 2
LF_STAGE_SHRINK, LF_STAGE_EXPAND, LF_STAGE_BASE, LF_STAGE_SINGLE_CTA, LF_STAGE_SEPARATE = 1, 2, 4, 8, 16
LF_BSTAGE_SHRINK, LF_BSTAGE_GRAD_X, LF_BSTAGE_GRAD_AB = 1, 2, 4
TILE_ROWS = 128

_c_i32 = ctypes.c_int32
_c_p = ctypes.c_void_p


class PlanInfo(ctypes.Structure):
    _fields_ = [(name, _c_i32) for name in (
        "total_rows", "n_routes", "n_slots", "n_tiles", "n_segtiles", "r_pad", "max_rank", "rank_total",
        "n_shrink_units", "table_words",
        "off_tile_st", "off_st_tile", "off_st_lo", "off_st_hi", "off_st_slot", "off_st_route", "off_st_scale",
        "off_slot_st", "off_slot_list", "off_slot_rank", "off_rank_prefix", "off_slot_order",
        "off_unit_tile", "off_unit_st0", "off_unit_nst",
        "n_pair_lora", "off_pair_lora", "off_pl_a", "off_pl_b", "off_pl_slot", "off_tile_unit")]


class Problem(ctypes.Structure):
    _fields_ = [
        ("dtype", _c_i32), ("T", _c_i32), ("K", _c_i32), ("N", _c_i32),
        ("x_dev", _c_p), ("w_dev", _c_p), ("a_pack_dev", _c_p), ("b_pack_dev", _c_p),
        ("bt_pack_dev", _c_p), ("at_pack_dev", _c_p),
    ]


class RowRun(ctypes.Structure):
    _fields_ = [("src", ctypes.c_uint64), ("dst", ctypes.c_uint64), ("src_stride", ctypes.c_int64),
                ("dst_stride", ctypes.c_int64), ("rows", ctypes.c_int64), ("row0", ctypes.c_int64)]


MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class PeerReduce(ctypes.Structure):
    """lf_peer_reduce: the gram kernel's exchange of spanning adapters' blocks between GPUs."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("exchange", ctypes.c_void_p * MAX_PEERS),
                ("slot_span_dev", ctypes.c_void_p), ("span_info_dev", ctypes.c_void_p), ("n_span", ctypes.c_int32),
                ("r_pad_x", ctypes.c_int32), ("gen", ctypes.c_uint64)]


class HostChunk(ctypes.Structure):
    _fields_ = [("row0", ctypes.c_int32), ("rows", ctypes.c_int32), ("info", ctypes.POINTER(PlanInfo)),
                ("table_dev", ctypes.c_void_p)]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def _declare(L: ctypes.CDLL) -> None:
    P = ctypes.POINTER
    L.lf_plan_table_words.argtypes = [_c_i32, _c_i32, _c_i32]
    L.lf_plan_table_words.restype = _c_i32
    L.lf_plan_tables.argtypes = [P(_c_i32), P(_c_i32), P(_c_i32), _c_i32, _c_i32, P(_c_i32),
                                 P(ctypes.c_float), _c_i32, P(_c_i32), _c_i32, P(PlanInfo)]
    L.lf_plan_tables.restype = ctypes.c_int
    L.lf_forward_workspace_bytes.argtypes = [P(PlanInfo), _c_i32]
    L.lf_forward_workspace_bytes.restype = ctypes.c_size_t
    L.lf_backward_workspace_bytes.argtypes = [P(PlanInfo), _c_i32]
    L.lf_backward_workspace_bytes.restype = ctypes.c_size_t
    L.lf_pack_adapters.argtypes = [_c_i32, _c_i32, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                   _c_p, _c_p]
    L.lf_pack_adapters.restype = ctypes.c_int
    L.lf_copy_rows.argtypes = [_c_p, _c_i32, ctypes.c_int64, ctypes.c_int64, _c_p]
    L.lf_forward_host.argtypes = [P(Problem), P(HostChunk), _c_i32, _c_p, _c_p, _c_p, _c_p, _c_p, ctypes.c_size_t,
                                  _c_p, _c_p, _c_p]
    L.lf_forward_host.restype = ctypes.c_int
    L.lf_release.argtypes = []
    L.lf_release.restype = ctypes.c_int
    L.lf_copy_rows.restype = ctypes.c_int
    L.lf_greedy_pack.argtypes = [P(_c_i32), P(_c_i32), _c_i32, _c_i32, _c_i32, P(_c_i32), P(_c_i32), P(_c_i32),
                                 P(_c_i32), P(_c_i32)]
    L.lf_greedy_pack.restype = ctypes.c_int
    L.lf_assign_rows.argtypes = [P(_c_i32), P(_c_i32), P(_c_i32), _c_i32, _c_i32, _c_i32, _c_i32,
                                 P(ctypes.c_int64), P(ctypes.c_int64), P(_c_i32), P(_c_i32)]
    L.lf_assign_rows.restype = ctypes.c_int
    L.lf_forward.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p, ctypes.c_size_t, _c_p]
    L.lf_forward.restype = ctypes.c_int
    L.lf_forward_stages.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p, ctypes.c_size_t, _c_i32, _c_p]
    L.lf_forward_stages.restype = ctypes.c_int
    L.lf_forward_launch_count.argtypes = [P(Problem), P(PlanInfo)]
    L.lf_forward_launch_count.restype = ctypes.c_int
    L.lf_backward_launch_count.argtypes = [P(Problem), P(PlanInfo)]
    L.lf_backward_launch_count.restype = ctypes.c_int
    L.lf_set_co_scheduling.argtypes = [_c_i32]
    L.lf_set_co_scheduling.restype = ctypes.c_int
    L.lf_get_co_scheduling.argtypes = [P(_c_i32), P(_c_i32)]
    L.lf_get_co_scheduling.restype = ctypes.c_int
    L.lf_forward_sf.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p, ctypes.c_size_t, _c_p, ctypes.c_size_t,
                                P(_c_i32), _c_p]
    L.lf_forward_sf.restype = ctypes.c_int
    L.lf_forward_fixed_workspace_bytes.argtypes = [P(PlanInfo), _c_i32]
    L.lf_forward_fixed_workspace_bytes.restype = ctypes.c_size_t
    L.lf_backward_ex.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_p, _c_p,
                                 ctypes.c_size_t, _c_p]
    L.lf_backward_ex.restype = ctypes.c_int
    L.lf_backward_peer.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_p,
                                   _c_p, ctypes.c_size_t, P(PeerReduce), _c_p]
    L.lf_backward_peer.restype = ctypes.c_int
    L.lf_peer_exchange_bytes.argtypes = [_c_i32, _c_i32, _c_i32]
    L.lf_peer_exchange_bytes.restype = ctypes.c_size_t
    L.lf_peer_alloc.argtypes = [ctypes.c_size_t, P(ctypes.c_void_p)]
    L.lf_peer_alloc.restype = ctypes.c_int
    L.lf_peer_free.argtypes = [_c_p]
    L.lf_peer_free.restype = ctypes.c_int
    L.lf_ipc_handle.argtypes = [_c_p, _c_p]
    L.lf_ipc_handle.restype = ctypes.c_int
    L.lf_ipc_open.argtypes = [_c_p, P(ctypes.c_void_p)]
    L.lf_ipc_open.restype = ctypes.c_int
    L.lf_ipc_close.argtypes = [_c_p]
    L.lf_ipc_close.restype = ctypes.c_int
    L.lf_backward_stages.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_p,
                                     _c_p, ctypes.c_size_t, _c_i32, _c_p]
    L.lf_backward_stages.restype = ctypes.c_int
    L.lf_backward.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, ctypes.c_size_t, _c_p]
    L.lf_backward.restype = ctypes.c_int
    L.lf_backward_sf.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p, _c_i32, _c_p, _c_p, _c_p, _c_p,
                                 ctypes.c_size_t, _c_p]
    L.lf_backward_sf.restype = ctypes.c_int
    L.lf_forward_noalloc.argtypes = [P(Problem), P(PlanInfo), _c_p, _c_p, _c_p]
    L.lf_forward_noalloc.restype = ctypes.c_int
    L.lf_set_wait_limit.argtypes = [ctypes.c_uint64]
    L.lf_set_wait_limit.restype = ctypes.c_int
    L.lf_inject_stale_ready.argtypes = [_c_i32]
    L.lf_inject_stale_ready.restype = ctypes.c_int
    L.lf_device_error.argtypes = [P(_c_i32)]
    L.lf_device_error.restype = ctypes.c_int
    L.lf_status_string.argtypes = [ctypes.c_int]
    L.lf_status_string.restype = ctypes.c_char_p
    L.lf_version.argtypes = []
    L.lf_version.restype = ctypes.c_char_p


def lib() -> ctypes.CDLL:
    """The loaded library; ``RuntimeError`` if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"lorafusion_b200 native library not found at {LIB_PATH}; "
                    "build it with `python -m lorafusion_b200.csrc.build` (needs nvcc for sm_100a)")
            L = ctypes.CDLL(LIB_PATH)
            _declare(L)
            _lib = L
    return _lib


def header_symbols() -> list[str]:
    """Names of every entry point the public header declares."""
    text = open(HEADER_PATH).read()
    return re.findall(r"^LF_API\s+[\w\s\*]+?\b(lf_\w+)\s*\(", text, flags=re.M)


def status_text(code: int) -> str:
    return lib().lf_status_string(code).decode()


def check(code: int, what: str) -> None:
    """Map a C status to the reference's exception types."""
    if code == LF_OK:
        return
    msg = f"{what}: {status_text(code)} (status {code})"
    if code in (LF_ERR_CUDA, LF_ERR_DEVICE):
        raise RuntimeError(msg)
    raise ValueError(msg)


def co_scheduling() -> tuple[int, int]:
    """(process-wide co-scheduling mode, cudaError_t of a refused cooperative launch on the current
    device or 0)."""
    mode, refused = _c_i32(0), _c_i32(0)
    check(lib().lf_get_co_scheduling(ctypes.byref(mode), ctypes.byref(refused)), "lf_get_co_scheduling")
    return int(mode.value), int(refused.value)


# device status codes of bounded waits that ran out (lf_ptx.cuh DeviceErr)
ERR_TIMEOUT_FULL, ERR_TIMEOUT_EMPTY, ERR_TIMEOUT_ACC, ERR_TIMEOUT_DRAIN, ERR_TIMEOUT_FLAG = 0x101, 0x102, 0x103, 0x104, 0x105


def set_wait_limit(limit_ns: int) -> None:
    """Bound of every in-kernel wait on the current device (0: the default, about 1 s)."""
    check(lib().lf_set_wait_limit(int(limit_ns)), "lf_set_wait_limit")


def device_error() -> int:
    """Read and clear the kernels' device status word (synchronizes the device)."""
    v = _c_i32(0)
    check(lib().lf_device_error(ctypes.byref(v)), "lf_device_error")
    return int(v.value)

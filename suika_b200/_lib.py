"""ctypes binding of libsuika_reshard.so (C ABI: include/suika_reshard.h).

The structures below mirror the header field for field. Loading never falls back to anything:
if the library is missing or cannot be built, every call into the reshard path raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

from . import build as _build

RS_MAX_DIMS = 8
RS_NO_SLICE = -1000

RS_OK = 0
RS_ERR_ARG = -1
RS_ERR_NO_OWNER = -2
RS_ERR_SHAPE = -3
RS_ERR_SLICE_DIM = -4
RS_ERR_EMPTY_SOURCE = -5
RS_ERR_CUDA = -6
RS_ERR_BOUNDS = -7
RS_ERR_CAPACITY = -8
RS_ERR_PEER = -9
RS_ERR_SUBFIELD = -10

RS_ORDER_REFERENCE = 0
RS_ORDER_SEMANTIC = 1
RS_SRC_REFERENCE = 0
RS_SRC_BALANCED = 1
RS_NOALLOC_MAX_ENTRIES = 16384
RS_RUN_STALL_FIRST_STAGE = 1


class RsTensorMeta(C.Structure):
    _fields_ = [("name_id", C.c_int32), ("ndim", C.c_int32), ("shape", C.c_int64 * RS_MAX_DIMS),
                ("itemsize", C.c_int32), ("slice_dim", C.c_int32), ("tp_index", C.c_int32), ("tp_deg", C.c_int32)]


class RsRankLayout(C.Structure):
    _fields_ = [("rank", C.c_int32), ("n_tensors", C.c_int32), ("tensors", C.POINTER(RsTensorMeta))]


class RsPlanOpts(C.Structure):
    _fields_ = [("minimum_est_peers", C.c_int32), ("order", C.c_int32), ("src_choice", C.c_int32), ("reserved", C.c_int32)]


class RsOp(C.Structure):
    _fields_ = [("name_id", C.c_int32), ("src_rank", C.c_int32), ("dst_rank", C.c_int32),
                ("src_slice_dim", C.c_int32), ("src_tp_index", C.c_int32), ("src_tp_deg", C.c_int32),
                ("dst_slice_dim", C.c_int32), ("dst_tp_index", C.c_int32), ("dst_tp_deg", C.c_int32),
                ("reserved", C.c_int32), ("numel", C.c_int64)]


RS_MAX_GROUPS = 4


class RsSliceGroup(C.Structure):
    _fields_ = [("offset", C.c_int64), ("size", C.c_int64), ("units", C.c_int64)]


class RsSliceRule(C.Structure):
    _fields_ = [("name_id", C.c_int32), ("n_groups", C.c_int32), ("groups", RsSliceGroup * RS_MAX_GROUPS)]


class RsSubfield(C.Structure):
    _fields_ = [("itemsize", C.c_int32), ("is_meta", C.c_int32)]


class RsProgramCounts(C.Structure):
    _fields_ = [("n_dst_slots", C.c_int64), ("n_src_slots", C.c_int64), ("n_meta_slots", C.c_int64),
                ("n_segments", C.c_int64), ("remote_bytes", C.c_uint64), ("local_bytes", C.c_uint64)]


class RsDstSlot(C.Structure):
    _fields_ = [("name_id", C.c_int32), ("subfield", C.c_int32), ("ndim", C.c_int32), ("reserved", C.c_int32),
                ("shape", C.c_int64 * RS_MAX_DIMS), ("nbytes", C.c_uint64)]


class RsSrcSlot(C.Structure):
    _fields_ = [("src_rank", C.c_int32), ("name_id", C.c_int32), ("subfield", C.c_int32), ("reserved", C.c_int32),
                ("nbytes", C.c_uint64)]


class RsMetaSlot(C.Structure):
    _fields_ = [("name_id", C.c_int32), ("subfield", C.c_int32), ("src_rank", C.c_int32), ("first_is_self", C.c_int32)]


class RsSegment(C.Structure):
    _fields_ = [("src_slot", C.c_int32), ("dst_slot", C.c_int32), ("src_offset", C.c_uint64), ("dst_offset", C.c_uint64),
                ("rows", C.c_uint64), ("row_bytes", C.c_uint64), ("src_pitch", C.c_uint64), ("dst_pitch", C.c_uint64)]


RS_COPY_REMOTE = 1


class RsCopyDesc(C.Structure):
    _fields_ = [("src_dev", C.c_uint64), ("dst_dev", C.c_uint64), ("rows", C.c_uint64), ("row_bytes", C.c_uint64),
                ("src_pitch", C.c_uint64), ("dst_pitch", C.c_uint64), ("flags", C.c_uint64)]


class RsLaunchInfo(C.Structure):
    _fields_ = [("n_tiles", C.c_uint64), ("total_bytes", C.c_uint64), ("n_entries", C.c_int64), ("n_tiles_remote", C.c_uint64),
                ("grid", C.c_int32), ("block", C.c_int32), ("variant", C.c_int32), ("reserved", C.c_int32),
                ("n_tensor_entries", C.c_int64), ("n_tensor_tiles", C.c_uint64), ("tensor_grid", C.c_int32),
                ("tensor_block", C.c_int32)]


class RsPeerHandle(C.Structure):
    _fields_ = [("ipc", C.c_uint8 * 64), ("alloc_base", C.c_uint64), ("alloc_bytes", C.c_uint64),
                ("device", C.c_int32), ("pid", C.c_int32)]


class RsStageMesh(C.Structure):
    _fields_ = [("n_groups", C.c_int32), ("reserved", C.c_int32), ("group_start", C.POINTER(C.c_int32)),
                ("ranks", C.POINTER(C.c_int32)), ("local_bsz", C.POINTER(C.c_int64))]


class RsActPiece(C.Structure):
    _fields_ = [("src_rank", C.c_int32), ("dst_rank", C.c_int32), ("src_batch", C.c_int64), ("dst_batch", C.c_int64),
                ("n_batch", C.c_int64), ("slice_start", C.c_int64), ("slice_len", C.c_int64)]


class RsActGeometry(C.Structure):
    _fields_ = [("ndim", C.c_int32), ("batch_dim", C.c_int32), ("slice_dim", C.c_int32), ("elem_bytes", C.c_int32),
                ("shape", C.c_int64 * RS_MAX_DIMS)]


# numpy mirrors used to fill large descriptor arrays without a Python loop per field.
TENSOR_META_DTYPE = np.dtype([("name_id", "<i4"), ("ndim", "<i4"), ("shape", "<i8", (RS_MAX_DIMS,)),
                              ("itemsize", "<i4"), ("slice_dim", "<i4"), ("tp_index", "<i4"), ("tp_deg", "<i4")])
COPY_DESC_DTYPE = np.dtype([("src_dev", "<u8"), ("dst_dev", "<u8"), ("rows", "<u8"), ("row_bytes", "<u8"),
                            ("src_pitch", "<u8"), ("dst_pitch", "<u8"), ("flags", "<u8")])
SEGMENT_DTYPE = np.dtype([("src_slot", "<i4"), ("dst_slot", "<i4"), ("src_offset", "<u8"), ("dst_offset", "<u8"),
                          ("rows", "<u8"), ("row_bytes", "<u8"), ("src_pitch", "<u8"), ("dst_pitch", "<u8")])
ACT_PIECE_DTYPE = np.dtype([("src_rank", "<i4"), ("dst_rank", "<i4"), ("src_batch", "<i8"), ("dst_batch", "<i8"),
                            ("n_batch", "<i8"), ("slice_start", "<i8"), ("slice_len", "<i8")])
assert TENSOR_META_DTYPE.itemsize == C.sizeof(RsTensorMeta)
assert ACT_PIECE_DTYPE.itemsize == C.sizeof(RsActPiece)
assert COPY_DESC_DTYPE.itemsize == C.sizeof(RsCopyDesc)
assert SEGMENT_DTYPE.itemsize == C.sizeof(RsSegment)

# Every symbol include/suika_reshard.h declares, with its ctypes signature.
_P = C.c_void_p
SIGNATURES = {
    "rs_last_error": (C.c_char_p, []),
    "rs_version": (C.c_int, [C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "rs_plan_build": (C.c_int, [C.POINTER(RsRankLayout), C.c_int32, C.POINTER(RsRankLayout), C.c_int32,
                                C.POINTER(RsPlanOpts), C.POINTER(_P)]),
    "rs_plan_build_rules": (C.c_int, [C.POINTER(RsRankLayout), C.c_int32, C.POINTER(RsRankLayout), C.c_int32,
                                      C.POINTER(RsSliceRule), C.c_int32, C.POINTER(RsPlanOpts), C.POINTER(_P)]),
    "rs_plan_num_ops": (C.c_int, [_P, C.POINTER(C.c_int64)]),
    "rs_plan_get_ops": (C.c_int, [_P, C.POINTER(RsOp), C.c_int64]),
    "rs_plan_free": (None, [_P]),
    "rs_program_build": (C.c_int, [_P, C.c_int32, C.POINTER(RsSubfield), C.c_int32, C.POINTER(_P)]),
    "rs_program_counts_get": (C.c_int, [_P, C.POINTER(RsProgramCounts)]),
    "rs_program_dst_slots": (C.c_int, [_P, C.POINTER(RsDstSlot), C.c_int64]),
    "rs_program_src_slots": (C.c_int, [_P, C.POINTER(RsSrcSlot), C.c_int64]),
    "rs_program_meta_slots": (C.c_int, [_P, C.POINTER(RsMetaSlot), C.c_int64]),
    "rs_program_segments": (C.c_int, [_P, _P, C.c_int64]),
    "rs_program_free": (None, [_P]),
    "rs_program_resolve": (C.c_int, [_P, _P, _P, _P, _P, _P, C.c_int64]),
    "rs_program_resolve_from": (C.c_int, [_P, C.c_int32, _P, _P, _P, _P, _P, C.c_int64, C.POINTER(C.c_int64)]),
    "rs_copy_workspace_bytes": (C.c_int, [C.c_int64, C.POINTER(C.c_uint64)]),
    "rs_copy_stage": (C.c_int, [_P, C.c_int64, _P, C.c_uint64, _P, C.POINTER(RsLaunchInfo)]),
    "rs_copy_run": (C.c_int, [_P, C.POINTER(RsLaunchInfo), _P]),
    "rs_copy_run_bounded": (C.c_int, [_P, C.POINTER(RsLaunchInfo), _P, C.c_uint64, C.c_uint32]),
    "rs_copy_status": (C.c_int, [_P, C.POINTER(RsLaunchInfo), _P, C.POINTER(C.c_uint32)]),
    "rs_copy_launch": (C.c_int, [_P, C.c_int64, _P, C.c_uint64, _P, C.POINTER(RsLaunchInfo)]),
    "rs_copy_launch_noalloc": (C.c_int, [_P, C.c_int64, _P, C.POINTER(RsLaunchInfo)]),
    "rs_host_device_pointer": (C.c_int, [_P, C.POINTER(_P)]),
    "rs_peer_export": (C.c_int, [_P, C.POINTER(RsPeerHandle), C.POINTER(C.c_uint64)]),
    "rs_peer_open": (C.c_int, [C.POINTER(RsPeerHandle), C.POINTER(_P)]),
    "rs_peer_close": (C.c_int, [_P]),
    "rs_act_plan": (C.c_int, [C.POINTER(RsStageMesh), C.POINTER(RsStageMesh), C.c_int64, _P, C.c_int64,
                              C.POINTER(C.c_int64)]),
    "rs_act_resolve": (C.c_int, [C.POINTER(RsStageMesh), C.POINTER(RsStageMesh), C.POINTER(RsActGeometry), _P, C.c_int64,
                                 _P, _P, C.c_int32, _P, C.c_int64, C.POINTER(C.c_int64)]),
}

_lock = threading.Lock()
_lib = None


def library_path() -> str:
    return _build.LIB_PATH


def load() -> C.CDLL:
    """Load (building first when the sources are newer) libsuika_reshard.so; raise if impossible."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if _build.is_stale():
            try:
                path = _build.build()
            except Exception as e:  # no toolchain: a prebuilt library is still fine
                if not os.path.exists(path):
                    raise RuntimeError(f"libsuika_reshard.so is missing and cannot be built: {e}") from e
        lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


class ReshardError(RuntimeError):
    """A non-assertion failure reported by libsuika_reshard (CUDA, peer memory, bounds)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[rs error {code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    """Raise the Python error matching the reference's behaviour for a failed call."""
    if rc == RS_OK:
        return
    msg = load().rs_last_error().decode(errors="replace")
    if rc in (RS_ERR_NO_OWNER, RS_ERR_SHAPE, RS_ERR_SLICE_DIM, RS_ERR_SUBFIELD):
        raise AssertionError(msg)  # the reference asserts in these cases (migration.py:293-294,311,356,441)
    if rc == RS_ERR_EMPTY_SOURCE:
        raise ValueError(msg)      # max() of an empty sequence (migration.py:335)
    raise ReshardError(rc, msg)

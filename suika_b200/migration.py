"""B200 drop-in for Suika's parameter-transfer path (Suika/migration.py).

The reference moves a job's merged {name: {sub_field: tensor}} state from one (TP, PP, DP)
layout to another with schedule_param_transfer (migration.py:322-381) and
execute_param_transfer (migration.py:397-556), glued by schedule_and_execute_param_transfer
(migration.py:558-598), which migration_save / migration_load call. This module keeps those
names, arguments, return values and error behaviour, and runs them on libsuika_reshard.so:

  * the schedule is computed by the C planner (rs_plan_build), op for op the reference's;
  * each target rank's op list becomes one table of strided copies (rs_program_build) that
    writes every piece straight into its final place in a freshly allocated target tensor;
  * one sm_100a kernel launch per rank executes the table, reading its own HBM and the HBM of
    the source ranks, mapped once per peer allocation through CUDA IPC, over NVLink.

There is no NCCL on the copy path and no CPU path: the device must be CUDA and the library
must load, or the call raises.
"""
from __future__ import annotations

import ctypes as C
import os
from collections import OrderedDict
from itertools import chain
from typing import Any, Callable, Dict, Iterable, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch
import torch.distributed as dist

from . import _lib as L

TPMeta = Tuple[int, int, int]  # slice_dim, tp_index, tp_deg


# ---------------------------------------------------------------------------------------------
# Layout objects. The reference's own TensorMeta / ParamLayout / TransferOp objects are accepted
# everywhere (they are read through .name/.dtype/.shape/.tp_meta and .layout only); these
# mirrors let a caller build layouts without the reference installed.
# ---------------------------------------------------------------------------------------------
class TensorMeta:
    """Mirror of Suika's TensorMeta (migration.py:29-131): dtype, FULL shape, tp_meta."""

    def __init__(self, tensor: Optional[torch.Tensor] = None, name: Optional[str] = None,
                 dtype: Optional[torch.dtype] = None, shape: Optional[Sequence[int]] = None,
                 tp_meta: Optional[TPMeta] = None):
        self.tp_meta = None
        if tensor is not None:
            self.dtype = tensor.dtype
            if hasattr(tensor, "slice_dim"):  # parallel linear: recover the full shape (migration.py:41-48)
                full = list(tensor.shape)
                full[tensor.slice_dim] *= tensor.tp_deg
                self.shape = torch.Size(full)
                self.tp_meta = (tensor.slice_dim, tensor.tp_index, tensor.tp_deg)
            else:
                self.shape = tensor.shape
        else:
            assert dtype is not None and shape is not None, "Either tensor or (dtype, shape) should be provided"
        self.name = name
        if dtype is not None:
            self.dtype = dtype
        if shape is not None:
            self.shape = torch.Size(shape)
        if tp_meta is not None:
            self.tp_meta = tuple(tp_meta)

    def is_tp(self) -> bool:
        return self.tp_meta is not None

    def slice_dim(self):
        return self.tp_meta[0] if self.is_tp() else None

    def tp_index(self) -> int:
        return self.tp_meta[1] if self.is_tp() else 0

    def tp_deg(self) -> int:
        return self.tp_meta[2] if self.is_tp() else 1

    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n // self.tp_deg()

    def volumn(self) -> int:
        return self.numel() * self.dtype.itemsize

    def actual_shape(self) -> torch.Size:
        if not self.is_tp():
            return torch.Size(self.shape)
        s = list(self.shape)
        s[self.slice_dim()] //= self.tp_deg()
        return torch.Size(s)

    def __repr__(self) -> str:
        return f"TensorMeta(name={self.name}, {self.dtype}, {self.shape}, {self.tp_meta})"


def get_named_parameters_and_persistent_buffers(model: torch.nn.Module):
    """Parameters then persistent buffers, as in migration.py:135-141."""
    state = model.state_dict()
    for name, p in chain(model.named_parameters(), model.named_buffers()):
        if name in state:
            yield name, p


def get_param_tensor_meta(model: torch.nn.Module) -> Dict[str, TensorMeta]:
    """name -> TensorMeta for a (TP-sliced) model, as in migration.py:147-151."""
    return {n: TensorMeta(tensor=p, name=n) for n, p in get_named_parameters_and_persistent_buffers(model)}


class ParamLayout:
    """Mirror of Suika's ParamLayout (migration.py:161-254): rank -> {name -> TensorMeta}."""

    def __init__(self):
        self.layout: Dict[int, Dict[str, Any]] = {}

    def gather(self, self_param_meta_or_module, world: Optional[dist.ProcessGroup] = None):
        if isinstance(self_param_meta_or_module, torch.nn.Module):
            meta = get_param_tensor_meta(self_param_meta_or_module)
        else:
            meta = self_param_meta_or_module
        metas = [None] * dist.get_world_size(world)
        dist.all_gather_object(metas, meta, group=world)
        for rank, m in enumerate(metas):
            self.layout[rank] = m

    def __repr__(self) -> str:
        return f"ParamLayout(\n  {self.layout}\n)"


class TransferOp:
    """Mirror of Suika's TransferOp (migration.py:257-283): one piece, source rank -> target rank."""

    def __init__(self, param_name: str, src_rank: int, dst_rank: int, src_meta, dst_meta=None):
        self.param_name = param_name
        self.src_rank = src_rank
        self.dst_rank = dst_rank
        self.src_meta = src_meta
        self.dst_meta = src_meta if dst_meta is None else dst_meta

    def __repr__(self) -> str:
        return f"TransferOp({self.param_name}, src={self.src_rank}, dst={self.dst_rank}, {self.src_meta.tp_meta}->{self.dst_meta.tp_meta})"


def is_ib_enabled() -> bool:
    """The reference's switch (Suika/utils.py:209-210); it changes the schedule (migration.py:340)."""
    return not (os.getenv("NCCL_IB_DISABLE", "False") in ["1", "true"])


def _itemsize(dtype) -> int:
    if isinstance(dtype, torch.dtype):
        return dtype.itemsize
    return np.dtype(dtype).itemsize


# ---------------------------------------------------------------------------------------------
# Plan / program wrappers over the C ABI.
# ---------------------------------------------------------------------------------------------
_ORDERS = {"reference": L.RS_ORDER_REFERENCE, "semantic": L.RS_ORDER_SEMANTIC}
_CHOICES = {"reference": L.RS_SRC_REFERENCE, "balanced": L.RS_SRC_BALANCED}

DST_SLOT_DTYPE = np.dtype([("name_id", "<i4"), ("subfield", "<i4"), ("ndim", "<i4"), ("reserved", "<i4"),
                           ("shape", "<i8", (L.RS_MAX_DIMS,)), ("nbytes", "<u8")])
SRC_SLOT_DTYPE = np.dtype([("src_rank", "<i4"), ("name_id", "<i4"), ("subfield", "<i4"), ("reserved", "<i4"),
                           ("nbytes", "<u8")])
META_SLOT_DTYPE = np.dtype([("name_id", "<i4"), ("subfield", "<i4"), ("src_rank", "<i4"), ("first_is_self", "<i4")])
OP_DTYPE = np.dtype([("name_id", "<i4"), ("src_rank", "<i4"), ("dst_rank", "<i4"),
                     ("src_slice_dim", "<i4"), ("src_tp_index", "<i4"), ("src_tp_deg", "<i4"),
                     ("dst_slice_dim", "<i4"), ("dst_tp_index", "<i4"), ("dst_tp_deg", "<i4"),
                     ("reserved", "<i4"), ("numel", "<i8")])
assert DST_SLOT_DTYPE.itemsize == C.sizeof(L.RsDstSlot)
assert SRC_SLOT_DTYPE.itemsize == C.sizeof(L.RsSrcSlot)
assert META_SLOT_DTYPE.itemsize == C.sizeof(L.RsMetaSlot)
assert OP_DTYPE.itemsize == C.sizeof(L.RsOp)


def _flatten_layout(layout: Dict[int, Dict[str, Any]], name_ids: Dict[str, int], names: List[str]):
    """ParamLayout.layout -> (rank array, per-rank TENSOR_META arrays) in dict order."""
    ranks, arrays = [], []
    for rank, metas in layout.items():
        arr = np.zeros(len(metas), dtype=L.TENSOR_META_DTYPE)
        for i, (name, m) in enumerate(metas.items()):
            nid = name_ids.get(name)
            if nid is None:
                nid = name_ids[name] = len(names)
                names.append(name)
            shape = tuple(int(s) for s in m.shape)
            if len(shape) > L.RS_MAX_DIMS:
                raise ValueError(f"{name}: more than {L.RS_MAX_DIMS} dims")
            tp = m.tp_meta
            rec = arr[i]
            rec["name_id"] = nid
            rec["ndim"] = len(shape)
            rec["shape"][: len(shape)] = shape
            rec["itemsize"] = _itemsize(m.dtype)
            if tp is None:
                rec["slice_dim"], rec["tp_index"], rec["tp_deg"] = L.RS_NO_SLICE, 0, 1
            else:
                rec["slice_dim"], rec["tp_index"], rec["tp_deg"] = int(tp[0]), int(tp[1]), int(tp[2])
        ranks.append(int(rank))
        arrays.append(arr)
    return ranks, arrays


def _rank_layouts(ranks, arrays):
    out = (L.RsRankLayout * max(1, len(ranks)))()
    for i, (r, a) in enumerate(zip(ranks, arrays)):
        out[i].rank = r
        out[i].n_tensors = len(a)
        out[i].tensors = C.cast(a.ctypes.data, C.POINTER(L.RsTensorMeta)) if len(a) else C.POINTER(L.RsTensorMeta)()
    return out


class Plan:
    """The transfer schedule of one reshard (schedule_param_transfer, migration.py:322-381).

    Built by the C planner from the source and target ParamLayouts. `order` selects the cat order
    of multi-piece targets ("reference" reproduces the reference's bytes, "semantic" writes pieces
    in slice order); `src_choice` selects among owners ("reference" = the reference's greedy rule).
    """

    def __init__(self, source_param_layout, target_param_layout, order: str = "reference",
                 src_choice: str = "reference", minimum_est_peers: Optional[int] = None):
        self._lib = L.load()
        self._h = None
        self.order = order
        self.spl, self.tpl = source_param_layout, target_param_layout
        self.names: List[str] = []
        self.name_ids: Dict[str, int] = {}
        s_ranks, s_arr = _flatten_layout(source_param_layout.layout, self.name_ids, self.names)
        d_ranks, d_arr = _flatten_layout(target_param_layout.layout, self.name_ids, self.names)
        self.src_ranks, self.dst_ranks = s_ranks, d_ranks
        opts = L.RsPlanOpts()
        opts.minimum_est_peers = (1 if is_ib_enabled() else 2) if minimum_est_peers is None else int(minimum_est_peers)
        opts.order = _ORDERS[order]
        opts.src_choice = _CHOICES[src_choice]
        h = C.c_void_p()
        L.check(self._lib.rs_plan_build(_rank_layouts(s_ranks, s_arr), len(s_ranks), _rank_layouts(d_ranks, d_arr),
                                        len(d_ranks), C.byref(opts), C.byref(h)))
        self._h = h
        n = C.c_int64()
        L.check(self._lib.rs_plan_num_ops(self._h, C.byref(n)))
        self.op_array = np.zeros(n.value, dtype=OP_DTYPE)
        L.check(self._lib.rs_plan_get_ops(self._h, C.cast(self.op_array.ctypes.data, C.POINTER(L.RsOp)), n.value))

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value:
            self._lib.rs_plan_free(self._h)
            self._h = None

    def __len__(self) -> int:
        return len(self.op_array)

    def transfer_ops(self) -> List[TransferOp]:
        """The schedule as TransferOp objects (for inspection and parity with the reference)."""
        out = []
        for o in self.op_array:
            name = self.names[o["name_id"]]
            src_m = self.spl.layout[int(o["src_rank"])][name]
            dst_full = self.tpl.layout[int(o["dst_rank"])][name]
            tp = None if o["dst_slice_dim"] == L.RS_NO_SLICE else (int(o["dst_slice_dim"]), int(o["dst_tp_index"]), int(o["dst_tp_deg"]))
            piece = TensorMeta(name=name, dtype=dst_full.dtype, shape=dst_full.shape, tp_meta=tp)
            out.append(TransferOp(name, int(o["src_rank"]), int(o["dst_rank"]), src_m, piece))
        return out

    def program(self, rank: int, subfields: Sequence[Tuple[int, bool]]) -> "Program":
        return Program(self, rank, subfields)

    def rank_bytes(self, subfield_itemsizes: Sequence[int]) -> Dict[str, Dict[int, int]]:
        """Per-rank ingress / egress / local bytes of all normal sub-fields (roofline accounting)."""
        per_elem = sum(subfield_itemsizes)
        ops = self.op_array
        nbytes = ops["numel"].astype(np.int64) * per_elem
        remote = ops["src_rank"] != ops["dst_rank"]
        res = {"ingress": {}, "egress": {}, "local": {}}
        for key, mask, col in (("ingress", remote, "dst_rank"), ("egress", remote, "src_rank"), ("local", ~remote, "dst_rank")):
            r = ops[col][mask]
            b = nbytes[mask]
            for rk in np.unique(r):
                res[key][int(rk)] = int(b[r == rk].sum())
        return res


class Program:
    """Everything one target rank executes (rs_program_build): slots, meta slots, copy segments."""

    def __init__(self, plan: Plan, rank: int, subfields: Sequence[Tuple[int, bool]]):
        self._lib = plan._lib
        self.plan = plan
        self.rank = rank
        self._h = None
        sf = (L.RsSubfield * max(1, len(subfields)))()
        for i, (isz, meta) in enumerate(subfields):
            sf[i].itemsize = int(isz)
            sf[i].is_meta = 1 if meta else 0
        h = C.c_void_p()
        L.check(self._lib.rs_program_build(plan._h, int(rank), sf, len(subfields), C.byref(h)))
        self._h = h
        cnt = L.RsProgramCounts()
        L.check(self._lib.rs_program_counts_get(self._h, C.byref(cnt)))
        self.remote_bytes = int(cnt.remote_bytes)
        self.local_bytes = int(cnt.local_bytes)
        self.dst_slots = np.zeros(cnt.n_dst_slots, dtype=DST_SLOT_DTYPE)
        self.src_slots = np.zeros(cnt.n_src_slots, dtype=SRC_SLOT_DTYPE)
        self.meta_slots = np.zeros(cnt.n_meta_slots, dtype=META_SLOT_DTYPE)
        self.segments = np.zeros(cnt.n_segments, dtype=L.SEGMENT_DTYPE)
        L.check(self._lib.rs_program_dst_slots(self._h, C.cast(self.dst_slots.ctypes.data, C.POINTER(L.RsDstSlot)), len(self.dst_slots)))
        L.check(self._lib.rs_program_src_slots(self._h, C.cast(self.src_slots.ctypes.data, C.POINTER(L.RsSrcSlot)), len(self.src_slots)))
        L.check(self._lib.rs_program_meta_slots(self._h, C.cast(self.meta_slots.ctypes.data, C.POINTER(L.RsMetaSlot)), len(self.meta_slots)))
        L.check(self._lib.rs_program_segments(self._h, self.segments.ctypes.data, len(self.segments)))

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value:
            self._lib.rs_program_free(self._h)
            self._h = None

    def resolve(self, src_dev: np.ndarray, src_ext: np.ndarray, dst_dev: np.ndarray, dst_ext: np.ndarray) -> np.ndarray:
        """Bind slots to addresses; returns the COPY_DESC table (bounds-checked in C)."""
        out = np.zeros(len(self.segments), dtype=L.COPY_DESC_DTYPE)
        arrs = [np.ascontiguousarray(a, dtype=np.uint64) for a in (src_dev, src_ext, dst_dev, dst_ext)]
        L.check(self._lib.rs_program_resolve(self._h, *[a.ctypes.data for a in arrs], out.ctypes.data, len(out)))
        return out


def launch_copies(descs: np.ndarray, device: torch.device, stream: Optional[torch.cuda.Stream] = None) -> L.RsLaunchInfo:
    """Run a COPY_DESC table with one sm_100a kernel launch on `stream` (asynchronous)."""
    lib = L.load()
    info = L.RsLaunchInfo()
    n = len(descs)
    if n == 0:
        return info
    descs = np.ascontiguousarray(descs, dtype=L.COPY_DESC_DTYPE)
    ws_bytes = C.c_uint64()
    L.check(lib.rs_copy_workspace_bytes(n, C.byref(ws_bytes)))
    ws = torch.empty(int(ws_bytes.value), dtype=torch.uint8, device=device)
    if stream is None:
        stream = torch.cuda.current_stream(device)
    # The workspace is freed into the stream-ordered caching allocator after the launch, so it is
    # reused only by work queued behind this kernel on the same stream.
    L.check(lib.rs_copy_launch(descs.ctypes.data, n, ws.data_ptr(), ws.numel(), C.c_void_p(stream.cuda_stream), C.byref(info)))
    return info

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
            assert dtype is not None and shape is not None, "a TensorMeta needs a tensor, or both a dtype and a shape"
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

    def scale_to_tp(self, target_tp_deg: int) -> List["TensorMeta"]:
        """The pieces of this shard at a finer TP degree (migration.py:103-118); itself otherwise."""
        if self.is_tp() and target_tp_deg > self.tp_deg():
            d, i, g = self.tp_meta
            k = target_tp_deg // g
            return [TensorMeta(name=self.name, dtype=self.dtype, shape=self.shape, tp_meta=(d, k * i + j, target_tp_deg))
                    for j in range(k)]
        return [self]

    def __eq__(self, other: Any) -> bool:
        """migration.py:120-124: same TP-ness and slice dim, dtype and full shape."""
        if not isinstance(other, TensorMeta):
            return False
        return (self.is_tp() == other.is_tp() and self.slice_dim() == other.slice_dim()
                and self.dtype == other.dtype and torch.Size(self.shape) == torch.Size(other.shape))

    __hash__ = None  # like the reference's class, which defines __eq__ only

    def __repr__(self) -> str:
        return f"<TensorMeta {self.name}: {self.dtype} full shape {tuple(self.shape)} tp_meta {self.tp_meta}>"

    __str__ = __repr__


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

    def is_owned(self, rank: int, param) -> bool:
        """migration.py:195-205: the rank holds the tensor (by name), or a shard that owns the
        given piece (by TensorMeta)."""
        if isinstance(param, str):
            return param in self.layout[rank]
        name = param.name
        return name in self.layout[rank] and self.is_tensor_tp_owned(self.layout[rank][name], param)

    def owners(self, param) -> List[int]:
        """migration.py:207-208."""
        return [rank for rank in self.layout if self.is_owned(rank, param)]

    @staticmethod
    def is_tensor_tp_overlap(meta1, meta2) -> bool:
        """migration.py:220-244 (the planner's C++ restates the same test)."""
        a = meta1.tp_meta if hasattr(meta1, "tp_meta") else meta1
        b = meta2.tp_meta if hasattr(meta2, "tp_meta") else meta2
        if a is None or b is None:
            return True
        assert a[0] == b[0], f"slice dim mismatch {a[0]} vs {b[0]}"
        (_, i1, g1), (_, i2, g2) = a, b
        if g1 > g2:
            i1, i2, g1, g2 = i2, i1, g2, g1
        return i2 // (g2 // g1) == i1

    @staticmethod
    def is_tensor_tp_owned(meta_src, meta_tgt) -> bool:
        """migration.py:246-254."""
        a = meta_src.tp_meta if hasattr(meta_src, "tp_meta") else meta_src
        b = meta_tgt.tp_meta if hasattr(meta_tgt, "tp_meta") else meta_tgt
        da = a[2] if a is not None else 1
        db = b[2] if b is not None else 1
        return da <= db and ParamLayout.is_tensor_tp_overlap(a, b)

    def __repr__(self) -> str:
        return f"ParamLayout(\n  {self.layout}\n)"

    __str__ = __repr__


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


def _flatten_layout(layout: Dict[int, Dict[str, Any]], name_ids: Dict[str, int], names: List[str],
                    rules: Optional[Dict[str, Any]] = None):
    """ParamLayout.layout -> (rank array, per-rank TENSOR_META arrays) in dict order. Slice rules
    (a `tp_rule` attribute on a meta: [(offset, size, units), ...]) are collected into `rules`."""
    ranks, arrays = [], []
    pad = (0,) * L.RS_MAX_DIMS
    itemsize_of: Dict[Any, int] = {}
    for rank, metas in layout.items():
        recs = []
        for name, m in metas.items():
            nid = name_ids.get(name)
            if nid is None:
                nid = name_ids[name] = len(names)
                names.append(name)
            rule = getattr(m, "tp_rule", None)
            if rule is not None and rules is not None:
                rule = tuple(tuple(int(x) for x in g) for g in rule)
                if rules.setdefault(name, rule) != rule:
                    raise ValueError(f"{name}: different slice rules in the source and target layouts")
            shape = tuple(int(x) for x in m.shape)
            if len(shape) > L.RS_MAX_DIMS:
                raise ValueError(f"{name}: more than {L.RS_MAX_DIMS} dims")
            isz = itemsize_of.get(m.dtype)
            if isz is None:
                isz = itemsize_of[m.dtype] = _itemsize(m.dtype)
            tp = m.tp_meta
            if tp is None:
                recs.append((nid, len(shape), shape + pad[len(shape):], isz, L.RS_NO_SLICE, 0, 1))
            else:
                recs.append((nid, len(shape), shape + pad[len(shape):], isz, int(tp[0]), int(tp[1]), int(tp[2])))
        ranks.append(int(rank))
        arrays.append(np.array(recs, dtype=L.TENSOR_META_DTYPE) if recs else np.zeros(0, dtype=L.TENSOR_META_DTYPE))
    return ranks, arrays


def _flatten_any(param_layout, name_ids: Dict[str, int], names: List[str], rules: Optional[Dict[str, Any]] = None):
    """A layout's records for the planner: a CompactLayout (suika_b200.metadata) hands over its
    records as they are; a ParamLayout's objects are read one by one."""
    if hasattr(param_layout, "flatten"):
        return param_layout.flatten(name_ids, names, rules)
    return _flatten_layout(param_layout.layout, name_ids, names, rules)


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
                 src_choice: str = "reference", minimum_est_peers: Optional[int] = None, mode: str = "auto"):
        self._lib = L.load()
        self._h = None
        self.spl, self.tpl = source_param_layout, target_param_layout
        self.names: List[str] = []
        self.name_ids: Dict[str, int] = {}
        rules: Dict[str, Any] = {}
        s_ranks, s_arr = _flatten_any(source_param_layout, self.name_ids, self.names, rules)
        d_ranks, d_arr = _flatten_any(target_param_layout, self.name_ids, self.names, rules)
        self.src_ranks, self.dst_ranks = s_ranks, d_ranks
        # "reference": the reference's schedule and cat order (chunk layouts only). "interval": slice
        # intersection, slice order, balanced replicas (any slice rules). "auto": interval iff rules.
        self.mode = ("interval" if rules else "reference") if mode == "auto" else mode
        self.order = order if self.mode == "reference" else "semantic"
        opts = L.RsPlanOpts()
        opts.minimum_est_peers = (1 if is_ib_enabled() else 2) if minimum_est_peers is None else int(minimum_est_peers)
        opts.order = _ORDERS[self.order]
        opts.src_choice = _CHOICES[src_choice]
        h = C.c_void_p()
        if self.mode == "reference":
            if rules:
                raise ValueError("slice rules need mode='interval' (the reference only cuts contiguous chunks)")
            L.check(self._lib.rs_plan_build(_rank_layouts(s_ranks, s_arr), len(s_ranks), _rank_layouts(d_ranks, d_arr),
                                            len(d_ranks), C.byref(opts), C.byref(h)))
        else:
            rr = (L.RsSliceRule * max(1, len(rules)))()
            for k, (name, groups) in enumerate(rules.items()):
                if len(groups) > L.RS_MAX_GROUPS:
                    raise ValueError(f"{name}: more than {L.RS_MAX_GROUPS} slice groups")
                rr[k].name_id = self.name_ids[name]
                rr[k].n_groups = len(groups)
                for g, (off, size, units) in enumerate(groups):
                    rr[k].groups[g].offset, rr[k].groups[g].size, rr[k].groups[g].units = off, size, units
            L.check(self._lib.rs_plan_build_rules(_rank_layouts(s_ranks, s_arr), len(s_ranks), _rank_layouts(d_ranks, d_arr),
                                                  len(d_ranks), rr, len(rules), C.byref(opts), C.byref(h)))
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


class PreparedCopies:
    """A copy table staged on the device once (rs_copy_stage) and launched any number of times
    (rs_copy_run), each launch one sm_100a kernel. The addresses in the table must stay valid."""

    def __init__(self, descs: np.ndarray, device: torch.device, stream: Optional[torch.cuda.Stream] = None):
        self._lib = L.load()
        self.device = device
        self.info = L.RsLaunchInfo()
        descs = np.ascontiguousarray(descs, dtype=L.COPY_DESC_DTYPE)
        ws_bytes = C.c_uint64()
        L.check(self._lib.rs_copy_workspace_bytes(len(descs), C.byref(ws_bytes)))
        self.workspace = torch.empty(max(int(ws_bytes.value), 256), dtype=torch.uint8, device=device)
        stream = self._stream(stream)
        L.check(self._lib.rs_copy_stage(descs.ctypes.data, len(descs), self.workspace.data_ptr(), self.workspace.numel(),
                                        C.c_void_p(stream.cuda_stream), C.byref(self.info)))

    def _stream(self, stream):
        current = torch.cuda.current_stream(self.device)
        if stream is None:
            return current
        if stream != current:
            stream.wait_stream(current)  # sources, targets and staging were produced on the current stream
            self.workspace.record_stream(stream)
        return stream

    def launch(self, stream: Optional[torch.cuda.Stream] = None) -> L.RsLaunchInfo:
        stream = self._stream(stream)
        L.check(self._lib.rs_copy_run(self.workspace.data_ptr(), C.byref(self.info), C.c_void_p(stream.cuda_stream)))
        return self.info

    def status(self, stream: Optional[torch.cuda.Stream] = None) -> int:
        """Status bits of the launches so far (synchronises the stream); 0 means no error."""
        stream = stream or torch.cuda.current_stream(self.device)
        v = C.c_uint32()
        L.check(self._lib.rs_copy_status(self.workspace.data_ptr(), C.byref(self.info), C.c_void_p(stream.cuda_stream), C.byref(v)))
        return int(v.value)

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        st = self.status(stream)
        if st:
            raise L.ReshardError(L.RS_ERR_CUDA, f"copy kernel reported status {st:#x} (a bounded wait ran out; targets incomplete)")


def launch_copies(descs: np.ndarray, device: torch.device, stream: Optional[torch.cuda.Stream] = None) -> L.RsLaunchInfo:
    """Stage a COPY_DESC table and run it with one sm_100a kernel launch on `stream` (asynchronous).
    The workspace returns to the stream-ordered caching allocator afterwards, so it is reused only
    by work queued behind this kernel."""
    if len(descs) == 0:
        return L.RsLaunchInfo()
    p = PreparedCopies(descs, device, stream)
    return p.launch(stream)


# ---------------------------------------------------------------------------------------------
# Shared execution helpers.
# ---------------------------------------------------------------------------------------------
def _is_meta_field(field_type) -> bool:
    """execute_param_transfer's is_meta_tensor (migration.py:423-424)."""
    return not (isinstance(field_type, str) and field_type == "normal")


class _NullProf:
    def start(self, *a, **k):
        pass

    def stop(self, *a, **k):
        pass


def _sub_dtypes(expected_sub_fields, states: Iterable[Dict[str, Dict[str, torch.Tensor]]]) -> Dict[str, torch.dtype]:
    """dtype of every normal sub-field, read from the first source entry that has it. The
    reference allocates received pieces in the layout dtype (migration.py:285-287), which only
    works when every sub-field has the param's dtype; here each sub-field keeps its own dtype."""
    out: Dict[str, torch.dtype] = {}
    want = [s for s, ft in expected_sub_fields if not _is_meta_field(ft)]
    for st in states:
        for ent in st.values():
            for s in want:
                if s not in out and s in ent:
                    out[s] = ent[s].dtype
            if len(out) == len(want):
                return out
    return out


def _program_spec(expected_sub_fields, dtypes: Dict[str, torch.dtype]):
    spec = []
    for s, ft in expected_sub_fields:
        if _is_meta_field(ft):
            spec.append((ft.dtype.itemsize, True))
        else:
            if s not in dtypes:
                raise AssertionError(f"expected_sub_fields mismatch: no source tensor carries sub-field {s}")
            spec.append((dtypes[s].itemsize, False))
    return spec


def _name_order(plan: Plan, rank: int) -> List[int]:
    """Target tensor order of a rank: first op per name (target_state_dict creation, migration.py:431-433)."""
    ops = plan.op_array
    ids = ops["name_id"][ops["dst_rank"] == rank]
    if len(ids) == 0:
        return []
    _, first = np.unique(ids, return_index=True)
    return [int(x) for x in ids[np.sort(first)]]


def _check_source(t: torch.Tensor, name: str, sub: str, device: torch.device, dtype: torch.dtype) -> torch.Tensor:
    if t.device != device:
        raise RuntimeError(f"source {name}[{sub}] is on {t.device}, expected {device}")
    if t.dtype.itemsize != dtype.itemsize:
        raise AssertionError(f"source {name}[{sub}] has dtype {t.dtype}, sub-field dtype is {dtype}")
    return t if t.is_contiguous() else t.contiguous()


class _MetaStage:
    """Singleton sub-fields (e.g. Adam's step), written into their own target tensors by entries
    of the same copy table: values already on the target device are copied device to device;
    host values are gathered, uploaded once, and copied from the staging buffer."""

    def __init__(self, device: torch.device):
        self.device = device
        self.values: List[bytes] = []
        self.targets: List[torch.Tensor] = []
        self.direct: List[Tuple[int, torch.Tensor, int]] = []  # (source address, target, bytes)
        self._keep: List[torch.Tensor] = []

    def add(self, value: torch.Tensor, out: torch.Tensor) -> None:
        v = value.detach().reshape(-1)
        if v.numel() != 1 or v.element_size() != out.element_size():
            raise AssertionError(f"singleton sub-field of {v.numel()} x {v.dtype} cannot fill {out.dtype}")
        if v.device == out.device:
            v = v.contiguous()
            self._keep.append(v)
            self.direct.append((v.data_ptr(), out, v.element_size()))
            return
        self.values.append(v.cpu().view(torch.uint8).numpy().tobytes())
        self.targets.append(out)

    def descs(self) -> Tuple[np.ndarray, Optional[List[torch.Tensor]]]:
        """The copy entries and the buffers they read, which must outlive the launches."""
        d = np.zeros(len(self.targets) + len(self.direct), dtype=L.COPY_DESC_DTYPE)
        for i, (src, t, n) in enumerate(self.direct):
            d[i] = (src, t.data_ptr(), 1, n, n, n, 0)
        if not self.targets:
            return d, (list(self._keep) if self._keep else None)
        sizes = [len(v) for v in self.values]
        offs = np.cumsum([0] + [(s + 15) // 16 * 16 for s in sizes])
        host = np.zeros(int(offs[-1]), dtype=np.uint8)
        for o, v in zip(offs, self.values):
            host[o:o + len(v)] = np.frombuffer(v, dtype=np.uint8)
        stage = torch.from_numpy(host).to(self.device)
        base = stage.data_ptr()
        k = len(self.direct)
        for i, (o, s, t) in enumerate(zip(offs, sizes, self.targets)):
            d[k + i] = (base + int(o), t.data_ptr(), 1, s, s, s, 0)
        self._keep.append(stage)
        return d, list(self._keep)


def _meta_target(value: torch.Tensor, first_is_self: bool, field_type, device: torch.device) -> torch.Tensor:
    """Shape/dtype the reference gives a singleton target: the source tensor's own when the first
    piece is a self transfer (migration.py:446), [1] in the field's dtype when received (:486-487)."""
    if first_is_self:
        return torch.empty(value.shape, dtype=value.dtype, device=device)
    return torch.empty((1,), dtype=field_type.dtype, device=device)


# ---------------------------------------------------------------------------------------------
# All ranks of a reshard on one device.
# ---------------------------------------------------------------------------------------------
def reshard_local(source_param_layout, target_param_layout, source_state_dicts: Dict[int, Dict[str, Dict[str, torch.Tensor]]],
                  expected_sub_fields, device=None, views: bool = False, order: str = "reference",
                  src_choice: str = "reference", minimum_est_peers: Optional[int] = None, plan: Optional[Plan] = None,
                  stream: Optional[torch.cuda.Stream] = None, return_info: bool = False):
    """Reshard every rank's state on one device: {src rank: state} -> {dst rank: state}.

    The target of each rank equals what execute_param_transfer returns on that rank. With
    views=True a target that is one contiguous range of one source tensor (a dim-0 TP slice or a
    replicated tensor) is returned as a view of it instead of a copy, so only row-strided pieces
    move (the "TP1 -> TP2 views" relayout); views=False copies everything like the reference.
    Asynchronous on `stream`; synchronise before reading the targets.
    """
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if device.type != "cuda":
        raise RuntimeError("suika_b200.reshard_local runs on a CUDA device only")
    plan = plan or Plan(source_param_layout, target_param_layout, order=order, src_choice=src_choice,
                        minimum_est_peers=minimum_est_peers)
    dtypes = _sub_dtypes(expected_sub_fields, source_state_dicts.values())
    spec = _program_spec(expected_sub_fields, dtypes)
    subs = [s for s, _ in expected_sub_fields]
    meta = _MetaStage(device)
    tables = []
    out: Dict[int, Dict[str, Dict[str, torch.Tensor]]] = {}
    for rank, metas in target_param_layout.layout.items():
        if not metas:
            continue
        prog = plan.program(rank, spec)
        srcs = []
        for ss in prog.src_slots:
            name, sub = plan.names[ss["name_id"]], subs[ss["subfield"]]
            srcs.append(_check_source(source_state_dicts[int(ss["src_rank"])][name][sub], name, sub, device, dtypes[sub]))
        seg_count = np.bincount(prog.segments["dst_slot"], minlength=len(prog.dst_slots)) if len(prog.segments) else np.zeros(len(prog.dst_slots), int)
        first_seg = {}
        for i, sg in enumerate(prog.segments):
            first_seg.setdefault(int(sg["dst_slot"]), i)
        dst_t, keep = [], np.ones(len(prog.segments), dtype=bool)
        for k, ds in enumerate(prog.dst_slots):
            sub = subs[ds["subfield"]]
            shape = tuple(int(x) for x in ds["shape"][: ds["ndim"]])
            t = None
            if views and seg_count[k] == 1:
                sg = prog.segments[first_seg[k]]
                if sg["rows"] == 1 and sg["row_bytes"] == ds["nbytes"]:
                    src = srcs[sg["src_slot"]]
                    e0 = int(sg["src_offset"]) // src.element_size()
                    t = src.reshape(-1)[e0:e0 + int(ds["nbytes"]) // src.element_size()].view(shape)
                    keep[first_seg[k]] = False
            if t is None:
                t = torch.empty(shape, dtype=dtypes[sub], device=device)
            dst_t.append(t)
        if len(prog.segments):
            d = prog.resolve(np.array([t.data_ptr() for t in srcs], np.uint64),
                             np.array([t.numel() * t.element_size() for t in srcs], np.uint64),
                             np.array([t.data_ptr() for t in dst_t], np.uint64),
                             np.array([t.numel() * t.element_size() for t in dst_t], np.uint64))
            d["flags"] &= ~np.uint64(L.RS_COPY_REMOTE)  # every rank is on this device: nothing crosses NVLink
            tables.append(d[keep])
        ent: Dict[str, Dict[str, torch.Tensor]] = {}
        for ds, t in zip(prog.dst_slots, dst_t):
            ent.setdefault(plan.names[ds["name_id"]], {})[subs[ds["subfield"]]] = t
        for ms in prog.meta_slots:
            name, sub = plan.names[ms["name_id"]], subs[ms["subfield"]]
            v = source_state_dicts[int(ms["src_rank"])][name][sub]
            t = _meta_target(v, bool(ms["first_is_self"]), expected_sub_fields[ms["subfield"]][1], device)
            meta.add(v, t)
            ent.setdefault(name, {})[sub] = t
        out[rank] = {plan.names[n]: {s: ent[plan.names[n]][s] for s in subs if s in ent[plan.names[n]]}
                     for n in _name_order(plan, rank)}
    md, stage = meta.descs()
    table = np.concatenate(tables + [md]) if (tables or len(md)) else np.zeros(0, dtype=L.COPY_DESC_DTYPE)
    prepared = PreparedCopies(table, device, stream) if len(table) else None
    info = prepared.launch(stream) if prepared is not None else L.RsLaunchInfo()
    if stage is not None and stream is not None:
        for t in stage:
            t.record_stream(stream)
    if return_info:
        return out, info, prepared
    return out


# ---------------------------------------------------------------------------------------------
# One rank per process: the drop-in for schedule_and_execute_param_transfer.
# ---------------------------------------------------------------------------------------------
class _PeerMaps:
    """Peer allocations mapped into this process for one call; closed together at the end."""

    def __init__(self):
        self._lib = L.load()
        self.bases: Dict[Tuple[int, int], int] = {}

    def base(self, peer: int, alloc: int, handle_bytes: bytes) -> int:
        key = (peer, alloc)
        if key not in self.bases:
            h = L.RsPeerHandle.from_buffer_copy(handle_bytes)
            p = C.c_void_p()
            L.check(self._lib.rs_peer_open(C.byref(h), C.byref(p)))
            self.bases[key] = int(p.value)
        return self.bases[key]

    def close(self) -> None:
        err = None
        for p in self.bases.values():
            rc = self._lib.rs_peer_close(C.c_void_p(p))
            if rc != L.RS_OK and err is None:
                err = rc
        self.bases.clear()
        if err is not None:
            L.check(err)


def _export(tensors: List[torch.Tensor]):
    """Export the allocations holding `tensors`: ([handle bytes per allocation], [(alloc, offset)])."""
    lib = L.load()
    handles: List[bytes] = []
    index: Dict[int, int] = {}
    where = []
    for t in tensors:
        h = L.RsPeerHandle()
        off = C.c_uint64()
        L.check(lib.rs_peer_export(C.c_void_p(t.data_ptr()), C.byref(h), C.byref(off)))
        if h.alloc_base not in index:
            index[h.alloc_base] = len(handles)
            handles.append(bytes(h))
        where.append((index[h.alloc_base], int(off.value)))
    return handles, where


def plan_phases(plan: "Plan", phased: bool = True) -> Tuple[Dict[Tuple[int, int], int], int]:
    """Phase of every remote (source, target) pair of a plan (transfer_phases), and the count."""
    if not phased:
        return {}, 1
    ops = plan.op_array
    m = ops["src_rank"] != ops["dst_rank"]
    pairs: Dict[Tuple[int, int], int] = {}
    for s, t, n in zip(ops["src_rank"][m], ops["dst_rank"][m], ops["numel"][m]):
        pairs[(int(s), int(t))] = pairs.get((int(s), int(t)), 0) + int(n)
    col = transfer_phases(pairs)
    return col, (max(col.values()) + 1) if col else 1


class _Phased:
    """Per-phase staged tables of one rank, run with a barrier between phases."""

    def _stage_phases(self, table: np.ndarray, peer_of_entry: np.ndarray, as_source: bool, phased: bool):
        self.phase_of_pair, self.n_phases = plan_phases(self.plan, phased)
        tables = _phase_tables(table, peer_of_entry, self.rank, self.phase_of_pair, self.n_phases, as_source)
        self.prepared_phases = [PreparedCopies(t, self.device) if len(t) else None for t in tables]
        self.prepared = self.prepared_phases[0] if self.n_phases == 1 else None

    def launch(self, stream: Optional[torch.cuda.Stream] = None) -> L.RsLaunchInfo:
        """Queue every phase of this rank back to back (asynchronous); no cross-rank pacing."""
        if getattr(self, "_paced", False):
            raise RuntimeError("a fan-out transfer reads in stage 2 what stage 1 wrote: use run()")
        info = L.RsLaunchInfo()
        for p in getattr(self, "prepared_phases", []):
            if p is not None:
                info = p.launch(stream)
        return info

    def run(self) -> None:
        """Run the phases in step with the other ranks: phase k+1 starts on every rank after every
        rank has finished phase k (host barrier), so each GPU talks to one peer per direction."""
        phases = getattr(self, "prepared_phases", [])
        for k in range(getattr(self, "n_phases", 1)):
            if k:
                torch.cuda.current_stream(self.device).synchronize()
                dist.barrier(group=self.world)
            if k < len(phases) and phases[k] is not None:
                phases[k].launch()

    def _status(self) -> int:
        st = 0
        for p in getattr(self, "prepared_phases", []):
            if p is not None:
                st |= p.status()
        return st


class RankTransfer(_Phased):
    """One rank's share of a reshard, split into prepare / launch / finish so that the data path
    (launch) can be run and timed on its own.

    prepare (constructor, collective over `world`): export the allocations of the source tensors
    other ranks read from this rank; exchange handles, offsets, sub-field dtypes and singleton
    values in one all_gather_object; map the peer allocations this rank reads (CUDA IPC); allocate
    the targets; bind the copy program to addresses (bounds-checked).
    launch: one kernel launch pulls every piece (peer HBM over NVLink, own HBM locally).
    finish (collective): a barrier after this rank's kernel has finished keeps every source alive
    until its last reader is done; then peer mappings are closed and source_state_dict is cleared
    (migration.py:527).
    """

    def __init__(self, plan: Plan, source_state_dict: Dict[str, Dict[str, torch.Tensor]], expected_sub_fields,
                 device: torch.device, world: Optional[dist.ProcessGroup] = None, log_func: Optional[Callable] = None,
                 phased: bool = True):
        self.plan, self.device, self.world = plan, device, world
        self.source_state_dict = source_state_dict
        self.log = log_func or (lambda m: None)
        self.rank = rank = dist.get_rank(world)
        ws = dist.get_world_size(world)
        subs = [s for s, _ in expected_sub_fields]
        sidx = {s: i for i, s in enumerate(subs)}
        ops = plan.op_array
        # 1. what peers read from this rank
        mask = (ops["src_rank"] == rank) & (ops["dst_rank"] != rank)
        served = [int(x) for x in np.unique(ops["name_id"][mask])]
        exp_tensors, exp_keys, meta_vals = [], [], {}
        for nid in served:
            name = plan.names[nid]
            if name not in source_state_dict:
                raise AssertionError(f"[{rank}]: param missing in source {name}")
            ent = source_state_dict[name]
            for s, ft in expected_sub_fields:
                if s not in ent:
                    raise AssertionError(f"expected_sub_fields mismatch: {name} has no {s}")
                v = ent[s]
                if _is_meta_field(ft):
                    meta_vals[(nid, sidx[s])] = (v.detach().reshape(-1).cpu().view(torch.uint8).numpy().tobytes(), str(v.dtype), tuple(v.shape))
                else:
                    if v.device != device:
                        raise RuntimeError(f"source {name}[{s}] is on {v.device}, expected {device}")
                    if not v.is_contiguous():
                        v = ent[s] = v.contiguous()
                    exp_tensors.append(v)
                    exp_keys.append((nid, sidx[s], v.numel() * v.element_size()))
        handles, where = _export(exp_tensors)
        my_dtypes = {s: str(d).replace("torch.", "") for s, d in _sub_dtypes(expected_sub_fields, [source_state_dict]).items()}
        torch.cuda.current_stream(device).synchronize()  # sources are complete before any peer reads them
        info = {"handles": handles, "tensors": {k[:2]: (a, o, k[2]) for k, (a, o) in zip(exp_keys, where)},
                "meta": meta_vals, "dtypes": my_dtypes}
        gathered: List[Any] = [None] * ws
        dist.all_gather_object(gathered, info, group=world)
        # 2. this rank's program, bound to local, peer and freshly allocated target addresses
        dtypes: Dict[str, torch.dtype] = {}
        for g in gathered:
            for s, d in g["dtypes"].items():
                dtypes.setdefault(s, getattr(torch, d))
        self.target: Dict[str, Dict[str, torch.Tensor]] = {}
        self.table = np.zeros(0, dtype=L.COPY_DESC_DTYPE)
        self.remote_bytes = self.local_bytes = 0
        self._stage = None
        self.prepared = None
        self.prepared_phases, self.n_phases = [], plan_phases(plan, phased)[1]
        self.peers = _PeerMaps()
        if not np.any(ops["dst_rank"] == rank):
            return
        try:
            spec = _program_spec(expected_sub_fields, dtypes)
            prog = plan.program(rank, spec)
            src_ptr = np.zeros(len(prog.src_slots), np.uint64)
            src_ext = np.zeros(len(prog.src_slots), np.uint64)
            for i, ss in enumerate(prog.src_slots):
                nid, sf, sr = int(ss["name_id"]), int(ss["subfield"]), int(ss["src_rank"])
                if sr == rank:
                    name = plan.names[nid]
                    if name not in source_state_dict:
                        raise AssertionError(f"[{rank}]: param missing in source {name}")
                    v = _check_source(source_state_dict[name][subs[sf]], name, subs[sf], device, dtypes[subs[sf]])
                    source_state_dict[name][subs[sf]] = v
                    src_ptr[i], src_ext[i] = v.data_ptr(), v.numel() * v.element_size()
                else:
                    a, o, nb = gathered[sr]["tensors"][(nid, sf)]
                    src_ptr[i] = self.peers.base(sr, a, gathered[sr]["handles"][a]) + o
                    src_ext[i] = nb
            dst_t = []
            for ds in prog.dst_slots:
                shape = tuple(int(x) for x in ds["shape"][: ds["ndim"]])
                dst_t.append(torch.empty(shape, dtype=dtypes[subs[ds["subfield"]]], device=device))
            table = prog.resolve(src_ptr, src_ext, np.array([x.data_ptr() for x in dst_t], np.uint64),
                                 np.array([x.numel() * x.element_size() for x in dst_t], np.uint64))
            ent: Dict[str, Dict[str, torch.Tensor]] = {}
            for ds, x in zip(prog.dst_slots, dst_t):
                ent.setdefault(plan.names[ds["name_id"]], {})[subs[ds["subfield"]]] = x
            meta = _MetaStage(device)
            for ms in prog.meta_slots:
                nid, sf, sr = int(ms["name_id"]), int(ms["subfield"]), int(ms["src_rank"])
                name, s = plan.names[nid], subs[sf]
                if sr == rank:
                    v = source_state_dict[name][s]
                else:
                    raw, dt, shape = gathered[sr]["meta"][(nid, sf)]
                    v = torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(getattr(torch, dt.replace("torch.", ""))).reshape(shape)
                x = _meta_target(v, bool(ms["first_is_self"]), expected_sub_fields[sf][1], device)
                meta.add(v, x)
                ent.setdefault(name, {})[s] = x
            md, self._stage = meta.descs()
            self.table = np.concatenate([table, md])
            peer = np.concatenate([prog.src_slots["src_rank"][prog.segments["src_slot"]].astype(np.int64),
                                   np.full(len(md), rank, np.int64)])
            self._stage_phases(self.table, peer, as_source=False, phased=phased)
            self.remote_bytes, self.local_bytes = prog.remote_bytes, prog.local_bytes
            self.target = {plan.names[n]: {s: ent[plan.names[n]][s] for s in subs if s in ent[plan.names[n]]}
                           for n in _name_order(plan, rank)}
        except BaseException:
            self.peers.close()
            raise

    def finish(self) -> Dict[str, Dict[str, torch.Tensor]]:
        """Wait for this rank's kernel, then for every rank (barrier); release peers and sources."""
        try:
            torch.cuda.current_stream(self.device).synchronize()
            st = self._status()
            dist.barrier(group=self.world)  # every reader of this rank's sources has finished
        finally:
            self.peers.close()
        if st:
            raise L.ReshardError(L.RS_ERR_CUDA, f"rank {self.rank}: copy kernel reported status {st:#x}; targets incomplete")
        self._stage = None
        self.prepared = None
        self.prepared_phases = []
        self.source_state_dict.clear()
        self.log(f"suika_b200: rank {self.rank} pulled {self.remote_bytes} B from peers and {self.local_bytes} B "
                 f"locally with {len(self.table)} copies")
        return self.target


def _arena_layout(dst_slots: np.ndarray):
    """256-byte aligned offsets of a rank's target slots inside one arena: (offsets, sizes, total)."""
    nb = dst_slots["nbytes"].astype(np.uint64)
    off = np.zeros(len(nb), np.uint64)
    if len(nb) > 1:
        off[1:] = np.cumsum((nb[:-1] + np.uint64(255)) // np.uint64(256) * np.uint64(256))
    total = int(off[-1] + nb[-1]) if len(nb) else 0
    return off, nb, total


def _push_table(prog: Program, rank: int, src_addr: Callable[[str, str], Tuple[int, int]], dst_base: int,
                dst_off: np.ndarray, dst_nb: np.ndarray, subs: Sequence[str]) -> np.ndarray:
    """COPY_DESC entries of `prog` (a target rank's program) whose source lives on `rank`, with
    targets at dst_base + dst_off[slot]; src_addr(name, sub) -> (address, bytes) of a local source."""
    src_ptr = np.zeros(len(prog.src_slots), np.uint64)
    src_ext = np.zeros(len(prog.src_slots), np.uint64)
    for i, ss in enumerate(prog.src_slots):
        if int(ss["src_rank"]) == rank:
            src_ptr[i], src_ext[i] = src_addr(prog.plan.names[int(ss["name_id"])], subs[int(ss["subfield"])])
    dst_ptr = np.asarray(dst_off, np.uint64) + np.uint64(dst_base)
    out = np.zeros(len(prog.segments), dtype=L.COPY_DESC_DTYPE)
    n = C.c_int64()
    arrs = [np.ascontiguousarray(a, dtype=np.uint64) for a in (src_ptr, src_ext, dst_ptr, dst_nb)]
    L.check(L.load().rs_program_resolve_from(prog._h, rank, *[a.ctypes.data for a in arrs], out.ctypes.data, len(out), C.byref(n)))
    return out[: n.value]


def _push_rank_tables(plan: Plan, rank: int, spec, subs: Sequence[str], src_addr: Callable[[str, str], Tuple[int, int]],
                      arena_base: Callable[[int], int], slot_off: Callable[[int], np.ndarray], slot_nb: Callable[[int], np.ndarray],
                      my_prog: Optional["Program"] = None, fanout=None):
    """What `rank` writes in a push reshard. Stage 1: the pieces it is the source of, for every
    target rank T (into arena_base(T) + slot_off(T)[slot]), minus the tensors T takes from a
    fan-out leader. Stage 2 (fan-out only): the assembled tensors it forwards as a leader.
    Returns (stage-1 table, target rank of each entry, {(follower, round): stage-2 table})."""
    from .fanout import forward_table, stage1_keep
    ops = plan.op_array
    tables, peers_of = [], []
    progs: Dict[int, Program] = {}

    def prog_of(t: int) -> "Program":
        if t == rank and my_prog is not None:
            return my_prog
        if t not in progs:
            progs[t] = plan.program(t, spec)
        return progs[t]

    for T in sorted(set(int(t) for t in ops["dst_rank"][ops["src_rank"] == rank])):
        prog = prog_of(T)
        d = _push_table(prog, rank, src_addr, arena_base(T), slot_off(T), slot_nb(T), subs)
        if fanout is not None and fanout.active:
            d = d[stage1_keep(prog, rank, fanout.forwarded_names(T))]
        tables.append(d)
        peers_of.append(np.full(len(d), T, np.int64))
    stage2: Dict[Tuple[int, int], np.ndarray] = {}
    if fanout is not None and fanout.active:
        for (F, rnd), names in fanout.children_of(rank).items():
            stage2[(F, rnd)] = forward_table(prog_of(rank), arena_base(rank), slot_off(rank), prog_of(F), arena_base(F),
                                             slot_off(F), slot_nb(F), names)
    table = np.concatenate(tables) if tables else np.zeros(0, dtype=L.COPY_DESC_DTYPE)
    peer = np.concatenate(peers_of) if peers_of else np.zeros(0, np.int64)
    return table, peer, stage2


class RankTransferPush(_Phased):
    """One rank's share of a reshard with targets written by their sources (same contract as
    RankTransfer: prepare / launch / finish, same targets byte for byte).

    prepare: one all_gather_object shares sub-field dtypes and singleton values; every target
    rank allocates its targets in ONE arena (returned tensors are views of it) and exports it;
    a second all_gather_object shares the arena handles and slot offsets; each rank maps the
    arenas of the ranks it sends to and binds a table of the pieces it is the source of (its own
    targets' pieces included), plus the singleton values of its own targets.
    launch: one kernel writes every piece this rank sources: local HBM reads, stores into peer
    HBM over NVLink (posted writes, no read requests on the reverse direction).
    finish: after this rank's kernel has finished, a barrier; past it every rank's pieces have
    landed, and the arena mappings are closed.
    fanout: a suika_b200.fanout.FanOut (plan_fanout of this plan, the same on every rank): stage
    1 sends a replicated tensor to its leader only, stage 2 has leaders forward it to the other
    replicas; run() paces the stages (launch() refuses).
    """

    def __init__(self, plan: Plan, source_state_dict: Dict[str, Dict[str, torch.Tensor]], expected_sub_fields,
                 device: torch.device, world: Optional[dist.ProcessGroup] = None, log_func: Optional[Callable] = None,
                 phased: bool = True, fanout=None):
        if fanout is not None and fanout.active and not phased:
            raise ValueError("fan-out runs in phases (stage 2 reads what stage 1 wrote)")
        self.plan, self.device, self.world = plan, device, world
        self.source_state_dict = source_state_dict
        self.log = log_func or (lambda m: None)
        self.rank = rank = dist.get_rank(world)
        ws = dist.get_world_size(world)
        subs = [s for s, _ in expected_sub_fields]
        sidx = {s: i for i, s in enumerate(subs)}
        ops = plan.op_array
        # 1. dtypes and the singleton values targets on other ranks take from this rank
        mask = (ops["src_rank"] == rank) & (ops["dst_rank"] != rank)
        meta_vals = {}
        for nid in np.unique(ops["name_id"][mask]):
            name = plan.names[int(nid)]
            if name not in source_state_dict:
                raise AssertionError(f"[{rank}]: param missing in source {name}")
            for s, ft in expected_sub_fields:
                if _is_meta_field(ft):
                    v = source_state_dict[name][s]
                    meta_vals[(int(nid), sidx[s])] = (v.detach().reshape(-1).cpu().view(torch.uint8).numpy().tobytes(), str(v.dtype), tuple(v.shape))
        my_dtypes = {s: str(d).replace("torch.", "") for s, d in _sub_dtypes(expected_sub_fields, [source_state_dict]).items()}
        torch.cuda.current_stream(device).synchronize()  # sources are complete before this rank's kernel reads them
        g1: List[Any] = [None] * ws
        dist.all_gather_object(g1, {"meta": meta_vals, "dtypes": my_dtypes}, group=world)
        dtypes: Dict[str, torch.dtype] = {}
        for g in g1:
            for s, d in g["dtypes"].items():
                dtypes.setdefault(s, getattr(torch, d))
        spec = _program_spec(expected_sub_fields, dtypes)
        # 2. this rank's targets, in one exported arena
        self.peers = _PeerMaps()
        self.target: Dict[str, Dict[str, torch.Tensor]] = {}
        self.remote_bytes = self.local_bytes = 0
        self.prepared = None
        self.prepared_phases, self.n_phases = [], plan_phases(plan, phased)[1]
        self._stage = None
        my_prog = plan.program(rank, spec) if np.any(ops["dst_rank"] == rank) else None
        arena_handle, arena_offset, slot_off, slot_nb = None, 0, np.zeros(0, np.uint64), np.zeros(0, np.uint64)
        dst_views = []
        if my_prog is not None and len(my_prog.dst_slots):
            slot_off, slot_nb, total = _arena_layout(my_prog.dst_slots)
            self.arena = torch.empty(max(total, 1), dtype=torch.uint8, device=device)
            for ds, o, nb in zip(my_prog.dst_slots, slot_off, slot_nb):
                shape = tuple(int(x) for x in ds["shape"][: ds["ndim"]])
                dt = dtypes[subs[ds["subfield"]]]
                dst_views.append(self.arena[int(o):int(o) + int(nb)].view(dt).view(shape))
            # the handle covers the whole allocation holding the arena; peers add the arena's offset
            hs, where = _export([self.arena])
            arena_handle, arena_offset = hs[0], where[0][1]
        g2: List[Any] = [None] * ws
        dist.all_gather_object(g2, {"arena": arena_handle, "arena_offset": arena_offset, "off": slot_off, "nb": slot_nb},
                               group=world)
        try:
            # 3. the pieces this rank sources, for every target rank (and, with fan-out, the
            # tensors it forwards as a leader)
            def src_addr(name, sub):
                if name not in source_state_dict:
                    raise AssertionError(f"[{rank}]: param missing in source {name}")
                v = _check_source(source_state_dict[name][sub], name, sub, device, dtypes[sub])
                source_state_dict[name][sub] = v
                return v.data_ptr(), v.numel() * v.element_size()

            def arena_base(T):
                return self.arena.data_ptr() if T == rank else self.peers.base(T, 0, g2[T]["arena"]) + g2[T]["arena_offset"]

            t1, peer1, stage2 = _push_rank_tables(plan, rank, spec, subs, src_addr, arena_base, lambda T: g2[T]["off"],
                                                  lambda T: g2[T]["nb"], my_prog, fanout)
            nb1 = (t1["rows"] * t1["row_bytes"]).astype(np.int64)
            self.local_bytes += int(nb1[peer1 == rank].sum())
            self.remote_bytes += int(nb1[peer1 != rank].sum()) + sum(int((d["rows"] * d["row_bytes"]).sum()) for d in stage2.values())
            tables, peers_of = [t1], [peer1]
            # 4. this rank's targets: dict in the reference's order, singleton values staged locally
            if my_prog is not None:
                ent: Dict[str, Dict[str, torch.Tensor]] = {}
                for ds, x in zip(my_prog.dst_slots, dst_views):
                    ent.setdefault(plan.names[ds["name_id"]], {})[subs[ds["subfield"]]] = x
                meta = _MetaStage(device)
                for ms in my_prog.meta_slots:
                    nid, sf, sr = int(ms["name_id"]), int(ms["subfield"]), int(ms["src_rank"])
                    name, s = plan.names[nid], subs[sf]
                    if sr == rank:
                        v = source_state_dict[name][s]
                    else:
                        raw, dt, shape = g1[sr]["meta"][(nid, sf)]
                        v = torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(getattr(torch, dt.replace("torch.", ""))).reshape(shape)
                    x = _meta_target(v, bool(ms["first_is_self"]), expected_sub_fields[sf][1], device)
                    meta.add(v, x)
                    ent.setdefault(name, {})[s] = x
                md, self._stage = meta.descs()
                tables.append(md)
                peers_of.append(np.full(len(md), rank, np.int64))
                self.target = {plan.names[n]: {s: ent[plan.names[n]][s] for s in subs if s in ent[plan.names[n]]}
                               for n in _name_order(plan, rank)}
            self.table = np.concatenate(tables) if tables else np.zeros(0, dtype=L.COPY_DESC_DTYPE)
            peer = np.concatenate(peers_of) if peers_of else np.zeros(0, np.int64)
            if fanout is not None and fanout.active:
                self._stage_fanout(self.table, peer, stage2, fanout)
            else:
                self._stage_phases(self.table, peer, as_source=True, phased=phased)
        except BaseException:
            self.peers.close()
            raise

    def _stage_fanout(self, table: np.ndarray, peer: np.ndarray, stage2: Dict[Tuple[int, int], np.ndarray], fanout) -> None:
        """Stage-1 phases (the plan's pairs without forwarded tensors), then stage-2 phases."""
        t1 = _phase_tables(table, peer, self.rank, fanout.phase1, fanout.n1, as_source=True)
        t2: List[List[np.ndarray]] = [[] for _ in range(fanout.n2)]
        for (F, rnd), d in stage2.items():
            t2[fanout.phase2[(self.rank, F, rnd)]].append(d)
        tables = t1 + [np.concatenate(x) if x else np.zeros(0, dtype=L.COPY_DESC_DTYPE) for x in t2]
        self.phase_of_pair, self.n_phases = dict(fanout.phase1), fanout.n_phases
        self.prepared_phases = [PreparedCopies(t, self.device) if len(t) else None for t in tables]
        self.prepared = None
        self._paced = True

    def finish(self) -> Dict[str, Dict[str, torch.Tensor]]:
        """Wait for this rank's kernel, then for every rank (barrier): all pieces have landed."""
        try:
            torch.cuda.current_stream(self.device).synchronize()
            st = self._status()
            dist.barrier(group=self.world)
        finally:
            self.peers.close()
        if st:
            raise L.ReshardError(L.RS_ERR_CUDA, f"rank {self.rank}: copy kernel reported status {st:#x}; targets incomplete")
        self._stage = None
        self.prepared = None
        self.prepared_phases = []
        self.source_state_dict.clear()
        self.log(f"suika_b200: rank {self.rank} wrote {self.remote_bytes} B to peers and {self.local_bytes} B locally")
        return self.target


def execute_plan_distributed(plan: Plan, source_state_dict: Dict[str, Dict[str, torch.Tensor]], expected_sub_fields,
                             device: torch.device, world: Optional[dist.ProcessGroup] = None,
                             log_func: Optional[Callable] = None, timers: Optional[dict] = None, direction: str = "pull",
                             phased: bool = True, fanout=False):
    """Run one rank's share of a reshard (execute_param_transfer, migration.py:397-556): prepare,
    one kernel launch, finish. Collective over `world`. direction="pull": each target rank reads
    its pieces (RankTransfer); "push": each source rank writes them (RankTransferPush).
    fanout (push only): False, True or "auto", as suika_b200.fanout.plan_fanout takes it."""
    if direction == "push":
        fo = None
        if fanout:
            from .fanout import plan_fanout
            fo = plan_fanout(plan, 1, mode=fanout)
        rt = RankTransferPush(plan, source_state_dict, expected_sub_fields, device, world, log_func, phased=phased, fanout=fo)
    elif direction == "pull":
        if fanout:
            raise ValueError("fan-out is implemented for the push direction")
        rt = RankTransfer(plan, source_state_dict, expected_sub_fields, device, world, log_func, phased=phased)
    else:
        raise ValueError(f"direction {direction!r}: 'pull' or 'push'")
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    rt.run()
    ev1.record()
    target = rt.finish()
    if timers is not None:
        timers["kernel_ms"] = ev0.elapsed_time(ev1)
        timers["phases"] = rt.n_phases
        timers["remote_bytes"], timers["local_bytes"] = rt.remote_bytes, rt.local_bytes
    return target


def self_pieces(plan: Plan, source_state_dict: Dict[str, Dict[str, torch.Tensor]], expected_sub_fields, rank: int,
                device: torch.device) -> List[torch.Tensor]:
    """The tensors the reference's forcefully_free releases on `rank` (migration.py:539-541): a
    self-transferred piece whose source TP degree is at least the target piece's is the source
    tensor itself (get_send_tensor, migration.py:297-300), and a singleton's piece is the source
    tensor when it already lives on `device` (tensor.to(device), :445-446)."""
    ops = plan.op_array
    m = (ops["src_rank"] == rank) & (ops["dst_rank"] == rank) & (ops["src_tp_deg"] >= ops["dst_tp_deg"])
    out: List[torch.Tensor] = []
    seen = set()
    for nid in ops["name_id"][m]:
        name = plan.names[int(nid)]
        if name in seen or name not in source_state_dict:
            continue
        seen.add(name)
        for sub, ft in expected_sub_fields:
            t = source_state_dict[name].get(sub)
            if not isinstance(t, torch.Tensor):
                continue
            if _is_meta_field(ft) and t.device != device:
                continue  # the reference frees its device copy, not the host source
            out.append(t)
    return out


def _forcefully_free(tensors: List[torch.Tensor]) -> None:
    """forcefully_free_tensor (Suika/utils.py:255-260) on each tensor."""
    for t in tensors:
        st = t.untyped_storage()
        if st.resizable():
            st.resize_(0)
        else:
            t.data = torch.empty(0, device="meta")


def _fanout_setting(value: str):
    """$SUIKA_RESHARD_FANOUT: "0" / "" (off), "auto", "1" (wherever exact)."""
    v = value.strip().lower()
    table = {"0": False, "": False, "off": False, "auto": "auto", "1": True, "on": True}
    if v not in table:
        raise ValueError(f"SUIKA_RESHARD_FANOUT={value!r}: use 0, auto or 1")
    return table[v]


def schedule_and_execute_param_transfer(source_param_layout, target_param_layout, source_state_dict: Dict[str, Dict[str, torch.Tensor]],
                                        other_context_dict: Dict[str, Any], device, world: Optional[dist.ProcessGroup],
                                        prof=None, forcefully_free: bool = False, log_func=None, direction: Optional[str] = None):
    """Drop-in for Suika's schedule_and_execute_param_transfer (migration.py:558-598).

    Same arguments, same return value ({name: {sub_field: tensor}} of this rank, tensors new and
    contiguous), same side effect (source_state_dict cleared). The targets are byte-identical to
    the reference's, including its order of concatenated pieces.

    forcefully_free: as in the reference (migration.py:539-541), the storages of this rank's
    self-sent pieces that are whole source tensors are released after the transfer (the shrink
    path of migration_save passes True, so the old state is gone before the hand-off).

    direction (default: $SUIKA_RESHARD_DIRECTION, else "push"): "push" has every source rank write
    its pieces into the target ranks' memory (targets of a rank are views of one arena); "pull" has
    every target rank read them (targets are separate allocations). Transfers run in phases in
    which every GPU sends to at most one peer and receives from at most one.
    $SUIKA_RESHARD_FANOUT ("0" by default, "auto" or "1"): DP-replica fan-out of the push
    direction (suika_b200.fanout).
    """
    if not isinstance(device, torch.device):
        device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("suika_b200 moves state on CUDA devices only (no CPU path)")
    prof = prof or _NullProf()
    prof.start("schedule")
    plan = Plan(source_param_layout, target_param_layout)
    prof.stop("schedule")
    prof.start("execute", require_memory=True)
    direction = direction or os.environ.get("SUIKA_RESHARD_DIRECTION", "push")
    release = getattr(source_state_dict, "release", None)
    if callable(release):
        # sources received in place from the old process (suika_b200.handoff) are memory another
        # process owns: they cannot be re-exported to peers, so this rank's own kernel reads them
        direction = "push"
    fanout = _fanout_setting(os.environ.get("SUIKA_RESHARD_FANOUT", "0"))
    exp = other_context_dict["expected_sub_fields"]
    to_free = self_pieces(plan, source_state_dict, exp, dist.get_rank(world), device) if forcefully_free else []
    target = execute_plan_distributed(plan, source_state_dict, exp, device, world, log_func,
                                      direction=direction, fanout=fanout if direction == "push" else False)
    torch.cuda.synchronize(device=device)
    if callable(release):
        release()  # every rank is past the barrier: the old process may free its memory
    _forcefully_free(to_free)  # past the barrier no rank reads them any more
    prof.stop("execute", require_memory=True)
    return target


class TransferSchedule(list):
    """The list of TransferOps schedule_param_transfer returns, carrying the C plan that
    execute_param_transfer runs."""

    def __init__(self, plan: Plan):
        super().__init__(plan.transfer_ops())
        self.plan = plan


def schedule_param_transfer(source_param_layout, target_param_layout, log_func: Optional[Callable] = None) -> TransferSchedule:
    """Drop-in for schedule_param_transfer (migration.py:322-381)."""
    plan = Plan(source_param_layout, target_param_layout)
    if log_func is not None:
        for o in plan.op_array[plan.op_array["src_rank"] != plan.op_array["dst_rank"]]:
            log_func(f"schedule_param_transfer: {int(o['src_rank'])} > {int(o['dst_rank'])} transfer {plan.names[o['name_id']]}")
    return TransferSchedule(plan)


def execute_param_transfer(transfer_ops: TransferSchedule, source_state_dict, device, expected_sub_fields, world=None,
                           log_func=None, prof=None, forcefully_free: bool = False, fake_source_state_dicts=None,
                           rank: Optional[int] = None):
    """Drop-in for execute_param_transfer (migration.py:397-556) on a schedule made by
    schedule_param_transfer above (the C plan travels with it).

    With fake_source_state_dicts (checkpoint resume, migration.py:1235-1244: every needed source
    shard loaded from disk into host memory) the targets are built on `device` (CUDA) straight from
    host memory: the needed source tensors are gathered into one page-locked arena and the copy
    kernel reads them over PCIe. No collective is used; `rank` overrides dist.get_rank(world)."""
    if not isinstance(transfer_ops, TransferSchedule):
        raise TypeError("execute_param_transfer needs the schedule returned by suika_b200's schedule_param_transfer")
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("suika_b200 moves state on CUDA devices only (no CPU path)")
    if fake_source_state_dicts is not None:
        r = dist.get_rank(world) if rank is None else rank
        return execute_from_host(transfer_ops.plan, r, source_state_dict, fake_source_state_dicts, expected_sub_fields, device)
    to_free = self_pieces(transfer_ops.plan, source_state_dict, expected_sub_fields, dist.get_rank(world), device) if forcefully_free else []
    target = execute_plan_distributed(transfer_ops.plan, source_state_dict, expected_sub_fields, device, world, log_func)
    torch.cuda.synchronize(device=device)
    _forcefully_free(to_free)
    return target


_HOST_CHUNK_BYTES = 256 << 20  # checkpoint resume: bytes of source shards gathered per launch


def execute_from_host(plan: Plan, rank: int, source_state_dict, fake_source_state_dicts, expected_sub_fields,
                      device: torch.device) -> Dict[str, Dict[str, torch.Tensor]]:
    """Checkpoint resume on B200: this rank's targets from host-resident source shards.

    Same bytes and cat order as the reference's checkpoint path; like it, every target takes its
    source's dtype, and a singleton target keeps its source's shape (recv_tensor =
    tensor_from_fake_source.to(device), migration.py:477-482)."""
    subs = [s for s, _ in expected_sub_fields]
    srcs = dict(fake_source_state_dicts)
    if source_state_dict:
        srcs.setdefault(rank, source_state_dict)
    dtypes = _sub_dtypes(expected_sub_fields, srcs.values())
    spec = _program_spec(expected_sub_fields, dtypes)
    if not np.any(plan.op_array["dst_rank"] == rank):
        return {}
    prog = plan.program(rank, spec)

    def host_src(sr, name, sub):
        st = srcs.get(sr)
        if st is None or name not in st:
            raise AssertionError(f"[{rank}]: param missing in source {name} of rank {sr}")
        t = st[name][sub]
        if t.device.type != "cpu":
            raise RuntimeError(f"checkpoint source {name}[{sub}] of rank {sr} is not in host memory")
        return t.contiguous()

    # 1. the needed source slots go into one page-locked arena the GPU reads directly
    hs = [host_src(int(ss["src_rank"]), plan.names[int(ss["name_id"])], subs[int(ss["subfield"])]) for ss in prog.src_slots]
    nb = np.array([t.numel() * t.element_size() for t in hs], np.uint64)
    off = np.zeros(len(hs), np.uint64)
    if len(hs) > 1:
        off[1:] = np.cumsum((nb[:-1] + np.uint64(255)) // np.uint64(256) * np.uint64(256))
    total = int(off[-1] + nb[-1]) if len(hs) else 0
    arena = torch.empty(max(total, 1), dtype=torch.uint8, pin_memory=True)
    dp = C.c_void_p()
    L.check(L.load().rs_host_device_pointer(C.c_void_p(arena.data_ptr()), C.byref(dp)))
    # 2. targets on the device; their copy table, reading host memory over PCIe
    dst_t = []
    for ds in prog.dst_slots:
        shape = tuple(int(x) for x in ds["shape"][: ds["ndim"]])
        dst_t.append(torch.empty(shape, dtype=dtypes[subs[ds["subfield"]]], device=device))
    table = prog.resolve(off + np.uint64(dp.value), nb, np.array([x.data_ptr() for x in dst_t], np.uint64),
                         np.array([x.numel() * x.element_size() for x in dst_t], np.uint64))
    table["flags"] = L.RS_COPY_REMOTE
    # 3. gather and copy in chunks of source slots: while the GPU reads chunk k over PCIe, the host
    #    gathers chunk k + 1 into the arena, so the two overlap
    chunk_of = np.zeros(len(hs), np.int64)
    acc, c = 0, 0
    for i in range(len(hs)):
        if acc >= _HOST_CHUNK_BYTES:
            c, acc = c + 1, 0
        chunk_of[i] = c
        acc += int(nb[i])
    seg_chunk = chunk_of[prog.segments["src_slot"]] if len(prog.segments) else np.zeros(0, np.int64)
    n_chunks = int(chunk_of.max()) + 1 if len(hs) else 0
    # every chunk's table is staged before the gather starts, so a chunk's launch is a kernel launch only
    chunks = [PreparedCopies(table[seg_chunk == k], device) if np.any(seg_chunk == k) else None for k in range(n_chunks)]
    launched = []
    try:
        for k in range(n_chunks):
            for i in np.nonzero(chunk_of == k)[0]:
                o, n = int(off[i]), int(nb[i])
                arena[o:o + n].copy_(hs[i].reshape(-1).view(torch.uint8))
            if chunks[k] is not None:
                chunks[k].launch()
                launched.append(chunks[k])
        ent: Dict[str, Dict[str, torch.Tensor]] = {}
        for ds, x in zip(prog.dst_slots, dst_t):
            ent.setdefault(plan.names[ds["name_id"]], {})[subs[ds["subfield"]]] = x
        meta = _MetaStage(device)
        for ms in prog.meta_slots:
            name, s = plan.names[int(ms["name_id"])], subs[int(ms["subfield"])]
            v = host_src(int(ms["src_rank"]), name, s)
            x = torch.empty(v.shape, dtype=v.dtype, device=device)
            meta.add(v, x)
            ent.setdefault(name, {})[s] = x
        md, stage = meta.descs()
        if len(md):
            p = PreparedCopies(md, device)
            p.launch()
            launched.append(p)
        for p in launched:
            p.check()  # synchronises: the arena and the staging buffer may go after this
    except BaseException:
        # the kernels read the arena through a device pointer the pinned-memory cache does not
        # track: none of them may still be reading it when it goes back to the cache
        if launched:
            try:
                torch.cuda.synchronize(device)
            except Exception:
                pass
        raise
    del arena, stage
    return {plan.names[n]: {s: ent[plan.names[n]][s] for s in subs if s in ent[plan.names[n]]} for n in _name_order(plan, rank)}


# ---------------------------------------------------------------------------------------------
# Transfer phases: at most one peer per direction per GPU at a time.
# ---------------------------------------------------------------------------------------------
def transfer_phases(pairs: Dict[Tuple[int, int], int]) -> Dict[Tuple[int, int], int]:
    """Phase of every remote (source, target) rank pair such that within a phase every rank sends
    to at most one peer and receives from at most one: a proper edge colouring of the bipartite
    source -> target multigraph with as many colours as its largest degree (Konig), found by
    alternating-path recolouring. Heavier pairs are coloured first. pairs: {(s, t): bytes}, s != t."""
    color: Dict[Tuple[int, int], int] = {}
    at_src: Dict[int, Dict[int, int]] = {}   # s -> {colour: t}
    at_dst: Dict[int, Dict[int, int]] = {}   # t -> {colour: s}
    deg: Dict[Tuple[str, int], int] = {}
    for s, t in pairs:
        deg[("s", s)] = deg.get(("s", s), 0) + 1
        deg[("t", t)] = deg.get(("t", t), 0) + 1
    ncol = max(deg.values(), default=0)
    for (s, t) in sorted(pairs, key=lambda p: (-pairs[p], p)):
        cs, ct = at_src.setdefault(s, {}), at_dst.setdefault(t, {})
        a = next(c for c in range(ncol) if c not in cs)   # free at the source
        b = next(c for c in range(ncol) if c not in ct)   # free at the target
        if a != b and a in ct:
            # flip the a/b alternating path that starts at target t along colour a
            path, node, side, c = [], t, "t", a
            while True:
                nxt = (at_dst if side == "t" else at_src).get(node, {}).get(c)
                if nxt is None:
                    break
                e = (nxt, node) if side == "t" else (node, nxt)
                path.append(e)
                node, side, c = nxt, ("s" if side == "t" else "t"), (b if c == a else a)
            for e in path:  # remove, then re-add with swapped colours
                old = color[e]
                del at_src[e[0]][old], at_dst[e[1]][old]
            for e in path:
                new = b if color[e] == a else a
                color[e] = new
                at_src[e[0]][new], at_dst[e[1]][new] = e[1], e[0]
        color[(s, t)] = a
        cs[a], ct[a] = t, s
    return color


def _phase_tables(table: np.ndarray, peer_of_entry: np.ndarray, rank: int, phase_of_pair, n_phases: int,
                  as_source: bool) -> List[np.ndarray]:
    """Split a rank's table by phase: a remote entry goes to the phase of its (source, target)
    pair; local entries are spread over the phases, each to the one with the fewest bytes so far."""
    if n_phases <= 1:
        return [table]
    nbytes = (table["rows"] * table["row_bytes"]).astype(np.int64)
    phase = np.zeros(len(table), np.int64)
    load = np.zeros(n_phases, np.int64)
    remote = peer_of_entry != rank
    for i in np.nonzero(remote)[0]:
        p = int(peer_of_entry[i])
        k = phase_of_pair[(rank, p) if as_source else (p, rank)]
        phase[i] = k
        load[k] += nbytes[i]
    for i in np.nonzero(~remote)[0]:
        k = int(np.argmin(load))
        phase[i] = k
        load[k] += nbytes[i]
    return [table[phase == k] for k in range(n_phases)]

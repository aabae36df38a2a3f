"""Compact metadata plane: parameter layouts as flat records instead of pickled objects.

Replaces, for the reshard, how Suika moves layouts between ranks:
  - ParamLayout.gather (Suika/migration.py:172-192): every rank's {name: TensorMeta} goes through
    dist.all_gather_object (pickle, a size exchange, the bytes, unpickle of every object);
  - broadcast_objects of the source layout (Suika/migration.py:1631-1633, Suika/utils.py:98-104):
    the whole layout pickled through broadcast_object_list.
Here a rank's layout is one byte blob: a header, one TENSOR_META record per tensor (the C
planner's own input format, include/suika_reshard.h rs_tensor_meta), a dtype code per tensor, the
names, and the slice rules of extension layouts (JSON, usually empty). Blobs travel through
all_gather_into_tensor / broadcast of uint8 tensors (on the GPU for NCCL groups, on the host for
gloo) and are decoded with numpy. A CompactLayout hands the records to the planner as they are
(no per-tensor Python objects on the way); its .layout builds the reference-shaped
{rank: {name: TensorMeta}} on first use, for code that wants it.
"""
from __future__ import annotations

import json
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from . import _lib as L

_MAGIC = 0x314C4B53  # "SKL1"
_HEADER = np.dtype([("magic", "<u4"), ("n", "<u4"), ("names_len", "<u4"), ("rules_len", "<u4"),
                    ("reserved", "<u8", (2,))])
_DTYPES = [torch.float32, torch.bfloat16, torch.float16, torch.float64, torch.int64, torch.int32, torch.int16,
           torch.int8, torch.uint8, torch.bool, torch.float8_e4m3fn, torch.float8_e5m2, torch.complex64]
_CODE = {d: i for i, d in enumerate(_DTYPES)}
_ITEMSIZE = [d.itemsize for d in _DTYPES]


def _dtype_code(dtype) -> int:
    code = _CODE.get(dtype)
    if code is None:
        raise ValueError(f"dtype {dtype} has no code in the metadata plane")
    return code


def encode_metas(metas: Dict[str, Any]) -> np.ndarray:
    """One rank's {name: TensorMeta} (the reference's class or this package's mirror: read through
    .shape, .dtype, .tp_meta and an optional .tp_rule) as a uint8 blob."""
    n = len(metas)
    recs, codes = [], np.zeros(n, dtype=np.int8)
    rules: Dict[str, Any] = {}
    pad = (0,) * L.RS_MAX_DIMS
    for i, (name, m) in enumerate(metas.items()):
        shape = tuple(int(x) for x in m.shape)
        if len(shape) > L.RS_MAX_DIMS:
            raise ValueError(f"{name}: more than {L.RS_MAX_DIMS} dims")
        code = _dtype_code(m.dtype)
        tp = m.tp_meta
        sd, ti, td = (L.RS_NO_SLICE, 0, 1) if tp is None else (int(tp[0]), int(tp[1]), int(tp[2]))
        recs.append((i, len(shape), shape + pad[len(shape):], _ITEMSIZE[code], sd, ti, td))
        codes[i] = code
        rule = getattr(m, "tp_rule", None)
        if rule is not None:
            rules[name] = [[int(x) for x in g] for g in rule]
    rec = np.array(recs, dtype=L.TENSOR_META_DTYPE) if recs else np.zeros(0, dtype=L.TENSOR_META_DTYPE)
    names = "\0".join(metas).encode()
    rj = json.dumps(rules).encode() if rules else b""
    head = np.zeros(1, dtype=_HEADER)
    head["magic"], head["n"], head["names_len"], head["rules_len"] = _MAGIC, n, len(names), len(rj)
    return np.concatenate([head.view(np.uint8), rec.view(np.uint8), codes.view(np.uint8),
                           np.frombuffer(names, np.uint8), np.frombuffer(rj, np.uint8)])


def decode_metas(blob: np.ndarray) -> Tuple[List[str], np.ndarray, np.ndarray, Dict[str, Any]]:
    """(names, TENSOR_META records with name_id = index into names, dtype codes, slice rules)."""
    blob = np.ascontiguousarray(blob, dtype=np.uint8)
    if blob.nbytes < _HEADER.itemsize:
        raise ValueError("metadata blob shorter than its header")
    head = blob[: _HEADER.itemsize].view(_HEADER)[0]
    if int(head["magic"]) != _MAGIC:
        raise ValueError("not a metadata blob")
    n, nl, rl = int(head["n"]), int(head["names_len"]), int(head["rules_len"])
    o = _HEADER.itemsize
    rec_end = o + n * L.TENSOR_META_DTYPE.itemsize
    if blob.nbytes < rec_end + n + nl + rl:
        raise ValueError("metadata blob truncated")
    rec = blob[o:rec_end].copy().view(L.TENSOR_META_DTYPE)
    codes = blob[rec_end:rec_end + n].view(np.int8).copy()
    names = bytes(blob[rec_end + n:rec_end + n + nl]).decode().split("\0") if n else []
    rules = json.loads(bytes(blob[rec_end + n + nl:rec_end + n + nl + rl]).decode()) if rl else {}
    if len(names) != n:
        raise ValueError("metadata blob: name count differs from record count")
    return names, rec, codes, rules


class CompactLayout:
    """A ParamLayout held as records: rank -> TENSOR_META array over one shared name table.
    Accepted wherever a ParamLayout is (Plan, schedule_and_execute_param_transfer)."""

    def __init__(self):
        self.names: List[str] = []
        self.name_ids: Dict[str, int] = {}
        self.ranks: List[int] = []
        self.records: List[np.ndarray] = []
        self.codes: List[np.ndarray] = []
        self.rules: Dict[str, Any] = {}
        self._layout: Optional[Dict[int, Dict[str, Any]]] = None

    def add_rank(self, rank: int, blob: np.ndarray) -> None:
        names, rec, codes, rules = decode_metas(blob)
        ids = np.empty(len(names), dtype=np.int32)
        for i, nm in enumerate(names):
            g = self.name_ids.get(nm)
            if g is None:
                g = self.name_ids[nm] = len(self.names)
                self.names.append(nm)
            ids[i] = g
        rec["name_id"] = ids[rec["name_id"]] if len(rec) else rec["name_id"]
        for nm, rule in rules.items():
            if self.rules.setdefault(nm, rule) != rule:
                raise ValueError(f"{nm}: ranks disagree on its slice rule")
        self.ranks.append(int(rank))
        self.records.append(rec)
        self.codes.append(codes)
        self._layout = None

    def flatten(self, name_ids: Dict[str, int], names: List[str], rules: Optional[Dict[str, Any]] = None):
        """(ranks, TENSOR_META arrays) with name ids remapped into the caller's table; the planner's
        input without a per-tensor Python object."""
        remap = np.empty(len(self.names), dtype=np.int32)
        for i, nm in enumerate(self.names):
            g = name_ids.get(nm)
            if g is None:
                g = name_ids[nm] = len(names)
                names.append(nm)
            remap[i] = g
        if rules is not None:
            for nm, rule in self.rules.items():
                rule = tuple(tuple(int(x) for x in g) for g in rule)
                if rules.setdefault(nm, rule) != rule:
                    raise ValueError(f"{nm}: different slice rules in the source and target layouts")
        arrays = []
        for rec in self.records:
            a = rec.copy()
            if len(a):
                a["name_id"] = remap[a["name_id"]]
            arrays.append(a)
        return list(self.ranks), arrays

    @property
    def layout(self) -> Dict[int, Dict[str, Any]]:
        """{rank: {name: TensorMeta}} in record order (built once, on first use)."""
        if self._layout is None:
            from .migration import TensorMeta
            out: Dict[int, Dict[str, Any]] = {}
            for rank, rec, codes in zip(self.ranks, self.records, self.codes):
                ent = {}
                for r, c in zip(rec, codes):
                    nm = self.names[int(r["name_id"])]
                    tp = None if int(r["slice_dim"]) == L.RS_NO_SLICE else (int(r["slice_dim"]), int(r["tp_index"]), int(r["tp_deg"]))
                    m = TensorMeta(name=nm, dtype=_DTYPES[int(c)], shape=[int(x) for x in r["shape"][: int(r["ndim"])]], tp_meta=tp)
                    if nm in self.rules:
                        m.tp_rule = [tuple(g) for g in self.rules[nm]]
                    ent[nm] = m
                out[rank] = ent
            self._layout = out
        return self._layout

    def encode(self) -> np.ndarray:
        """The whole layout as one blob: a rank index, then each rank's blob."""
        blobs = [encode_metas(self.layout[r]) for r in self.ranks]
        index = np.array([len(self.ranks)] + [x for r, b in zip(self.ranks, blobs) for x in (r, b.nbytes)], dtype=np.int64)
        return np.concatenate([index.view(np.uint8), *blobs]) if blobs else index.view(np.uint8)

    @classmethod
    def decode(cls, blob: np.ndarray) -> "CompactLayout":
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        n = int(blob[:8].view(np.int64)[0])
        index = blob[8:8 + 16 * n].view(np.int64).reshape(n, 2)
        out, o = cls(), 8 + 16 * n
        for rank, size in index:
            out.add_rank(int(rank), blob[o:o + int(size)])
            o += int(size)
        return out

    @classmethod
    def from_layout(cls, layout) -> "CompactLayout":
        """From a ParamLayout (the reference's or the mirror) or a {rank: {name: meta}} dict."""
        src = getattr(layout, "layout", layout)
        out = cls()
        for rank, metas in src.items():
            out.add_rank(int(rank), encode_metas(metas))
        return out


def _transport_device(group) -> torch.device:
    return torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")


def gather_param_layout(self_param_meta_or_module, world: Optional[dist.ProcessGroup] = None) -> CompactLayout:
    """ParamLayout.gather (Suika/migration.py:172-192) over records: every rank's layout, in group
    rank order, from one size all-gather and one byte all-gather. Collective over `world`."""
    if isinstance(self_param_meta_or_module, torch.nn.Module):
        from .migration import get_param_tensor_meta
        metas = get_param_tensor_meta(self_param_meta_or_module)
    else:
        metas = self_param_meta_or_module
    blob = encode_metas(metas)
    dev = _transport_device(world)
    n = dist.get_world_size(world)
    sizes = torch.zeros(n, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(sizes, torch.tensor([blob.nbytes], dtype=torch.int64, device=dev), group=world)
    sizes_h = sizes.cpu().numpy()
    width = int(sizes_h.max())
    mine = torch.zeros(width, dtype=torch.uint8)
    mine[: blob.nbytes] = torch.from_numpy(blob)
    allb = torch.empty(n * width, dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(allb, mine.to(dev), group=world)
    allh = allb.cpu().numpy().reshape(n, width)
    out = CompactLayout()
    for r in range(n):
        out.add_rank(r, allh[r, : int(sizes_h[r])])
    return out


def broadcast_param_layout(layout, src: int = 0, group: Optional[dist.ProcessGroup] = None) -> Optional[CompactLayout]:
    """The layout part of broadcast_objects (Suika/utils.py:98-104) over records: rank `src` holds
    the layout (a ParamLayout, CompactLayout or None); every rank returns it. Collective."""
    dev = _transport_device(group)
    size = torch.zeros(1, dtype=torch.int64, device=dev)
    blob = None
    if dist.get_rank(group) == src:
        if layout is not None:
            cl = layout if isinstance(layout, CompactLayout) else CompactLayout.from_layout(layout)
            blob = cl.encode()
            size[0] = blob.nbytes
        else:
            size[0] = -1  # "no checkpoint" (migration.py:1635-1637 tests the layout for None)
    dist.broadcast(size, src=dist.get_global_rank(group, src) if group is not None else src, group=group)
    n = int(size.item())
    if n < 0:
        return None
    buf = torch.from_numpy(blob).to(dev) if blob is not None else torch.empty(n, dtype=torch.uint8, device=dev)
    dist.broadcast(buf, src=dist.get_global_rank(group, src) if group is not None else src, group=group)
    if blob is not None and isinstance(layout, CompactLayout):
        return layout
    return CompactLayout.decode(buf.cpu().numpy())

"""CPU restatement of Suika's reshard path (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Layouts are read the way the reference reads a ParamLayout: `.layout` is {rank: {name: meta}}
in dict order, each meta exposing `.shape` (FULL shape), `.dtype` and `.tp_meta`
((slice_dim, tp_index, tp_deg) or None). States are {rank: {name: {sub_field: np.ndarray}}},
arrays holding the rank's actual shard (bf16 as uint16 bit patterns).
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


def _itemsize(dtype) -> int:
    return getattr(dtype, "itemsize", None) or np.dtype(dtype).itemsize


def _deg(tp):
    return 1 if tp is None else tp[2]


def _idx(tp):
    return 0 if tp is None else tp[1]


@dataclass(frozen=True)
class Op:
    """One TransferOp (Suika/migration.py:257-283), with the rescaled target piece's tp_meta."""
    name: str
    src: int
    dst: int
    src_tp: Optional[Tuple[int, int, int]]
    dst_tp: Optional[Tuple[int, int, int]]
    numel: int


def _numel(shape, tp) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n // _deg(tp)  # TensorMeta.numel, migration.py:66-67


def _overlap(a, b) -> bool:
    """ParamLayout.is_tensor_tp_overlap, migration.py:220-244."""
    if a is None or b is None:
        return True
    assert a[0] == b[0], f"slice dim mismatch {a[0]} vs {b[0]}"
    (_, i1, g1), (_, i2, g2) = a, b
    if g1 > g2:
        i1, i2, g1, g2 = i2, i1, g2, g1
    return i2 // (g2 // g1) == i1


def _owned(src_tp, tgt_tp) -> bool:
    """ParamLayout.is_tensor_tp_owned, migration.py:246-254."""
    return _deg(src_tp) <= _deg(tgt_tp) and _overlap(src_tp, tgt_tp)


def _scale_to_tp(tp, target):
    """TensorMeta.scale_to_tp, migration.py:103-118 (tp_meta only)."""
    if tp is not None and target > tp[2]:
        scale = target // tp[2]
        return [(tp[0], scale * tp[1] + i, target) for i in range(scale)]
    return [tp]


def schedule(spl, tpl, minimum_est_peers: int = 2) -> List[Op]:
    """schedule_param_transfer, Suika/migration.py:322-381."""
    src = spl.layout
    max_tp = max(_deg(m.tp_meta) for metas in src.values() for m in metas.values())
    latency = [0.0 for _ in src.keys()]
    ops: List[Op] = []
    for dst, params in tpl.layout.items():
        est = set()
        for name, m in params.items():
            vol_unit = _itemsize(m.dtype)
            for piece in _scale_to_tp(m.tp_meta, max_tp):
                srcs = [r for r, metas in src.items() if name in metas and _owned(metas[name].tp_meta, piece)]
                assert len(srcs) > 0, f"illegal transfer, target param {name} {piece} is not present in any source"
                vol = _numel(m.shape, piece) * vol_unit
                if dst in srcs:
                    best = dst
                else:
                    est_srcs = [s for s in srcs if s in est]
                    pool = est_srcs if (len(est_srcs) > 0 and len(est) >= minimum_est_peers) else srcs
                    best = min(pool, key=lambda s: latency[s] + vol)
                est.add(best)
                ops.append(Op(name, best, dst, src[best][name].tp_meta, piece, _numel(m.shape, piece)))
                latency[best] += vol
    return ops


def send_piece(arr: np.ndarray, src_tp, dst_tp) -> np.ndarray:
    """TransferOp.get_send_tensor, migration.py:290-312."""
    assert (src_tp is None) == (dst_tp is None) and (src_tp is None or src_tp[0] == dst_tp[0]), "slice dim mismatch"
    if _deg(src_tp) >= _deg(dst_tp):
        return arr
    d, si, sg = src_tp
    _, di, dg = dst_tp
    k = dg // sg
    return np.ascontiguousarray(np.split(arr, k, axis=d)[di - si * k])


def execute_rank(ops: Sequence[Op], states, subfields: Sequence[Tuple[str, bool]], rank: int,
                 order: str = "reference") -> Dict[str, Dict[str, np.ndarray]]:
    """execute_param_transfer for one rank, migration.py:397-556.

    subfields: (name, is_meta) in expected_sub_fields order. order="reference" keeps the
    reference's piece order (received pieces first, self pieces after them, migration.py:448-509);
    "semantic" orders pieces by their TP index. The receive buffer of a normal sub-field takes
    that sub-field's own dtype (the reference allocates it in the layout dtype,
    migration.py:285-287, which only works when every sub-field has the param's dtype).
    """
    target: Dict[str, Dict[str, list]] = {}
    slice_dim: Dict[str, Optional[int]] = {}
    tp_of: Dict[str, list] = {}
    deferred = []
    for op in ops:
        if op.dst == rank and op.name not in target:
            target[op.name] = {s: [] for s, _ in subfields}
            slice_dim[op.name] = None if op.dst_tp is None else op.dst_tp[0]
            tp_of[op.name] = []
        if op.src == rank:
            if op.dst == rank:  # self transfer, appended after all remote pieces
                for s, meta in subfields:
                    a = states[rank][op.name][s]
                    deferred.append((op.name, s, a if meta else send_piece(a, op.src_tp, op.dst_tp), _idx(op.dst_tp)))
        elif op.dst == rank:
            for s, meta in subfields:
                a = states[op.src][op.name][s]
                v = a.reshape(1) if meta else send_piece(a, op.src_tp, op.dst_tp)  # recv into [1] / actual shape
                target[op.name][s].append((v, _idx(op.dst_tp)))
    for name, s, v, ti in deferred:
        target[name][s].append((v, ti))
    out: Dict[str, Dict[str, np.ndarray]] = {}
    for name, fields in target.items():
        out[name] = {}
        for s, meta in subfields:
            pieces = fields[s]
            if order == "semantic":
                pieces = sorted(pieces, key=lambda p: p[1])
            arrs = [p[0] for p in pieces]
            if not meta and len(arrs) > 1:
                out[name][s] = np.concatenate(arrs, axis=slice_dim[name])
            else:
                out[name][s] = np.array(arrs[0], copy=True)
    return out


def execute_world(ops, states, subfields, ranks: Sequence[int], order: str = "reference", threads: int = 1):
    """execute_rank for every target rank. With threads > 1 the work is split by (rank, tensor)
    over a thread pool: every target tensor depends only on its own ops, and numpy's copies
    release the GIL."""
    if threads <= 1:
        return {r: execute_rank(ops, states, subfields, r, order) for r in ranks}
    tasks = []
    for r in ranks:
        names = list(dict.fromkeys(o.name for o in ops if o.dst == r))
        for k in range(threads):
            part = set(names[k::threads])
            if part:
                tasks.append((r, [o for o in ops if o.name in part and (o.dst == r or o.src == r)]))
    with ThreadPoolExecutor(max_workers=threads) as ex:
        futs = [(r, ex.submit(execute_rank, sub_ops, states, subfields, r, order)) for r, sub_ops in tasks]
        out = {r: {} for r in ranks}
        for r, f in futs:
            out[r].update(f.result())
    for r in ranks:  # restore the reference's tensor order
        order_r = list(dict.fromkeys(o.name for o in ops if o.dst == r))
        out[r] = {n: out[r][n] for n in order_r}
    return out


def _spans(full_shape, tp, rule):
    """Slice-dim intervals of a shard: the reference's chunk, or per group of a slice rule the
    units [i*u/T, (i+1)*u/T) (u >= T) or the unit floor(i*u/T) (u < T, replicated)."""
    d, i, g = tp
    F = int(full_shape[d])
    if not rule:
        return [(i * F // g, (i + 1) * F // g)]
    out = []
    for off, size, units in rule:
        usz = size // units
        lo = i * (units // g) if units >= g else (i * units // g)
        n = units // g if units >= g else 1
        out.append((off + lo * usz, off + (lo + n) * usz))
    return out


def semantic_target(states, spl, tpl, subfields, rank: int) -> Dict[str, Dict[str, np.ndarray]]:
    """Gather each full tensor from the source shards and re-slice it by the target rule (chunks,
    or a `tp_rule` attribute on the metas)."""
    out = {}
    for name, m in tpl.layout[rank].items():
        out[name] = {}
        owners = [(r, metas[name]) for r, metas in spl.layout.items() if name in metas]
        for s, meta in subfields:
            if meta:
                out[name][s] = np.array(states[owners[0][0]][name][s], copy=True)
                continue
            tps = [mm.tp_meta for _, mm in owners if mm.tp_meta is not None]
            if not tps:
                full = states[owners[0][0]][name][s]
            else:
                d = tps[0][0]
                a0 = states[owners[0][0]][name][s]
                shape = list(int(x) for x in m.shape)
                full = np.zeros(shape, dtype=a0.dtype)
                for r, mm in owners:
                    a = states[r][name][s]
                    if mm.tp_meta is None:
                        full = a.copy()
                        break
                    at = 0
                    for lo, hi in _spans(shape, mm.tp_meta, getattr(mm, "tp_rule", None)):
                        idx = [slice(None)] * len(shape)
                        sidx = [slice(None)] * len(shape)
                        idx[d], sidx[d] = slice(lo, hi), slice(at, at + hi - lo)
                        full[tuple(idx)] = a[tuple(sidx)]
                        at += hi - lo
            if m.tp_meta is None:
                out[name][s] = np.array(full, copy=True)
            else:
                d = m.tp_meta[0]
                parts = [np.take(full, np.arange(lo, hi), axis=d) for lo, hi in _spans(m.shape, m.tp_meta, getattr(m, "tp_rule", None))]
                out[name][s] = np.ascontiguousarray(np.concatenate(parts, axis=d))
    return out

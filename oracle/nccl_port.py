"""The reference's execute_param_transfer as it runs on GPUs: one torch.distributed P2P op per
tensor and sub-field (TEST AND BENCHMARK-BASELINE INFRASTRUCTURE ONLY; see oracle/__init__.py).

Restates Suika/migration.py:397-556, with the P2P helper of Suika/utils.py:212-234 (non-batched
isend/irecv, issued in op order), on torch tensors:
  - a piece a rank sends is get_send_tensor's .contiguous() chunk (migration.py:290-312);
  - a piece a rank receives lands in a fresh buffer of the piece's shape (get_recv_tensor, :285-287);
  - self pieces are appended after the received ones (the deferred closures, :448-459, :508-509);
  - after the waits, the source dict is cleared, and each target is torch.cat of its pieces along
    the slice dim, or a clone of its single piece (:531-545); cuda_gc runs where the reference
    runs it (:529, :547; Suika/utils.py:248-253).
One forced difference: a received sub-field's buffer takes that sub-field's dtype, where the
reference allocates every sub-field in the layout dtype (:285-287), which breaks when fp32 Adam
state sits next to a bf16 param.

bench.py times this on B200s over NCCL as the library baseline of the reshard (the reference's
own GPU path); tests/test_reference_port.py pins it on gloo CPU ranks against the reference's
golden digests.
"""
from __future__ import annotations

import gc
from typing import Dict, Sequence, Tuple

import torch
import torch.distributed as dist

from .restate import Op, _deg


def _cuda_gc() -> None:
    """Suika/utils.py:248-253."""
    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
        torch.cuda.synchronize()
        torch.cuda.ipc_collect()


def send_piece(t: torch.Tensor, src_tp, dst_tp) -> torch.Tensor:
    """TransferOp.get_send_tensor (migration.py:290-312) on a torch tensor."""
    if _deg(src_tp) >= _deg(dst_tp):
        return t
    d, si, sg = src_tp
    _, di, dg = dst_tp
    k = dg // sg
    return t.chunk(k, dim=d)[di - si * k].contiguous()


def _piece_shape(full_shape, dst_tp):
    """TensorMeta.actual_shape of the (rescaled) target piece (migration.py:92-98)."""
    s = [int(x) for x in full_shape]
    if dst_tp is not None:
        s[dst_tp[0]] //= dst_tp[2]
    return s


def execute_rank(ops: Sequence[Op], source_state_dict: Dict[str, Dict[str, torch.Tensor]],
                 subfields: Sequence[Tuple[str, bool, torch.dtype]], full_shapes: Dict[str, Sequence[int]],
                 rank: int, device: torch.device, world=None, cuda_gc: bool = True) -> Dict[str, Dict[str, torch.Tensor]]:
    """One rank's execute_param_transfer. subfields: (name, is_meta, dtype) in expected_sub_fields
    order; full_shapes: the full (unsharded) shape of every target tensor."""
    p2p = []
    deferred = []
    target: Dict[str, Dict[str, list]] = {}
    slice_dim: Dict[str, int] = {}
    for op in ops:
        if op.dst == rank and op.name not in target:
            target[op.name] = {s: [] for s, _m, _d in subfields}
            slice_dim[op.name] = None if op.dst_tp is None else op.dst_tp[0]
        if op.src == rank:
            if op.name not in source_state_dict:
                raise AssertionError(f"[{rank}]: param missing in source {op.name}")
            for s, meta, _dt in subfields:
                t = source_state_dict[op.name][s]
                send = t.to(device) if meta else send_piece(t, op.src_tp, op.dst_tp).to(device)
                if op.dst == rank:
                    deferred.append((op.name, s, send))
                else:
                    p2p.append((dist.isend, send, op.dst))
        elif op.dst == rank:
            for s, meta, dt in subfields:
                if meta:
                    recv = torch.tensor([0], dtype=dt, device=device)
                else:
                    recv = torch.empty(_piece_shape(full_shapes[op.name], op.dst_tp), dtype=dt, device=device)
                p2p.append((dist.irecv, recv, op.src))
                target[op.name][s].append(recv)
    reqs = [fn(t, peer, group=world) for fn, t, peer in p2p]  # Suika/utils.py:223-234, in op order
    for name, s, send in deferred:
        target[name][s].append(send)
    for r in reqs:
        r.wait()
    del p2p, deferred, reqs
    source_state_dict.clear()
    if cuda_gc:
        _cuda_gc()
    out: Dict[str, Dict[str, torch.Tensor]] = {}
    for name, fields in target.items():
        out[name] = {}
        for s, meta, _dt in subfields:
            pieces = fields[s]
            out[name][s] = torch.cat(pieces, dim=slice_dim[name]) if (not meta and len(pieces) > 1) else pieces[0].clone()
    if cuda_gc:
        _cuda_gc()
    return out


def checkpoint_rank(ops: Sequence[Op], fake_source_state_dicts: Dict[int, Dict[str, Dict[str, torch.Tensor]]],
                    subfields: Sequence[Tuple[str, bool, torch.dtype]], rank: int) -> Dict[str, Dict[str, torch.Tensor]]:
    """One rank's checkpoint resume as the reference runs it: execute_param_transfer with
    fake_source_state_dicts on device "cpu" (Suika/migration.py:1235-1244). A piece from another
    rank is get_send_tensor of that rank's host shard (the fake-source branch, :475-482); a piece of
    the rank's own source goes through the deferred self branch (:448-459), so it lands after the
    others; each target is torch.cat of its pieces along the slice dim, or a clone (:531-545). A
    piece this rank would send to another is still cut out (get_send_tensor, :442-446) and then not
    sent (:461-463), as the reference does."""
    own = fake_source_state_dicts.get(rank, {})
    deferred = []
    target: Dict[str, Dict[str, list]] = {}
    slice_dim: Dict[str, int] = {}
    for op in ops:
        if op.dst != rank and op.src != rank:
            continue
        if op.dst == rank and op.name not in target:
            target[op.name] = {s: [] for s, _m, _d in subfields}
            slice_dim[op.name] = None if op.dst_tp is None else op.dst_tp[0]
        if op.src == rank:
            if op.name not in own:
                raise AssertionError(f"[{rank}]: param missing in source {op.name}")
            for s, meta, _dt in subfields:
                t = own[op.name][s]
                piece = t if meta else send_piece(t, op.src_tp, op.dst_tp)
                if op.dst == rank:
                    deferred.append((op.name, s, piece))
        else:
            src = fake_source_state_dicts[op.src][op.name]
            for s, meta, _dt in subfields:
                target[op.name][s].append(src[s] if meta else send_piece(src[s], op.src_tp, op.dst_tp))
    for name, s, t in deferred:
        target[name][s].append(t)
    out: Dict[str, Dict[str, torch.Tensor]] = {}
    for name, fields in target.items():
        out[name] = {}
        for s, meta, _dt in subfields:
            pieces = fields[s]
            out[name][s] = torch.cat(pieces, dim=slice_dim[name]) if (not meta and len(pieces) > 1) else pieces[0].clone()
    return out

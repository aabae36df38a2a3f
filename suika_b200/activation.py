"""Activation hand-over between adjacent pipeline stages whose DP/TP shapes differ, on B200.

Drop-in for the cross-stage communication of Suika's PipelineExecModule
(Suika/pipeline_parallel.py:665-836). The reference issues, per rank and micro-batch, one NCCL P2P
op per (batch overlap x slice chunk) block, each staged through a .contiguous() copy and copied
back into place afterwards (:748-756); a receiving TP group then all-gathers the chunks and cats
them (:817-832). Here the planner (rs_act_plan, C++) lists every block a receiver ends up with and
where it comes from, and one launch of the copy kernel writes them all into their final positions:
  - exchange_local: every rank's tensors on one device (one launch; tests and single-GPU use);
  - ActivationExchange: one process per GPU. Each receiver owns a persistent window (two slots,
    mapped by its senders once through CUDA IPC); a sender's send() pushes its blocks straight
    from its activation into the receivers' windows over NVLink (one launch), and a receiver's
    recv() copies its blocks from the window into the caller's tensor (one local launch). No
    all-gather: a receiver gets every chunk from its sender directly.
Ordering is stream-ordered, never host-blocking: each exchange ends with a one-element NCCL
all-reduce over the two stages' ranks, issued by senders after their push and by receivers before
their copy, so a receiver's copy starts after every push into its window has finished, and a
sender reuses a window slot only after the receiver has copied out of it (two exchanges later).

Bytes written are the reference's, from the same sender rank (tests/golden/act_golden.json holds
the reference's own results). Rows no sender covers are not written (the reference's engine
allocates receive tensors with zeros, so they stay zero in both).
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

from . import _lib as L
from .migration import PreparedCopies, _export, _PeerMaps

MeshLike = Sequence[Sequence[int]]


def mesh_lists(mesh) -> List[List[int]]:
    """A stage mesh as lists of ranks per DP group: a reference DeviceMesh2D (or RawDeviceMesh2D)
    through its to_list(), or nested lists as they are."""
    if hasattr(mesh, "to_list"):
        mesh = mesh.to_list()
    return [[int(r) for r in group] for group in mesh]


class _Stage:
    """rs_stage_mesh with the arrays it points to kept alive."""

    def __init__(self, mesh, bszs: Sequence[int]):
        self.groups = mesh_lists(mesh)
        if len(bszs) != len(self.groups):
            raise ValueError(f"{len(bszs)} local batch sizes for {len(self.groups)} DP groups")
        self.start = np.concatenate([[0], np.cumsum([len(g) for g in self.groups])]).astype(np.int32)
        self.ranks = np.array([r for g in self.groups for r in g], dtype=np.int32)
        self.bsz = np.array([int(b) for b in bszs], dtype=np.int64)
        self.c = L.RsStageMesh(len(self.groups), 0,
                               self.start.ctypes.data_as(C.POINTER(C.c_int32)),
                               self.ranks.ctypes.data_as(C.POINTER(C.c_int32)),
                               self.bsz.ctypes.data_as(C.POINTER(C.c_int64)))

    def rank_bsz(self) -> Dict[int, int]:
        return {r: int(b) for g, b in zip(self.groups, self.bsz) for r in g}


def _geometry(shape: Sequence[int], batch_dim: int, slice_dim: int, elem_bytes: int) -> L.RsActGeometry:
    nd = len(shape)
    if not 2 <= nd <= L.RS_MAX_DIMS:
        raise ValueError(f"activation of {nd} dims: 2 to {L.RS_MAX_DIMS} supported")
    g = L.RsActGeometry()
    g.ndim, g.batch_dim, g.slice_dim, g.elem_bytes = nd, batch_dim % nd, slice_dim % nd, elem_bytes
    for i, x in enumerate(shape):
        g.shape[i] = max(int(x), 0) if i != g.batch_dim else 0
    return g


def plan_activation_exchange(mesh_src, mesh_dst, bszs_src: Sequence[int], bszs_dst: Sequence[int],
                             slice_size: int) -> np.ndarray:
    """Every block the receiving stage gets (rs_act_plan), as an ACT_PIECE_DTYPE array."""
    return _plan(_Stage(mesh_src, bszs_src), _Stage(mesh_dst, bszs_dst), slice_size)


def _plan(src: _Stage, dst: _Stage, slice_size: int) -> np.ndarray:
    lib = L.load()
    n = C.c_int64()
    L.check(lib.rs_act_plan(C.byref(src.c), C.byref(dst.c), int(slice_size), None, 0, C.byref(n)))
    out = np.zeros(int(n.value), dtype=L.ACT_PIECE_DTYPE)
    if len(out):
        L.check(lib.rs_act_plan(C.byref(src.c), C.byref(dst.c), int(slice_size), out.ctypes.data, len(out), C.byref(n)))
    return out


def _resolve(src: _Stage, dst: _Stage, geo: L.RsActGeometry, pieces: np.ndarray,
             src_dev: Dict[int, int], dst_dev: Dict[int, int]) -> np.ndarray:
    """Copy descriptors of `pieces` (rs_act_resolve) for the given per-rank base addresses."""
    lib = L.load()
    n_ranks = max([0, *src_dev, *dst_dev]) + 1
    sa = np.zeros(n_ranks, dtype=np.uint64)
    da = np.zeros(n_ranks, dtype=np.uint64)
    for r, a in src_dev.items():
        sa[r] = a
    for r, a in dst_dev.items():
        da[r] = a
    pieces = np.ascontiguousarray(pieces, dtype=L.ACT_PIECE_DTYPE)
    n = C.c_int64()
    args = (C.byref(src.c), C.byref(dst.c), C.byref(geo), pieces.ctypes.data, len(pieces),
            sa.ctypes.data, da.ctypes.data, n_ranks)
    L.check(lib.rs_act_resolve(*args, None, 0, C.byref(n)))
    out = np.zeros(int(n.value), dtype=L.COPY_DESC_DTYPE)
    if len(out):
        L.check(lib.rs_act_resolve(*args, out.ctypes.data, len(out), C.byref(n)))
    return out


def rotated_pieces(pieces: np.ndarray, rank: int) -> np.ndarray:
    """The pieces `rank` sends, ordered so that the senders start at different receivers.

    The copy kernel's CTAs walk the table in order, so a sender's bytes leave one receiver at a
    time. Had every sender the same receiver order, all of them would write to the first
    receiver together, two or more links into one ingress, while the others idled. Sender i of
    n (ascending rank) starts instead at receiver i * m // n of the m receivers and goes round:
    with n == m each receiver has one writer at a time. The order within a receiver is kept."""
    mine = pieces[pieces["src_rank"] == rank]
    senders = sorted(set(pieces["src_rank"].tolist()))
    receivers = sorted(set(pieces["dst_rank"].tolist()))
    if len(mine) < 2 or len(receivers) < 2:
        return mine
    start = senders.index(rank) * len(receivers) // len(senders)
    turn = {r: (i - start) % len(receivers) for i, r in enumerate(receivers)}
    keys = np.array([turn[int(r)] for r in mine["dst_rank"]])
    return mine[np.argsort(keys, kind="stable")]


def send_table(src: _Stage, dst: _Stage, geo: L.RsActGeometry, pieces: np.ndarray, rank: int,
               activation_ptr: int, windows: Dict[int, int]) -> np.ndarray:
    """What a sending rank writes in one exchange: its blocks, from its activation at
    activation_ptr into each receiver's window slot (windows: receiver rank -> slot address in
    this process), laid out as the receiver's tensor, receivers in rotated_pieces' order."""
    mine = rotated_pieces(pieces, rank)
    return _resolve(src, dst, geo, mine, {rank: activation_ptr}, {r: windows[r] for r in set(mine["dst_rank"].tolist())})


def recv_table(dst: _Stage, geo: L.RsActGeometry, pieces: np.ndarray, rank: int, window_ptr: int, target_ptr: int) -> np.ndarray:
    """What a receiving rank copies in one exchange: its blocks, from its window slot into the
    caller's tensor (both in its own layout); rows no sender covers are left alone."""
    own = pieces[pieces["dst_rank"] == rank].copy()
    own["src_rank"] = rank
    own["src_batch"] = own["dst_batch"]
    return _resolve(dst, dst, geo, own, {rank: window_ptr}, {rank: target_ptr})


def _check_tensor(t: torch.Tensor, shape: Sequence[int], what: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{what} must be contiguous")
    if list(t.shape) != list(shape):
        raise AssertionError(f"{what} has shape {list(t.shape)}, expected {list(shape)}")


def _local_shape(shape: Sequence[int], batch_dim: int, bsz: int) -> List[int]:
    s = list(shape)
    s[batch_dim % len(s)] = int(bsz)
    return s


def exchange_local(mesh_src, mesh_dst, bszs_src: Sequence[int], bszs_dst: Sequence[int],
                   sources: Dict[int, torch.Tensor], targets: Dict[int, torch.Tensor],
                   batch_dim: int = 0, slice_dim: int = -1, stream: Optional[torch.cuda.Stream] = None) -> L.RsLaunchInfo:
    """One hand-over with every rank's tensors on one device: {sender rank: activation} into
    {receiver rank: tensor} (written in place), one copy launch on `stream` (asynchronous)."""
    src, dst = _Stage(mesh_src, bszs_src), _Stage(mesh_dst, bszs_dst)
    any_t = next(iter(targets.values()))
    nd = any_t.dim()
    bd, sd = batch_dim % nd, slice_dim % nd
    geo = _geometry(list(any_t.shape), bd, sd, any_t.element_size())
    for r, b in src.rank_bsz().items():
        if r not in sources:
            raise AssertionError(f"no activation for sending rank {r}")
        _check_tensor(sources[r], _local_shape(any_t.shape, bd, b), f"activation of rank {r}")
        if sources[r].dtype != any_t.dtype or sources[r].device != any_t.device:
            raise AssertionError("activations and targets must share dtype and device")
    for r, b in dst.rank_bsz().items():
        if r not in targets:
            raise AssertionError(f"no target for receiving rank {r}")
        _check_tensor(targets[r], _local_shape(any_t.shape, bd, b), f"target of rank {r}")
    pieces = _plan(src, dst, int(any_t.shape[sd]))
    descs = _resolve(src, dst, geo, pieces, {r: t.data_ptr() for r, t in sources.items()},
                     {r: t.data_ptr() for r, t in targets.items()})
    if len(descs) == 0:
        return L.RsLaunchInfo()
    return PreparedCopies(descs, any_t.device, stream).launch(stream)


class ActivationExchange:
    """One direction of the hand-over between two adjacent stages, one process per GPU.

    Collective: every rank of `group` (default: the world) constructs it with the same arguments;
    the group must hold every rank of both stages. `shape` is the activation's local shape with
    any value at batch_dim (each rank's local batch size applies). Then, once per micro-batch, in
    the same order on every rank of the group:
      - a sending rank calls send(activation);
      - a receiving rank calls recv(target) (target is written in place and returned);
      - any other rank of the group calls exchange() (it only takes part in the ordering step).
    The roles mirror the reference's send_op / recv_op pair (pipeline_parallel.py:780-870).
    """

    def __init__(self, rank: int, mesh_src, mesh_dst, bszs_src: Sequence[int], bszs_dst: Sequence[int],
                 shape: Sequence[int], dtype: torch.dtype, batch_dim: int = 0, slice_dim: int = -1,
                 group: Optional[dist.ProcessGroup] = None, device: Optional[torch.device] = None, slots: int = 2):
        if slots < 2:
            raise ValueError("two window slots at least: a slot is reused only two exchanges later")
        self.rank, self.group, self.slots = int(rank), group, slots
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.src, self.dst = _Stage(mesh_src, bszs_src), _Stage(mesh_dst, bszs_dst)
        self.shape, self.dtype = list(shape), dtype
        nd = len(self.shape)
        self.bd, self.sd = batch_dim % nd, slice_dim % nd
        self.elem = torch.empty(0, dtype=dtype).element_size()
        self.geo = _geometry(self.shape, self.bd, self.sd, self.elem)
        self.pieces = _plan(self.src, self.dst, int(self.shape[self.sd]))
        src_bsz, dst_bsz = self.src.rank_bsz(), self.dst.rank_bsz()
        if set(src_bsz) & set(dst_bsz):
            raise AssertionError("the two stages share ranks")
        members = set(dist.get_process_group_ranks(group)) if group is not None else set(range(dist.get_world_size()))
        missing = (set(src_bsz) | set(dst_bsz)) - members
        if missing:
            raise AssertionError(f"ranks {sorted(missing)} of the two stages are not in the exchange's process group")
        self.is_sender, self.is_receiver = self.rank in src_bsz, self.rank in dst_bsz
        self.my_src_shape = _local_shape(self.shape, self.bd, src_bsz.get(self.rank, 0))
        self.my_dst_shape = _local_shape(self.shape, self.bd, dst_bsz.get(self.rank, 0))
        self._count = 0
        self._token = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._tables: Dict[Tuple[int, int], Optional[PreparedCopies]] = {}
        self._peers = _PeerMaps()
        self._window: Optional[torch.Tensor] = None
        self._slot_bytes = int(np.prod(self.my_dst_shape)) * self.elem
        mine: Dict[str, object] = {}
        if self.is_receiver:
            self._window = torch.zeros([slots, *self.my_dst_shape], dtype=dtype, device=self.device)
            handles, where = _export([self._window])
            mine = {"handle": handles[0], "offset": where[0][1], "slot_bytes": self._slot_bytes}
        everyone: List[Dict[str, object]] = [None] * dist.get_world_size(group)  # type: ignore[list-item]
        dist.all_gather_object(everyone, (self.rank, mine), group=group)
        self._remote_window: Dict[int, Tuple[int, int]] = {}  # receiver -> (window address here, slot bytes)
        if self.is_sender:
            wanted = set(int(r) for r in self.pieces["dst_rank"][self.pieces["src_rank"] == self.rank])
            with torch.cuda.device(self.device):
                for r, info in everyone:
                    if r in wanted:
                        base = self._peers.base(r, 0, info["handle"])
                        self._remote_window[r] = (base + int(info["offset"]), int(info["slot_bytes"]))
            missing = wanted - set(self._remote_window)
            if missing:
                raise AssertionError(f"receivers {sorted(missing)} did not publish a window")

    # -- per micro-batch ---------------------------------------------------------------------
    _MAX_TABLES = 64

    def _remember(self, key, descs: np.ndarray) -> Optional[PreparedCopies]:
        """Staged tables by (tensor address, slot): steady-state training reuses a few addresses.
        The oldest is dropped past _MAX_TABLES (its workspace returns to the allocator on the
        current stream, behind the launches that read it)."""
        table = PreparedCopies(descs, self.device) if len(descs) else None
        if len(self._tables) >= self._MAX_TABLES:
            self._tables.pop(next(iter(self._tables)))
        self._tables[key] = table
        return table

    def _slot(self) -> int:
        return self._count % self.slots

    def _order(self) -> None:
        """The ordering step: a one-element all-reduce, stream-ordered on every rank."""
        dist.all_reduce(self._token, group=self.group)
        self._count += 1

    def send(self, activation: torch.Tensor) -> None:
        if not self.is_sender:
            raise AssertionError(f"rank {self.rank} is not in the sending stage")
        _check_tensor(activation, self.my_src_shape, "activation")
        if activation.dtype != self.dtype:
            raise AssertionError(f"activation dtype {activation.dtype}, expected {self.dtype}")
        slot = self._slot()
        key = (activation.data_ptr(), slot)
        table = self._tables.get(key, False)
        if table is False:
            # each receiver's slot stride is its own tensor's size (published with its window)
            windows = {r: base + slot * stride for r, (base, stride) in self._remote_window.items()}
            descs = send_table(self.src, self.dst, self.geo, self.pieces, self.rank, activation.data_ptr(), windows)
            table = self._remember(key, descs)
        if table is not None:
            table.launch()
        self._order()

    def recv(self, target: torch.Tensor) -> torch.Tensor:
        if not self.is_receiver:
            raise AssertionError(f"rank {self.rank} is not in the receiving stage")
        _check_tensor(target, self.my_dst_shape, "target")
        if target.dtype != self.dtype:
            raise AssertionError(f"target dtype {target.dtype}, expected {self.dtype}")
        slot = self._slot()
        self._order()
        key = (target.data_ptr(), -1 - slot)
        table = self._tables.get(key, False)
        if table is False:
            descs = recv_table(self.dst, self.geo, self.pieces, self.rank, self._window[slot].data_ptr(), target.data_ptr())
            table = self._remember(key, descs)
        if table is not None:
            table.launch()
        return target

    def exchange(self, activation: Optional[torch.Tensor] = None, target: Optional[torch.Tensor] = None):
        """send() and/or recv() by role; a rank in neither stage only takes the ordering step."""
        if self.is_sender:
            self.send(activation)
        if self.is_receiver:
            return self.recv(target)
        if not self.is_sender:
            self._order()
        return None

    def check(self) -> None:
        """Status of every launch so far (synchronises); raises if a kernel reported an error."""
        for t in self._tables.values():
            if t is not None:
                t.check()

    def close(self) -> None:
        """Collective: unmap the peers' windows after every launch is done, then free this rank's."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._tables.clear()
        with torch.cuda.device(self.device):
            self._peers.close()
        dist.barrier(group=self.group)
        self._window = None


def get_send_op(exchange: ActivationExchange):
    """send_op(tensor) in the shape of PipelineExecModule._get_send_op (pipeline_parallel.py:840-870)."""
    def send_op(tensor: torch.Tensor) -> None:
        exchange.send(tensor.contiguous())
    return send_op


def get_recv_op(exchange: ActivationExchange):
    """recv_op(target) in the shape of PipelineExecModule._get_recv_op (pipeline_parallel.py:780-836)."""
    def recv_op(target: torch.Tensor) -> None:
        exchange.recv(target)
    return recv_op

"""CPU restatement of Suika's cross-stage activation exchange (TEST INFRASTRUCTURE ONLY; see
oracle/__init__.py).

Follows PipelineExecModule._get_recv_or_send_P2P_ops (Suika/pipeline_parallel.py:665-776), the
P2P pairing of _perform_p2pops (:503-526: sends and receives between one pair of ranks match in
issue order) and the receive side's TP all-gather (:780-836). Meshes are lists of DP groups, each
a list of ranks (a TP group), as DeviceMesh2D.to_list() gives them. Activations are numpy arrays
whose batch dim holds the rank's local batch.

Pinned by tests/golden/act_golden.json: op lists and received bytes produced by running the
reference's own generator on one gloo rank (tests/golden/make_act_golden.py).
"""
from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import numpy as np

Mesh = Sequence[Sequence[int]]


def _coord(mesh: Mesh, rank: int) -> Tuple[int, int]:
    """RawDeviceMesh2D.get_coord (Suika/device_mesh.py:170-176)."""
    for dp, group in enumerate(mesh):
        if rank in group:
            return dp, list(group).index(rank)
    raise AssertionError(f"rank {rank} not in mesh {mesh}")


def p2p_ops(rank: int, mesh_src: Mesh, mesh_dst: Mesh, bszs_src: Sequence[int], bszs_dst: Sequence[int],
            op: str) -> List[Tuple[int, int, int, int, int]]:
    """The P2P ops one rank issues, in the reference's order (pipeline_parallel.py:687-761):
    [(peer, batch offset in the rank's own tensor, batch rows, tp_deg, tp_rank)]. The block moved
    is rows [offset, offset + rows) by chunk tp_rank of tp_deg along the slice dim. op is "send"
    (rank in mesh_src) or "recv" (rank in mesh_dst)."""
    if op == "send":  # :691-693: the sender plans as a receiver with the two stages swapped
        mesh_src, mesh_dst = mesh_dst, mesh_src
        bszs_src, bszs_dst = list(bszs_dst), list(bszs_src)
    elif op != "recv":
        raise AssertionError(op)
    dst_dp, dst_tp = _coord(mesh_dst, rank)
    d = len(mesh_dst[dst_dp])
    starts_src = np.concatenate([[0], np.cumsum(bszs_src)]).astype(int)
    starts_dst = np.concatenate([[0], np.cumsum(bszs_dst)]).astype(int)
    l_dst, r_dst = int(starts_dst[dst_dp]), int(starts_dst[dst_dp + 1])
    out = []
    for src_dp in range(len(mesh_src)):
        l_src, r_src = int(starts_src[src_dp]), int(starts_src[src_dp + 1])
        lo, hi = max(l_src, l_dst), min(r_src, r_dst)
        if lo >= hi:
            continue
        s = len(mesh_src[src_dp])
        begin = dst_tp * s // d
        end = (dst_tp + 1) * s // d if s >= d else begin + 1
        for src_tp in range(begin, end):
            tp_deg, tp_rank = (s, src_tp) if s >= d else (d, dst_tp)
            out.append((int(mesh_src[src_dp][src_tp]), lo - l_dst, hi - lo, tp_deg, tp_rank))
    return out


def _block(a: np.ndarray, b0: int, nb: int, tp_deg: int, tp_rank: int, batch_dim: int, slice_dim: int):
    """target.narrow(batch_dim, b0, nb).narrow(slice_dim, tp_rank * chunk, chunk)
    (pipeline_parallel.py:748-756); a view."""
    idx = [slice(None)] * a.ndim
    idx[batch_dim] = slice(b0, b0 + nb)
    chunk = a.shape[slice_dim] // tp_deg
    idx[slice_dim] = slice(tp_rank * chunk, (tp_rank + 1) * chunk)
    return a[tuple(idx)]


def _torch_chunk(a: np.ndarray, n: int, i: int, dim: int):
    """torch.chunk(a, n, dim)[i]: ceil-sized chunks (pipeline_parallel.py:824)."""
    size = -(-a.shape[dim] // n)
    idx = [slice(None)] * a.ndim
    idx[dim] = slice(i * size, min((i + 1) * size, a.shape[dim]))
    return a[tuple(idx)]


def exchange_world(sources: Dict[int, np.ndarray], targets: Dict[int, np.ndarray], mesh_src: Mesh, mesh_dst: Mesh,
                   bszs_src: Sequence[int], bszs_dst: Sequence[int], batch_dim: int = 0, slice_dim: int = -1) -> None:
    """Run one exchange on numpy arrays: every sender's sends, every receiver's receives, paired in
    issue order per (sender, receiver), then each receiving TP group's all-gather. targets are
    filled in place (rows no sender covers keep their values)."""
    nd = next(iter(targets.values())).ndim if targets else 0
    bd, sd = batch_dim % nd if nd else 0, slice_dim % nd if nd else 0
    queues: Dict[Tuple[int, int], List[np.ndarray]] = {}
    for group in mesh_src:
        for r in group:
            for peer, b0, nb, deg, tr in p2p_ops(r, mesh_src, mesh_dst, bszs_src, bszs_dst, "send"):
                # transmit_tensor = block.contiguous() (:754)
                queues.setdefault((r, peer), []).append(np.ascontiguousarray(_block(sources[r], b0, nb, deg, tr, bd, sd)))
    for group in mesh_dst:
        for r in group:
            for peer, b0, nb, deg, tr in p2p_ops(r, mesh_src, mesh_dst, bszs_src, bszs_dst, "recv"):
                q = queues.get((peer, r))
                assert q, f"receive of rank {r} from {peer} has no matching send"
                blk = _block(targets[r], b0, nb, deg, tr, bd, sd)
                sent = q.pop(0)
                assert sent.shape == blk.shape, (sent.shape, blk.shape)
                blk[...] = sent  # restore_transmit_tensor (:755-756)
    assert all(not q for q in queues.values()), "sends without a matching receive"
    for group in mesh_dst:  # TP all-gather of each receiving group (:817-832)
        d = len(group)
        if d == 1:
            continue
        parts = [np.array(_torch_chunk(targets[r], d, j, sd)) for j, r in enumerate(group)]
        full = np.concatenate(parts, axis=sd)
        for r in group:
            targets[r][...] = full


def provenance(mesh_src: Mesh, mesh_dst: Mesh, bszs_src: Sequence[int], bszs_dst: Sequence[int],
               slice_size: int) -> List[Tuple[int, int, int, int, int, int, int]]:
    """Where each received block comes from after the all-gather, in rs_act_plan's order:
    [(src_rank, dst_rank, src_batch, dst_batch, n_batch, slice_start, slice_len)]."""
    out = []
    starts_src = np.concatenate([[0], np.cumsum(bszs_src)]).astype(int)
    starts_dst = np.concatenate([[0], np.cumsum(bszs_dst)]).astype(int)
    for dst_dp, group in enumerate(mesh_dst):
        for r in group:
            per_src: Dict[int, List] = {}
            # every member of the group ends with the union of the members' P2P blocks
            for member in group:
                for peer, b0, nb, deg, tr in p2p_ops(member, mesh_src, mesh_dst, bszs_src, bszs_dst, "recv"):
                    src_dp, _ = _coord(mesh_src, peer)
                    chunk = slice_size // deg
                    lo_global = b0 + int(starts_dst[dst_dp])
                    per_src.setdefault(src_dp, []).append(
                        (peer, r, lo_global - int(starts_src[src_dp]), b0, nb, tr * chunk, chunk))
            for src_dp in sorted(per_src):
                out.extend(sorted(per_src[src_dp], key=lambda p: p[5]))
    return out

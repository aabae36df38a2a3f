"""DP-replica fan-out for the push direction of a reshard.

When several target ranks are DP replicas of the same tensor (a DP grow, or a TP shrink into
DP > 1), the reference has every replica receive every piece from a source rank
(Suika/migration.py:355-379 picks one owner per replica and piece), so a source shard may leave
its GPU once per replica. With fan-out:
  - stage 1: one replica per tensor, the leader, receives the pieces from the sources;
  - stage 2: the leader forwards the assembled tensor (every normal sub-field) to the other
    replicas, its followers, in phases in which every GPU sends to at most one peer and receives
    from at most one.
Leaders rotate over the tensors of a replica group, so stage 2 is an exchange among replicas and
each source sends a tensor's pieces once.

Forwarding is exact only where the follower would have assembled the same bytes:
  - its pieces come from the same source pieces (the same source TP coordinates, read from any DP
    replica of the source; replicas of a synchronised DP job hold the same state), and
  - they sit in the same positions (in the reference's cat order, received pieces come before the
    rank's own, so a replica that owns a piece of the tensor itself assembles a different order).
Replicas that own a piece of the tensor keep their direct pieces and are never followers.

`plan_fanout(plan, bytes_per_elem, mode)` decides. Its cost model is the sum over phases of the
largest pair's bytes (each GPU talks to one peer per direction within a phase). mode "auto" keeps
fan-out only when that sum drops; True forces it wherever it is exact; False turns it off.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Set, Tuple

import numpy as np

from . import _lib as L


@dataclass
class FanOut:
    # (follower rank, name_id) -> (rank it receives the tensor from, broadcast round)
    forward: Dict[Tuple[int, int], Tuple[int, int]] = field(default_factory=dict)
    phase1: Dict[Tuple[int, int], int] = field(default_factory=dict)        # stage-1 (source, target) -> phase
    n1: int = 1
    phase2: Dict[Tuple[int, int, int], int] = field(default_factory=dict)   # (sender, follower, round) -> phase of stage 2
    n2: int = 0
    est_direct: int = 0    # cost model, in bytes: sum over phases of the largest pair
    est_fanout: int = 0

    @property
    def n_phases(self) -> int:
        return self.n1 + self.n2

    @property
    def active(self) -> bool:
        return bool(self.forward)

    def forwarded_names(self, follower: int) -> Set[int]:
        return {n for (f, n) in self.forward if f == follower}

    def children_of(self, rank: int) -> Dict[Tuple[int, int], List[int]]:
        """{(follower, round): [name_id]} of the tensors `rank` forwards in stage 2."""
        out: Dict[Tuple[int, int], List[int]] = {}
        for (f, n), (p, r) in sorted(self.forward.items()):
            if p == rank:
                out.setdefault((f, r), []).append(n)
        return out

    def stage1_mask(self, ops: np.ndarray) -> np.ndarray:
        """Ops that stage 1 still carries (False: the target gets that tensor in stage 2)."""
        if not self.forward:
            return np.ones(len(ops), bool)
        drop = np.array([(int(d), int(n)) in self.forward for d, n in zip(ops["dst_rank"], ops["name_id"])], bool)
        return ~drop


def _phases_cost(pairs: Dict[Tuple[int, int], int]) -> Tuple[Dict[Tuple[int, int], int], int, int]:
    from .migration import transfer_phases
    if not pairs:
        return {}, 0, 0
    col = transfer_phases(pairs)
    n = max(col.values()) + 1
    worst = [0] * n
    for p, c in col.items():
        worst[c] = max(worst[c], pairs[p])
    return col, n, sum(worst)


def _signature(ops: np.ndarray, idx: np.ndarray, semantic: bool) -> tuple:
    """The pieces of one (target rank, tensor) in the order they are written."""
    sig = [(int(ops["src_slice_dim"][i]), int(ops["src_tp_index"][i]), int(ops["src_tp_deg"][i]),
            int(ops["dst_slice_dim"][i]), int(ops["dst_tp_index"][i]), int(ops["dst_tp_deg"][i])) for i in idx]
    if semantic:
        return tuple(sorted(sig, key=lambda s: (s[4], s)))
    self_op = [int(ops["src_rank"][i]) == int(ops["dst_rank"][i]) for i in idx]
    # the reference's cat order: received pieces in op order, then the rank's own (migration.py:448-509)
    return tuple([s for s, me in zip(sig, self_op) if not me] + [s for s, me in zip(sig, self_op) if me])


def plan_fanout(plan, bytes_per_elem: int, mode="auto") -> FanOut:
    """Leaders, broadcast trees and the phases of both stages for every replicated target tensor.

    Within a group of exact replicas, the leader is the member that holds most of the tensor
    already (its own pieces cost no NVLink); ties rotate over the tensors. Followers get the
    tensor along a binomial tree: in round r every member that holds it sends it to one that does
    not, so k replicas are served in ceil(log2 k) rounds."""
    ops = plan.op_array
    remote = ops["src_rank"] != ops["dst_rank"]
    nbytes = ops["numel"].astype(np.int64) * int(bytes_per_elem)

    def pairs_of(mask) -> Dict[Tuple[int, int], int]:
        pr: Dict[Tuple[int, int], int] = {}
        for s, t, b in zip(ops["src_rank"][mask], ops["dst_rank"][mask], nbytes[mask]):
            pr[(int(s), int(t))] = pr.get((int(s), int(t)), 0) + int(b)
        return pr

    col0, n0, cost0 = _phases_cost(pairs_of(remote))
    direct = FanOut(phase1=col0, n1=max(n0, 1), est_direct=cost0, est_fanout=cost0)
    if mode is False:
        return direct
    semantic = plan.order == "semantic"
    # group every (target rank, tensor) by the target's meta: DP replicas share name, shape, tp_meta
    by_key: Dict[tuple, List[int]] = {}
    rows: Dict[Tuple[int, int], np.ndarray] = {}
    order = np.lexsort((np.arange(len(ops)), ops["name_id"], ops["dst_rank"]))
    d_sorted, n_sorted = ops["dst_rank"][order], ops["name_id"][order]
    starts = np.flatnonzero(np.r_[True, (d_sorted[1:] != d_sorted[:-1]) | (n_sorted[1:] != n_sorted[:-1])]) if len(order) else []
    bounds = np.r_[starts, len(order)]
    for a, b in zip(bounds[:-1], bounds[1:]):
        idx = np.sort(order[a:b])  # op order within the (rank, tensor)
        t, n = int(ops["dst_rank"][idx[0]]), int(ops["name_id"][idx[0]])
        rows[(t, n)] = idx
        meta = plan.tpl.layout[t][plan.names[n]]
        tp = tuple(meta.tp_meta) if meta.tp_meta is not None else None
        by_key.setdefault((n, tuple(int(x) for x in meta.shape), tp), []).append(t)
    # broadcast groups: tensors with the same leader and followers travel together along one tree
    groups: Dict[Tuple[int, Tuple[int, ...]], List[int]] = {}
    turn = 0
    for (n, _shape, _tp), members in sorted(by_key.items()):
        if len(members) < 2:
            continue
        classes: Dict[tuple, List[int]] = {}
        for t in sorted(members):
            classes.setdefault(_signature(ops, rows[(t, n)], semantic), []).append(t)
        for cls in classes.values():
            if len(cls) < 2:
                continue
            local = {t: int(nbytes[rows[(t, n)]][~remote[rows[(t, n)]]].sum()) for t in cls}
            best = max(local.values())
            cands = [t for t in cls if local[t] == best]
            leader = cands[turn % len(cands)]
            turn += 1
            followers = tuple(t for t in cls if t != leader and local[t] == 0)
            if followers:
                groups.setdefault((leader, followers), []).append(n)
    if not groups:
        return direct
    forward: Dict[Tuple[int, int], Tuple[int, int]] = {}
    round_pairs: Dict[int, Dict[Tuple[int, int], int]] = {}
    for (leader, followers), names in sorted(groups.items()):
        size = {f: sum(int(nbytes[rows[(f, n)]].sum()) for n in names) for f in followers}
        holders, pending, r = [leader], list(followers), 0
        while pending:
            new = []
            for h in holders:
                if not pending:
                    break
                f = pending.pop(0)
                for n in names:
                    forward[(f, n)] = (h, r)
                rp = round_pairs.setdefault(r, {})
                rp[(h, f)] = rp.get((h, f), 0) + size[f]
                new.append(f)
            holders += new
            r += 1
    fo = FanOut(forward=forward)
    keep = fo.stage1_mask(ops)
    col1, n1, cost1 = _phases_cost(pairs_of(remote & keep))
    phase2: Dict[Tuple[int, int, int], int] = {}
    n2 = cost2 = 0
    for r in sorted(round_pairs):  # rounds in order; each round coloured into matchings
        col, n, cost = _phases_cost(round_pairs[r])
        for (h, f), c in col.items():
            phase2[(h, f, r)] = n2 + c
        n2 += n
        cost2 += cost
    fo.phase1, fo.n1, fo.phase2, fo.n2 = col1, max(n1, 1), phase2, n2
    fo.est_direct, fo.est_fanout = cost0, cost1 + cost2
    if mode == "auto" and fo.est_fanout >= fo.est_direct:
        return direct
    return fo


def forward_table(leader_prog, leader_base: int, leader_off: np.ndarray, follower_prog, follower_base: int,
                  follower_off: np.ndarray, follower_nb: np.ndarray, names: Sequence[int]) -> np.ndarray:
    """COPY_DESC entries a leader writes in stage 2: for every normal sub-field slot of `names`, its
    own assembled target (leader_base + leader_off[slot]) into the follower's slot of the same
    tensor and sub-field."""
    want = set(int(n) for n in names)
    fslot = {(int(s["name_id"]), int(s["subfield"])): i for i, s in enumerate(follower_prog.dst_slots)}
    out = []
    for i, s in enumerate(leader_prog.dst_slots):
        key = (int(s["name_id"]), int(s["subfield"]))
        if key[0] not in want:
            continue
        j = fslot.get(key)
        if j is None or int(follower_nb[j]) != int(s["nbytes"]):
            raise AssertionError(f"follower slot for tensor {key[0]} sub-field {key[1]} missing or of another size")
        nb = int(s["nbytes"])
        if nb:
            out.append((leader_base + int(leader_off[i]), follower_base + int(follower_off[j]), 1, nb, nb, nb, L.RS_COPY_REMOTE))
    return np.array(out, dtype=L.COPY_DESC_DTYPE) if out else np.zeros(0, dtype=L.COPY_DESC_DTYPE)


def stage1_keep(prog, rank: int, forwarded: Set[int]) -> np.ndarray:
    """Mask over the entries rs_program_resolve_from(prog, rank) returns (the segments of a
    target's program whose source is `rank`, in segment order): False for a tensor the target
    receives from its leader instead."""
    seg = prog.segments
    if len(seg) == 0:
        return np.zeros(0, bool)
    src_rank = prog.src_slots["src_rank"][seg["src_slot"]]
    mine = seg[src_rank == rank]
    if not forwarded:
        return np.ones(len(mine), bool)
    names = prog.dst_slots["name_id"][mine["dst_slot"]]
    return ~np.isin(names, np.array(sorted(forwarded), dtype=names.dtype))

"""Activation hand-over between pipeline stages, on the CPU:
  - the oracle (oracle/activation.py) against the reference's own op lists and received bytes
    (tests/golden/act_golden.json, made by tests/golden/make_act_golden.py);
  - the C planner (rs_act_plan) against the oracle's provenance of every received block;
  - the copy descriptors (rs_act_resolve), applied to emulated memory, against the golden bytes:
    the one-device table, and the two tables of the one-process-per-GPU protocol (sender ->
    receiver window, window -> receiver tensor);
  - the planner's errors."""
import json
import os

import numpy as np
import pytest

from oracle import activation as OA
from suika_b200 import activation as A
from suika_b200 import _lib as L
from tests.golden.act_cases import ACT_CASES, source_arrays, zero_targets
from tests.helpers import GOLDEN_DIR, Memory, digest

with open(os.path.join(GOLDEN_DIR, "act_golden.json")) as _f:
    GOLDEN = json.load(_f)


def _sd(case):
    return case["slice_dim"] % len(case["shape"])


def _slice_size(case):
    return case["shape"][_sd(case)]


def _apply(mem: Memory, descs: np.ndarray) -> None:
    mem.apply(descs)


def test_golden_covers_every_case():
    assert set(GOLDEN) == set(ACT_CASES)


@pytest.mark.parametrize("name", sorted(ACT_CASES))
def test_oracle_op_lists_match_reference(name):
    case, g = ACT_CASES[name], GOLDEN[name]
    sd, bd = _sd(case), case["batch_dim"] % len(case["shape"])
    for r_s, ops in g["ops"].items():
        r = int(r_s)
        kind = "send" if "send" in ops else "recv"
        mine = OA.p2p_ops(r, case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"], kind)
        assert [p for p, *_ in mine] == [p for p, _ in ops[kind]], (r, kind)
        for (peer, b0, nb, deg, tr), (_, shape) in zip(mine, ops[kind]):
            assert shape[bd] == nb and shape[sd] == case["shape"][sd] // deg, (r, peer, shape)


@pytest.mark.parametrize("name", sorted(ACT_CASES))
def test_oracle_exchange_matches_reference_bytes(name):
    case, g = ACT_CASES[name], GOLDEN[name]
    tg = zero_targets(case)
    OA.exchange_world(source_arrays(case), tg, case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"],
                      case["batch_dim"], case["slice_dim"])
    assert {str(r): digest(a) for r, a in tg.items()} == g["digests"]


@pytest.mark.parametrize("name", sorted(ACT_CASES))
def test_planner_matches_oracle_provenance(name):
    case = ACT_CASES[name]
    got = A.plan_activation_exchange(case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"], _slice_size(case))
    want = OA.provenance(case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"], _slice_size(case))
    assert [tuple(int(x) for x in p) for p in got] == want


def _stages(case):
    return A._Stage(case["mesh_src"], case["bszs_src"]), A._Stage(case["mesh_dst"], case["bszs_dst"])


def _geo(case, itemsize):
    return A._geometry(case["shape"], case["batch_dim"], case["slice_dim"], itemsize)


@pytest.mark.parametrize("name", sorted(ACT_CASES))
def test_one_device_table_rebuilds_reference_bytes(name):
    case, g = ACT_CASES[name], GOLDEN[name]
    src, dst = _stages(case)
    srcs, tgts = source_arrays(case), zero_targets(case)
    mem = Memory()
    sa = {r: mem.add(a.reshape(-1).view(np.uint8)) for r, a in srcs.items()}
    da = {r: mem.add(a.reshape(-1).view(np.uint8)) for r, a in tgts.items()}
    pieces = A._plan(src, dst, _slice_size(case))
    _apply(mem, A._resolve(src, dst, _geo(case, srcs[next(iter(srcs))].itemsize), pieces, sa, da))
    assert {str(r): digest(a) for r, a in tgts.items()} == g["digests"]


@pytest.mark.parametrize("name", sorted(ACT_CASES))
def test_window_protocol_tables_rebuild_reference_bytes(name):
    """Senders write into receivers' window slots (their tables only), then each receiver copies
    its blocks from the window into its tensor; run twice into the two slots."""
    case, g = ACT_CASES[name], GOLDEN[name]
    src, dst = _stages(case)
    srcs = source_arrays(case)
    geo = _geo(case, srcs[next(iter(srcs))].itemsize)
    pieces = A._plan(src, dst, _slice_size(case))
    mem = Memory()
    sa = {r: mem.add(a.reshape(-1).view(np.uint8)) for r, a in srcs.items()}
    for slot in range(2):
        windows = {r: np.full((2, *a.shape), 7, dtype=a.dtype) for r, a in zero_targets(case).items()}
        wa = {r: mem.add(w.reshape(-1).view(np.uint8)) for r, w in windows.items()}
        slot_bytes = {r: w[0].nbytes for r, w in windows.items()}
        for r in srcs:
            _apply(mem, A.send_table(src, dst, geo, pieces, r, sa[r], {q: wa[q] + slot * slot_bytes[q] for q in wa}))
        tgts = zero_targets(case)
        for r, t in tgts.items():
            ta = mem.add(t.reshape(-1).view(np.uint8))
            _apply(mem, A.recv_table(dst, geo, pieces, r, wa[r] + slot * slot_bytes[r], ta))
        assert {str(r): digest(a) for r, a in tgts.items()} == g["digests"], slot


def test_planner_rejects_non_power_of_two_tp():
    with pytest.raises(AssertionError, match="powers of two"):
        A.plan_activation_exchange([[0, 1, 2]], [[3, 4]], [4], [4], 12)


def test_planner_rejects_indivisible_slice():
    with pytest.raises(AssertionError, match="does not divide"):
        A.plan_activation_exchange([[0, 1, 2, 3]], [[4]], [2], [2], 6)


def test_resolve_rejects_out_of_range_pieces():
    src, dst = A._Stage([[0]], [2]), A._Stage([[1]], [2])
    geo = A._geometry([2, 4], 0, 1, 4)
    bad = np.zeros(1, dtype=L.ACT_PIECE_DTYPE)
    bad[0] = (0, 1, 1, 0, 2, 0, 4)  # rows 1..3 of a 2-row source
    with pytest.raises(L.ReshardError, match="leaves its tensors"):
        A._resolve(src, dst, geo, bad, {0: 1 << 20}, {1: 1 << 21})


def test_resolve_needs_every_address():
    src, dst = A._Stage([[0]], [2]), A._Stage([[1]], [2])
    pieces = A._plan(src, dst, 4)
    with pytest.raises(L.ReshardError, match="address"):
        A._resolve(src, dst, A._geometry([2, 4], 0, 1, 4), pieces, {0: 1 << 20}, {})


def test_mesh_from_reference_object():
    class Raw:  # what RawDeviceMesh2D.to_list() hands over
        def to_list(self):
            return [[0, 1], [2, 3]]
    assert A.mesh_lists(Raw()) == [[0, 1], [2, 3]]


def _random_stage(rng, first_rank):
    groups, r = [], first_rank
    for _ in range(int(rng.integers(1, 4))):
        tp = int(rng.choice([1, 2, 4]))
        groups.append(list(range(r, r + tp)))
        r += tp
    bszs = [int(rng.integers(0, 4)) for _ in groups]
    return groups, bszs, r


def random_act_cases(n=40, seed=77):
    rng = np.random.default_rng(seed)
    out = []
    while len(out) < n:
        ms, bs, nxt = _random_stage(rng, 0)
        md, bd, _ = _random_stage(rng, nxt)
        nd = int(rng.integers(2, 5))
        batch_dim, slice_dim = (int(x) for x in rng.choice(nd, size=2, replace=False))
        shape = [int(rng.integers(1, 4)) for _ in range(nd)]
        shape[slice_dim] = 4 * int(rng.integers(1, 4))  # divisible by every TP degree used
        shape[batch_dim] = -1
        out.append(dict(mesh_src=ms, bszs_src=bs, mesh_dst=md, bszs_dst=bd, shape=shape, batch_dim=batch_dim,
                        slice_dim=slice_dim, dtype="float32"))
    return out


@pytest.mark.parametrize("k", range(40))
def test_random_exchanges_match_the_oracle(k):
    """Seeded random stage pairs (DP groups of unequal TP, empty and uneven batches, 2-4 dims, any
    batch / slice dim): the one-device table equals the oracle's exchange."""
    case = random_act_cases()[k]
    src, dst = _stages(case)
    srcs, tgts = source_arrays(case, seed=k), zero_targets(case)
    want = zero_targets(case)
    OA.exchange_world(srcs, want, case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"],
                      case["batch_dim"], case["slice_dim"])
    mem = Memory()
    sa = {r: mem.add(a.reshape(-1).view(np.uint8)) for r, a in srcs.items()}
    da = {r: mem.add(a.reshape(-1).view(np.uint8)) for r, a in tgts.items()}
    pieces = A._plan(src, dst, _slice_size(case))
    assert [tuple(int(x) for x in p) for p in pieces] == OA.provenance(case["mesh_src"], case["mesh_dst"], case["bszs_src"],
                                                                         case["bszs_dst"], _slice_size(case))
    _apply(mem, A._resolve(src, dst, _geo(case, 4), pieces, sa, da))
    for r in tgts:
        assert np.array_equal(tgts[r], want[r]), r


def _turns(pieces):
    """For each sender, its receivers in send order (one entry per receiver, first visit)."""
    out = {}
    for s in sorted(set(pieces["src_rank"].tolist())):
        seen = []
        for r in A.rotated_pieces(pieces, s)["dst_rank"].tolist():
            if r not in seen:
                seen.append(int(r))
        out[s] = seen
    return out


@pytest.mark.parametrize("k", range(40))
def test_rotated_send_order_is_a_permutation(k):
    """rotated_pieces only reorders: each sender keeps exactly its own pieces, and the pieces of
    one receiver stay together in their planner order."""
    case = random_act_cases()[k]
    src, dst = _stages(case)
    pieces = A._plan(src, dst, _slice_size(case))
    for s in set(pieces["src_rank"].tolist()):
        mine = pieces[pieces["src_rank"] == s]
        rot = A.rotated_pieces(pieces, s)
        assert sorted(map(tuple, rot.tolist())) == sorted(map(tuple, mine.tolist()))
        for r in set(mine["dst_rank"].tolist()):
            assert rot[rot["dst_rank"] == r].tolist() == mine[mine["dst_rank"] == r].tolist()
        firsts = [i for i, r in enumerate(rot["dst_rank"].tolist()) if i == 0 or rot["dst_rank"][i - 1] != r]
        assert len(firsts) == len(set(rot["dst_rank"].tolist())), "a receiver's pieces are split"


@pytest.mark.parametrize("tp", [2, 4])
def test_rotated_send_order_gives_each_receiver_one_writer(tp):
    """A TP group handing over to as many DP ranks, and back: at every turn of the send order
    each receiver is written by exactly one sender (the stage pairs of bench.py --activation)."""
    ma, mb = [list(range(tp))], [[tp + i] for i in range(tp)]
    ba, bb = [8], [8 // tp] * tp
    for ms, md, bs, bd in ((ma, mb, ba, bb), (mb, ma, bb, ba)):
        pieces = A.plan_activation_exchange(ms, md, bs, bd, 5120)
        turns = _turns(pieces)
        for t in range(tp):
            assert sorted(order[t] for order in turns.values()) == sorted(set(pieces["dst_rank"].tolist())), (ms, md, turns)

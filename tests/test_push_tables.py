"""The push direction's copy tables, executed on the CPU against emulated memory: every rank's
tables (built by the same function RankTransferPush uses) applied to numpy buffers must rebuild
the reference's targets (tests/golden digests). Covers the table logic of RankTransferPush without
GPUs or IPC, with and without DP-replica fan-out (suika_b200/fanout.py): with fan-out, stage 1
runs first, then stage 2's phases in order, each phase a matching."""
import numpy as np
import pytest

from suika_b200 import migration as M
from suika_b200.fanout import plan_fanout
from tests.golden.cases import CASES
from tests.helpers import SUB_ITEMSIZE, SUBS, Memory, digest, golden_states, load_golden

SPEC = [(SUB_ITEMSIZE[s], kind == "meta") for s, kind in SUBS]
SUBNAMES = [s for s, _ in SUBS]


def _apply(mem: Memory, table: np.ndarray) -> None:
    mem.apply(table)


def run_push(case, fanout=False):
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    plan = M.Plan(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    fo = plan_fanout(plan, 1, mode=True) if fanout else None
    mem = Memory()
    src_addr = {}
    for r, st in states.items():
        for name, ent in st.items():
            for sub, a in ent.items():
                b = np.ascontiguousarray(a).reshape(-1).view(np.uint8).copy()
                src_addr[(r, name, sub)] = (mem.add(b), b.nbytes)
    arenas, progs = {}, {}
    for T, metas in tpl.layout.items():
        if not metas:
            continue
        progs[T] = plan.program(T, SPEC)
        off, nb, total = M._arena_layout(progs[T].dst_slots)
        arr = np.full(max(total, 1), 0xAB, dtype=np.uint8)
        arenas[T] = (mem.add(arr), off, nb)
    ops = plan.op_array
    stage2 = []
    for rank in sorted(set(int(x) for x in ops["src_rank"]) | set(arenas)):
        t1, peer, s2 = M._push_rank_tables(plan, rank, SPEC, SUBNAMES, lambda n, s, r=rank: src_addr[(r, n, s)],
                                           lambda T: arenas[T][0], lambda T: arenas[T][1], lambda T: arenas[T][2],
                                           progs.get(rank), fo)
        _apply(mem, t1)
        for (F, rnd), d in s2.items():
            stage2.append((fo.phase2[(rank, F, rnd)], rank, F, d))
    if fo is not None:
        for k in range(fo.n2):  # phases in order: a later round reads what an earlier one wrote
            in_phase = [(s, f) for p, s, f, _ in stage2 if p == k]
            assert len({s for s, _ in in_phase}) == len(in_phase) and len({f for _, f in in_phase}) == len(in_phase), in_phase
            for p, _s, _f, d in stage2:
                if p == k:
                    _apply(mem, d)
    return g, plan, progs, arenas, mem, fo


def _check(case, fanout):
    g, plan, progs, arenas, mem, fo = run_push(case, fanout)
    for rank_s, want in g["ranks"].items():
        T = int(rank_s)
        base, off, nb = arenas[T]
        got = {}
        for ds, o, n in zip(progs[T].dst_slots, off, nb):
            got[(plan.names[ds["name_id"]], SUBNAMES[ds["subfield"]])] = mem.view(base + int(o), int(n))
        for name, fields in want["digests"].items():
            for sub, (shape, _dt, sha) in fields.items():
                if sub == "step":
                    continue
                assert digest(got[(name, sub)]) == sha, (rank_s, name, sub)
    return fo


@pytest.mark.parametrize("case", ["odd_mini", "cfg2b_mini", "cfg3_mini", "cfg4_mini", "shrink_mini", "hetero_mini",
                                  "pp_deepen_mini", "gpt_shrink_mini", "grow_dp_tp_mini", "qwen_grow_mini"])
def test_push_tables_rebuild_reference_targets(case):
    _check(case, fanout=False)


@pytest.mark.parametrize("case", ["cfg2_mini", "cfg4_mini", "cfg5_mini", "hetero_mini", "shrink_mini", "grow_dp_tp_mini"])
def test_fanout_tables_rebuild_reference_targets(case):
    """Forced fan-out (every exact replica forwarded): still the reference's bytes everywhere."""
    fo = _check(case, fanout=True)
    assert fo.active and fo.n2 >= 1

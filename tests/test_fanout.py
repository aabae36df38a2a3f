"""DP-replica fan-out planning (suika_b200/fanout.py), on the CPU: where it applies and what its
cost model decides, the broadcast trees' shape, the switch of the drop-in, and a DP grow x4 run
through the push tables on emulated memory against the oracle."""
import math

import numpy as np
import pytest

from oracle import restate as O
from suika_b200 import migration as M
from suika_b200 import synthetic as S
from suika_b200.fanout import plan_fanout
from suika_b200.layouts import CONFIGS, SPECS, ReshardConfig, scaled_spec
from tests.helpers import SUB_META, SUBS, Memory
from tests.test_push_tables import SPEC, SUBNAMES, _apply

STATE_BYTES = 14  # bf16 param + fp32 master, m, v per element


def _plan(src, dst, spec=SPECS["llama2-7b"], order="reference"):
    spl, tpl = ReshardConfig("t", spec, src, dst).layouts()
    return spl, tpl, M.Plan(spl, tpl, order=order, minimum_est_peers=1)


def _emulate_push(plan, tpl, states, fo):
    """Both stages of a push transfer on emulated memory: every rank's stage-1 table, then the
    stage-2 phases in order. Returns (memory, arenas, programs)."""
    mem = Memory()
    src_addr = {}
    for r, st in states.items():
        for name, ent in st.items():
            for sub, a in ent.items():
                b = np.ascontiguousarray(a).reshape(-1).view(np.uint8).copy()
                src_addr[(r, name, sub)] = (mem.add(b), b.nbytes)
    arenas, progs = {}, {}
    for T in tpl.layout:
        progs[T] = plan.program(T, SPEC)
        off, nb, total = M._arena_layout(progs[T].dst_slots)
        arenas[T] = (mem.add(np.full(max(total, 1), 0xAB, dtype=np.uint8)), off, nb)
    stage2 = []
    for rank in sorted(arenas):
        t1, _peer, s2 = M._push_rank_tables(plan, rank, SPEC, SUBNAMES, lambda n, s, r=rank: src_addr[(r, n, s)],
                                            lambda T: arenas[T][0], lambda T: arenas[T][1], lambda T: arenas[T][2],
                                            progs[rank], fo)
        _apply(mem, t1)
        stage2 += [(fo.phase2[(rank, F, rnd)], d) for (F, rnd), d in s2.items()]
    for k in range(fo.n2):
        for p, d in stage2:
            if p == k:
                _apply(mem, d)
    return mem, arenas, progs


def test_auto_keeps_direct_transfers_on_the_baseline_reshards():
    """On cfg2-cfg5 no source sends more than the busiest target receives: fan-out cannot help."""
    for c in ("cfg2", "cfg3", "cfg4", "cfg5"):
        spl, tpl = CONFIGS[c].layouts()
        fo = plan_fanout(M.Plan(spl, tpl, minimum_est_peers=1), STATE_BYTES, "auto")
        assert not fo.active, c


def test_auto_fans_out_a_dp_grow_by_eight():
    _, _, plan = _plan([[[0]]], [[[i] for i in range(8)]])
    fo = plan_fanout(plan, STATE_BYTES, "auto")
    assert fo.active
    assert fo.est_fanout * 2 < fo.est_direct  # 7 sends of the state from one GPU vs a 3-round tree
    rounds = {r for (_f, _n), (_p, r) in fo.forward.items()}
    assert rounds == {0, 1, 2}  # ceil(log2 8) rounds
    # every follower gets each tensor exactly once, from a rank that holds it by then
    holders = {}
    for (f, n), (p, r) in sorted(fo.forward.items(), key=lambda kv: kv[1][1]):
        assert p == 0 or holders.get((p, n), math.inf) < r, (f, n, p, r)
        holders[(f, n)] = r


def test_mode_false_and_no_replicas_mean_direct():
    _, _, plan = _plan([[[0]]], [[[i] for i in range(4)]])
    assert not plan_fanout(plan, STATE_BYTES, False).active
    spl, tpl = CONFIGS["cfg3"].layouts()  # no DP replicas among the targets
    assert not plan_fanout(M.Plan(spl, tpl, minimum_est_peers=1), STATE_BYTES, True).active


def test_replicas_that_own_a_piece_are_never_followers():
    """cfg5's TP4 -> TP2 x DP2: a target that was a source assembles its own piece last in the
    reference's cat order, so its bytes differ from its replica's and it keeps direct pieces."""
    spl, tpl = CONFIGS["cfg5"].layouts()
    plan = M.Plan(spl, tpl, minimum_est_peers=1)
    fo = plan_fanout(plan, STATE_BYTES, True)
    ops = plan.op_array
    for (f, n) in fo.forward:
        mine = (ops["dst_rank"] == f) & (ops["name_id"] == n)
        assert not np.any(ops["src_rank"][mine] == f)


@pytest.mark.parametrize("order", ["reference", "semantic"])
def test_dp_grow_tables_with_fanout_match_the_oracle(order):
    spec = scaled_spec(SPECS["llama2-7b"], name="grow", hidden=64, n_layers=2, n_heads=4, ffn=128, vocab=96)
    spl, tpl, plan = _plan([[[0, 1]]], [[[0, 1], [2, 3], [4, 5], [6, 7]]], spec, order)  # TP2 x DP1 -> TP2 x DP4
    fo = plan_fanout(plan, STATE_BYTES, True)
    assert fo.active
    states = S.host_states(spl, SUBS, seed=11, distinct_steps=True)
    mem, arenas, progs = _emulate_push(plan, tpl, states, fo)
    ops = O.schedule(spl, tpl, minimum_est_peers=1)
    for T in tpl.layout:
        want = O.execute_rank(ops, states, SUB_META, T, order=order)
        base, off, nb = arenas[T]
        for ds, o, n in zip(progs[T].dst_slots, off, nb):
            name, sub = plan.names[ds["name_id"]], SUBNAMES[ds["subfield"]]
            if sub == "step":
                continue
            got = mem.view(base + int(o), int(n))
            assert np.array_equal(got, want[name][sub].reshape(-1).view(np.uint8)), (T, name, sub)


def test_fanout_switch_values():
    assert M._fanout_setting("0") is False and M._fanout_setting("") is False
    assert M._fanout_setting(" AUTO ") == "auto" and M._fanout_setting("1") is True
    with pytest.raises(ValueError, match="SUIKA_RESHARD_FANOUT"):
        M._fanout_setting("yes")


def test_fanout_on_an_interval_plan_equals_reslice():
    """GQA with fused QKV and vocab-parallel wte (interval planner), TP4 -> TP2 x DP2 with forced
    fan-out: every target equals the re-sliced full tensor."""
    from tests.test_extension_layouts import EXT_CASES
    cfg = EXT_CASES["gqa_rep_src"]
    spl, tpl = cfg.layouts()
    plan = M.Plan(spl, tpl)
    assert plan.mode == "interval"
    fo = plan_fanout(plan, STATE_BYTES, True)
    assert fo.active
    states = S.host_states(spl, SUBS, seed=3, distinct_steps=True)
    mem, arenas, progs = _emulate_push(plan, tpl, states, fo)
    for T in tpl.layout:
        want = O.semantic_target(states, spl, tpl, SUB_META, T)
        base, off, nb = arenas[T]
        for ds, o, n in zip(progs[T].dst_slots, off, nb):
            name, sub = plan.names[ds["name_id"]], SUBNAMES[ds["subfield"]]
            assert np.array_equal(mem.view(base + int(o), int(n)), want[name][sub].reshape(-1).view(np.uint8)), (T, name, sub)

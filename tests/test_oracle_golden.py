"""The CPU oracle restates the reference: checked against digests of the reference's own run
(tests/golden/*.json, made by tests/golden/make_golden.py on CPU/gloo ranks)."""
import pytest

from oracle import restate as O
from tests.golden.cases import CASES
from tests.helpers import SUB_META, digest, golden_states, load_golden, schedule_as_lists

NAMES = sorted(CASES)


@pytest.mark.parametrize("case", NAMES)
def test_oracle_schedule_matches_reference(case):
    g = load_golden(case)
    spl, tpl = CASES[case]["config"].layouts()
    ops = O.schedule(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    assert schedule_as_lists(ops) == g["schedule"]


@pytest.mark.parametrize("case", NAMES)
def test_oracle_execute_matches_reference(case):
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    ops = O.schedule(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    for rank_s, want in g["ranks"].items():
        got = O.execute_rank(ops, states, SUB_META, int(rank_s), order="reference")
        assert list(got) == want["order"]
        for name, fields in want["digests"].items():
            for sub, (shape, _dtype, sha) in fields.items():
                arr = got[name][sub]
                assert list(arr.shape) == shape, (rank_s, name, sub)
                assert digest(arr) == sha, (rank_s, name, sub)


def test_ib_switch_changes_schedule():
    assert load_golden("cfg2_mini")["schedule"] != load_golden("cfg2_mini_noib")["schedule"]


def test_semantic_order_fixes_shrink_quirk():
    """TP shrink: the reference concatenates received pieces before the rank's own piece; the
    semantic order equals gathering the full tensor and re-slicing it."""
    cfg = CASES["cfg3_mini"]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg)
    ops = O.schedule(spl, tpl, minimum_est_peers=1)
    quirk = 0
    for rank in tpl.layout:
        ref = O.execute_rank(ops, states, SUB_META, rank, "reference")
        sem = O.execute_rank(ops, states, SUB_META, rank, "semantic")
        want = O.semantic_target(states, spl, tpl, SUB_META, rank)
        for name in want:
            for sub, _ in SUB_META:
                assert digest(sem[name][sub]) == digest(want[name][sub])
                quirk += digest(ref[name][sub]) != digest(want[name][sub])
    assert quirk > 0

"""forcefully_free of the drop-in, on the CPU: the tensors it releases are the ones the
reference's execute_param_transfer releases (its self pieces that are whole source tensors,
Suika/migration.py:297-300,539-541), and releasing empties their storage."""
import pytest
import torch

from oracle import restate as O
from suika_b200 import migration as M
from suika_b200 import synthetic as S
from tests.golden.cases import CASES
from tests.helpers import SUBS, golden_states, load_golden


def _reference_freed(ops, rank):
    """Names whose self piece is the source tensor itself in the reference's schedule."""
    return {o.name for o in ops if o.src == rank and o.dst == rank and O._deg(o.src_tp) >= O._deg(o.dst_tp)}


@pytest.mark.parametrize("case", ["shrink_mini", "cfg3_mini", "cfg2b_mini", "hetero_mini"])
def test_self_pieces_are_the_reference_frees(case):
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    plan = M.Plan(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    ops = O.schedule(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    kinds = dict(SUBS)
    exp = S.expected_sub_fields()
    for rank, st in states.items():
        src = {n: {s: S.to_torch(a, kinds[s]) for s, a in e.items()} for n, e in st.items()}
        got = M.self_pieces(plan, src, exp, rank, torch.device("cpu"))
        names = {n for n, e in src.items() for t in got if any(t is x for x in e.values())}
        assert names == _reference_freed(ops, rank), rank
        # every normal sub-field of a freed tensor, and the singleton only when it is on the device
        for n in names:
            ids = {id(t) for t in got}
            assert all(id(src[n][s]) in ids for s, k in SUBS)


def test_singletons_on_the_host_stay():
    cfg = CASES["shrink_mini"]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=load_golden("shrink_mini")["seed"])
    plan = M.Plan(spl, tpl, minimum_est_peers=1)
    kinds = dict(SUBS)
    rank = next(iter(states))
    src = {n: {s: S.to_torch(a, kinds[s]) for s, a in e.items()} for n, e in states[rank].items()}
    got = M.self_pieces(plan, src, S.expected_sub_fields(), rank, torch.device("cuda", 0))  # sources are not on it
    assert got and not any(t is e["step"] for e in src.values() for t in got)


def test_forcefully_free_empties_storage():
    a, b = torch.ones(1000), torch.ones(10)
    view = b[2:5]
    M._forcefully_free([a, view])
    assert a.untyped_storage().nbytes() == 0 and b.untyped_storage().nbytes() == 0

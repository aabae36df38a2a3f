"""The C planner (libsuika_reshard.so) against the reference: its schedule equals the reference's
op for op, and each rank's copy program, applied with numpy on the CPU, reproduces the
reference's output bytes (tests/golden) and, in semantic order, the re-sliced full tensors."""
import numpy as np
import pytest

from oracle import restate as O
from suika_b200 import migration as M
from tests.golden.cases import CASES
from tests.helpers import (SUB_ITEMSIZE, SUB_META, SUBS, digest, emulate_program, golden_states, load_golden)

NAMES = sorted(CASES)
SUBFIELD_SPEC = [(SUB_ITEMSIZE[s], kind == "meta") for s, kind in SUBS]


def plan_schedule_lists(plan):
    out = []
    for o in plan.op_array:
        tp = lambda d, i, g: None if d == -1000 else [int(d), int(i), int(g)]
        out.append([plan.names[o["name_id"]], int(o["src_rank"]), int(o["dst_rank"]),
                    tp(o["src_slice_dim"], o["src_tp_index"], o["src_tp_deg"]),
                    tp(o["dst_slice_dim"], o["dst_tp_index"], o["dst_tp_deg"])])
    return out


@pytest.mark.parametrize("case", NAMES)
def test_plan_matches_reference_schedule(case):
    g = load_golden(case)
    spl, tpl = CASES[case]["config"].layouts()
    plan = M.Plan(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    assert plan_schedule_lists(plan) == g["schedule"]


@pytest.mark.parametrize("case", NAMES)
def test_program_reproduces_reference_bytes(case):
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    plan = M.Plan(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    for rank_s, want in g["ranks"].items():
        prog = plan.program(int(rank_s), SUBFIELD_SPEC)
        got = emulate_program(prog, plan.names, states, int(rank_s))
        assert list(got) == want["order"]
        for name, fields in want["digests"].items():
            assert list(got[name]) == list(fields)
            for sub, (shape, _dtype, sha) in fields.items():
                assert list(got[name][sub].shape) == shape, (rank_s, name, sub)
                assert digest(got[name][sub]) == sha, (rank_s, name, sub)


@pytest.mark.parametrize("case", ["cfg3_mini", "cfg5_mini", "shrink_mini", "hetero_mini", "odd_mini"])
def test_semantic_program_equals_reslice(case):
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg)
    plan = M.Plan(spl, tpl, order="semantic", minimum_est_peers=1)
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        got = emulate_program(plan.program(rank, SUBFIELD_SPEC), plan.names, states, rank)
        want = O.semantic_target(states, spl, tpl, SUB_META, rank)
        for name in want:
            for sub, meta in SUB_META:
                if not meta:
                    assert np.array_equal(got[name][sub].view(np.uint8), want[name][sub].view(np.uint8)), (rank, name, sub)


@pytest.mark.parametrize("case", ["cfg2_mini", "cfg5_mini", "cfg4_mini"])
def test_balanced_choice_same_bytes_lower_egress(case):
    """Any owner of a piece holds the same bytes, so the balanced source choice changes who sends,
    not what arrives; its max egress is never above the reference's greedy choice."""
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg)
    ref = M.Plan(spl, tpl, minimum_est_peers=1)
    bal = M.Plan(spl, tpl, src_choice="balanced", minimum_est_peers=1)
    its = [SUB_ITEMSIZE[s] for s, k in SUBS if k != "meta"]
    assert max(bal.rank_bytes(its)["egress"].values()) <= max(ref.rank_bytes(its)["egress"].values())
    for rank, metas in tpl.layout.items():
        a = emulate_program(ref.program(rank, SUBFIELD_SPEC), ref.names, states, rank)
        b = emulate_program(bal.program(rank, SUBFIELD_SPEC), bal.names, states, rank)
        for name in a:
            for sub in a[name]:
                assert digest(a[name][sub]) == digest(b[name][sub])


def _meta(name, shape, tp, dtype=None):
    import torch
    return M.TensorMeta(name=name, dtype=dtype or torch.bfloat16, shape=shape, tp_meta=tp)


def _lay(d):
    lay = M.ParamLayout()
    lay.layout = d
    return lay


def test_no_owner_raises_assertion():
    spl = _lay({0: {"w": _meta("w", (8, 4), (0, 0, 2))}, 1: {}})
    tpl = _lay({0: {"w": _meta("w", (8, 4), (0, 0, 1))}})
    with pytest.raises(AssertionError, match="illegal transfer"):
        M.Plan(spl, tpl)


def test_slice_dim_mismatch_raises_assertion():
    spl = _lay({0: {"w": _meta("w", (8, 4), (0, 0, 1))}})
    tpl = _lay({0: {"w": _meta("w", (8, 4), (-1, 0, 2))}})
    with pytest.raises(AssertionError, match="slice dim"):
        M.Plan(spl, tpl)


def test_empty_source_raises_value_error():
    spl = _lay({0: {}})
    tpl = _lay({0: {"w": _meta("w", (8, 4), None)}})
    with pytest.raises(ValueError):
        M.Plan(spl, tpl)


def test_replicated_to_sliced_mismatch_raises_at_program_build():
    spl = _lay({0: {"w": _meta("w", (8, 4), None)}})
    tpl = _lay({0: {"w": _meta("w", (8, 4), (0, 0, 2))}, 1: {"w": _meta("w", (8, 4), (0, 1, 2))}})
    plan = M.Plan(spl, tpl)  # the reference's schedule accepts it too (overlap with None is True)
    with pytest.raises(AssertionError, match="slice dim"):
        plan.program(0, [(2, False)])


def test_indivisible_shape_raises():
    spl = _lay({0: {"w": _meta("w", (7, 4), (0, 0, 1))}})
    tpl = _lay({0: {"w": _meta("w", (7, 4), (0, 0, 2))}, 1: {"w": _meta("w", (7, 4), (0, 1, 2))}})
    plan = M.Plan(spl, tpl)
    with pytest.raises(AssertionError, match="divisible"):
        plan.program(0, [(2, False)])


def test_empty_target_rank_has_empty_program():
    spl = _lay({0: {"w": _meta("w", (8, 4), None)}, 1: {}})
    tpl = _lay({0: {"w": _meta("w", (8, 4), None)}, 1: {}})
    prog = M.Plan(spl, tpl).program(1, [(2, False), (4, True)])
    assert len(prog.dst_slots) == len(prog.segments) == len(prog.meta_slots) == 0


def test_resolve_rejects_out_of_bounds():
    spl = _lay({0: {"w": _meta("w", (8, 4), (-1, 0, 1))}})
    tpl = _lay({0: {"w": _meta("w", (8, 4), (-1, 0, 2))}, 1: {"w": _meta("w", (8, 4), (-1, 1, 2))}})
    prog = M.Plan(spl, tpl).program(1, [(2, False)])
    assert len(prog.segments) == 1 and prog.segments[0]["rows"] == 8
    n = len(prog.src_slots)
    ok = prog.resolve(np.full(n, 4096, np.uint64), np.full(n, 64, np.uint64), np.full(1, 8192, np.uint64), np.full(1, 32, np.uint64))
    assert ok[0]["src_dev"] == 4096 + 4 and ok[0]["src_pitch"] == 8 and ok[0]["dst_pitch"] == 4
    from suika_b200._lib import ReshardError
    with pytest.raises(ReshardError, match="leaves"):
        prog.resolve(np.full(n, 4096, np.uint64), np.full(n, 63, np.uint64), np.full(1, 8192, np.uint64), np.full(1, 32, np.uint64))


def test_resolve_marks_remote_pieces():
    """Entries whose source is another rank carry RS_COPY_REMOTE; the executor stages them first
    and interleaves them with local entries in every CTA."""
    cfg = CASES["cfg3_mini"]["config"]
    spl, tpl = cfg.layouts()
    plan = M.Plan(spl, tpl, minimum_est_peers=1)
    for rank in range(8):
        prog = plan.program(rank, SUBFIELD_SPEC)
        n = len(prog.src_slots)
        m = len(prog.dst_slots)
        out = prog.resolve(np.full(n, 1 << 40, np.uint64), np.full(n, 1 << 40, np.uint64),
                           np.full(m, 1 << 41, np.uint64), np.full(m, 1 << 40, np.uint64))
        want = (prog.src_slots["src_rank"][prog.segments["src_slot"]] != rank).astype(np.uint64)
        assert np.array_equal(out["flags"], want)
        assert want.any()


# The state the reference's own worker migrates: bf16 param, step, bf16 exp_avg / exp_avg_sq
# (no fp32 master; tasks/task.py keeps bf16 as the default dtype and uses torch.optim.AdamW).
WORKER_SUBS = [("param", "bf16"), ("step", "meta"), ("exp_avg", "bf16"), ("exp_avg_sq", "bf16")]


@pytest.mark.parametrize("case", ["cfg3_mini", "cfg5_mini", "shrink_mini", "hetero_mini"])
def test_program_on_the_reference_worker_state(case):
    """Every sub-field moves as bytes of its own size: the worker's 6-byte state through the same
    programs, against the oracle (pinned on the benchmark's sub-fields)."""
    from suika_b200 import synthetic as S
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, WORKER_SUBS, seed=2, distinct_steps=True)
    plan = M.Plan(spl, tpl, minimum_est_peers=1)
    spec = [(2, False), (4, True), (2, False), (2, False)]
    ops = O.schedule(spl, tpl, minimum_est_peers=1)
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        got = emulate_program(plan.program(rank, spec), plan.names, states, rank, WORKER_SUBS)
        want = O.execute_rank(ops, states, [(s, k == "meta") for s, k in WORKER_SUBS], rank)
        assert list(got) == list(want)
        for name, ent in want.items():
            for sub, a in ent.items():
                g = got[name][sub]
                assert g.shape == a.shape and np.array_equal(g.reshape(-1).view(np.uint8), a.reshape(-1).view(np.uint8)), (rank, name, sub)

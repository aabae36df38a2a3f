"""The C planner against the oracle on seeded random reshards: random (TP, PP, DP) meshes on both
sides, unequal TP degrees inside a stage, worlds that grow and shrink, both peer rules. For each,
the op list must equal the oracle's schedule op for op, and every target rank's program, applied
with numpy, must reproduce the oracle's bytes in the reference's cat order (and in slice order)."""
import numpy as np
import pytest

from oracle import restate as O
from suika_b200 import migration as M
from suika_b200 import synthetic as S
from suika_b200.layouts import SPECS, ReshardConfig, scaled_spec
from tests.helpers import SUB_ITEMSIZE, SUB_META, SUBS, emulate_program
from tests.test_planner import plan_schedule_lists

SPEC = scaled_spec(SPECS["llama2-13b"], name="rand", hidden=32, n_layers=4, n_heads=4, ffn=64, vocab=64)
SUBFIELD_SPEC = [(SUB_ITEMSIZE[s], kind == "meta") for s, kind in SUBS]


def random_mesh(rng, max_world=8):
    """stages -> DP groups -> ranks, ranks numbered consecutively; TP degrees are powers of two
    dividing the model's heads, and may differ between the DP groups of a stage."""
    pp = int(rng.choice([1, 2, 4]))
    stages, r = [], 0
    for _ in range(pp):
        groups = []
        for _ in range(int(rng.integers(1, 3))):
            tp = int(rng.choice([1, 2, 4]))
            if r + tp > max_world:
                tp = 1
            if r + tp > max_world:
                break
            groups.append(list(range(r, r + tp)))
            r += tp
        if not groups:
            return None
        stages.append(groups)
    return stages


def cases(n=48, seed=1234):
    rng = np.random.default_rng(seed)
    out = []
    while len(out) < n:
        src, dst = random_mesh(rng), random_mesh(rng)
        if src is None or dst is None:
            continue
        out.append((src, dst, int(rng.choice([1, 2]))))
    return out


def _to_schedule_lists(ops):
    return [[o.name, o.src, o.dst, list(o.src_tp) if o.src_tp else None, list(o.dst_tp) if o.dst_tp else None] for o in ops]


@pytest.mark.parametrize("src,dst,peers", cases())
def test_random_reshard_matches_oracle(src, dst, peers):
    spl, tpl = ReshardConfig("rand", SPEC, src, dst).layouts()
    states = S.host_states(spl, SUBS, seed=9, distinct_steps=True, threads=1)
    ops = O.schedule(spl, tpl, minimum_est_peers=peers)
    plan = M.Plan(spl, tpl, minimum_est_peers=peers)
    assert plan_schedule_lists(plan) == _to_schedule_lists(ops)
    sem = M.Plan(spl, tpl, order="semantic", minimum_est_peers=peers)
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        for p, order in ((plan, "reference"), (sem, "semantic")):
            got = emulate_program(p.program(rank, SUBFIELD_SPEC), p.names, states, rank)
            want = O.execute_rank(ops, states, SUB_META, rank, order=order)
            assert list(got) == list(want), (rank, order)
            for name, ent in want.items():
                for sub, a in ent.items():
                    g = got[name][sub]
                    assert g.shape == a.shape and np.array_equal(g.reshape(-1).view(np.uint8), a.reshape(-1).view(np.uint8)), \
                        (rank, order, name, sub)

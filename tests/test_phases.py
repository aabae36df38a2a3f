"""Transfer phases: every phase is a matching (each rank sends to at most one peer and receives
from at most one), and the number of phases equals the largest per-rank degree."""
import collections

import numpy as np
import pytest

from suika_b200 import migration as M
from suika_b200.layouts import CONFIGS


def _check(pairs):
    col = M.transfer_phases(pairs)
    assert set(col) == set(pairs)
    deg = collections.Counter()
    for s, t in pairs:
        deg[("s", s)] += 1
        deg[("t", t)] += 1
    n = max(col.values()) + 1 if col else 0
    assert n == max(deg.values(), default=0)
    for k in range(n):
        src = [s for (s, t), c in col.items() if c == k]
        dst = [t for (s, t), c in col.items() if c == k]
        assert len(src) == len(set(src)) and len(dst) == len(set(dst))


@pytest.mark.parametrize("seed", range(40))
def test_random_bipartite_graphs(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(2, 12))
    pairs = {}
    for s in range(n):
        for t in range(n):
            if s != t and rng.random() < 0.4:
                pairs[(s, t)] = int(rng.integers(1, 1000))
    _check(pairs)


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
def test_config_phases(name):
    spl, tpl = CONFIGS[name].layouts()
    plan = M.Plan(spl, tpl, minimum_est_peers=1)
    col, n = M.plan_phases(plan)
    ops = plan.op_array
    pairs = {(int(s), int(t)): 1 for s, t in zip(ops["src_rank"], ops["dst_rank"]) if s != t}
    _check(pairs)
    assert n == (max(col.values()) + 1 if col else 1)


def test_phase_tables_spread_local_entries():
    table = np.zeros(6, dtype=M.L.COPY_DESC_DTYPE)
    table["rows"] = 1
    table["row_bytes"] = [100, 100, 50, 50, 50, 50]
    peer = np.array([1, 2, 0, 0, 0, 0])  # rank 0 reads from 1 (phase 0) and 2 (phase 1); 4 local
    parts = M._phase_tables(table, peer, 0, {(1, 0): 0, (2, 0): 1}, 2, as_source=False)
    assert [len(p) for p in parts] == [3, 3]
    assert sum(int(p["row_bytes"].sum()) for p in parts) == 400

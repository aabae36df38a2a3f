"""The push direction's copy tables, executed on the CPU against emulated memory: every rank's
table (the pieces it sources, for every target rank) applied to numpy buffers must rebuild the
reference's targets (tests/golden digests). Covers the table logic of RankTransferPush without
GPUs or IPC."""
import numpy as np
import pytest

from suika_b200 import migration as M
from tests.golden.cases import CASES
from tests.helpers import SUB_ITEMSIZE, SUBS, Memory, digest, golden_states, load_golden

SPEC = [(SUB_ITEMSIZE[s], kind == "meta") for s, kind in SUBS]
SUBNAMES = [s for s, _ in SUBS]


def run_push(case):
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    plan = M.Plan(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
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
    for rank in sorted(set(int(x) for x in ops["src_rank"])):
        for T in sorted(set(int(t) for t in ops["dst_rank"][ops["src_rank"] == rank])):
            base, off, nb = arenas[T]
            table = M._push_table(progs[T], rank, lambda n, s, r=rank: src_addr[(r, n, s)], base, off, nb, SUBNAMES)
            for d in table:
                for row in range(int(d["rows"])):
                    rb = int(d["row_bytes"])
                    mem.view(int(d["dst_dev"]) + row * int(d["dst_pitch"]), rb)[:] = mem.view(int(d["src_dev"]) + row * int(d["src_pitch"]), rb)
    return g, plan, progs, arenas, mem


@pytest.mark.parametrize("case", ["odd_mini", "cfg2b_mini", "cfg3_mini", "cfg4_mini", "shrink_mini", "hetero_mini"])
def test_push_tables_rebuild_reference_targets(case):
    g, plan, progs, arenas, mem = run_push(case)
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

"""The NCCL-path port of the reference's execute_param_transfer (oracle/nccl_port.py), run on gloo
CPU ranks: every target must match the reference's golden digests, so the GPU baseline that
bench.py times moves the same bytes as the reference."""
import json
import os
import tempfile
import traceback

import pytest
import torch

from tests.golden.cases import CASES
from tests.helpers import load_golden


def _worker(rank, world, case, port, outdir):
    res = {"rank": rank}
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as dist
        from oracle import nccl_port as P
        from oracle import restate as O
        from suika_b200 import synthetic as S
        from tests.helpers import SUBS, digest
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = load_golden(case)
        cfg = CASES[case]["config"]
        spl, tpl = cfg.layouts()
        states = S.host_states(spl, SUBS, seed=g["seed"], distinct_steps=True, ranks=[rank])
        src = {n: {s: S.to_torch(a, k) for (s, k), a in zip(SUBS, e.values())} for n, e in states.get(rank, {}).items()}
        subfields = [(s, k == "meta", S.TORCH_DTYPE[k]) for s, k in SUBS]
        shapes = {n: m.shape for metas in tpl.layout.values() for n, m in metas.items()}
        ops = O.schedule(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
        out = P.execute_rank(ops, src, subfields, shapes, rank, torch.device("cpu"), cuda_gc=False)
        assert len(src) == 0
        dig = {}
        for name, ent in out.items():
            dig[name] = {}
            for s, t in ent.items():
                h = t.view(torch.uint16) if t.dtype == torch.bfloat16 else t
                dig[name][s] = [list(t.shape), str(t.dtype).replace("torch.", ""), digest(h.numpy())]
        res.update(order=list(out), digests=dig)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        res["error"] = traceback.format_exc()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


PORT_CASES = ["odd_mini", "hetero_mini", "grow_dp_tp_mini"]


@pytest.mark.parametrize("case", PORT_CASES)
def test_nccl_port_matches_reference_digests(case):
    import torch.multiprocessing as mp
    spl, tpl = CASES[case]["config"].layouts()
    world = max(len(spl.layout), len(tpl.layout))
    g = load_golden(case)
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, case, 29730 + 7 * PORT_CASES.index(case), d), nprocs=world, join=True)
        results = {r: json.load(open(os.path.join(d, f"rank{r}.json"))) for r in range(world)}
    for r, res in results.items():
        assert "error" not in res, res.get("error")
    for rank_s, want in g["ranks"].items():
        got = results[int(rank_s)]
        assert got["order"] == want["order"]
        for name, fields in want["digests"].items():
            for sub, (shape, dtype, sha) in fields.items():
                gs, gd, gh = got["digests"][name][sub]
                if sub == "step":  # compared by value elsewhere; the port's dtype follows the sub-field
                    continue
                assert (gs, gd, gh) == (shape, dtype, sha), (rank_s, name, sub)


@pytest.mark.parametrize("case", ["cfg3_mini", "odd_mini", "hetero_mini", "grow_dp_tp_mini", "next_step"])
def test_checkpoint_port_matches_reference_digests(case):
    """The port of the reference's checkpoint resume (execute on the CPU from every rank's host
    shard), which bench.py --checkpoint times as the reference's path, rebuilds the golden targets."""
    from oracle import nccl_port as P
    from oracle import restate as O
    from suika_b200 import synthetic as S
    from tests.helpers import SUBS, digest
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, SUBS, seed=g["seed"], distinct_steps=True)
    fake = {r: {n: {s: S.to_torch(a, k) for (s, k), a in zip(SUBS, e.values())} for n, e in st.items()} for r, st in states.items()}
    subfields = [(s, k == "meta", S.TORCH_DTYPE[k]) for s, k in SUBS]
    ops = O.schedule(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    for rank_s, want in g["ranks"].items():
        out = P.checkpoint_rank(ops, fake, subfields, int(rank_s))
        assert list(out) == want["order"]
        for name, fields in want["digests"].items():
            for sub, (shape, dtype, sha) in fields.items():
                t = out[name][sub]
                h = t.view(torch.uint16) if t.dtype == torch.bfloat16 else t
                if sub == "step":
                    continue
                assert [list(t.shape), str(t.dtype).replace("torch.", ""), digest(h.numpy())] == [shape, dtype, sha], (rank_s, name, sub)

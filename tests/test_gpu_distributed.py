"""The drop-in schedule_and_execute_param_transfer with one process per rank: peers' source
allocations are mapped through CUDA IPC and read (pull) or written (push) by one kernel per rank
and phase, over NVLink with a GPU per rank. Every target must equal the reference's own output
(tests/golden digests). With fewer GPUs than ranks, all ranks share cuda:0 (gloo process group,
CUDA IPC between processes on one device), which runs the same code path minus NVLink."""
import datetime
import json
import os
import tempfile
import traceback

import numpy as np
import pytest
import torch

from tests.golden.cases import CASES
from tests.helpers import load_golden

pytestmark = pytest.mark.gpu


def _worker(rank, world, case, port, outdir, directions):
    res = {"rank": rank}
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        from suika_b200 import migration as M
        from suika_b200 import synthetic as S
        from tests.helpers import SUBS, digest, rank_device
        dev, backend = rank_device(rank, world)
        torch.cuda.set_device(dev)
        dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
        res["backend"] = backend
        g = load_golden(case)
        cfg = CASES[case]["config"]
        spl, tpl = cfg.layouts()
        states = S.host_states(spl, SUBS, seed=g["seed"], distinct_steps=True, ranks=[rank])
        kinds = dict(SUBS)
        if g["minimum_est_peers"] == 2:
            os.environ["NCCL_IB_DISABLE"] = "1"
        for direction in directions:
            src = {n: {s: S.to_torch(a, kinds[s], dev if kinds[s] != "meta" else None) for s, a in e.items()}
                   for n, e in states.get(rank, {}).items()}
            timers = {}
            plan = M.Plan(spl, tpl)
            out = M.execute_plan_distributed(plan, src, S.expected_sub_fields(), dev, None, timers=timers, direction=direction)
            torch.cuda.synchronize()
            assert len(src) == 0  # cleared like the reference's source_state_dict
            dig = {}
            for name, ent in out.items():
                dig[name] = {}
                for s, t in ent.items():
                    assert t.device == dev and t.is_contiguous()
                    h = t.detach().cpu()
                    if h.dtype == torch.bfloat16:
                        h = h.view(torch.uint16)
                    dig[name][s] = [list(t.shape), str(t.dtype).replace("torch.", ""), digest(h.numpy())]
            res[direction] = dict(order=list(out), digests=dig, timers={k: v for k, v in timers.items() if k != "launch"})
            del out
            dist.barrier()
        dist.destroy_process_group()
    except Exception:
        res["error"] = traceback.format_exc()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


def run_case(case, port, directions=("pull", "push")):
    world = CASES[case]["config"].world_size
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, case, port, d, tuple(directions)), nprocs=world, join=True)
        return [json.load(open(os.path.join(d, f"rank{r}.json"))) for r in range(world)]


@pytest.mark.parametrize("case", ["cfg2b_mini", "odd_mini", "cfg1", "cfg2_mini", "cfg3_mini", "cfg4_mini", "cfg5_mini",
                                  "shrink_mini", "hetero_mini", "cfg2_mini_noib", "pp_deepen_mini", "gpt_shrink_mini",
                                  "grow_dp_tp_mini", "qwen_grow_mini", "wide_mini", "wide_shrink_mini", "next_step"])
def test_drop_in_matches_reference(case):
    """Pull, then push, in the same processes; both against the reference's digests."""
    g = load_golden(case)
    results = run_case(case, 29800 + 2 * sorted(CASES).index(case))
    for r in results:
        assert "error" not in r, r.get("error")
    for direction in ("pull", "push"):
        for rank_s, want in g["ranks"].items():
            got = results[int(rank_s)][direction]
            assert got["order"] == want["order"], direction
            for name, fields in want["digests"].items():
                for sub, exp in fields.items():
                    assert got["digests"][name][sub] == exp, (direction, rank_s, name, sub)
        for r in results:  # ranks without targets return an empty dict
            if str(r["rank"]) not in g["ranks"]:
                assert r[direction]["order"] == []

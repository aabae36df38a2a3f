"""DP-replica fan-out on B200s (one process per GPU, push direction): a DP grow from one GPU to
four (TP1 x DP1 -> TP1 x DP4) runs stage 1 (the source to each tensor's leader) and a binomial
broadcast among the replicas (stage 2). Every target must equal the oracle's, in the reference's
cat order. With fewer than 4 GPUs the four ranks share cuda:0 (gloo process group, CUDA IPC
between processes on one device)."""
import datetime
import json
import os
import tempfile
import traceback

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = 4


def _cfg():
    from suika_b200.layouts import SPECS, ReshardConfig, scaled_spec
    spec = scaled_spec(SPECS["llama2-7b"], name="grow4", hidden=128, n_layers=2, n_heads=4, ffn=256, vocab=192)
    return ReshardConfig("grow4", spec, [[[0]]], [[[0], [1], [2], [3]]])


def _worker(rank, world, port, outdir):
    res = {"rank": rank}
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        from oracle import restate as O
        from suika_b200 import migration as M
        from suika_b200 import synthetic as S
        from tests.helpers import SUB_META, SUBS, rank_device
        dev, backend = rank_device(rank, world)
        torch.cuda.set_device(dev)
        dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        spl, tpl = _cfg().layouts()
        states = S.host_states(spl, SUBS, seed=5, distinct_steps=True)
        kinds = dict(SUBS)
        src = {n: {s: S.to_torch(a, kinds[s], dev if kinds[s] != "meta" else None) for s, a in e.items()}
               for n, e in states.get(rank, {}).items()}
        plan = M.Plan(spl, tpl, minimum_est_peers=1)
        timers = {}
        out = M.execute_plan_distributed(plan, src, S.expected_sub_fields(), dev, None, timers=timers,
                                         direction="push", fanout=True)
        torch.cuda.synchronize()
        want = O.execute_rank(O.schedule(spl, tpl, minimum_est_peers=1), states, SUB_META, rank)
        assert list(out) == list(want)
        for name, ent in want.items():
            for sub, a in ent.items():
                t = out[name][sub].detach().cpu().contiguous()
                if t.dtype == torch.bfloat16:
                    t = t.view(torch.uint16)
                assert np.array_equal(t.numpy().reshape(-1).view(np.uint8), a.reshape(-1).view(np.uint8)), (name, sub)
        res["phases"] = timers["phases"]
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        res["error"] = traceback.format_exc()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


def test_fanout_dp_grow_matches_oracle():
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(WORLD, 29960, d), nprocs=WORLD, join=True)
        results = [json.load(open(os.path.join(d, f"rank{r}.json"))) for r in range(WORLD)]
    for r in results:
        assert "error" not in r, r.get("error")
    assert all(r["phases"] >= 3 for r in results)  # stage 1 plus two broadcast rounds

"""Activation hand-over between pipeline stages on B200.
  - exchange_local: every golden case on one GPU must reproduce the reference's received bytes
    (tests/golden/act_golden.json); a larger bf16 case is checked against the oracle.
  - ActivationExchange, one process per GPU (2 and 4 GPUs): several micro-batches through both
    window slots, forward and backward exchanges alive together, each checked against the oracle."""
import datetime
import json
import os
import tempfile
import traceback

import numpy as np
import pytest
import torch

from oracle import activation as OA
from tests.golden.act_cases import ACT_CASES, rank_bsz, source_arrays, zero_targets
from tests.helpers import GOLDEN_DIR, digest

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

with open(os.path.join(GOLDEN_DIR, "act_golden.json")) as _f:
    GOLDEN = json.load(_f)


def _dev(a: np.ndarray, dtype: str, device) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a))
    return (t.view(torch.bfloat16) if dtype == "bfloat16" else t).to(device)


def _host(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    return (t.view(torch.uint16) if t.dtype == torch.bfloat16 else t).numpy()


@pytest.mark.parametrize("name", sorted(ACT_CASES))
def test_exchange_local_matches_reference(name):
    from suika_b200 import activation as A
    case = ACT_CASES[name]
    srcs = {r: _dev(a, case["dtype"], DEV) for r, a in source_arrays(case).items()}
    tgts = {r: _dev(a, case["dtype"], DEV) for r, a in zero_targets(case).items()}
    info = A.exchange_local(case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"], srcs, tgts,
                            case["batch_dim"], case["slice_dim"])
    torch.cuda.synchronize()
    assert info.n_entries + info.n_tensor_entries > 0
    assert {str(r): digest(_host(t)) for r, t in tgts.items()} == GOLDEN[name]["digests"]


def test_exchange_local_large_bf16_against_oracle():
    """TP4 -> DP2 x TP2 at a 13B stage boundary width (micro-batch 8, seq 512, hidden 5120)."""
    from suika_b200 import activation as A
    case = dict(mesh_src=[[0, 1, 2, 3]], bszs_src=[8], mesh_dst=[[4, 5], [6, 7]], bszs_dst=[4, 4],
                shape=[-1, 512, 5120], batch_dim=0, slice_dim=-1, dtype="bfloat16")
    srcs_np, tg_np = source_arrays(case, seed=5), zero_targets(case)
    srcs = {r: _dev(a, "bfloat16", DEV) for r, a in srcs_np.items()}
    tgts = {r: _dev(a, "bfloat16", DEV) for r, a in tg_np.items()}
    A.exchange_local(case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"], srcs, tgts)
    torch.cuda.synchronize()
    OA.exchange_world(srcs_np, tg_np, case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"])
    for r, t in tgts.items():
        assert np.array_equal(_host(t), tg_np[r]), r


# ---- one process per GPU ------------------------------------------------------------------
DIST_CASES = {
    "pp_1to1": dict(mesh_src=[[0]], bszs_src=[4], mesh_dst=[[1]], bszs_dst=[4],
                    shape=[-1, 64, 256], batch_dim=0, slice_dim=-1, dtype="float32"),
    "tp2_to_dp2": dict(mesh_src=[[0, 1]], bszs_src=[4], mesh_dst=[[2], [3]], bszs_dst=[2, 2],
                       shape=[-1, 32, 512], batch_dim=0, slice_dim=-1, dtype="bfloat16"),
    "dp2_to_tp2": dict(mesh_src=[[0], [1]], bszs_src=[3, 1], mesh_dst=[[2, 3]], bszs_dst=[4],
                       shape=[-1, 32, 512], batch_dim=0, slice_dim=-1, dtype="float32"),
}
MICRO_BATCHES = 5


def _worker(rank, world, name, port, outdir):
    res = {"rank": rank}
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        from suika_b200 import activation as A
        from tests.helpers import rank_device
        dev, backend = rank_device(rank, world)
        torch.cuda.set_device(dev)
        dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        case = DIST_CASES[name]
        back = dict(case, mesh_src=case["mesh_dst"], bszs_src=case["bszs_dst"], mesh_dst=case["mesh_src"], bszs_dst=case["bszs_src"])
        tdtype = torch.bfloat16 if case["dtype"] == "bfloat16" else torch.float32
        fwd = A.ActivationExchange(rank, case["mesh_src"], case["mesh_dst"], case["bszs_src"], case["bszs_dst"],
                                   case["shape"], tdtype, case["batch_dim"], case["slice_dim"], device=dev)
        bwd = A.ActivationExchange(rank, back["mesh_src"], back["mesh_dst"], back["bszs_src"], back["bszs_dst"],
                                   back["shape"], tdtype, back["batch_dim"], back["slice_dim"], device=dev)
        send_op, recv_op = A.get_send_op(fwd), A.get_recv_op(fwd)
        checked = 0
        for mb in range(MICRO_BATCHES):
            for ex, c, seed in ((fwd, case, 100 + mb), (bwd, back, 200 + mb)):
                srcs_np = source_arrays(c, seed=seed)
                tg_np = zero_targets(c)
                target = None
                if ex.is_sender:
                    act = _dev(srcs_np[rank], c["dtype"], dev)
                    if ex is fwd:
                        send_op(act)  # the reference-shaped wrapper
                    else:
                        ex.send(act)
                if ex.is_receiver:
                    target = _dev(tg_np[rank], c["dtype"], dev)
                    if ex is fwd:
                        recv_op(target)
                    else:
                        ex.recv(target)
                if target is not None:
                    OA.exchange_world(srcs_np, tg_np, c["mesh_src"], c["mesh_dst"], c["bszs_src"], c["bszs_dst"],
                                      c["batch_dim"], c["slice_dim"])
                    got = _host(target)
                    assert np.array_equal(got, tg_np[rank]), (mb, "fwd" if ex is fwd else "bwd")
                    checked += 1
        fwd.check()
        bwd.check()
        fwd.close()
        bwd.close()
        res["checked"] = checked
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        res["error"] = traceback.format_exc()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


@pytest.mark.parametrize("name", sorted(DIST_CASES))
def test_activation_exchange_distributed(name):
    case = DIST_CASES[name]
    world = len(rank_bsz(case["mesh_src"], case["bszs_src"])) + len(rank_bsz(case["mesh_dst"], case["bszs_dst"]))
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, name, 29900 + 3 * sorted(DIST_CASES).index(name), d), nprocs=world, join=True)
        results = [json.load(open(os.path.join(d, f"rank{r}.json"))) for r in range(world)]
    for r in results:
        assert "error" not in r, r.get("error")
    # every rank receives in exactly one of the two directions, once per micro-batch
    assert all(r["checked"] == MICRO_BATCHES for r in results)

"""Generate tests/golden/act_golden.json by running Suika's own activation-exchange generator.

Run where the reference checkout (read-only) is importable; $SUIKA_REFERENCE names its directory:

    python tests/golden/make_act_golden.py

For each case of act_cases.py, PipelineExecModule._get_recv_or_send_P2P_ops
(Suika/pipeline_parallel.py:665-776, a static method) runs unmodified on one gloo rank:
  - every sender calls it with dist.isend on its activation; the P2POp tensors it returns are the
    blocks it would send (the reference's .contiguous() copies);
  - every receiver calls it with dist.irecv on a zero tensor; each returned P2POp's tensor gets the
    matching sent block (sends and receives of one rank pair match in issue order, as NCCL P2P
    does), then the returned restore function copies the blocks into place;
  - each receiving TP group of more than one rank then does what recv_op does after the P2P
    (pipeline_parallel.py:817-832): every member contributes target.chunk(d, slice_dim)[its TP
    index], and every member's target becomes the concatenation. The collective itself is done in
    this process (torch.cat of the members' chunks), since all ranks live here.
Output: per case, every rank's op list ([peer, shape of the block]) and the sha256 of every
receiver's final tensor.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from tests.golden.act_cases import ACT_CASES, source_arrays, zero_targets  # noqa: E402


def _torch(a, dtype):
    import torch
    t = torch.from_numpy(a.copy())
    return t.view(torch.bfloat16) if dtype == "bfloat16" else t


def _digest(t) -> str:
    import torch
    return hashlib.sha256(t.contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


def run_case(case: dict, P, RawDeviceMesh2D, dist) -> dict:
    import torch
    ms, md = RawDeviceMesh2D(case["mesh_src"]), RawDeviceMesh2D(case["mesh_dst"])
    bd, sd = case["batch_dim"], case["slice_dim"]
    srcs = {r: _torch(a, case["dtype"]) for r, a in source_arrays(case).items()}
    tgts = {r: _torch(a, case["dtype"]) for r, a in zero_targets(case).items()}
    ops = {}
    queues = {}
    for r, t in srcs.items():
        gen = P._get_recv_or_send_P2P_ops(r, ms, md, case["bszs_src"], case["bszs_dst"], dist.isend, batch_dim=bd, slice_dim=sd)
        sent, _ = gen(t)
        ops[str(r)] = {"send": [[o.peer, list(o.tensor.shape)] for o in sent]}
        for o in sent:
            queues.setdefault((r, o.peer), []).append(o.tensor.clone())
    for r, t in tgts.items():
        gen = P._get_recv_or_send_P2P_ops(r, ms, md, case["bszs_src"], case["bszs_dst"], dist.irecv, batch_dim=bd, slice_dim=sd)
        recv, restore = gen(t)
        ops[str(r)] = {"recv": [[o.peer, list(o.tensor.shape)] for o in recv]}
        for o in recv:
            blk = queues[(o.peer, r)].pop(0)
            assert blk.shape == o.tensor.shape
            o.tensor.copy_(blk)
        restore()
    assert all(not q for q in queues.values()), "unmatched sends"
    for group in case["mesh_dst"]:
        d = len(group)
        if d == 1:
            continue
        parts = [tgts[r].chunk(d, dim=sd)[j].contiguous() for j, r in enumerate(group)]
        full = torch.cat(parts, dim=sd)
        for r in group:
            tgts[r].copy_(full)
    return {"ops": ops, "digests": {str(r): _digest(t) for r, t in tgts.items()}}


def main() -> None:
    ref = os.environ.get("SUIKA_REFERENCE")
    if not ref:
        raise SystemExit("set SUIKA_REFERENCE to the directory of the reference checkout (the one holding Suika/)")
    sys.path.insert(0, ref)
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29631", rank=0, world_size=1)
    from Suika.device_mesh import RawDeviceMesh2D
    from Suika.pipeline_parallel import PipelineExecModule as P
    out = {name: run_case(case, P, RawDeviceMesh2D, dist) for name, case in ACT_CASES.items()}
    dist.destroy_process_group()
    with open(os.path.join(HERE, "act_golden.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print(f"wrote {len(out)} cases")


if __name__ == "__main__":
    main()

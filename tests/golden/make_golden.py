"""Generate golden digests by running Suika's own reshard code on CPU/gloo ranks.

Run where the reference checkout (read-only) is importable; $SUIKA_REFERENCE names its directory:

    python tests/golden/make_golden.py [case ...]

For each case the reference's schedule_param_transfer + execute_param_transfer
(Suika/migration.py:322-556) run unmodified on world_size gloo processes, on source state built by
suika_b200.synthetic (numpy, platform independent). Each case runs twice:
  A. layout dtype bf16, sub-fields [param (bf16), step (meta)];
  B. layout dtype fp32, sub-fields [step (meta), master, exp_avg, exp_avg_sq] (fp32).
The reference cannot carry fp32 sub-fields next to a bf16 param (its receive buffer takes the
layout dtype, migration.py:285-287, and gloo aborts on the size mismatch), so the fp32 sub-fields
are pinned by run B; both runs must produce the same schedule, which is stored with the digests.
Output: tests/golden/<case>.json with, per target rank, name and sub-field: shape, dtype, sha256.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
import traceback

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from tests.golden.cases import CASES  # noqa: E402


def _digest(t) -> str:
    import torch
    b = t.detach().contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()
    return hashlib.sha256(b).hexdigest()


def _worker(rank, world, case_name, port, ref_path, outdir):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        case = CASES[case_name]
        if case.get("ib_disabled"):
            os.environ["NCCL_IB_DISABLE"] = "1"
        else:
            os.environ.pop("NCCL_IB_DISABLE", None)
        import torch
        import torch.distributed as dist
        sys.path.insert(0, ref_path)
        import Suika.migration as M
        from suika_b200 import synthetic as S
        dist.init_process_group("gloo", rank=rank, world_size=world)
        cfg = case["config"]
        result = {"rank": rank, "runs": {}}
        for run, (ldtype, subs) in {
            "A": (torch.bfloat16, [("param", "bf16"), ("step", "meta")]),
            "B": (torch.float32, [("step", "meta"), ("master", "f32"), ("exp_avg", "f32"), ("exp_avg_sq", "f32")]),
        }.items():
            ours_s, ours_t = cfg.layouts(dtype=ldtype)

            def to_ref(lay):
                # TensorMeta(dtype=, shape=) leaves tp_meta unset when it is None (migration.py:58-64);
                # metas built from tensors always carry it, so set it explicitly.
                out = M.ParamLayout()
                for r, metas in lay.layout.items():
                    out.layout[r] = {}
                    for n, m in metas.items():
                        rm = M.TensorMeta(name=n, dtype=m.dtype, shape=m.shape)
                        rm.tp_meta = m.tp_meta
                        out.layout[r][n] = rm
                return out

            spl, tpl = to_ref(ours_s), to_ref(ours_t)
            states = S.host_states(ours_s, subs, seed=case.get("seed", 0), distinct_steps=True)
            src = {}
            if rank in states:
                for name, ent in states[rank].items():
                    src[name] = {s: S.to_torch(ent[s], kind) for s, kind in subs}
            expected = [(s, M.TensorMeta(tensor=torch.tensor(1.0, dtype=torch.float32)) if kind == "meta" else "normal")
                        for s, kind in subs]
            ops = M.schedule_param_transfer(spl, tpl)
            sched = [[o.param_name, o.src_rank, o.dst_rank, list(o.src_meta.tp_meta) if o.src_meta.tp_meta else None,
                      list(o.dst_meta.tp_meta) if o.dst_meta.tp_meta else None] for o in ops]
            out = M.execute_param_transfer(ops, src, torch.device("cpu"), expected, world=None)
            dig = {}
            for name, ent in out.items():
                dig[name] = {s: [list(t.shape), str(t.dtype).replace("torch.", ""), _digest(t)] for s, t in ent.items()}
            result["runs"][run] = {"schedule": sched, "digests": dig, "order": list(out.keys())}
            dist.barrier()
        dist.destroy_process_group()
    except Exception:
        result = {"rank": rank, "error": traceback.format_exc()}
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(result, f)


def run_case(name: str, port: int) -> dict:
    import torch.multiprocessing as mp
    case = CASES[name]
    cfg = case["config"]
    world = cfg.world_size
    ref = os.environ.get("SUIKA_REFERENCE")
    if not ref:
        raise SystemExit("set SUIKA_REFERENCE to the directory of the reference checkout (the one holding Suika/)")
    results = {}
    with tempfile.TemporaryDirectory() as outdir:
        mp.spawn(_worker, args=(world, name, port, ref, outdir), nprocs=world, join=True)
        for rank in range(world):
            with open(os.path.join(outdir, f"rank{rank}.json")) as f:
                r = json.load(f)
            if "error" in r:
                raise RuntimeError(f"rank {rank} failed:\n{r['error']}")
            results[rank] = r
    sched_a = results[0]["runs"]["A"]["schedule"]
    sched_b = results[0]["runs"]["B"]["schedule"]
    assert sched_a == sched_b, "the bf16 and fp32 runs produced different schedules"
    ranks = {}
    for rank, r in sorted(results.items()):
        a, b = r["runs"]["A"], r["runs"]["B"]
        if not a["digests"]:
            continue
        merged = {}
        for n in a["order"]:
            merged[n] = dict(a["digests"][n])
            assert b["digests"][n]["step"][2] == a["digests"][n]["step"][2], f"step differs between runs for {n}"
            for s in ("master", "exp_avg", "exp_avg_sq"):
                merged[n][s] = b["digests"][n][s]
        ranks[str(rank)] = {"order": a["order"], "digests": merged}
    return {"case": name, "description": case["description"], "world_size": world,
            "minimum_est_peers": 2 if case.get("ib_disabled") else 1, "seed": case.get("seed", 0),
            "distinct_steps": True, "schedule": sched_a, "ranks": ranks}


def main(argv):
    names = argv or list(CASES)
    port = 29610
    for n in names:
        out = run_case(n, port)
        port += 1
        path = os.path.join(HERE, f"{n}.json")
        with open(path, "w") as f:
            json.dump(out, f, separators=(",", ":"))
        print(f"{n}: {len(out['schedule'])} ops, {sum(len(v['digests']) for v in out['ranks'].values())} target tensors -> {path}", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])

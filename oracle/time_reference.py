"""Time the reference's own CPU/gloo migration next to the oracle port on the same sample
(TEST AND BENCHMARK INFRASTRUCTURE; needs the reference checkout, $SUIKA_REFERENCE).

    SUIKA_REFERENCE=/path/to/Suika python oracle/time_reference.py [--layers 1] [--reps 3]

The sample is bench.py's cpu_baseline sample at N = 1: `layers` decoder layers of Llama2-7B (with
embedding and head), TP1 -> TP2, full training state (bf16 param, fp32 master / exp_avg /
exp_avg_sq, step).
  * reference: Suika.migration.schedule_param_transfer + execute_param_transfer
    (Suika/migration.py:322-556), unmodified, on 2 gloo processes (the reshard's world), each with
    half of the host's threads. The reference receives every sub-field in the layout's dtype
    (migration.py:285-287), so it runs twice, as the golden generator does: layout bf16 with
    [param, step], then layout fp32 with [step, master, exp_avg, exp_avg_sq]; the time is the sum.
    Wall time between barriers, max over ranks.
  * port: oracle/restate.py (what bench.py --impl reference times on the GPU box) on all threads.
Both write every target tensor, as the reference does; rates are given in bench.py's unit (bytes
of the row-split pieces, which the views relayout moves, per second) and as seconds per sample.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)


def _worker(rank, world, layers, reps, port, ref_path, threads, outdir):
    res = {"rank": rank}
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        torch.set_num_threads(threads)
        sys.path.insert(0, ref_path)
        import Suika.migration as RM
        from suika_b200 import synthetic as S
        from suika_b200.layouts import CONFIGS, ReshardConfig, scaled_spec
        dist.init_process_group("gloo", rank=rank, world_size=world)
        base = CONFIGS["cfg2b"]
        cfg = ReshardConfig("cfg2b", scaled_spec(base.spec, n_layers=layers), base.src_mesh, base.dst_mesh)
        runs = []
        for ldtype, subs in ((torch.bfloat16, [("param", "bf16"), ("step", "meta")]),
                             (torch.float32, [("step", "meta"), ("master", "f32"), ("exp_avg", "f32"), ("exp_avg_sq", "f32")])):
            ours_s, ours_t = cfg.layouts(dtype=ldtype)

            def to_ref(lay):
                out = RM.ParamLayout()
                for r, metas in lay.layout.items():
                    out.layout[r] = {}
                    for n, m in metas.items():
                        rm = RM.TensorMeta(name=n, dtype=m.dtype, shape=m.shape)
                        rm.tp_meta = m.tp_meta
                        out.layout[r][n] = rm
                return out

            spl, tpl = to_ref(ours_s), to_ref(ours_t)
            states = S.host_states(ours_s, subs, seed=0, ranks=[rank], threads=threads)
            expected = [(s, RM.TensorMeta(tensor=torch.tensor(1.0, dtype=torch.float32)) if k == "meta" else "normal") for s, k in subs]
            runs.append((spl, tpl, states, subs, expected))
        times, written = [], 0
        for rep in range(reps + 1):
            total = 0.0
            for spl, tpl, states, subs, expected in runs:
                src = {n: {s: S.to_torch(e[s], k) for s, k in subs} for n, e in states.get(rank, {}).items()}
                dist.barrier()
                t0 = time.perf_counter()
                ops = RM.schedule_param_transfer(spl, tpl)
                out = RM.execute_param_transfer(ops, src, torch.device("cpu"), expected, world=None)
                dist.barrier()
                total += time.perf_counter() - t0
                if rep == 0:
                    written += sum(t.numel() * t.element_size() for e in out.values() for s, t in e.items() if s != "step")
            if rep:  # the first repetition is the warm-up
                times.append(total)
        res.update(times=times, written=written)
        dist.destroy_process_group()
    except Exception:
        import traceback
        res["error"] = traceback.format_exc()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    ref_path = os.environ.get("SUIKA_REFERENCE")
    if not ref_path:
        raise SystemExit("set SUIKA_REFERENCE to the reference checkout")
    import statistics

    import torch.multiprocessing as mp
    cores = os.cpu_count() or 1
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, args.layers, args.reps, 29590, ref_path, max(1, cores // world), d), nprocs=world, join=True)
        rs = [json.load(open(os.path.join(d, f"rank{r}.json"))) for r in range(world)]
    for r in rs:
        if "error" in r:
            raise RuntimeError(r["error"])
    t_ref = statistics.median(max(r["times"][i] for r in rs) for i in range(args.reps))
    written = sum(r["written"] for r in rs)

    sys.argv = [sys.argv[0]]
    import bench
    smp = bench.OracleSample(bench.workload(1, args.layers), 1, cores)
    smp.step()
    t_port = statistics.median(smp.step() for _ in range(args.reps))
    # GB/s in bench.py's unit: bytes of row-split pieces (what the views relayout moves) per second;
    # both sides write every target, as the reference does.
    print(json.dumps({"sample": f"{args.layers} layer(s) of Llama2-7B TP1 -> TP2 (cfg2b), full training state",
                      "host_cores": cores, "bench_unit_bytes": smp.units, "all_target_bytes": written,
                      "reference": {"gbs": round(smp.units / t_ref / 1e9, 3), "s": round(t_ref, 3), "ranks": world,
                                    "threads_per_rank": max(1, cores // world)},
                      "port": {"gbs": round(smp.units / t_port / 1e9, 3), "s": round(t_port, 3), "threads": cores}}))


if __name__ == "__main__":
    main()

"""Benchmark of the B200 live-reshard path (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  (N > 1: torchrun --nproc-per-node N bench.py --gpus N ...)

Workloads (synthetic seeded state, sub-fields bf16 param + fp32 master/m/v + step):
  N = 1  cfg2b: Llama2-7B full state, TP1 -> TP2 on one GPU, dim-0 slices and replicated tensors
         as views, row-split (dim -1) pieces packed; a step is one launch of the pack kernel.
  N > 1  Llama2-13B-shaped, 5*N layers, TP N x PP1 -> TP N/2 x PP2 (N = 8 is cfg3 exactly:
         Llama2-13B TP8 -> TP4 x PP2); per-GPU state is fixed as N grows (weak scaling); a step
         is one launch of each rank's pull kernel (peer HBM over NVLink + own HBM).
`value` is the state moved by all ranks per second (GB/s, bytes that must be written into
target tensors); the time of a step is the max over ranks of the device time.

Other modes (not the driver's contract lines): --impl reference-nccl (the reference's own GPU
path, execute_param_transfer over NCCL, on the N > 1 workload), --handoff (old -> new process
hand-off, 1 GPU), --activation (pipeline activation hand-over, N >= 2), --metadata (layout
exchange and planning, any N; gloo without GPUs), --fanout (DP-replica fan-out of the push path).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from suika_b200 import migration as M  # noqa: E402
from suika_b200 import synthetic as S  # noqa: E402
from suika_b200.layouts import CONFIGS, EXTRA_CONFIGS, SPECS, ReshardConfig, scaled_spec  # noqa: E402

METRIC = "state-migration time (s) and NVLink GB/s per GPU for 3D-layout reshard"
FALLBACK_HBM_GBS = 6650.0
NVLINK_GBS = 900.0               # NVLink 5 per direction per GPU: the roofline of remote traffic
NVLINK_MEASURED_PEER_GBS = 770.0  # a peer copy per direction measured on this pool, for context
L2_BYTES = 126 * 2 ** 20


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------------------------
def workload(n_gpus: int, layers: int = 0, config: str = "") -> ReshardConfig:
    """The reshard a run of n_gpus ranks measures: cfg2b at N = 1, the Llama2-13B TP N -> TP N/2 x
    PP2 family at N > 1 (cfg3 at N = 8), or a named configuration whose rank count is N."""
    if config:
        cfg = CONFIGS.get(config) or EXTRA_CONFIGS[config]
        if cfg.world_size != n_gpus:
            raise SystemExit(f"{config} runs on {cfg.world_size} ranks, not {n_gpus}")
        if layers:
            cfg = ReshardConfig(cfg.name, scaled_spec(cfg.spec, n_layers=layers), cfg.src_mesh, cfg.dst_mesh, cfg.note)
        return cfg
    if n_gpus == 1:
        cfg = CONFIGS["cfg2b"]
        if layers:
            cfg = ReshardConfig("cfg2b", scaled_spec(cfg.spec, n_layers=layers), cfg.src_mesh, cfg.dst_mesh, cfg.note)
        return cfg
    if n_gpus % 2:
        raise SystemExit("N > 1 must be even (TP N -> TP N/2 x PP2)")
    spec = scaled_spec(SPECS["llama2-13b"], n_layers=layers or 5 * n_gpus)
    src = [[list(range(n_gpus))]]
    half = n_gpus // 2
    dst = [[list(range(half))], [list(range(half, n_gpus))]]
    name = "cfg3" if (n_gpus == 8 and spec.n_layers == 40) else f"llama2-13b-{spec.n_layers}L"
    return ReshardConfig(name, spec, src, dst, f"Llama2-13B-shaped {spec.n_layers} layers TP{n_gpus} -> TP{half}xPP2")


def workload_config(cfg: ReshardConfig, n_gpus: int) -> dict:
    """The `config` object of a result line; both arms print the same one for the same workload."""
    if n_gpus == 1:
        what = (f"{cfg.name}: {cfg.spec.name} ({cfg.spec.n_layers} layers) full training state (bf16 param + fp32 "
                f"master/m/v + step), TP1 -> TP2 on one GPU, dim-0 slices and replicated tensors as views, row-split "
                f"pieces packed")
    else:
        what = f"{cfg.name}: {cfg.note}, full training state (bf16 param + fp32 master/m/v + step)"
    return {"workload": what, "l2": "inputs larger than L2 (no flush needed)", "order": "reference"}


# ---------------------------------------------------------------------------------------------
# Clocks during the timed region (nvidia-smi sampler)
# ---------------------------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# CPU baseline: the oracle (a restatement of the reference's algorithm) on the host cores
# ---------------------------------------------------------------------------------------------
STATE_BYTES_PER_ELEM = 2 + 4 + 4 + 4  # bf16 param + fp32 master, exp_avg, exp_avg_sq


def moved_bytes_views(plan: M.Plan, spl, tpl) -> int:
    """Bytes a TP1 -> TP2 'views' relayout must write: every piece that is not one contiguous range
    of its source (row-split pieces); the reference writes all target bytes."""
    total = 0
    for o in plan.op_array:
        if o["dst_slice_dim"] == -1 and o["src_tp_deg"] < o["dst_tp_deg"]:
            total += int(o["numel"]) * STATE_BYTES_PER_ELEM
    return total


def moved_bytes_views_ops(ops) -> int:
    """moved_bytes_views over the oracle's op list (the reference arm loads no product code)."""
    return sum(o.numel * STATE_BYTES_PER_ELEM for o in ops
               if o.dst_tp is not None and o.dst_tp[0] == -1 and (o.src_tp[2] if o.src_tp else 1) < o.dst_tp[2])


def cpu_sample(cfg: ReshardConfig, n_gpus: int):
    """A bounded sample of the workload for the host-core baseline: one decoder layer per stage."""
    if n_gpus == 1:
        spec = scaled_spec(cfg.spec, n_layers=1)
        return ReshardConfig(cfg.name + "-1L", spec, cfg.src_mesh, cfg.dst_mesh, "1 layer of " + cfg.note)
    spec = scaled_spec(cfg.spec, n_layers=2)
    return ReshardConfig(cfg.name + "-2L", spec, cfg.src_mesh, cfg.dst_mesh, "2 layers (1 per target stage) of " + cfg.note)


class OracleSample:
    """A bounded sample of the workload run by the oracle (oracle/restate.py, a restatement of
    Suika/migration.py:322-556) on host cores; inputs are generated once, outside the timing.
    N = 1: one layer of cfg2b, both target ranks. N > 1: one target rank's share of two layers
    (one per target stage, no embeddings): the rank with the most remote ingress, fed by the
    source ranks it reads from."""

    def __init__(self, cfg: ReshardConfig, n_gpus: int, threads: int):
        from oracle import restate as O
        self.O = O
        self.sample = cpu_sample(cfg, n_gpus)
        self.spl, self.tpl = self.sample.layouts(with_embeddings=(n_gpus == 1))
        self.subs = [(s, k == "meta") for s, k in S.SUBFIELDS]
        self.threads = threads
        # units and ranks come from the oracle's own schedule: nothing here loads the product library
        ops = O.schedule(self.spl, self.tpl, minimum_est_peers=1)
        if n_gpus == 1:
            self.units = moved_bytes_views_ops(ops)
            self.ranks = [r for r, m in self.tpl.layout.items() if m]
            src_ranks = None
            self.what = self.sample.note
        else:
            ing = {}
            for o in ops:
                ing[o.dst] = ing.get(o.dst, 0) + (o.numel if o.src != o.dst else 0)
            r = max(ing, key=lambda k: (ing[k], -k))
            self.ranks = [r]
            src_ranks = sorted({o.src for o in ops if o.dst == r})
            self.units = sum(o.numel for o in ops if o.dst == r) * STATE_BYTES_PER_ELEM
            self.what = f"target rank {r}'s share of 2 layers (1 per target stage, no embeddings) of {cfg.note}"
        self.states = S.host_states(self.spl, S.SUBFIELDS, seed=0, ranks=src_ranks, threads=threads)

    def step(self) -> float:
        t0 = time.perf_counter()
        ops = self.O.schedule(self.spl, self.tpl, 1)
        out = self.O.execute_world(ops, self.states, self.subs, self.ranks, threads=self.threads)
        dt = time.perf_counter() - t0
        del out
        return dt

    def describe(self, steps: int) -> str:
        return (f"{self.what}: {self.units / 1e9:.3f} GB of target state per step, {steps} steps, "
                f"oracle/restate.py (restatement of Suika/migration.py:322-556) on {self.threads} host threads")


def cpu_baseline_block(cfg, n_gpus, threads, budget_s=20.0):
    smp = OracleSample(cfg, n_gpus, threads)
    t1 = smp.step()
    reps = max(1, min(20, int(budget_s / max(t1, 1e-3))))
    t = sum(smp.step() for _ in range(reps))
    return {"value": round(smp.units * reps / t / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": smp.describe(reps)}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per moved byte of the one-GPU pack
# (the split launch: the banded vector copy and the tensor-map copy, one launch each per step),
# from one ncu capture of both launches of one step on a 2-layer cfg2b case (1.732 GB moved per
# step, above L2), taken with shape 15 as the default: `ncu --set full --clock-control none -k
# regex:rs_copy -s 8 -c 2 python bench.py --layers 2 --steps 3 --warmup 3 --no-e2e
# --no-cpu-baseline --no-check` gave 0.470 + 1.263 GB read and 0.419 + 1.221 GB written. Shape 17
# (the default now) moves the same rows with larger boxes, each byte again read once and written
# once. Traffic grows with the moved bytes, so a full step's traffic is this ratio x moved.
DRAM_BYTES_PER_MOVED_BYTE = 1.947


def rank_bytes_ops(ops) -> dict:
    """Per-rank ingress / egress / local bytes of an oracle op list (14 B per element)."""
    out = {"ingress": {}, "egress": {}, "local": {}}
    for o in ops:
        b = o.numel * STATE_BYTES_PER_ELEM
        if o.src == o.dst:
            out["local"][o.dst] = out["local"].get(o.dst, 0) + b
        else:
            out["ingress"][o.dst] = out["ingress"].get(o.dst, 0) + b
            out["egress"][o.src] = out["egress"].get(o.src, 0) + b
    return out


# ---------------------------------------------------------------------------------------------
# N = 1: cfg2b, TP1 -> TP2 views on one GPU
# ---------------------------------------------------------------------------------------------
def verify_views(spl, tpl, src, out) -> dict:
    """Size-independent checks on the full state: every row-split target, re-concatenated along
    its slice dim, equals its source; every other target is a view of its source with equal bytes."""
    n_checked = n_views = 0
    for name, m in tpl.layout[0].items():
        sd = m.tp_meta[0] if m.tp_meta else None
        for sub, kind in S.SUBFIELDS:
            if kind == "meta":
                assert float(out[0][name][sub]) == float(src[name][sub]) == float(out[1][name][sub])
                continue
            a, b, full = out[0][name][sub], out[1][name][sub], src[name][sub]
            if sd == -1:
                assert torch.equal(torch.cat([a, b], dim=-1), full), (name, sub)
            else:
                same = a.untyped_storage().data_ptr() == full.untyped_storage().data_ptr()
                assert same and b.untyped_storage().data_ptr() == full.untyped_storage().data_ptr(), (name, sub)
                assert torch.equal(torch.cat([a, b], dim=0), full) if sd == 0 else (torch.equal(a, full) and torch.equal(b, full))
                n_views += 2
            n_checked += 1
    return {"tensors_checked": n_checked, "views": n_views, "status": "pass"}


def run_single(args):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = workload(1, args.layers)
    spl, tpl = cfg.layouts()
    t0 = time.perf_counter()
    state = S.DeviceState(spl.layout[0], dev)
    torch.cuda.synchronize()
    log(f"generated {state.nbytes() / 1e9:.1f} GB of source state in {time.perf_counter() - t0:.1f} s")
    exp = S.expected_sub_fields()
    plan = M.Plan(spl, tpl, minimum_est_peers=1)
    out, info, prepared = M.reshard_local(spl, tpl, {0: state.state}, exp, dev, views=True, plan=plan, return_info=True)
    torch.cuda.synchronize()
    check = verify_views(spl, tpl, state.state, out) if not args.no_check else {"status": "skipped"}
    moved = int(info.total_bytes)
    units = moved_bytes_views(plan, spl, tpl)
    launches_per_step = int(info.n_entries > 0) + int(info.n_tensor_entries > 0)
    log(f"pack table: {info.n_entries} vector copies in {info.n_tiles} tiles (grid {info.grid}x{info.block}), "
        f"{info.n_tensor_entries} tensor-map copies in {info.n_tensor_tiles} boxes (grid {info.tensor_grid}x{info.tensor_block}); "
        f"launch shape {info.variant + 1}, {launches_per_step} kernel(s) per step; "
        f"{moved / 1e9:.2f} GB per step")
    with Clocks(0) as ck:
        for _ in range(args.warmup):
            prepared.launch()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        for a, b in evs:
            a.record()
            prepared.launch()
            b.record()
        end.record()
        torch.cuda.synchronize()
    total_s = start.elapsed_time(end) / 1e3
    launch_ms = [a.elapsed_time(b) for a, b in evs]
    kern_s = statistics.mean(launch_ms) / 1e3
    peak, peak_src = peaks()
    achieved = 2 * moved / kern_s / 1e9
    tpu = DRAM_BYTES_PER_MOVED_BYTE
    res = {
        "metric": METRIC, "value": round(moved * args.steps / total_s / 1e9, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_s / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded N(0,0.02) weights, norms 1.0, m~N(0,1e-3), v~|N(0,1e-6)|)",
        "config": workload_config(cfg, 1),
        "workload_bytes": {"source_state_gb": round(state.nbytes() / 1e9, 2), "moved_gb_per_step": round(moved / 1e9, 3)},
        "migration_s": round(total_s / args.steps, 6),
        "nvlink_gbs_per_gpu": 0.0,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
                     "traffic": int(tpu * moved),
                     "algorithmic_bytes_per_launch": 2 * moved, "kernel_ms": round(kern_s * 1e3, 4)},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": ck.summary(),
        "check": check,
    }
    del out, prepared, state
    torch.cuda.empty_cache()
    if not args.no_e2e:
        res["e2e"] = e2e_single(args, dev)
    if not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_block(cfg, 1, os.cpu_count() or 1)
    return res


def layer_groups(spl, tpl, per_group: int):
    """(source, target) sub-layouts of consecutive decoder layers, per_group at a time; the
    embedding joins the first group and the head and final norm the last."""
    names = list(spl.layout[0])
    layer_of = {n: int(n.split(".")[1]) if n.startswith("h.") else None for n in names}
    layers = sorted({v for v in layer_of.values() if v is not None})
    chunks = [layers[i:i + per_group] for i in range(0, len(layers), per_group)]
    out = []
    for gi, chunk in enumerate(chunks):
        keep = {n for n, l in layer_of.items() if l in chunk}
        if gi == 0:
            keep |= {n for n, l in layer_of.items() if l is None and n.startswith(("wte", "wpe"))}
        if gi == len(chunks) - 1:
            keep |= {n for n, l in layer_of.items() if l is None and not n.startswith(("wte", "wpe"))}
        sub = []
        for lay in (spl, tpl):
            g = M.ParamLayout()
            for r, metas in lay.layout.items():
                g.layout[r] = {n: m for n, m in metas.items() if n in keep}
            sub.append(g)
        out.append(tuple(sub))
    return out


def e2e_single(args, dev):
    """The same metric through the public API (reshard_local) with host buffers. Each step copies
    the source state in from pinned host memory, reshards it and reads the packed targets back,
    by groups of layers on three streams: the host-to-device copy of group k+1, the reshard of
    group k and the device-to-host copy of group k-1 overlap, so both PCIe directions and the
    kernel run at once. Runs on a layer sample so the pinned buffers stay well inside host memory."""
    cfg = workload(1, args.e2e_layers)
    spl, tpl = cfg.layouts()
    exp = S.expected_sub_fields()
    groups = []
    for gspl, gtpl in layer_groups(spl, tpl, args.e2e_group_layers):
        state = S.DeviceState(gspl.layout[0], dev)
        host = {k: torch.empty(a.shape, dtype=a.dtype, pin_memory=True) for k, a in state.arenas.items()}
        for k, a in state.arenas.items():
            host[k].copy_(a)
        groups.append((gspl, gtpl, state, host))
    torch.cuda.synchronize()

    def packed_targets(out, state):
        arena_ptrs = {a.untyped_storage().data_ptr() for a in state.arenas.values()}
        return [t for r in out.values() for e in r.values() for s, t in e.items()
                if s != "step" and t.untyped_storage().data_ptr() not in arena_ptrs]

    h2d = sum(a.numel() * a.element_size() for g in groups for a in g[3].values())
    d2h = 0
    for gspl, gtpl, state, _ in groups:
        out = M.reshard_local(gspl, gtpl, {0: state.state}, exp, dev, views=True)
        d2h += sum(t.numel() * t.element_size() for t in packed_targets(out, state))
        del out
    res_host = torch.empty(d2h, dtype=torch.uint8, pin_memory=True)
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    times = []
    for i in range(args.e2e_warmup + args.e2e_steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ev_in = []
        with torch.cuda.stream(s_in):
            for _, _, state, host in groups:
                for k, a in state.arenas.items():
                    a.copy_(host[k], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_in)
                ev_in.append(ev)
        keep, off = [], 0
        for (gspl, gtpl, state, _), ev in zip(groups, ev_in):
            s_cmp.wait_event(ev)
            with torch.cuda.stream(s_cmp):
                out = M.reshard_local(gspl, gtpl, {0: state.state}, exp, dev, views=True)
            done = torch.cuda.Event()
            done.record(s_cmp)
            s_out.wait_event(done)
            with torch.cuda.stream(s_out):
                for t in packed_targets(out, state):
                    n = t.numel() * t.element_size()
                    res_host[off:off + n].copy_(t.reshape(-1).view(torch.uint8), non_blocking=True)
                    off += n
            keep.append(out)
        torch.cuda.synchronize()
        if i >= args.e2e_warmup:
            times.append(time.perf_counter() - t0)
        del keep
    t = statistics.mean(times)
    del groups, res_host
    torch.cuda.empty_cache()
    return {"value": round(d2h / t / 1e9, 3), "unit": "GB/s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(t * 1e3, 3), "steps": args.e2e_steps,
            "pcie_gbs_h2d": round(h2d / t / 1e9, 2),
            "sample": f"{args.e2e_layers} of 32 layers of cfg2b, {args.e2e_group_layers} layers per pipelined group "
                      f"(pinned host buffers of the source arenas and packed targets)",
            "api": "suika_b200.migration.reshard_local(views=True) per layer group: plan (C ABI) + program + one kernel launch"}


# ---------------------------------------------------------------------------------------------
# N > 1: one process per GPU, TP N -> TP N/2 x PP2 (N = 8: cfg3)
# ---------------------------------------------------------------------------------------------
def run_dist(args):
    rank, world = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    cfg = workload(world, args.layers, args.config)
    spl, tpl = cfg.layouts()
    state = S.DeviceState(spl.layout.get(rank, {}), dev)
    torch.cuda.synchronize()
    exp = S.expected_sub_fields()
    plan = M.Plan(spl, tpl, minimum_est_peers=1)
    src = {n: dict(e) for n, e in state.state.items()}
    if args.direction == "pull":
        rt = M.RankTransfer(plan, src, exp, dev, phased=not args.no_phases)
    else:
        from suika_b200.fanout import plan_fanout
        fo = plan_fanout(plan, STATE_BYTES_PER_ELEM, mode={"off": False, "auto": "auto", "on": True}[args.fanout])
        rt = M.RankTransferPush(plan, src, exp, dev, phased=not args.no_phases, fanout=fo if fo.active else None)
    its = [2, 4, 4, 4]
    rb = plan.rank_bytes(its)
    moved_all = int(plan.op_array["numel"].sum()) * sum(its)
    ingress = rb["ingress"].get(rank, 0)
    # warm-up, then K timed steps between barriers; device time per rank, max over ranks
    # a step: every phase of the reshard (phases separated by host barriers), device time from the
    # first launch to the end of the last kernel on this rank; the step time is the max over ranks
    with Clocks(local) as ck:
        for _ in range(args.warmup):
            dist.barrier()
            rt.run()
            torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        kern = []
        for _ in range(args.steps):
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            rt.run()
            b.record()
            torch.cuda.synchronize()
            kern.append(a.elapsed_time(b))
        torch.cuda.synchronize()
        dist.barrier()
    per_rank = [None] * world
    # kernels per step on this rank: one per phase, two where a phase's table is split between the
    # vector and the tensor-map kernel (a phase with only local pieces, under the default shape)
    n_launch = sum(int(p.info.n_entries > 0) + int(p.info.n_tensor_entries > 0) for p in rt.prepared_phases if p is not None)
    dist.all_gather_object(per_rank, (round(statistics.mean(kern), 4), int(rt.remote_bytes), int(rt.local_bytes), n_launch))
    rt_phase_counts = [p[3] for p in per_rank]
    t = max(p[0] for p in per_rank) / 1e3  # the step ends when the slowest rank's kernel ends
    check = verify_dist(plan, rt, rank, state.state, exp) if not args.no_check else {"status": "skipped"}
    target = rt.finish()
    del target
    max_dir = max(max(rb["ingress"].values(), default=0), max(rb["egress"].values(), default=0))
    e2e = None if args.no_e2e else e2e_dist(args, world, rank, dev)
    res = None
    if rank == 0:
        achieved = max_dir / t / 1e9
        res = {
            "metric": METRIC, "value": round(moved_all / t / 1e9, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded N(0,0.02) weights, norms 1.0, m~N(0,1e-3), v~|N(0,1e-6)|)",
            "config": workload_config(cfg, world),
            "workload_bytes": {"cross_gb": round(sum(rb["ingress"].values()) / 1e9, 3),
                               "local_gb": round(sum(rb["local"].values()) / 1e9, 3),
                               "max_ingress_gb": round(max(rb["ingress"].values(), default=0) / 1e9, 3),
                               "max_egress_gb": round(max(rb["egress"].values(), default=0) / 1e9, 3),
                               "src_choice": "reference", "direction": args.direction, "phases": rt.n_phases},
            "migration_s": round(t, 6),
            "nvlink_gbs_per_gpu": round(max(rb["ingress"].values(), default=0) / t / 1e9, 2),
            "roofline": {"bound": "nvlink", "achieved": round(achieved, 1), "peak": NVLINK_GBS, "unit": "GB/s",
                         "frac": round(achieved / NVLINK_GBS, 4),
                         "peak_source": "NVLink 5, 900 GB/s per direction per GPU",
                         "frac_of_measured_peer_copy": round(achieved / NVLINK_MEASURED_PEER_GBS, 4),
                         "traffic": None, "algorithmic_bytes_per_launch": int(max_dir), "kernel_ms": round(t * 1e3, 4)},
            "gpu_launches": args.steps * sum(rt_phase_counts),
            "per_rank": [{"rank": r, "kernel_ms": p[0], "remote_gb": round(p[1] / 1e9, 3), "local_gb": round(p[2] / 1e9, 3)}
                         for r, p in enumerate(per_rank)],
            "clocks": ck.summary(),
            "check": check,
        }
        if e2e is not None:
            res["e2e"] = e2e
    return res


def run_reference_nccl(args):
    """The reference's own GPU data path on run_dist's workload: oracle/nccl_port.py restates
    execute_param_transfer (Suika/migration.py:397-556) with one NCCL isend/irecv per tensor and
    sub-field, .contiguous() chunks, then cat / clone and cuda_gc. A step is one execute on every
    rank from a fresh shallow copy of the source dict (the reference clears it); device time from
    before the first op to after the last cat, max over ranks."""
    from oracle import nccl_port as P
    from oracle import restate as O
    rank, world = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    cfg = workload(world, args.layers, args.config)
    spl, tpl = cfg.layouts()
    state = S.DeviceState(spl.layout.get(rank, {}), dev)
    torch.cuda.synchronize()
    ops = O.schedule(spl, tpl, minimum_est_peers=1)
    subfields = [(s, k == "meta", S.TORCH_DTYPE[k]) for s, k in S.SUBFIELDS]
    shapes = {n: m.shape for metas in tpl.layout.values() for n, m in metas.items()}
    rb = rank_bytes_ops(ops)  # the reference's path loads no product code
    moved_all = sum(o.numel for o in ops) * STATE_BYTES_PER_ELEM
    times = []
    with Clocks(local) as ck:
        for i in range(args.warmup + args.steps):
            src = {n: dict(e) for n, e in state.state.items()}
            dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            out = P.execute_rank(ops, src, subfields, shapes, rank, dev)
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                times.append(a.elapsed_time(b))
            del out
    per_rank = [None] * world
    dist.all_gather_object(per_rank, round(statistics.mean(times), 4))
    t = max(per_rank) / 1e3
    if rank != 0:
        return None
    max_dir = max(max(rb["ingress"].values(), default=0), max(rb["egress"].values(), default=0))
    return {
        "metric": METRIC, "impl": "reference-nccl", "value": round(moved_all / t / 1e9, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic (as the ours arm)",
        "config": workload_config(cfg, world),
        "path": "oracle/nccl_port.py: execute_param_transfer over NCCL P2P per tensor, cat/clone, cuda_gc",
        "migration_s": round(t, 6), "nvlink_gbs_per_gpu": round(max(rb["ingress"].values(), default=0) / t / 1e9, 2),
        "roofline": {"bound": "nvlink", "achieved": round(max_dir / t / 1e9, 1), "peak": NVLINK_GBS, "unit": "GB/s",
                     "frac": round(max_dir / t / 1e9 / NVLINK_GBS, 4)},
        "per_rank_ms": per_rank, "clocks": ck.summary(),
    }


def region_checksum(t: torch.Tensor, offset: int, rows: int, row_bytes: int, pitch: int) -> int:
    """Position-weighted checksum (mod 2^64) of a strided byte region of tensor t's storage."""
    b = t.reshape(-1).view(torch.uint8) if t.dim() else t.reshape(1).view(torch.uint8)
    offset += b.storage_offset()  # as_strided offsets count from the start of the storage
    acc = 0
    step = max(1, (64 << 20) // max(row_bytes, 1))
    for r0 in range(0, rows, step):
        nr = min(step, rows - r0)
        v = b.as_strided((nr, row_bytes), (pitch, 1), offset + r0 * pitch).to(torch.int64)
        w = (torch.arange(r0 * row_bytes, (r0 + nr) * row_bytes, device=t.device, dtype=torch.int64) % 65521 + 1).view(nr, row_bytes)
        acc += int((v * w).sum().item())
    return acc % (1 << 64)


def verify_dist(plan, rt, rank, src_state, exp) -> dict:
    """Full-size check of every piece this rank pulled: a position-weighted checksum of the piece
    in its target tensor (computed here) must equal the checksum of the same region of the source
    tensor (computed by the source rank on its own copy). Pieces land in their cat position by the
    same program the small-size parity tests pin against the reference."""
    subs = [s for s, _ in exp]
    kinds = dict(S.SUBFIELDS)  # a rank may hold no source (a DP grow's new ranks)
    spec = [(4, True) if kinds[s] == "meta" else (S.TORCH_DTYPE[kinds[s]].itemsize, False) for s in subs]
    mine = []
    if rt.target:
        prog = plan.program(rank, spec)
        for sg in prog.segments:
            ss, ds = prog.src_slots[sg["src_slot"]], prog.dst_slots[sg["dst_slot"]]
            name = plan.names[ds["name_id"]]
            t = rt.target[name][subs[ds["subfield"]]]
            c = region_checksum(t, int(sg["dst_offset"]), int(sg["rows"]), int(sg["row_bytes"]), int(sg["dst_pitch"]))
            mine.append((int(ss["src_rank"]), plan.names[ss["name_id"]], subs[ss["subfield"]], int(sg["src_offset"]),
                         int(sg["rows"]), int(sg["row_bytes"]), int(sg["src_pitch"]), c))
    allc = [None] * dist.get_world_size()
    dist.all_gather_object(allc, mine)
    bad = checked = 0
    for lst in allc:
        for sr, name, sub, off, rows, rb, pitch, c in lst:
            if sr != rank:
                continue
            checked += 1
            bad += region_checksum(src_state[name][sub], off, rows, rb, pitch) != c
    tot = torch.tensor([checked, bad], dtype=torch.int64, device=rt.device)
    dist.all_reduce(tot)
    return {"pieces_checked": int(tot[0]), "mismatches": int(tot[1]), "status": "pass" if int(tot[1]) == 0 else "FAIL",
            "how": "position-weighted checksum of every piece, target side vs source side"}


def e2e_dist(args, world, rank, dev):
    """The drop-in schedule_and_execute_param_transfer end to end on a layer sample: per step the
    source shard is copied in from pinned host memory, the call plans, exchanges handles, maps
    peers, pulls and syncs, and the targets are read back to pinned host memory."""
    cfg = workload(world, 2, args.config)  # one decoder layer per target stage keeps every rank's pinned buffers small
    spl, tpl = cfg.layouts()
    state = S.DeviceState(spl.layout.get(rank, {}), dev)
    host = {k: torch.empty(a.shape, dtype=a.dtype, pin_memory=True) for k, a in state.arenas.items()}
    for k, a in state.arenas.items():
        host[k].copy_(a)
    exp = S.expected_sub_fields()
    h2d = sum(a.numel() * a.element_size() for a in host.values())
    ctx = {"expected_sub_fields": exp}
    times, d2h, moved = [], 0, 0
    res_host = None
    for i in range(args.e2e_warmup + args.e2e_steps):
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for k, a in state.arenas.items():
            a.copy_(host[k], non_blocking=True)
        src = {n: dict(e) for n, e in state.state.items()}
        out = M.schedule_and_execute_param_transfer(spl, tpl, src, ctx, dev, None, direction=args.direction)
        ts = [t for e in out.values() for s, t in e.items() if s != "step"]
        n = sum(t.numel() * t.element_size() for t in ts)
        if res_host is None:
            res_host = torch.empty(max(n, 1), dtype=torch.uint8, pin_memory=True)
        off = 0
        for t in ts:
            k = t.numel() * t.element_size()
            res_host[off:off + k].copy_(t.reshape(-1).view(torch.uint8), non_blocking=True)
            off += k
        torch.cuda.synchronize()
        dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
        dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        if i >= args.e2e_warmup:
            times.append(float(dt.item()))
        d2h = n
        del out, ts
    tot = torch.tensor([d2h, h2d], dtype=torch.float64, device=dev)
    dist.all_reduce(tot)
    t = statistics.mean(times)
    del state, host, res_host
    torch.cuda.empty_cache()
    return {"value": round(float(tot[0]) / t / 1e9, 3), "unit": "GB/s", "h2d_bytes_per_step": int(tot[1]),
            "d2h_bytes_per_step": int(tot[0]), "ms_per_step": round(t * 1e3, 3), "steps": args.e2e_steps,
            "sample": f"{cfg.spec.n_layers} layers of the workload (pinned host buffers on every rank)",
            "api": "suika_b200.migration.schedule_and_execute_param_transfer (drop-in for Suika/migration.py:558)"}


# ---------------------------------------------------------------------------------------------
# Reference arm: the oracle port on the host cores (rank 0 only)
# ---------------------------------------------------------------------------------------------
def run_reference(args, world):
    cfg = workload(world, args.layers, args.config)
    threads = os.cpu_count() or 1
    smp = OracleSample(cfg, world, threads)
    for _ in range(args.warmup):
        smp.step()
    t = sum(smp.step() for _ in range(args.steps))
    v = smp.units * args.steps / t / 1e9
    return {
        "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic (seeded N(0,0.02) weights, norms 1.0, m~N(0,1e-3), v~|N(0,1e-6)|)", "impl": "reference",
        "config": workload_config(cfg, world),
        "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": threads, "kind": "port", "sample": smp.describe(args.steps)},
        "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-nccl"], default="ours",
                    help="reference: the CPU oracle (the driver's reference arm); reference-nccl: the reference's "
                         "own GPU path (execute_param_transfer over NCCL P2P per tensor, N > 1 under torchrun)")
    ap.add_argument("--layers", type=int, default=0, help="override the workload's layer count (smaller cases)")
    ap.add_argument("--config", default="", choices=["", "cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "dpgrow8"],
                    help="N > 1: measure this named reshard instead of the default family (its rank count must be N); "
                         "dpgrow8 is the DP grow from one GPU to eight where --fanout applies")
    ap.add_argument("--e2e-layers", type=int, default=8)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--e2e-warmup", type=int, default=1)
    ap.add_argument("--e2e-group-layers", type=int, default=1,
                    help="N = 1 e2e: layers per pipelined group (copy in, reshard, copy out overlap across groups)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true")
    ap.add_argument("--no-phases", action="store_true", help="N > 1: run all transfers at once instead of in matching phases")
    ap.add_argument("--handoff", action="store_true", help="time the old -> new process hand-off instead (1 GPU)")
    ap.add_argument("--metadata", action="store_true",
                    help="time the layout exchange before a reshard instead (N ranks under torchrun; gloo without GPUs)")
    ap.add_argument("--activation", action="store_true",
                    help="time the pipeline activation hand-over between two stages instead (N >= 2 under torchrun)")
    ap.add_argument("--fanout", choices=["off", "auto", "on"], default="off",
                    help="N > 1, push: DP-replica fan-out (suika_b200.fanout); the default workloads have no replicas")
    ap.add_argument("--direction", choices=["pull", "push"], default="push",
                    help="N > 1: target ranks read their pieces (pull) or source ranks write them (push)")
    ap.add_argument("--checkpoint", action="store_true",
                    help="time checkpoint resume instead: one target rank's state built on the GPU from host shards "
                         "(1 GPU; ours against the reference's CPU execute plus a copy to the GPU)")
    ap.add_argument("--peer-probe", action="store_true",
                    help="time the copy kernel's peer patterns between GPU 0 and GPU 1 instead (one process, 2 GPUs)")
    ap.add_argument("--peer-gib", type=float, default=2.0)
    ap.add_argument("--peer-variants", default="2,6")
    ap.add_argument("--peer-one", action="store_true",
                    help="with --peer-probe: one pull launch then one push launch on GPU 0 against GPU 1 (for a profiler)")
    ap.add_argument("--pack-probe", action="store_true",
                    help="time the copy kernel's one-GPU patterns (column slices of one source, one contiguous run) instead")
    ap.add_argument("--pack-gib", type=float, default=8.0)
    ap.add_argument("--pack-variants", default="8,9,11,14")
    args = ap.parse_args()
    if args.peer_probe:
        run_peer_probe(args)
        return
    if args.pack_probe:
        run_pack_probe(args)
        return
    if args.checkpoint:
        print(json.dumps(run_checkpoint(args)), flush=True)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.handoff:
        print(json.dumps(run_handoff(args)), flush=True)
        return
    if args.metadata:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group(backend)
        try:
            res = run_metadata(args)
        finally:
            dist.barrier()
            dist.destroy_process_group()
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.activation:
        import datetime
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        try:
            res = run_activation(args)
        finally:
            dist.barrier()
            dist.destroy_process_group()
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, max(world, args.gpus))), flush=True)
        return
    if args.impl == "reference-nccl" and world < 2:
        raise SystemExit("--impl reference-nccl times the reference's P2P path: run N >= 2 ranks under torchrun")
    if world > 1:
        import datetime
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        try:
            res = run_reference_nccl(args) if args.impl == "reference-nccl" else run_dist(args)
        finally:
            dist.barrier()
            dist.destroy_process_group()
    else:
        res = run_single(args)
    if res is not None:
        print(json.dumps(res), flush=True)



# ---------------------------------------------------------------------------------------------
# --checkpoint: checkpoint resume, one target rank built from host-resident source shards (1 GPU)
# ---------------------------------------------------------------------------------------------
def run_checkpoint(args):
    """Checkpoint resume (Suika/migration.py:1156-1305): every source shard a target rank needs is
    in host memory (loaded from disk; loading is not timed), and the rank's new state must end up on
    its GPU. Workload: target rank 0 of the cfg3 family (Llama2-13B-shaped, TP8 -> TP4 x PP2) on a
    layer sample. A step:
      ours: execute_param_transfer(..., fake_source_state_dicts=...) -- the needed shards are
        gathered into one page-locked arena and one launch writes every target on the GPU, reading
        host memory over PCIe;
      reference: its execute_param_transfer on device "cpu" (migration.py:1235-1244; restated in
        oracle/nccl_port.checkpoint_rank, pinned to the golden digests), then every target copied
        to the GPU.
    Wall time per step after a synchronize on both sides; the two results are compared byte for
    byte once, outside the timing."""
    from oracle import nccl_port as P
    from oracle import restate as O
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = workload(8, args.layers or 8)
    spl, tpl = cfg.layouts()
    rank = 0
    mep = 1 if M.is_ib_enabled() else 2
    ops = O.schedule(spl, tpl, minimum_est_peers=mep)
    src_ranks = sorted({o.src for o in ops if o.dst == rank})
    states = S.host_states(spl, S.SUBFIELDS, seed=0, ranks=src_ranks)
    fake = {r: {n: {s: S.to_torch(a, k) for (s, k), a in zip(S.SUBFIELDS, e.values())} for n, e in st.items()}
            for r, st in states.items()}
    del states
    exp = S.expected_sub_fields()
    subfields = [(s, k == "meta", S.TORCH_DTYPE[k]) for s, k in S.SUBFIELDS]
    sched = M.schedule_param_transfer(spl, tpl)
    target_bytes = sum(o.numel for o in ops if o.dst == rank) * STATE_BYTES_PER_ELEM

    def ours():
        return M.execute_param_transfer(sched, fake.get(rank, {}), dev, exp, fake_source_state_dicts=fake, rank=rank)

    def reference():
        out = P.checkpoint_rank(ops, fake, subfields, rank)
        return {n: {s: t.to(dev) for s, t in e.items()} for n, e in out.items()}

    res = {}
    for name, fn in (("ours", ours), ("reference", reference)):
        times = []
        for i in range(args.warmup + args.steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            out = fn()
            torch.cuda.synchronize()
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
            if i < args.warmup + args.steps - 1:
                del out
        res[name] = (statistics.median(times), out)
    a, b = res["ours"][1], res["reference"][1]
    same = list(a) == list(b) and all(torch.equal(a[n][s].reshape(-1), b[n][s].reshape(-1)) for n in a for s in a[n])
    t_ours, t_ref = res["ours"][0], res["reference"][0]
    return {"metric": "checkpoint resume: one target rank's training state built on its GPU from host shards",
            "value": round(target_bytes / t_ours / 1e9, 3), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ours * 1e3, 2), "higher_is_better": True,
            "config": {"workload": f"target rank {rank} of {cfg.note} ({cfg.spec.n_layers} layers), full training state, "
                                   f"source shards of ranks {src_ranks} in host memory"},
            "target_gb": round(target_bytes / 1e9, 3), "reference_ms_per_step": round(t_ref * 1e3, 2),
            "reference_gbs": round(target_bytes / t_ref / 1e9, 3), "speedup": round(t_ref / t_ours, 2),
            "check": {"byte_equal": bool(same)},
            "reference_path": "oracle/nccl_port.checkpoint_rank (execute on device cpu, Suika/migration.py:1235-1244) + .to(cuda)",
            "host_threads": torch.get_num_threads()}


# ---------------------------------------------------------------------------------------------
# --peer-probe: peer patterns between two GPUs (one process)
# ---------------------------------------------------------------------------------------------
def _peer_enable_access() -> None:
    import ctypes
    import glob
    libs = glob.glob(os.path.join(os.path.dirname(torch.__file__), "..", "nvidia", "cuda_runtime", "lib", "libcudart.so*"))
    if not libs:
        raise RuntimeError("libcudart not found next to torch")
    rt = ctypes.CDLL(libs[0])
    for a, b in ((0, 1), (1, 0)):
        rt.cudaSetDevice(a)
        rt.cudaDeviceEnablePeerAccess(b, 0)  # an "already enabled" return is fine


def _peer_row(src, dst, n, strided, remote):
    if strided:
        return (src, dst, n // 2560, 1280, 2560, 2560, remote)
    return (src, dst, 1, n, n, n, remote)


def _peer_time(per_dev, reps=5):
    preps = {}
    for dev, ents in per_dev.items():
        with torch.cuda.device(dev):
            t = np.array([_peer_row(*e) for e in ents], dtype=M.L.COPY_DESC_DTYPE)
            preps[dev] = M.PreparedCopies(t, torch.device("cuda", dev))
    for dev, p in preps.items():
        with torch.cuda.device(dev):
            p.launch()
    for d in (0, 1):
        torch.cuda.synchronize(d)
    ev = {}
    for dev, p in preps.items():
        with torch.cuda.device(dev):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(reps):
                p.launch()
            b.record()
            ev[dev] = (a, b)
    for d in (0, 1):
        torch.cuda.synchronize(d)
    for p in preps.values():
        p.check()
    return max(a.elapsed_time(b) for a, b in ev.values()) / reps


def run_peer_probe(args):
    """Peer-bandwidth patterns between GPU 0 and GPU 1 for the copy kernel (one process). For each
    launch shape (SUIKA_RS_VARIANT) and piece shape (one contiguous run; 1280-byte rows at a
    2560-byte pitch, like a TP8 -> TP4 row-parallel piece) it times, per direction:
      pull: the kernel on GPU a reads GPU b's memory;  push: it writes GPU b's memory;
      1-way: one GPU copies;  2-way: both copy at once in opposite directions;
      +local: the same table also holds an equal local copy (interleaved with the remote one).
    These are the patterns a reshard is made of; they decide its direction and phasing."""
    if torch.cuda.device_count() < 2:
        raise SystemExit("needs two GPUs")
    _peer_enable_access()
    n = int(args.peer_gib * (1 << 30))
    if args.peer_one:
        d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
        a0, b0 = torch.ones(n, dtype=torch.uint8, device=d0), torch.empty(n, dtype=torch.uint8, device=d0)
        a1 = torch.full((n,), 2, dtype=torch.uint8, device=d1)
        b1 = torch.empty(n, dtype=torch.uint8, device=d1)
        for name, (s_, d_) in (("pull", (a1, b0)), ("push", (a0, b1))):
            p = M.PreparedCopies(np.array([_peer_row(s_.data_ptr(), d_.data_ptr(), n, False, 1)], dtype=M.L.COPY_DESC_DTYPE), d0)
            p.launch()
            p.check()
            assert torch.equal(d_[:1024].cpu(), s_[:1024].cpu())
            print(f"{name}: {n} bytes copied", flush=True)
        return
    b = {d: [torch.empty(n, dtype=torch.uint8, device=torch.device("cuda", d)) for _ in range(4)] for d in (0, 1)}
    p = {d: [t.data_ptr() for t in b[d]] for d in (0, 1)}
    for var in args.peer_variants.split(","):
        os.environ["SUIKA_RS_VARIANT"] = var
        for st in (False, True):
            moved = n // 2 if st else n
            pats = {
                "pull 1-way": {0: [(p[1][0], p[0][1], n, st, 1)]},
                "pull 2-way": {0: [(p[1][0], p[0][1], n, st, 1)], 1: [(p[0][0], p[1][1], n, st, 1)]},
                "push 1-way": {0: [(p[0][0], p[1][1], n, st, 1)]},
                "push 2-way": {0: [(p[0][0], p[1][1], n, st, 1)], 1: [(p[1][0], p[0][1], n, st, 1)]},
                "pull 2-way +local": {0: [(p[1][0], p[0][1], n, st, 1), (p[0][2], p[0][3], n, st, 0)],
                                      1: [(p[0][0], p[1][1], n, st, 1), (p[1][2], p[1][3], n, st, 0)]},
                "push 2-way +local": {0: [(p[0][0], p[1][1], n, st, 1), (p[0][2], p[0][3], n, st, 0)],
                                      1: [(p[1][0], p[0][1], n, st, 1), (p[1][2], p[1][3], n, st, 0)]},
            }
            for name, cfg in pats.items():
                ms = _peer_time(cfg)
                print(f"variant {var} {'strided' if st else 'contig '} {name:18s}: {ms:7.3f} ms  "
                      f"{moved / ms / 1e6:6.0f} GB/s per direction", flush=True)


# ---------------------------------------------------------------------------------------------
# --pack-probe: one-GPU copy patterns (one process)
# ---------------------------------------------------------------------------------------------
def _median_event_s(fn, reps=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in evs:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return float(np.median([a.elapsed_time(b) for a, b in evs])) / 1e3


def run_pack_probe(args):
    """One-GPU patterns of a relayout, per launch shape (SUIKA_RS_VARIANT). A "halves" pattern is
    the TP-grow pieces of row-parallel weights: source matrices of 4096 rows (Llama2-7B's hidden
    size) with rows of twice row_bytes, each cut into its two column slices, written to two
    contiguous targets, as many matrices as the buffer holds (22016-byte slices are fp32 down_proj
    half-rows, 11008 their bf16 copy, 8192 fp32 o_proj half-rows). "contiguous" is one run over
    the whole buffer. The buffer is larger than L2; rates are read + write bytes over the median
    CUDA-event time of 10 launches, beside torch's own copy of the whole buffer."""
    dev = torch.device("cuda", 0)
    n = int(args.pack_gib * (1 << 30)) & ~((1 << 20) - 1)
    src = torch.randint(0, 255, (n,), dtype=torch.uint8, device=dev)
    dst = torch.empty(n, dtype=torch.uint8, device=dev)
    t = _median_event_s(lambda: dst.copy_(src))
    print(f"torch copy_: {2 * n / t / 1e9:.0f} GB/s", flush=True)
    rows = 4096
    pats = {}
    for rb in (22016, 11008, 8192, 4096):
        mat = rows * 2 * rb
        descs = []
        for m in range(n // mat):
            for h in (0, 1):
                descs.append((src.data_ptr() + m * mat + h * rb, dst.data_ptr() + m * mat + h * rows * rb, rows, rb, 2 * rb, rb, 0))
        pats[f"halves {rb}/{2 * rb} x{n // mat}"] = descs
    pats["contiguous"] = [(src.data_ptr(), dst.data_ptr(), 1, n, n, n, 0)]
    for v in args.pack_variants.split(","):
        os.environ["SUIKA_RS_VARIANT"] = v
        for name, descs in pats.items():
            moved = sum(d[2] * d[3] for d in descs)
            dst.zero_()
            p = M.PreparedCopies(np.array(descs, dtype=M.L.COPY_DESC_DTYPE), dev)
            t = _median_event_s(p.launch)
            p.check()
            for d in (descs[0], descs[-1]):
                got = torch.empty(d[2] * d[3], dtype=torch.uint8, device=dev)
                got.copy_(dst[d[1] - dst.data_ptr():][:d[2] * d[3]])
                want = src[d[0] - src.data_ptr():][:(d[2] - 1) * d[4] + d[3]].as_strided((d[2], d[3]), (d[4], 1))
                if not torch.equal(got.view(d[2], d[3]), want):
                    raise RuntimeError(f"variant {v} {name}: target differs from source")
            print(f"variant {v:>2} {name:26s}: {t * 1e3:7.3f} ms {2 * moved / t / 1e9:6.0f} GB/s  "
                  f"(vector entries {p.info.n_entries}, tensor-map entries {p.info.n_tensor_entries}, boxes {p.info.n_tensor_tiles})",
                  flush=True)
            del p


# ---------------------------------------------------------------------------------------------
# --handoff: old -> new process hand-off of one rank's state on one GPU
# ---------------------------------------------------------------------------------------------
def _ref_send(queues, tensors):
    """Suika's per-tensor protocol (Suika/utils.py:325-386): one queue message and one ack per
    CUDA tensor, freeing each after its ack."""
    queues[0].put(len(tensors))
    for t in tensors:
        queues[0].put(t, block=True)
        queues[1].get(block=True)
        t.untyped_storage().resize_(0)


def _ref_recv(queues):
    """Suika/utils.py:389-406: receive, clone, ack, one tensor at a time."""
    n = queues[0].get(block=True)
    out = []
    for _ in range(n):
        t = queues[0].get(block=True)
        out.append(t.clone())
        del t
        queues[1].put(None, block=True)
    torch.cuda.synchronize()
    return out


def _handoff_old(queues, mode, layers, ready):
    from suika_b200 import handoff
    torch.cuda.set_device(0)
    cfg = workload(8, layers)
    spl, _ = cfg.layouts()
    st = {}
    for name, m in spl.layout[1].items():  # one rank's source shard, one allocation per tensor
        shape = S._actual_shape(m)
        st[name] = {s: torch.empty(shape, dtype=S.TORCH_DTYPE[k], device="cuda:0").fill_(1) for s, k in S.SUBFIELDS if k != "meta"}
        st[name]["step"] = torch.tensor(1.0)
    torch.cuda.synchronize()
    ready.put(sum(t.numel() * t.element_size() for e in st.values() for t in e.values() if t.is_cuda))
    if mode == "reference":
        _ref_send(queues, [t for e in st.values() for t in e.values() if t.is_cuda])
    else:
        handoff.interactive_IPC_state_dict_send(queues, {"source_param_layout": None, "source_state_dict": st, "other_context_dict": {}})


def _handoff_new(queues, mode, result):
    from suika_b200 import handoff
    torch.cuda.set_device(0)
    torch.zeros(1, device="cuda:0")
    t0 = time.perf_counter()
    if mode == "reference":
        out = _ref_recv(queues)
        n = len(out)
    else:
        state = handoff.interactive_IPC_state_dict_recv(queues)
        sd = state["source_state_dict"]
        n = sum(1 for e in sd.values() for t in e.values() if t.is_cuda)
        torch.cuda.synchronize()
        sd.clear()
        sd.release()
    result.put((time.perf_counter() - t0, n))


def _get_or_fail(q, procs, timeout_s=600.0):
    """Queue get that gives up as soon as one of `procs` has died, or after timeout_s."""
    import queue as _queue
    t0 = time.perf_counter()
    while True:
        try:
            return q.get(timeout=1.0)
        except _queue.Empty:
            dead = [p.exitcode for p in procs if not p.is_alive()]
            if dead or time.perf_counter() - t0 > timeout_s:
                for p in procs:
                    if p.is_alive():
                        p.kill()
                raise RuntimeError(f"hand-off process failed (exit codes {[p.exitcode for p in procs]})")


def run_handoff(args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    res = {"metric": "old->new process hand-off of one rank's migration state (s)", "unit": "s", "higher_is_better": False,
           "n_gpus": 1, "config": {"workload": f"one cfg3 source rank: Llama2-13B TP8 shard, {args.layers or 40} layers, "
                                               "bf16 param + fp32 master/m/v, one allocation per tensor, old and new process on one GPU"}}
    for mode in ("reference", "batched-zero-copy"):
        times = []
        for rep in range(max(1, args.steps)):
            queues, ready, result = (ctx.Queue(), ctx.Queue()), ctx.Queue(), ctx.Queue()
            po = ctx.Process(target=_handoff_old, args=(queues, mode, args.layers, ready))
            po.start()
            nbytes = _get_or_fail(ready, [po])
            pn = ctx.Process(target=_handoff_new, args=(queues, mode, result))
            pn.start()
            dt, n = _get_or_fail(result, [po, pn])
            pn.join(120)
            po.join(120)
            if pn.exitcode != 0 or po.exitcode != 0:
                raise RuntimeError(f"hand-off processes exited with {pn.exitcode}, {po.exitcode}")
            times.append(dt)
        res[mode] = {"seconds": round(statistics.median(times), 4), "tensors": n, "bytes": int(nbytes), "runs": len(times)}
    res["value"] = res["batched-zero-copy"]["seconds"]
    res["speedup_vs_reference_protocol"] = round(res["reference"]["seconds"] / max(res["value"], 1e-9), 1)
    return res


# ---------------------------------------------------------------------------------------------
# --activation: pipeline activation hand-over between two stages (N GPUs under torchrun)
# ---------------------------------------------------------------------------------------------
ACT_BATCH, ACT_SEQ, ACT_HIDDEN = 8, 2048, 5120


def activation_stages(world: int):
    """Stage A: the first N/2 ranks as one TP group; stage B: the other N/2 as DP N/2 x TP1 (the
    boundary a TP -> DP re-plan makes). Global micro-batch 8 x 2048 tokens, hidden 5120 (13B), bf16."""
    half = world // 2
    return [list(range(half))], [ACT_BATCH], [[half + i] for i in range(half)], [ACT_BATCH // half] * half


def _ref_port_exchange(rank, mesh_s, mesh_d, bsz_s, bsz_d, act, target, tp_groups):
    """The reference's sequence for one direction (Suika/pipeline_parallel.py:687-836, with
    Suika/utils.py:212-234): per block a .contiguous() staging copy, non-batched isend/irecv
    (sends first), copy back into place, then the receiving TP group's all-gather + cat + copy."""
    from oracle import activation as OA
    sends, recvs, restore = [], [], []
    if act is not None:
        for peer, b0, nb, deg, tr in OA.p2p_ops(rank, mesh_s, mesh_d, bsz_s, bsz_d, "send"):
            c = act.shape[-1] // deg
            sends.append((act.narrow(0, b0, nb).narrow(-1, tr * c, c).contiguous(), peer))
    if target is not None:
        for peer, b0, nb, deg, tr in OA.p2p_ops(rank, mesh_s, mesh_d, bsz_s, bsz_d, "recv"):
            c = target.shape[-1] // deg
            view = target.narrow(0, b0, nb).narrow(-1, tr * c, c)
            buf = view.contiguous()
            recvs.append((buf, peer))
            restore.append((view, buf))
    reqs = [dist.isend(t, dst=p) for t, p in sends] + [dist.irecv(t, src=p) for t, p in recvs]
    for q in reqs:
        q.wait()
    for view, buf in restore:
        view.copy_(buf)
    if target is not None:
        for group, pg in tp_groups:
            if rank in group and len(group) > 1:
                j = group.index(rank)
                part = target.chunk(len(group), dim=-1)[j]
                parts = [torch.empty_like(part) for _ in group]
                dist.all_gather(parts, part.contiguous(), group=pg)
                target.copy_(torch.cat(parts, dim=-1))


def run_activation(args):
    from suika_b200 import activation as A
    rank, world = dist.get_rank(), dist.get_world_size()
    if world < 2 or world % 2 or ACT_BATCH % (world // 2):
        raise SystemExit("--activation needs an even number of ranks (2, 4 or 8)")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    ma, ba, mb, bb = activation_stages(world)
    shape, dtype = [-1, ACT_SEQ, ACT_HIDDEN], torch.bfloat16
    in_a = rank in ma[0]
    in_b = not in_a

    def mine(rows: int) -> torch.Tensor:
        g = torch.Generator(dev).manual_seed(rank)
        return torch.randn(rows, ACT_SEQ, ACT_HIDDEN, device=dev, generator=g).to(dtype)
    b_rows = bb[0]
    act_f = mine(ACT_BATCH) if in_a else None           # forward: A sends, B receives
    act_b = mine(b_rows) if in_b else None              # backward: B sends, A receives
    tgt_f = torch.zeros(b_rows, ACT_SEQ, ACT_HIDDEN, dtype=dtype, device=dev) if in_b else None
    tgt_b = torch.zeros(ACT_BATCH, ACT_SEQ, ACT_HIDDEN, dtype=dtype, device=dev) if in_a else None
    tp_groups = [(g, dist.new_group(g)) for g in ma + mb]  # every rank creates every group
    if args.impl == "reference":
        def step():
            _ref_port_exchange(rank, ma, mb, ba, bb, act_f, tgt_f, tp_groups)
            _ref_port_exchange(rank, mb, ma, bb, ba, act_b, tgt_b, tp_groups)
        launches = None
    else:
        fwd = A.ActivationExchange(rank, ma, mb, ba, bb, shape, dtype, device=dev)
        bwd = A.ActivationExchange(rank, mb, ma, bb, ba, shape, dtype, device=dev)

        def step():
            fwd.exchange(act_f, tgt_f)
            bwd.exchange(act_b, tgt_b)
        launches = 2  # per rank and step: one send launch in one direction, one receive copy in the other
    with Clocks(dev.index) as ck:
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        times = []
        for _ in range(args.steps):
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            step()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        dist.barrier()
    check = {"status": "skipped"}
    if args.impl != "reference":
        # the same inputs through the reference's sequence must give the same bytes
        ref_f = torch.zeros_like(tgt_f) if tgt_f is not None else None
        ref_b = torch.zeros_like(tgt_b) if tgt_b is not None else None
        _ref_port_exchange(rank, ma, mb, ba, bb, act_f, ref_f, tp_groups)
        _ref_port_exchange(rank, mb, ma, bb, ba, act_b, ref_b, tp_groups)
        torch.cuda.synchronize()
        ok = all(torch.equal(x, y) for x, y in ((tgt_f, ref_f), (tgt_b, ref_b)) if x is not None)
        flags = [None] * world
        dist.all_gather_object(flags, ok)
        check = {"status": "pass" if all(flags) else "FAIL", "what": "every received tensor equals the reference sequence's"}
        fwd.check()
        bwd.check()
        fwd.close()
        bwd.close()
    per_rank = [None] * world
    dist.all_gather_object(per_rank, round(statistics.mean(times), 4))
    t = max(per_rank) / 1e3
    elem = 2
    fwd_bytes = ACT_BATCH * ACT_SEQ * ACT_HIDDEN * elem            # every B rank gets its rows once
    bwd_bytes = len(ma[0]) * ACT_BATCH * ACT_SEQ * ACT_HIDDEN * elem  # every A rank gets the whole batch
    pf = A.plan_activation_exchange(ma, mb, ba, bb, ACT_HIDDEN)
    pb = A.plan_activation_exchange(mb, ma, bb, ba, ACT_HIDDEN)
    # the two directions run one after the other: the step's NVLink bound is the sum over them of
    # the busiest GPU direction (ingress or egress) of each
    max_dir = 0
    for pcs in (pf, pb):
        io = {}
        for p in pcs:
            nb = int(p["n_batch"]) * ACT_SEQ * int(p["slice_len"]) * elem
            if p["src_rank"] != p["dst_rank"]:
                io.setdefault(int(p["src_rank"]), [0, 0])[1] += nb
                io.setdefault(int(p["dst_rank"]), [0, 0])[0] += nb
        max_dir += max(max(v) for v in io.values())
    if rank != 0:
        return None
    res = {
        "metric": "pipeline activation hand-over between stages (forward + backward per micro-batch)",
        "value": round((fwd_bytes + bwd_bytes) / t / 1e9, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(t * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded normal activations)",
        "config": {"workload": f"stage A TP{len(ma[0])} -> stage B DP{len(mb)} x TP1 and back; micro-batch "
                               f"{ACT_BATCH} x {ACT_SEQ} tokens, hidden {ACT_HIDDEN}, bf16",
                   "received_mb_per_step": round((fwd_bytes + bwd_bytes) / 1e6, 1),
                   "l2": "buffers reused each step; per-step bytes above L2 only at N >= 4"},
        "roofline": {"bound": "nvlink", "achieved": round(max_dir / t / 1e9, 1), "peak": NVLINK_GBS, "unit": "GB/s",
                     "frac": round(max_dir / t / 1e9 / NVLINK_GBS, 4), "algorithmic_bytes_per_step": int(max_dir),
                     "peak_source": "NVLink 5, 900 GB/s per direction per GPU",
                     "frac_of_measured_peer_copy": round(max_dir / t / 1e9 / NVLINK_MEASURED_PEER_GBS, 4), "traffic": None},
        "per_rank_ms": per_rank, "clocks": ck.summary(), "check": check,
    }
    if launches is not None:
        res["gpu_launches"] = launches * args.steps
    if args.impl == "reference":
        res["impl"] = "reference"
        res["reference_kind"] = "port of the reference's NCCL sequence (torch.distributed isend/irecv + all_gather)"
    return res


# ---------------------------------------------------------------------------------------------
# --metadata: the layout exchange before a reshard (N ranks under torchrun; gloo without GPUs)
# ---------------------------------------------------------------------------------------------
def run_metadata(args):
    """What precedes the copies of a reshard: both layouts gathered from every rank, then the plan.
    The reference gathers {name: TensorMeta} objects with all_gather_object (ParamLayout.gather,
    Suika/migration.py:172-192) and plans from them; suika_b200.metadata gathers records
    (gather_param_layout) and plans from the records. cfg3's layouts when the world has 8 ranks,
    otherwise the Llama2-13B TP N -> TP N/2 x PP2 layouts."""
    from suika_b200 import metadata as MD
    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = CONFIGS["cfg3"] if world == 8 else workload(world)
    spl, tpl = cfg.layouts()
    src_mine, dst_mine = spl.layout.get(rank, {}), tpl.layout.get(rank, {})
    ref_t, ours_t = [], []
    for i in range(args.warmup + args.steps):
        dist.barrier()
        t0 = time.perf_counter()
        layouts = []
        for mine in (src_mine, dst_mine):
            objs = [None] * world
            dist.all_gather_object(objs, mine)
            pl = M.ParamLayout()
            pl.layout = dict(enumerate(objs))
            layouts.append(pl)
        ref_plan = M.Plan(*layouts, minimum_est_peers=1)
        t1 = time.perf_counter()
        dist.barrier()
        t2 = time.perf_counter()
        ours_plan = M.Plan(MD.gather_param_layout(src_mine), MD.gather_param_layout(dst_mine), minimum_est_peers=1)
        t3 = time.perf_counter()
        if i >= args.warmup:
            ref_t.append(t1 - t0)
            ours_t.append(t3 - t2)
        if i == 0 and not np.array_equal(ref_plan.op_array, ours_plan.op_array):
            raise RuntimeError("plans from records and from objects differ")
    stats = [None] * world
    dist.all_gather_object(stats, [statistics.median(ref_t), statistics.median(ours_t)])
    if rank != 0:
        return None
    ref_s, ours_s = max(s[0] for s in stats), max(s[1] for s in stats)
    return {"metric": "layout exchange and planning before a reshard (s, max over ranks, median of steps)", "unit": "s",
            "higher_is_better": False, "backend": dist.get_backend(), "world": world,
            "steps": args.steps, "warmup": args.warmup,
            "config": {"workload": f"{cfg.name} source and target layouts, {len(src_mine)} tensors on rank 0 before"},
            "value": round(ours_s, 6), "reference_objects_s": round(ref_s, 6), "records_s": round(ours_s, 6),
            "speedup": round(ref_s / ours_s, 2), "check": "plans equal"}


if __name__ == "__main__":
    main()

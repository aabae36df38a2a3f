"""Host-side pieces of bench.py, on the CPU: which reshard each run measures, the activation
stages, and the port of the reference's activation sequence (the baseline of `--activation`)
against the oracle on 4 gloo ranks."""
import os

import numpy as np
import pytest
import torch

import bench


def test_workloads():
    assert bench.workload(1).name == "cfg2b"
    c8 = bench.workload(8)
    assert c8.name == "cfg3" and c8.spec.n_layers == 40 and c8.world_size == 8
    assert bench.workload(4).spec.n_layers == 20 and bench.workload(2).spec.n_layers == 10
    with pytest.raises(SystemExit):
        bench.workload(3)
    for c in ("cfg2", "cfg4", "cfg5"):
        cfg = bench.workload(8, 2, c)
        assert cfg.world_size == 8 and cfg.spec.n_layers == 2
    with pytest.raises(SystemExit, match="runs on 8 ranks"):
        bench.workload(4, 0, "cfg3")
    assert bench.workload(8, 0, "dpgrow8").spec.n_layers == 16


def test_activation_stages():
    assert bench.activation_stages(4) == ([[0, 1]], [8], [[2], [3]], [4, 4])
    assert bench.activation_stages(8) == ([[0, 1, 2, 3]], [8], [[4], [5], [6], [7]], [2, 2, 2, 2])


def _port_worker(rank, world, port, q):
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from oracle import activation as OA
        ma, ba, mb, bb = bench.activation_stages(world)
        S, H = 3, 16

        def act(r, rows):
            return torch.randn(rows, S, H, generator=torch.Generator().manual_seed(r))

        in_a = rank in ma[0]
        groups = [(g, dist.new_group(g)) for g in ma + mb]
        tgt_f = torch.zeros(bb[0], S, H) if not in_a else None
        tgt_b = torch.zeros(8, S, H) if in_a else None
        bench._ref_port_exchange(rank, ma, mb, ba, bb, act(rank, 8) if in_a else None, tgt_f, groups)
        bench._ref_port_exchange(rank, mb, ma, bb, ba, act(rank, bb[0]) if not in_a else None, tgt_b, groups)
        if in_a:
            want = {r: np.zeros((8, S, H), np.float32) for r in ma[0]}
            OA.exchange_world({r: act(r, bb[0]).numpy() for g in mb for r in g}, want, mb, ma, bb, ba)
            ok = np.array_equal(tgt_b.numpy(), want[rank])
        else:
            want = {r: np.zeros((bb[0], S, H), np.float32) for g in mb for r in g}
            OA.exchange_world({r: act(r, 8).numpy() for r in ma[0]}, want, ma, mb, ba, bb)
            ok = np.array_equal(tgt_f.numpy(), want[rank])
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if ok else "mismatch"))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


def test_reference_activation_sequence_matches_oracle():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_port_worker, args=(r, 4, 29745, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(4):
            r, v = q.get(timeout=180)
            res[r] = v
    finally:
        for p in procs:
            p.join(30)
            if p.is_alive():
                p.kill()
    assert all(v == "ok" for v in res.values()), res


def test_e2e_layer_groups_partition_the_layouts():
    """The one-GPU e2e pipelines by layer groups: every tensor of both layouts lands in exactly one
    group, the embedding with the first layers and the head and final norm with the last."""
    cfg = bench.workload(1, 8)
    spl, tpl = cfg.layouts()
    for per in (1, 3):
        groups = bench.layer_groups(spl, tpl, per)
        assert len(groups) == -(-8 // per)
        for which, lay in ((0, spl), (1, tpl)):
            for r, metas in lay.layout.items():
                names = [n for g in groups for n in g[which].layout[r]]
                assert sorted(names) == sorted(metas), (per, which, r)
        assert "wte.weight" in groups[0][0].layout[0] and "lm_head.weight" in groups[-1][0].layout[0]
        assert "norm.weight" in groups[-1][1].layout[1]


def test_reference_arm_plans_without_the_product_library():
    """The reference arm's sample is planned by the oracle; nothing loads libsuika_reshard.so (in a
    fresh process: other tests of this session load it). The sample's synthetic state (several GB
    of numpy arrays, made by suika_b200.synthetic without the library) is not needed for the
    plan, so the subprocess skips generating it."""
    import subprocess
    import sys
    code = ("import sys; sys.argv = ['bench.py']; import bench; "
            "bench.S.host_states = lambda *a, **k: {}; "
            "smp = bench.OracleSample(bench.workload(1, 1), 1, 2); "
            "print(smp.units, smp.ranks, 'libsuika_reshard' in open('/proc/self/maps').read())")
    out = subprocess.run([sys.executable, "-c", code], cwd=os.path.dirname(os.path.abspath(bench.__file__)),
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.split() == ["866123776", "[0,", "1]", "False"], out.stdout


def test_result_config_is_the_same_for_both_arms():
    for n in (1, 8):
        cfg = bench.workload(n)
        assert bench.workload_config(cfg, n) == bench.workload_config(bench.workload(n), n)
    assert "cfg2b" in bench.workload_config(bench.workload(1), 1)["workload"]

"""The compact metadata plane (suika_b200/metadata.py), on the CPU:
  - a layout survives encode -> decode exactly (shapes, dtypes, tp_meta, slice rules, order);
  - the planner gives the same schedule from records as from ParamLayout objects;
  - gather_param_layout / broadcast_param_layout over 4 gloo ranks rebuild the layout that
    ParamLayout.gather / broadcast_objects would (Suika/migration.py:172-192, Suika/utils.py:98-104);
  - malformed blobs are rejected."""
import os

import numpy as np
import pytest
import torch

from suika_b200 import metadata as MD
from suika_b200 import migration as M
from suika_b200.layouts import CONFIGS
from tests.golden.cases import CASES


def _same_layout(a, b):
    assert list(a.layout) == list(b.layout)
    for r in a.layout:
        assert list(a.layout[r]) == list(b.layout[r]), r
        for name, m in a.layout[r].items():
            n = b.layout[r][name]
            assert tuple(int(x) for x in m.shape) == tuple(int(x) for x in n.shape), (r, name)
            assert m.dtype == n.dtype and (tuple(m.tp_meta) if m.tp_meta else None) == (tuple(n.tp_meta) if n.tp_meta else None)
            rm, rn = getattr(m, "tp_rule", None), getattr(n, "tp_rule", None)
            assert (rm is None) == (rn is None) and (rm is None or [list(g) for g in rm] == [list(g) for g in rn]), (r, name)


@pytest.mark.parametrize("cfg", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "cfg2b"])
def test_roundtrip_baseline_layouts(cfg):
    for pl in CONFIGS[cfg].layouts():
        cl = MD.CompactLayout.from_layout(pl)
        _same_layout(pl, cl)
        _same_layout(pl, MD.CompactLayout.decode(cl.encode()))


def test_roundtrip_extension_layouts_keep_slice_rules():
    from tests.test_extension_layouts import EXT_CASES
    for cfg in EXT_CASES.values():
        for pl in cfg.layouts():
            _same_layout(pl, MD.CompactLayout.decode(MD.CompactLayout.from_layout(pl).encode()))


@pytest.mark.parametrize("case", ["cfg1", "cfg3_mini", "cfg4_mini", "cfg5_mini", "hetero_mini", "shrink_mini"])
def test_plan_from_records_equals_plan_from_objects(case):
    spl, tpl = CASES[case]["config"].layouts()
    a = M.Plan(spl, tpl, minimum_est_peers=1)
    b = M.Plan(MD.CompactLayout.from_layout(spl), MD.CompactLayout.from_layout(tpl), minimum_est_peers=1)
    assert a.names == b.names
    assert np.array_equal(a.op_array, b.op_array)


def test_unknown_dtype_and_bad_blobs_are_rejected():
    m = M.TensorMeta(name="x", dtype=torch.complex128, shape=[2])
    with pytest.raises(ValueError, match="no code"):
        MD.encode_metas({"x": m})
    good = MD.encode_metas({"x": M.TensorMeta(name="x", dtype=torch.float32, shape=[2, 3], tp_meta=(0, 1, 2))})
    with pytest.raises(ValueError, match="truncated"):
        MD.decode_metas(good[:-3])
    bad = good.copy()
    bad[0] ^= 0xFF
    with pytest.raises(ValueError, match="not a metadata blob"):
        MD.decode_metas(bad)


def _worker(rank, world, port, cfg_name, q):
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        spl, _ = CONFIGS[cfg_name].layouts()
        got = MD.gather_param_layout(spl.layout[rank])
        _same_layout(spl, got)
        # broadcast of a layout held by rank 0 only, and of "no layout"
        b = MD.broadcast_param_layout(spl if rank == 0 else None, src=0)
        _same_layout(spl, b)
        assert MD.broadcast_param_layout(None, src=0) is None
        # a subgroup: its ranks are numbered within the group (as ParamLayout.gather numbers them)
        sub = dist.new_group([1, 3])
        if rank in (1, 3):
            part = MD.gather_param_layout(spl.layout[rank], world=sub)
            assert part.ranks == [0, 1]
            assert list(part.layout[0]) == list(spl.layout[1]) and list(part.layout[1]) == list(spl.layout[3])
            got = MD.broadcast_param_layout(part if rank == 3 else None, src=1, group=sub)  # group rank 1 = rank 3
            assert got.ranks == [0, 1] and list(got.layout[1]) == list(spl.layout[3])
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        import traceback
        q.put((rank, traceback.format_exc()))
        raise e


def test_gather_and_broadcast_over_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 4, 29711, "cfg4", q)) for r in range(4)]  # cfg4 sources: 4 ranks
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


def _dying_worker(rank, world, port, q):
    import datetime
    import time
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # a rank that dies before the layout exchange
    spl, _ = CONFIGS["cfg1"].layouts()
    t0 = time.perf_counter()
    try:
        MD.gather_param_layout(spl.layout[rank])
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, f"raised {type(e).__name__} after {time.perf_counter() - t0:.1f}s"))


def test_gather_fails_loudly_when_a_rank_dies():
    """A rank that dies before the exchange makes the others' gather raise (gloo error or the
    process group's 5 s timeout), never hang."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, 29719, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        rank, msg = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(30)
            if p.is_alive():
                p.kill()
    assert rank == 0 and msg.startswith("raised"), msg

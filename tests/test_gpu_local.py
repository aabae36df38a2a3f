"""GPU parity of the copy kernel: every golden case resharded on one B200 (all ranks emulated on
one device through reshard_local) must reproduce the reference's bytes, and the oracle's."""
import os

import numpy as np
import pytest
import torch

from oracle import restate as O
from suika_b200 import migration as M
from suika_b200 import synthetic as S
from tests.golden.cases import CASES
from tests.helpers import SUB_META, SUBS, digest, golden_states, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def to_device(states, step_on_device: bool = False):
    kinds = dict(SUBS)
    return {r: {n: {s: S.to_torch(a, kinds[s], DEV if (kinds[s] != "meta" or step_on_device) else None)
                    for s, a in ent.items()}
                for n, ent in st.items()} for r, st in states.items()}


def host(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.uint16)
    return t.numpy()


@pytest.mark.parametrize("case,step_on_device",
                         [(c, False) for c in sorted(CASES)] + [("cfg3_mini", True), ("odd_mini", True)])
def test_reshard_local_matches_reference_digests(case, step_on_device):
    """step_on_device: Adam's step lives in HBM (fused/capturable optimisers); it is then copied
    device to device by the same launch instead of being staged from the host."""
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    plan = M.Plan(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    out = M.reshard_local(spl, tpl, to_device(states, step_on_device), S.expected_sub_fields(), DEV, plan=plan)
    torch.cuda.synchronize()
    for rank_s, want in g["ranks"].items():
        got = out[int(rank_s)]
        assert list(got) == want["order"]
        for name, fields in want["digests"].items():
            assert list(got[name]) == list(fields)
            for sub, (shape, dtype, sha) in fields.items():
                t = got[name][sub]
                assert list(t.shape) == shape and str(t.dtype).replace("torch.", "") == dtype, (rank_s, name, sub)
                assert t.device == DEV and t.is_contiguous()
                assert digest(host(t)) == sha, (rank_s, name, sub)


@pytest.mark.parametrize("case", ["cfg3_mini", "cfg5_mini", "odd_mini", "hetero_mini"])
def test_reshard_local_semantic_order_matches_oracle(case):
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg)
    out = M.reshard_local(spl, tpl, to_device(states), S.expected_sub_fields(), DEV, order="semantic", minimum_est_peers=1)
    torch.cuda.synchronize()
    ops = O.schedule(spl, tpl, minimum_est_peers=1)
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        want = O.execute_rank(ops, states, SUB_META, rank, order="semantic")
        for name, ent in want.items():
            for sub, a in ent.items():
                assert np.array_equal(host(out[rank][name][sub]).reshape(-1).view(np.uint8), a.reshape(-1).view(np.uint8)), (rank, name, sub)


def test_views_move_only_row_split_pieces():
    cfg = CASES["cfg2b_mini"]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg)
    dev_states = to_device(states)
    out, info, _ = M.reshard_local(spl, tpl, dev_states, S.expected_sub_fields(), DEV, views=True, return_info=True)
    torch.cuda.synchronize()
    ops = O.schedule(spl, tpl, minimum_est_peers=1)
    moved = 0
    for rank in (0, 1):
        want = O.execute_rank(ops, states, SUB_META, rank)
        for name, ent in want.items():
            for sub, a in ent.items():
                t = out[rank][name][sub]
                assert np.array_equal(host(t).reshape(-1).view(np.uint8), a.reshape(-1).view(np.uint8))
                if sub != "step":
                    shares = t.untyped_storage().data_ptr() == dev_states[0][name][sub].untyped_storage().data_ptr()
                    row_split = spl.layout[0][name].tp_meta is not None and spl.layout[0][name].tp_meta[0] == -1
                    assert shares != row_split, (name, sub)
                    moved += 0 if shares else t.numel() * t.element_size()
    assert info.total_bytes == moved + 4 * len([1 for r in (0, 1) for _ in out[r]])  # + one 4-byte step per tensor


@pytest.mark.parametrize("variant", ["1", "2", "3", "4", "5", "6", "7", "8", "9", "10", "11", "12", "13", "14", "15", "16",
                                     "17"])
@pytest.mark.parametrize("tile", ["256", "4096", "131072"])
def test_copy_kernel_random_rectangles(tile, variant, monkeypatch):
    """Strided copies with random alignment, pitch and size (every vector width, column-split rows),
    for every launch shape (vector copies and TMA bulk copies), against torch's own copy."""
    monkeypatch.setenv("SUIKA_RS_TILE_BYTES", tile)
    monkeypatch.setenv("SUIKA_RS_VARIANT", variant)
    rng = np.random.default_rng(int(tile) + int(variant))
    src = torch.randint(0, 255, (8 << 20,), dtype=torch.uint8, device=DEV)
    dst = torch.zeros(16 << 20, dtype=torch.uint8, device=DEV)
    want = torch.zeros_like(dst)
    descs, dpos = [], 0
    for _ in range(300):
        rows = int(rng.integers(1, 40))
        rb = int(rng.choice([1, 2, 3, 4, 6, 8, 16, 48, 100, 1024, 5000, 20000]))
        sp = rb + int(rng.integers(0, 64))
        dp = rb + int(rng.integers(0, 64))
        so = int(rng.integers(0, src.numel() - rows * sp - 1))
        if rng.random() < 0.5:
            so -= so % 16
        dpos += int(rng.integers(0, 17))
        if dpos + rows * dp >= dst.numel():
            break
        descs.append((src.data_ptr() + so, dst.data_ptr() + dpos, rows, rb, sp, dp, int(rng.integers(0, 2))))
        for r in range(rows):
            want[dpos + r * dp: dpos + r * dp + rb] = src[so + r * sp: so + r * sp + rb]
        dpos += rows * dp
    table = np.array(descs, dtype=M.L.COPY_DESC_DTYPE)
    prepared = M.PreparedCopies(table, DEV)
    info = prepared.launch()
    assert info.variant == int(variant) - 1
    torch.cuda.synchronize()
    assert prepared.status() == 0
    assert torch.equal(dst, want)


@pytest.mark.parametrize("variant", ["5", "6", "7"])
def test_tma_wait_that_runs_out_reports_status_and_returns(variant, monkeypatch):
    """The bounded-wait error path of the TMA launch shapes, made to happen without a fault: every
    CTA arms its first stage's barrier for bytes that no copy delivers (RS_RUN_STALL_FIRST_STAGE),
    with a 1 ms limit. The wait runs out, the kernel drains what it issued and returns, and the
    status word reads 1. The context stays usable: the same table, staged again and run normally,
    then copies correctly with status 0."""
    import ctypes as C
    monkeypatch.setenv("SUIKA_RS_VARIANT", variant)
    lib = M.L.load()
    rows, rb, pitch = 2048, 4096, 8192  # 16-byte aligned rows: all of them go through the bulk copies
    src = torch.randint(0, 255, (rows * pitch,), dtype=torch.uint8, device=DEV)  # the two halves cover every byte
    dst = torch.zeros_like(src)
    table = np.array([(src.data_ptr() + h * rb, dst.data_ptr() + h * rb, rows, rb, pitch, pitch, 0) for h in (0, 1)],
                     dtype=M.L.COPY_DESC_DTYPE)
    prepared = M.PreparedCopies(table, DEV)
    stream = C.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    M.L.check(lib.rs_copy_run_bounded(prepared.workspace.data_ptr(), C.byref(prepared.info), stream, 1_000_000,
                                      M.L.RS_RUN_STALL_FIRST_STAGE))
    torch.cuda.synchronize()
    assert prepared.status() == 1
    with pytest.raises(M.L.ReshardError):
        prepared.check()
    assert not torch.equal(dst, src)  # the stalled stages were never copied
    again = M.PreparedCopies(table, DEV)  # staging clears the status block
    again.launch()
    torch.cuda.synchronize()
    assert again.status() == 0
    assert torch.equal(dst, src)


def test_stall_flag_needs_a_tma_shape(monkeypatch):
    import ctypes as C
    monkeypatch.setenv("SUIKA_RS_VARIANT", "2")
    lib = M.L.load()
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=DEV)
    table = np.array([(buf.data_ptr(), buf.data_ptr() + 32768, 1, 4096, 4096, 4096, 0)], dtype=M.L.COPY_DESC_DTYPE)
    prepared = M.PreparedCopies(table, DEV)
    rc = lib.rs_copy_run_bounded(prepared.workspace.data_ptr(), C.byref(prepared.info), None, 1_000_000,
                                 M.L.RS_RUN_STALL_FIRST_STAGE)
    assert rc == M.L.RS_ERR_ARG and b"TMA" in lib.rs_last_error()
    assert lib.rs_copy_run_bounded(prepared.workspace.data_ptr(), C.byref(prepared.info), None, 0, 0) == M.L.RS_ERR_ARG


@pytest.mark.parametrize("variant", ["9", "10", "11", "12", "13", "14"])
def test_tensor_map_kernel_edges(variant, monkeypatch):
    """The 3-D tensor-map kernel on the geometry its boxes have to clip: rows narrower than a box,
    widths that are not a multiple of the box width (odd element counts), row counts that leave a
    partial last box, one-row runs, and long contiguous runs cut into 2 KB rows plus a remainder.
    Every entry is local and 16-byte aligned, so all of them go to the tensor-map kernel."""
    monkeypatch.setenv("SUIKA_RS_VARIANT", variant)
    g = torch.Generator(device=DEV).manual_seed(int(variant))
    src = torch.randint(0, 255, (48 << 20,), dtype=torch.uint8, device=DEV, generator=g)
    dst = torch.zeros(64 << 20, dtype=torch.uint8, device=DEV)
    want = torch.zeros_like(dst)
    shapes = [(1, 8, 16, 16), (3, 24, 32, 48), (17, 2056, 4096, 2064), (5, 4104, 8208, 4112), (1000, 11008, 22016, 11008),
              (37, 1280, 2560, 1280), (1, 40000, 40000, 40000), (1, 4096 * 3 + 8, 0, 0), (64, 2048, 2048, 2048),
              (250, 16, 32, 16), (300, 22016, 44032, 22016), (1, 2 << 20, 0, 0)]
    descs, so, do = [], 0, 0
    for rows, rb, sp, dp in shapes:
        sp, dp = sp or rb, dp or rb
        descs.append((src.data_ptr() + so, dst.data_ptr() + do, rows, rb, sp, dp, 0))
        for r in range(rows):
            want[do + r * dp: do + r * dp + rb] = src[so + r * sp: so + r * sp + rb]
        so = (so + (rows - 1) * sp + rb + 4095) // 4096 * 4096 + 16
        do = (do + (rows - 1) * dp + rb + 4095) // 4096 * 4096 + 32
    assert so < src.numel() and do < dst.numel()
    prepared = M.PreparedCopies(np.array(descs, dtype=M.L.COPY_DESC_DTYPE), DEV)
    info = prepared.launch()
    assert info.n_entries == 0 and info.n_tensor_entries >= len(shapes)  # contiguous runs may add a remainder entry
    torch.cuda.synchronize()
    assert prepared.status() == 0
    assert torch.equal(dst, want)


def test_split_shape_gives_wide_rows_to_tensor_maps(monkeypatch):
    """Launch shape 15: local, aligned slices wider than 8 KB and contiguous runs of 1 MB or more
    take the tensor-map kernel; narrower slices, short runs and unaligned entries take the banded
    vector copy, in the same run. Every target gets exactly its bytes."""
    monkeypatch.setenv("SUIKA_RS_VARIANT", "15")
    monkeypatch.delenv("SUIKA_RS_BAND_BYTES", raising=False)
    g = torch.Generator(device=DEV).manual_seed(15)
    src = torch.randint(0, 255, (64 << 20,), dtype=torch.uint8, device=DEV, generator=g)
    dst = torch.zeros(64 << 20, dtype=torch.uint8, device=DEV)
    want = torch.zeros_like(dst)
    # (rows, row_bytes, src pitch, dst pitch, source offset misalignment, takes tensor maps)
    shapes = [(700, 11008, 22016, 11008, 0, True), (300, 8192, 16384, 8192, 0, False), (1, 3 << 20, 0, 0, 0, True),
              (1, 64 << 10, 0, 0, 0, False), (50, 16384, 32768, 16384, 8, False), (2048, 4096, 8192, 4096, 0, False),
              (9, 40000, 80000, 40000, 0, True), (200, 4096, 4096, 4096, 0, False)]
    descs, so, do, wide = [], 0, 0, 0
    for rows, rb, sp, dp, mis, tma in shapes:
        sp, dp = sp or rb, dp or rb
        descs.append((src.data_ptr() + so + mis, dst.data_ptr() + do, rows, rb, sp, dp, 0))
        want[do:do + rows * dp].view(rows, dp)[:, :rb] = src[so + mis:so + mis + rows * sp].view(rows, sp)[:, :rb]
        wide += tma
        so = (so + mis + rows * sp + 4095) // 4096 * 4096
        do = (do + rows * dp + 4095) // 4096 * 4096
    assert so <= src.numel() and do <= dst.numel()
    prepared = M.PreparedCopies(np.array(descs, dtype=M.L.COPY_DESC_DTYPE), DEV)
    info = prepared.launch()
    assert info.variant == 14
    assert info.n_tensor_entries >= wide and info.n_entries >= len(descs) - wide  # runs may add a remainder entry
    torch.cuda.synchronize()
    assert prepared.status() == 0
    assert torch.equal(dst, want)


@pytest.mark.parametrize("band", ["4096", "65536", "8388608"])
@pytest.mark.parametrize("variant", ["2", "8", "9", "11", "12", "14", "15", "16", "17"])
def test_groups_of_column_slices(variant, band, monkeypatch):
    """Column slices of the same source rows (the pieces of a TP grow by 2, 3, 4 and 8) are grouped:
    the vector copy cuts them into row bands of SUIKA_RS_BAND_BYTES and interleaves the bands, the
    tensor-map copy interleaves their boxes band by band. Every target must still get exactly its
    slice, whatever the table order."""
    monkeypatch.setenv("SUIKA_RS_VARIANT", variant)
    monkeypatch.setenv("SUIKA_RS_BAND_BYTES", band)
    g = torch.Generator(device=DEV).manual_seed(7)
    src = torch.randint(0, 255, (64 << 20,), dtype=torch.uint8, device=DEV, generator=g)
    dst = torch.zeros(64 << 20, dtype=torch.uint8, device=DEV)
    want = torch.zeros_like(dst)
    descs, so, do = [], 0, 0
    for k, rows, rb in ((2, 1000, 11008), (4, 517, 4096), (3, 64, 2064), (8, 77, 1280), (2, 5, 40000)):
        pitch = k * rb
        for h in range(k):
            descs.append((src.data_ptr() + so + h * rb, dst.data_ptr() + do, rows, rb, pitch, rb, 0))
            want[do:do + rows * rb] = src[so + h * rb: so + h * rb + rows * pitch].view(rows, pitch)[:, :rb].reshape(-1)
            do = (do + rows * rb + 4095) // 4096 * 4096
        so = (so + rows * pitch + 4095) // 4096 * 4096
    assert so <= src.numel() and do <= dst.numel()
    rng = np.random.default_rng(int(variant))
    table = np.array([descs[i] for i in rng.permutation(len(descs))], dtype=M.L.COPY_DESC_DTYPE)  # any table order
    prepared = M.PreparedCopies(table, DEV)
    info = prepared.launch()
    if int(variant) >= 15:  # slices wider than 8 KB (11008 and 40000 bytes) take tensor maps
        assert info.n_tensor_entries == 4 and info.n_entries >= len(descs) - 4
    elif int(variant) >= 9:
        assert info.n_entries == 0 and info.n_tensor_entries == len(descs)
    else:
        assert info.n_tensor_entries == 0 and info.n_entries >= len(descs)  # band-split entries
    torch.cuda.synchronize()
    assert prepared.status() == 0
    assert torch.equal(dst, want)


@pytest.mark.parametrize("band", ["1024", "65536"])
@pytest.mark.parametrize("case", ["cfg2b_mini", "grow_dp_tp_mini", "qwen_grow_mini", "cfg3_mini", "odd_mini", "next_step"])
def test_reshard_local_band_interleaved_matches_reference(case, band, monkeypatch):
    """The vector copy of one-GPU tables (shape 8: TP-grow slices cut into row bands and
    interleaved), with bands small enough to cut the reduced-width golden cases, equals the
    reference's digests."""
    monkeypatch.setenv("SUIKA_RS_VARIANT", "8")
    monkeypatch.setenv("SUIKA_RS_BAND_BYTES", band)
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    out, info, _ = M.reshard_local(spl, tpl, to_device(states), S.expected_sub_fields(), DEV,
                                   minimum_est_peers=g["minimum_est_peers"], return_info=True)
    torch.cuda.synchronize()
    assert info.n_tensor_entries == 0
    for rank_s, want in g["ranks"].items():
        got = out[int(rank_s)]
        assert list(got) == want["order"]
        for name, fields in want["digests"].items():
            for sub, exp in fields.items():
                t = got[name][sub]
                assert [list(t.shape), str(t.dtype).replace("torch.", ""), digest(host(t))] == exp, (rank_s, name, sub)


@pytest.mark.parametrize("variant", ["9", "11", "14", "15", "0"])
@pytest.mark.parametrize("case", ["cfg2b_mini", "cfg3_mini", "odd_mini", "qwen_grow_mini", "wide_mini", "wide_shrink_mini"])
def test_reshard_local_tensor_map_shapes_match_reference(case, variant, monkeypatch):
    """A whole reshard through the tensor-map launch shapes equals the reference's digests ("0":
    the default, shape 17; the wide cases give the split shapes rows for both of their kernels)."""
    if variant == "0":
        monkeypatch.delenv("SUIKA_RS_VARIANT", raising=False)
    else:
        monkeypatch.setenv("SUIKA_RS_VARIANT", variant)
    g = load_golden(case)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    out, info, _ = M.reshard_local(spl, tpl, to_device(states), S.expected_sub_fields(), DEV,
                                   minimum_est_peers=g["minimum_est_peers"], return_info=True)
    torch.cuda.synchronize()
    if case.startswith("wide") and variant in ("0", "15"):
        assert info.variant == (16 if variant == "0" else 14)
        assert info.n_tensor_entries > 0 and info.n_entries > 0  # both kernels ran
    for rank_s, want in g["ranks"].items():
        got = out[int(rank_s)]
        assert list(got) == want["order"]
        for name, fields in want["digests"].items():
            for sub, exp in fields.items():
                t = got[name][sub]
                assert [list(t.shape), str(t.dtype).replace("torch.", ""), digest(host(t))] == exp, (rank_s, name, sub)


@pytest.mark.parametrize("variant", ["9", "12", "14"])
def test_tensor_map_wait_that_runs_out_reports_status(variant, monkeypatch):
    """The bounded-wait error path of the tensor-map kernel (same hook as the bulk-copy shapes)."""
    import ctypes as C
    monkeypatch.setenv("SUIKA_RS_VARIANT", variant)
    lib = M.L.load()
    src = torch.randint(0, 255, (2048 * 8192,), dtype=torch.uint8, device=DEV)  # the two halves cover every byte
    dst = torch.zeros_like(src)
    table = np.array([(src.data_ptr() + h * 4096, dst.data_ptr() + h * 4096, 2048, 4096, 8192, 8192, 0) for h in (0, 1)],
                     dtype=M.L.COPY_DESC_DTYPE)
    prepared = M.PreparedCopies(table, DEV)
    assert prepared.info.n_tensor_entries == 2
    stream = C.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    M.L.check(lib.rs_copy_run_bounded(prepared.workspace.data_ptr(), C.byref(prepared.info), stream, 1_000_000,
                                      M.L.RS_RUN_STALL_FIRST_STAGE))
    torch.cuda.synchronize()
    assert prepared.status() == 1
    again = M.PreparedCopies(table, DEV)
    again.launch()
    torch.cuda.synchronize()
    assert again.status() == 0 and torch.equal(dst, src)


def test_empty_table_is_a_noop():
    info = M.launch_copies(np.zeros(0, dtype=M.L.COPY_DESC_DTYPE), DEV)
    assert info.n_tiles == 0


@pytest.mark.parametrize("case", ["cfg3_fused_mini", "gqa_rep_src", "gqa_rep_dst", "gqa_pp"])
def test_reshard_local_extension_layouts_match_reslice(case):
    """Fused QKV split by head, GQA KV-head replication, vocab-parallel wte (layouts the reference
    lacks): the kernel's targets equal gathering the full tensors and re-slicing them."""
    from tests.test_extension_layouts import EXT_CASES
    cfg = EXT_CASES[case]
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, SUBS, seed=3, distinct_steps=True)
    out = M.reshard_local(spl, tpl, to_device(states), S.expected_sub_fields(), DEV)
    torch.cuda.synchronize()
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        want = O.semantic_target(states, spl, tpl, SUB_META, rank)
        for name, ent in want.items():
            for sub, a in ent.items():
                if sub == "step":
                    continue
                assert np.array_equal(host(out[rank][name][sub]).reshape(-1).view(np.uint8), a.reshape(-1).view(np.uint8)), (rank, name, sub)


WORKER_SUBS = [("param", "bf16"), ("step", "meta"), ("exp_avg", "bf16"), ("exp_avg_sq", "bf16")]


@pytest.mark.parametrize("case", ["cfg3_mini", "cfg5_mini"])
def test_reshard_local_on_the_reference_worker_state(case):
    """The state the reference's worker migrates (bf16 param and Adam moments, no master): the
    kernel's targets equal the oracle's."""
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, WORKER_SUBS, seed=2, distinct_steps=True)
    kinds = dict(WORKER_SUBS)
    dev_states = {r: {n: {s: S.to_torch(a, kinds[s], DEV if kinds[s] != "meta" else None) for s, a in e.items()}
                      for n, e in st.items()} for r, st in states.items()}
    out = M.reshard_local(spl, tpl, dev_states, S.expected_sub_fields(WORKER_SUBS), DEV, minimum_est_peers=1)
    torch.cuda.synchronize()
    ops = O.schedule(spl, tpl, minimum_est_peers=1)
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        want = O.execute_rank(ops, states, [(s, k == "meta") for s, k in WORKER_SUBS], rank)
        for name, ent in want.items():
            for sub, a in ent.items():
                assert np.array_equal(host(out[rank][name][sub]).reshape(-1).view(np.uint8), a.reshape(-1).view(np.uint8)), (rank, name, sub)


@pytest.mark.parametrize("k", range(8))
def test_random_reshards_on_the_kernel(k):
    """Seeded random (TP, PP, DP) reshards through the kernel, every rank on one GPU: targets equal
    the oracle's in the reference's cat order."""
    from tests.test_planner_random import SPEC as RSPEC, cases
    from suika_b200.layouts import ReshardConfig
    src, dst, peers = cases(n=8, seed=99)[k]
    spl, tpl = ReshardConfig("rand", RSPEC, src, dst).layouts()
    states = S.host_states(spl, SUBS, seed=k, distinct_steps=True, threads=1)
    out = M.reshard_local(spl, tpl, to_device(states), S.expected_sub_fields(), DEV, minimum_est_peers=peers)
    torch.cuda.synchronize()
    ops = O.schedule(spl, tpl, minimum_est_peers=peers)
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        want = O.execute_rank(ops, states, SUB_META, rank)
        assert list(out[rank]) == list(want)
        for name, ent in want.items():
            for sub, a in ent.items():
                assert np.array_equal(host(out[rank][name][sub]).reshape(-1).view(np.uint8), a.reshape(-1).view(np.uint8)), (rank, name, sub)

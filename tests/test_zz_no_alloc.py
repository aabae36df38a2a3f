"""rs_copy_launch_noalloc: the copy launch for callers that cannot allocate device memory while
they reshard. During a live migration HBM is at its fullest (both layouts resident, and the
framework's caching allocator may hold the rest), so a cudaMalloc for the copy table can fail or
force the allocator to release memory and synchronise. This entry point keeps its copy table in an
array built into the library instead.

Checked through the C ABI on two calls in a row: the bytes it writes must equal an expected buffer
built on the host with numpy from the same descriptors, and must equal what rs_copy_launch (the
existing entry point, with caller workspace) writes. Also checked: tables of exactly 128 * k
entries (the host stages the table in chunks of 128) and of the maximum size, every launch shape
the entry point accepts, and that warm calls take no device memory.

This file is collected last on purpose: if it fails, a run that stops at the first failure has
already run every other test.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from suika_b200 import _lib as L
from suika_b200 import migration as M
from tests.helpers import copy_rect

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rectangles(n_src, n_dst, seed, count=400, sizes=(1, 2, 3, 4, 6, 8, 16, 48, 100, 1024, 5000, 40000, 200000), max_rows=48):
    """(src offset, dst offset, rows, row bytes, src pitch, dst pitch) of strided copies with random
    sizes, pitches and alignments (every vector width); targets do not overlap."""
    rng = np.random.default_rng(seed)
    descs, pos = [], 0
    for _ in range(count):
        rows = int(rng.integers(1, max_rows))
        rb = int(rng.choice(sizes))
        sp, dp = rb + int(rng.integers(0, 64)), rb + int(rng.integers(0, 64))
        so = int(rng.integers(0, n_src - rows * sp - 1))
        if rng.random() < 0.6:
            so -= so % 16
        pos += int(rng.integers(0, 17))
        if pos + rows * dp >= n_dst:
            break
        descs.append((so, pos, rows, rb, sp, dp))
        pos += rows * dp
    return descs


def _expected(src_host: np.ndarray, fill: int, n_dst: int, descs) -> np.ndarray:
    """The target buffer the copies must produce, built with numpy on the host."""
    out = np.full(n_dst, fill, dtype=np.uint8)
    for so, do, rows, rb, sp, dp in descs:
        copy_rect(out, do, dp, src_host, so, sp, rows, rb)
    return out


def _table(src, dst, descs):
    return np.array([(src.data_ptr() + so, dst.data_ptr() + do, r, rb, sp, dp, k % 2)
                     for k, (so, do, r, rb, sp, dp) in enumerate(descs)], dtype=L.COPY_DESC_DTYPE)


def _noalloc(table) -> L.RsLaunchInfo:
    lib = L.load()
    stream = C.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    info = L.RsLaunchInfo()
    L.check(lib.rs_copy_launch_noalloc(table.ctypes.data if len(table) else None, len(table), stream, C.byref(info)))
    return info


def _both_against_expected(src, descs, fill_a=0, fill_b=7, n_dst=96 << 20):
    """Run the copies with rs_copy_launch into one buffer and with rs_copy_launch_noalloc into
    another; both must equal the host-built expectation (outside the targets: the fill)."""
    dst_a = torch.full((n_dst,), fill_a, dtype=torch.uint8, device=DEV)
    dst_b = torch.full((n_dst,), fill_b, dtype=torch.uint8, device=DEV)
    M.launch_copies(_table(src, dst_a, descs), DEV)
    info = _noalloc(_table(src, dst_b, descs))
    torch.cuda.synchronize()
    src_host = src.cpu().numpy()
    assert np.array_equal(dst_a.cpu().numpy(), _expected(src_host, fill_a, n_dst, descs))
    assert np.array_equal(dst_b.cpu().numpy(), _expected(src_host, fill_b, n_dst, descs))
    return info


@pytest.fixture
def variant(request):
    old = os.environ.get("SUIKA_RS_VARIANT")
    os.environ["SUIKA_RS_VARIANT"] = request.param
    yield int(request.param)
    if old is None:
        os.environ.pop("SUIKA_RS_VARIANT", None)
    else:
        os.environ["SUIKA_RS_VARIANT"] = old


@pytest.mark.parametrize("variant", ["2", "1", "8", "6"], indirect=True)
def test_noalloc_matches_expected_and_rs_copy_launch_twice(variant):
    g = torch.Generator(device=DEV).manual_seed(11)
    src = torch.randint(0, 256, (64 << 20,), dtype=torch.uint8, device=DEV, generator=g)
    # first call: a large table with long and short rows
    d1 = _rectangles(src.numel(), 96 << 20, seed=1)
    info1 = _both_against_expected(src, d1)
    assert info1.n_entries == len(d1) and info1.n_tiles > 0
    # the TMA shapes (5-7) are not taken: the entry point keeps to the vector copies
    assert info1.variant == (1 if variant in (5, 6, 7) else variant - 1)
    # second call in a row: a smaller table over new source bytes; the shared array still holds
    # the first call's entries beyond the new ones, which must not matter
    src.copy_(torch.randint(0, 256, src.shape, dtype=torch.uint8, device=DEV, generator=g))
    d2 = _rectangles(src.numel(), 96 << 20, seed=2, count=60)
    info2 = _both_against_expected(src, d2, fill_a=3, fill_b=9)
    assert info2.n_entries == len(d2) < info1.n_entries


@pytest.mark.parametrize("n", [128, 256, 384, 129, L.RS_NOALLOC_MAX_ENTRIES])
def test_noalloc_chunk_multiples_and_the_maximum(n):
    """The table is staged in chunks of 128 entries: exact multiples, one more, and the maximum."""
    src = torch.randint(0, 256, (8 << 20,), dtype=torch.uint8, device=DEV, generator=torch.Generator(device=DEV).manual_seed(n))
    descs = _rectangles(src.numel(), 32 << 20, seed=n, count=n, sizes=(1, 4, 16, 48, 256, 1000), max_rows=5)
    assert len(descs) == n
    info = _both_against_expected(src, descs, n_dst=32 << 20)
    assert info.n_entries == n


def test_noalloc_empty_descriptors_are_skipped():
    src = torch.arange(4096, device=DEV, dtype=torch.int32).view(torch.uint8)
    descs = _rectangles(src.numel(), 1 << 16, seed=5, count=40, sizes=(4, 16, 64), max_rows=4)
    dst = torch.zeros(1 << 16, dtype=torch.uint8, device=DEV)
    t = _table(src, dst, descs)
    empty = np.zeros(3, dtype=L.COPY_DESC_DTYPE)  # rows == 0 / row_bytes == 0: nothing to copy
    empty["src_dev"], empty["dst_dev"], empty["rows"], empty["row_bytes"] = src.data_ptr(), dst.data_ptr(), [0, 5, 0], [8, 0, 0]
    info = _noalloc(np.concatenate([empty[:1], t[:20], empty[1:], t[20:]]))
    torch.cuda.synchronize()
    assert info.n_entries == len(descs)
    assert np.array_equal(dst.cpu().numpy(), _expected(src.cpu().numpy(), 0, 1 << 16, descs))


def test_noalloc_warm_calls_take_no_device_memory():
    src = torch.randint(0, 256, (16 << 20,), dtype=torch.uint8, device=DEV)
    dst = torch.zeros(32 << 20, dtype=torch.uint8, device=DEV)
    t = _table(src, dst, _rectangles(src.numel(), dst.numel(), seed=3, count=300))
    _noalloc(t)  # warm: the first call on a device looks up the array's address
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(DEV)
    for _ in range(20):
        _noalloc(t)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(DEV)
    assert free1 >= free0, (free0, free1)


def test_noalloc_rejects_tables_over_the_limit():
    lib = L.load()
    n = L.RS_NOALLOC_MAX_ENTRIES + 1
    buf = torch.zeros(16, dtype=torch.uint8, device=DEV)
    t = np.zeros(n, dtype=L.COPY_DESC_DTYPE)
    t["src_dev"], t["dst_dev"], t["rows"], t["row_bytes"], t["src_pitch"], t["dst_pitch"] = buf.data_ptr(), buf.data_ptr() + 8, 1, 4, 4, 4
    rc = lib.rs_copy_launch_noalloc(t.ctypes.data, n, None, None)
    assert rc == L.RS_ERR_CAPACITY
    assert b"at most" in lib.rs_last_error()
    assert torch.all(buf == 0)  # nothing was launched

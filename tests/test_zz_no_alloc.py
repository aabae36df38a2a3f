"""rs_copy_launch_noalloc: the copy launch for callers that cannot allocate device memory while
they reshard (HBM is fullest during a live migration). It keeps its copy table in an array built
into the library, so it must produce exactly what rs_copy_launch produces with caller-provided
workspace. Checked through the C ABI on two calls in a row, each against rs_copy_launch.

This file is collected last on purpose: if it fails, a run that stops at the first failure has
already run every other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from suika_b200 import _lib as L
from suika_b200 import migration as M

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rectangles(src, dst, seed, count=400):
    """Strided copies with random sizes, pitches and alignments (every vector width)."""
    rng = np.random.default_rng(seed)
    descs, pos = [], 0
    for _ in range(count):
        rows = int(rng.integers(1, 48))
        rb = int(rng.choice([1, 2, 3, 4, 6, 8, 16, 48, 100, 1024, 5000, 40000, 200000]))
        sp, dp = rb + int(rng.integers(0, 64)), rb + int(rng.integers(0, 64))
        so = int(rng.integers(0, src.numel() - rows * sp - 1))
        if rng.random() < 0.6:
            so -= so % 16
        pos += int(rng.integers(0, 17))
        if pos + rows * dp >= dst.numel():
            break
        descs.append((src.data_ptr() + so, pos, rows, rb, sp, dp))
        pos += rows * dp
    return descs


def _run_both(descs_rel, dst_a, dst_b):
    """Same copies into dst_a with rs_copy_launch and into dst_b with rs_copy_launch_noalloc."""
    lib = L.load()
    stream = C.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    ta = np.array([(s, dst_a.data_ptr() + o, r, rb, sp, dp, k % 2) for k, (s, o, r, rb, sp, dp) in enumerate(descs_rel)],
                  dtype=L.COPY_DESC_DTYPE)
    tb = np.array([(s, dst_b.data_ptr() + o, r, rb, sp, dp, k % 2) for k, (s, o, r, rb, sp, dp) in enumerate(descs_rel)],
                  dtype=L.COPY_DESC_DTYPE)
    M.launch_copies(ta, DEV)
    info = L.RsLaunchInfo()
    L.check(lib.rs_copy_launch_noalloc(tb.ctypes.data, len(tb), stream, C.byref(info)))
    torch.cuda.synchronize()
    return info


def test_noalloc_matches_rs_copy_launch_twice():
    src = torch.randint(0, 256, (64 << 20,), dtype=torch.uint8, device=DEV)
    dst_a = torch.zeros(96 << 20, dtype=torch.uint8, device=DEV)
    dst_b = torch.full_like(dst_a, 7)
    # first call: a large table with long and short rows
    d1 = _rectangles(src, dst_a, seed=1)
    info1 = _run_both(d1, dst_a, dst_b)
    assert info1.n_entries == len(d1) and info1.n_tiles > 0
    written = torch.zeros_like(dst_a, dtype=torch.bool)
    for _, o, r, rb, _, dp in d1:
        idx = (torch.arange(r, device=DEV) * dp + o)[:, None] + torch.arange(rb, device=DEV)[None, :]
        written[idx.reshape(-1)] = True
    assert torch.equal(dst_a[written], dst_b[written])
    # second call in a row: a different, smaller table over new source bytes; the shared array
    # still holds the first call's entries beyond the new ones, which must not matter
    src.copy_(torch.randint(0, 256, src.shape, dtype=torch.uint8, device=DEV))
    dst_a.zero_()
    dst_b.fill_(9)
    d2 = _rectangles(src, dst_a, seed=2, count=60)
    info2 = _run_both(d2, dst_a, dst_b)
    assert info2.n_entries == len(d2) < info1.n_entries
    written.zero_()
    for _, o, r, rb, _, dp in d2:
        idx = (torch.arange(r, device=DEV) * dp + o)[:, None] + torch.arange(rb, device=DEV)[None, :]
        written[idx.reshape(-1)] = True
    assert torch.equal(dst_a[written], dst_b[written])
    assert torch.all(dst_b[~written] == 9)  # nothing outside the table's targets was touched


def test_noalloc_rejects_tables_over_the_limit():
    lib = L.load()
    n = L.RS_NOALLOC_MAX_ENTRIES + 1
    buf = torch.zeros(16, dtype=torch.uint8, device=DEV)
    t = np.zeros(n, dtype=L.COPY_DESC_DTYPE)
    t["src_dev"], t["dst_dev"], t["rows"], t["row_bytes"], t["src_pitch"], t["dst_pitch"] = buf.data_ptr(), buf.data_ptr() + 8, 1, 4, 4, 4
    rc = lib.rs_copy_launch_noalloc(t.ctypes.data, n, None, None)
    assert rc == L.RS_ERR_CAPACITY
    assert b"at most" in lib.rs_last_error()

"""Host side of rs_copy_stage, on a machine without a GPU: the table it builds is counted in
rs_launch_info before the first CUDA call (the copy of the table to the device), which then fails
with RS_ERR_CUDA because there is no device. So the row-band cutting of column slices (the pieces
of a TP grow) can be checked here: how many entries it makes, and that it stays within the
caller's workspace. These tests skip wherever a GPU is visible, so the made-up workspace address
never reaches a device."""
import ctypes

import numpy as np
import pytest
import torch

from suika_b200 import _lib as L

pytestmark = pytest.mark.skipif(torch.cuda.is_available(), reason="host-only check; needs a machine without a GPU")

BASE = 1 << 40  # made-up, 256-byte aligned addresses: nothing is dereferenced on the host


def _stage(descs, workspace_bytes=None, env=None, monkeypatch=None):
    lib = L.load()
    for k, v in (env or {}).items():
        monkeypatch.setenv(k, v)
    t = np.array(descs, dtype=L.COPY_DESC_DTYPE)
    if workspace_bytes is None:
        b = ctypes.c_uint64()
        L.check(lib.rs_copy_workspace_bytes(len(t), ctypes.byref(b)))
        workspace_bytes = b.value
    info = L.RsLaunchInfo()
    rc = lib.rs_copy_stage(t.ctypes.data, len(t), ctypes.c_void_p(BASE), workspace_bytes, None, ctypes.byref(info))
    assert rc == L.RS_ERR_CUDA, lib.rs_last_error()  # the table was built; only the device copy failed
    return info


def _tp_grow(k, rows, rb):
    """k column slices of one source matrix [rows, k * rb] into k separate targets."""
    return [(BASE + h * rb, BASE + (1 << 36) + h * (rows * rb), rows, rb, k * rb, rb, 0) for h in range(k)]


def test_tp_grow_slices_are_cut_into_8_mb_bands(monkeypatch):
    monkeypatch.delenv("SUIKA_RS_BAND_BYTES", raising=False)
    monkeypatch.setenv("SUIKA_RS_VARIANT", "8")
    info = _stage(_tp_grow(2, 4096, 22016))
    band_rows = (8 << 20) // 22016  # 381 rows per band
    bands = -(-4096 // band_rows)
    assert info.n_entries == 2 * bands and info.variant == 7  # the evict-first vector shape
    assert info.total_bytes == 2 * 4096 * 22016


def test_band_size_follows_the_setting(monkeypatch):
    info = _stage(_tp_grow(4, 1000, 4096), env={"SUIKA_RS_BAND_BYTES": str(100 * 4096), "SUIKA_RS_VARIANT": "2"},
                  monkeypatch=monkeypatch)
    assert info.n_entries == 4 * 10 and info.variant == 1


def test_bands_shrink_to_fit_the_workspace(monkeypatch):
    """A workspace with room for 7 entries: the two slices get 3 bands each instead of 11."""
    monkeypatch.delenv("SUIKA_RS_BAND_BYTES", raising=False)
    monkeypatch.setenv("SUIKA_RS_VARIANT", "8")
    info = _stage(_tp_grow(2, 4096, 22016), workspace_bytes=256 + 256 + 7 * 72)
    assert info.n_entries == 6


def test_unrelated_entries_are_not_cut(monkeypatch):
    monkeypatch.delenv("SUIKA_RS_BAND_BYTES", raising=False)
    monkeypatch.setenv("SUIKA_RS_VARIANT", "8")
    descs = [(BASE + i * (1 << 30), BASE + (1 << 36) + i * (1 << 30), 4096, 22016, 44032, 22016, 0) for i in range(3)]
    info = _stage(descs)  # same geometry, but each slice comes from its own source matrix
    assert info.n_entries == 3


def test_default_one_gpu_shape_bands_its_narrow_rows(monkeypatch):
    """Unset, a local table takes shape 17; its rows of 8 KB and less stay with the vector copy,
    shape 8, and are cut into bands the same way (wide rows would go to the tensor-map kernel,
    whose maps need a GPU to encode)."""
    monkeypatch.delenv("SUIKA_RS_BAND_BYTES", raising=False)
    monkeypatch.delenv("SUIKA_RS_VARIANT", raising=False)
    info = _stage(_tp_grow(2, 4096, 8192))
    band_rows = (8 << 20) // 8192  # 1024 rows per band
    assert info.variant == 16 and info.n_tensor_entries == 0
    assert info.n_entries == 2 * (4096 // band_rows)


def test_remote_tables_keep_the_vector_shape(monkeypatch):
    monkeypatch.delenv("SUIKA_RS_VARIANT", raising=False)
    descs = [d[:6] + (L.RS_COPY_REMOTE,) for d in _tp_grow(2, 4096, 22016)]
    info = _stage(descs)
    assert info.variant == 1 and info.n_tensor_entries == 0 and info.n_entries == 2


@pytest.mark.parametrize("variant", ["15", "16", "17"])
def test_split_shapes_band_narrow_rows_like_shape_8(variant, monkeypatch):
    """The split shapes hand rows of 8 KB and less to the vector copy, cut into the same bands as
    shape 8 gives them, and leave the tensor-map part empty."""
    monkeypatch.delenv("SUIKA_RS_BAND_BYTES", raising=False)
    monkeypatch.setenv("SUIKA_RS_VARIANT", "8")
    want = _stage(_tp_grow(4, 8192, 4096))
    monkeypatch.setenv("SUIKA_RS_VARIANT", variant)
    info = _stage(_tp_grow(4, 8192, 4096))
    assert info.variant == int(variant) - 1 and info.n_tensor_entries == 0
    assert (info.n_entries, info.n_tiles, info.total_bytes) == (want.n_entries, want.n_tiles, want.total_bytes)
    assert info.n_entries == 16  # four 8 MB bands per 32 MB slice

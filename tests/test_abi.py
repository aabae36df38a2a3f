"""The C-ABI library loads on a CPU-only host and exports every function include/*.h declares."""
import ctypes
import glob
import os
import re

from suika_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(rs_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_the_path():
    names = declared_functions()
    for n in ("rs_plan_build", "rs_program_build", "rs_program_resolve", "rs_copy_launch", "rs_peer_open"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding knows the signature of each of them
    assert declared_functions() <= set(_lib.SIGNATURES)


def test_version_and_error_string():
    lib = _lib.load()
    a, b = ctypes.c_int32(), ctypes.c_int32()
    assert lib.rs_version(ctypes.byref(a), ctypes.byref(b)) == 0 and (a.value, b.value) >= (1, 1)
    assert lib.rs_plan_num_ops(None, None) == _lib.RS_ERR_ARG
    assert b"NULL" in lib.rs_last_error()


def test_copy_workspace_size_without_gpu():
    lib = _lib.load()
    n = ctypes.c_uint64()
    assert lib.rs_copy_workspace_bytes(1000, ctypes.byref(n)) == 0
    assert n.value >= 1000 * 72 and n.value % 256 == 0


def _descs(rows):
    import numpy as np
    return np.array(rows, dtype=_lib.COPY_DESC_DTYPE)


def test_copy_staging_validates_before_any_cuda_call():
    """Malformed copy descriptors are rejected on the host, before the device is touched (so
    these checks run without a GPU); an all-empty table is a no-op."""
    lib = _lib.load()
    info = _lib.RsLaunchInfo()
    ws = ctypes.c_void_p(1 << 20)  # never dereferenced: validation fails first
    bad_pitch = _descs([(1 << 20, 2 << 20, 4, 512, 256, 512, 0)])  # 512-byte rows at a 256-byte source pitch
    assert lib.rs_copy_stage(bad_pitch.ctypes.data, 1, ws, 1 << 20, None, ctypes.byref(info)) == _lib.RS_ERR_ARG
    assert b"longer than their pitch" in lib.rs_last_error()
    null_src = _descs([(0, 2 << 20, 1, 64, 64, 64, 0)])
    assert lib.rs_copy_stage(null_src.ctypes.data, 1, ws, 1 << 20, None, ctypes.byref(info)) == _lib.RS_ERR_ARG
    assert b"NULL address" in lib.rs_last_error()
    huge_rows = _descs([(1 << 20, 2 << 20, 1 << 33, 1, 1, 1, 0)])
    assert lib.rs_copy_stage(huge_rows.ctypes.data, 1, ws, 1 << 20, None, ctypes.byref(info)) == _lib.RS_ERR_ARG
    empty = _descs([(1 << 20, 2 << 20, 0, 64, 64, 64, 0), (1 << 20, 2 << 20, 3, 0, 64, 64, 0)])
    assert lib.rs_copy_stage(empty.ctypes.data, 2, None, 0, None, ctypes.byref(info)) == _lib.RS_OK
    assert info.n_entries == 0 and info.n_tiles == 0
    assert lib.rs_copy_run(None, ctypes.byref(info), None) == _lib.RS_OK  # nothing staged: nothing to launch


def test_noalloc_capacity_and_empty_tables_without_gpu():
    lib = _lib.load()
    over = _descs([(1 << 20, 2 << 20, 1, 16, 16, 16, 0)] * (_lib.RS_NOALLOC_MAX_ENTRIES + 1))
    assert lib.rs_copy_launch_noalloc(over.ctypes.data, len(over), None, None) == _lib.RS_ERR_CAPACITY
    empty = _descs([(1 << 20, 2 << 20, 0, 16, 16, 16, 0)] * 4)
    assert lib.rs_copy_launch_noalloc(empty.ctypes.data, len(empty), None, None) == _lib.RS_OK


def test_header_is_plain_c():
    """FFI users (ctypes, cgo, JNI) bind the header as C: it must compile as C99 on its own,
    without warnings, and as C++."""
    import shutil
    import subprocess
    import pytest
    hdr = os.path.join(REPO, "include", "suika_reshard.h")
    if not shutil.which("gcc"):
        pytest.skip("gcc not found")
    for cmd in (["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-fsyntax-only", "-x", "c", hdr],
                ["g++", "-std=c++11", "-Wall", "-Werror", "-fsyntax-only", "-x", "c++", hdr]):
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_ctypes_structs_match_the_header_layout(tmp_path):
    """Every ctypes structure in the binding has the size and field offsets the C compiler gives
    the header's struct of the same name (a header / binding drift would corrupt calls)."""
    import shutil
    import subprocess
    import pytest
    if not shutil.which("gcc"):
        pytest.skip("gcc not found")
    pairs = {
        "rs_tensor_meta": _lib.RsTensorMeta, "rs_rank_layout": _lib.RsRankLayout, "rs_plan_opts": _lib.RsPlanOpts,
        "rs_op": _lib.RsOp, "rs_slice_group": _lib.RsSliceGroup, "rs_slice_rule": _lib.RsSliceRule,
        "rs_subfield": _lib.RsSubfield, "rs_program_counts": _lib.RsProgramCounts, "rs_dst_slot": _lib.RsDstSlot,
        "rs_src_slot": _lib.RsSrcSlot, "rs_meta_slot": _lib.RsMetaSlot, "rs_segment": _lib.RsSegment,
        "rs_copy_desc": _lib.RsCopyDesc, "rs_launch_info": _lib.RsLaunchInfo, "rs_peer_handle": _lib.RsPeerHandle,
        "rs_stage_mesh": _lib.RsStageMesh, "rs_act_piece": _lib.RsActPiece, "rs_act_geometry": _lib.RsActGeometry,
    }
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{os.path.join(REPO, "include", "suika_reshard.h")}"',
             "int main(void) {"]
    for cname, cls in pairs.items():
        lines.append(f'  printf("{cname} (sizeof) %zu\\n", sizeof({cname}));')
        for f, _t in cls._fields_:
            lines.append(f'  printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    r = subprocess.run(["gcc", "-std=c99", str(src), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        name, field, value = line.split()
        got[(name, field)] = int(value)
    for cname, cls in pairs.items():
        assert got[(cname, "(sizeof)")] == ctypes.sizeof(cls), cname
        for f, _t in cls._fields_:
            assert got[(cname, f)] == getattr(cls, f).offset, (cname, f)


def test_numpy_mirrors_match_the_ctypes_structures():
    """The numpy dtypes used to fill large tables have the ctypes structures' field offsets."""
    from suika_b200 import migration as M
    for dt, cls in ((_lib.TENSOR_META_DTYPE, _lib.RsTensorMeta), (_lib.COPY_DESC_DTYPE, _lib.RsCopyDesc),
                    (_lib.SEGMENT_DTYPE, _lib.RsSegment), (_lib.ACT_PIECE_DTYPE, _lib.RsActPiece),
                    (M.DST_SLOT_DTYPE, _lib.RsDstSlot), (M.SRC_SLOT_DTYPE, _lib.RsSrcSlot),
                    (M.META_SLOT_DTYPE, _lib.RsMetaSlot), (M.OP_DTYPE, _lib.RsOp)):
        assert dt.itemsize == ctypes.sizeof(cls)
        assert list(dt.names) == [f for f, _ in cls._fields_]
        for f, _ in cls._fields_:
            assert dt.fields[f][1] == getattr(cls, f).offset, (cls.__name__, f)


def test_binding_arities_match_the_header():
    """Each ctypes signature takes as many arguments as the header's prototype, and returns int
    unless the prototype returns void or a string."""
    src = open(os.path.join(REPO, "include", "suika_reshard.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    protos = {}
    for m in re.finditer(r"^([A-Za-z_][\w\s\*]*?)\b(rs_\w+)\s*\(([^;{]*?)\)\s*;", src, flags=re.M | re.S):
        ret, name, params = m.group(1).strip(), m.group(2), " ".join(m.group(3).split())
        n = 0 if params in ("", "void") else params.count(",") + 1
        protos[name] = (ret, n)
    assert set(protos) == declared_functions(), "every declared function parsed"
    for name, (ret, n) in protos.items():
        res, args = _lib.SIGNATURES[name]
        assert len(args) == n, (name, len(args), n)
        if ret == "int":
            assert res is ctypes.c_int, name
        elif ret == "void":
            assert res is None, name


C_CLIENT = r"""
#include <stdio.h>
#include <string.h>
#include "suika_reshard.h"

/* A C client of the ABI: plan TP1 -> TP2 of one [8, 4] fp32 weight split on dim 0 and of one
   replicated [4] norm, then the activation pieces of a TP2 -> TP1 x DP2 stage boundary. */
int main(void) {
  rs_tensor_meta src_t[2], dst0[2], dst1[2];
  memset(src_t, 0, sizeof src_t); memset(dst0, 0, sizeof dst0); memset(dst1, 0, sizeof dst1);
  for (int i = 0; i < 2; ++i) {
    rs_tensor_meta* all[3] = {&src_t[i], &dst0[i], &dst1[i]};
    for (int k = 0; k < 3; ++k) {
      all[k]->name_id = i; all[k]->itemsize = 4;
      all[k]->ndim = i == 0 ? 2 : 1; all[k]->shape[0] = i == 0 ? 8 : 4; all[k]->shape[1] = 4;
      all[k]->slice_dim = RS_NO_SLICE; all[k]->tp_index = 0; all[k]->tp_deg = 1;
    }
  }
  dst0[0].slice_dim = 0; dst0[0].tp_index = 0; dst0[0].tp_deg = 2;
  dst1[0].slice_dim = 0; dst1[0].tp_index = 1; dst1[0].tp_deg = 2;
  rs_rank_layout src = {0, 2, src_t};
  rs_rank_layout dst[2] = {{0, 2, dst0}, {1, 2, dst1}};
  rs_plan_opts opts = {1, RS_ORDER_REFERENCE, RS_SRC_REFERENCE, 0};
  rs_plan* plan = NULL;
  if (rs_plan_build(&src, 1, dst, 2, &opts, &plan) != RS_OK) { printf("plan: %s\n", rs_last_error()); return 1; }
  int64_t n = 0;
  rs_plan_num_ops(plan, &n);
  rs_op ops[8];
  if (n != 4 || rs_plan_get_ops(plan, ops, 8) != RS_OK) { printf("ops: %lld\n", (long long)n); return 2; }
  rs_plan_free(plan);

  int32_t gs_src[2] = {0, 2}, ranks_src[2] = {0, 1}; int64_t b_src[1] = {4};
  int32_t gs_dst[3] = {0, 1, 2}, ranks_dst[2] = {2, 3}; int64_t b_dst[2] = {2, 2};
  rs_stage_mesh ms = {1, 0, gs_src, ranks_src, b_src}, md = {2, 0, gs_dst, ranks_dst, b_dst};
  int64_t np_ = 0;
  if (rs_act_plan(&ms, &md, 16, NULL, 0, &np_) != RS_OK || np_ != 4) { printf("act: %lld\n", (long long)np_); return 3; }
  if (rs_act_plan(&ms, &md, 15, NULL, 0, &np_) != RS_ERR_SHAPE) return 4;  /* 15 does not split in two */
  int32_t maj = 0, min = 0;
  rs_version(&maj, &min);
  printf("ok %d.%d ops=%lld pieces=4\n", maj, min, (long long)n);
  return 0;
}
"""


def test_a_c_program_links_and_plans(tmp_path):
    """The boundary is C: a C program links libsuika_reshard.so and plans through it (no GPU
    needed for planning)."""
    import shutil
    import subprocess
    import pytest
    if not shutil.which("gcc"):
        pytest.skip("gcc not found")
    lib = _lib.library_path()
    _lib.load()  # builds the library when it is stale
    src = tmp_path / "client.c"
    src.write_text(C_CLIENT)
    exe = tmp_path / "client"
    libdir = os.path.dirname(lib)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{os.path.join(REPO, 'include')}", str(src), "-o", str(exe),
                        f"-L{libdir}", "-l:" + os.path.basename(lib), f"-Wl,-rpath,{libdir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True)
    assert run.returncode == 0 and run.stdout.startswith("ok 1."), (run.returncode, run.stdout, run.stderr)

"""The drop-in takes the reference's own layout objects (needs the reference checkout: $SUIKA_REFERENCE).

Suika passes its own ParamLayout / TensorMeta objects to schedule_and_execute_param_transfer
(Suika/migration.py:558-598); they are built by get_param_tensor_meta from parameters that carry
slice_dim / tp_index / tp_deg attributes (Suika/migration.py:29-64,147-151). Here such objects are
built with the reference's classes from meta tensors carrying those attributes, fed to
suika_b200's Plan and schedule_param_transfer, and the op lists must equal the reference's own
schedule_param_transfer on the same objects, op for op (name, source, target, both tp_metas).
The data path of the same call needs a GPU; on the GPU box the layouts are this package's mirror
objects, which these tests show plan identically.
"""
import os
import sys

import pytest
import torch

from suika_b200 import migration as M
from tests.golden.cases import CASES

pytestmark = pytest.mark.skipif(not os.environ.get("SUIKA_REFERENCE"), reason="needs the reference checkout ($SUIKA_REFERENCE)")


def _ref():
    p = os.environ["SUIKA_REFERENCE"]
    if p not in sys.path:
        sys.path.insert(0, p)
    import Suika.migration as RM
    return RM


def _reference_layout(RM, lay):
    """A reference ParamLayout whose TensorMetas come from tensors, as get_param_tensor_meta builds them."""
    out = RM.ParamLayout()
    for rank, metas in lay.layout.items():
        out.layout[rank] = {}
        for name, m in metas.items():
            shape = list(m.shape)
            if m.tp_meta is not None:
                shape[m.tp_meta[0]] //= m.tp_meta[2]
            t = torch.empty(shape, dtype=m.dtype, device="meta")
            if m.tp_meta is not None:
                t.slice_dim, t.tp_index, t.tp_deg = m.tp_meta
            out.layout[rank][name] = RM.TensorMeta(tensor=t, name=name)
    return out


def _ops(ops):
    return [(o.param_name, o.src_rank, o.dst_rank, tuple(o.src_meta.tp_meta) if o.src_meta.tp_meta else None,
             tuple(o.dst_meta.tp_meta) if o.dst_meta.tp_meta else None) for o in ops]


@pytest.mark.parametrize("case", ["cfg1", "cfg2_mini", "cfg3_mini", "cfg4_mini", "cfg5_mini", "hetero_mini", "shrink_mini",
                                  "pp_deepen_mini", "next_step"])
@pytest.mark.parametrize("ib", [True, False])
def test_plan_of_reference_objects_equals_reference_schedule(case, ib, monkeypatch):
    RM = _ref()
    if ib:
        monkeypatch.delenv("NCCL_IB_DISABLE", raising=False)
    else:
        monkeypatch.setenv("NCCL_IB_DISABLE", "1")
    spl, tpl = CASES[case]["config"].layouts()
    rspl, rtpl = _reference_layout(RM, spl), _reference_layout(RM, tpl)
    want = _ops(RM.schedule_param_transfer(rspl, rtpl))
    assert _ops(M.schedule_param_transfer(rspl, rtpl)) == want
    assert _ops(M.Plan(rspl, rtpl).transfer_ops()) == want


def test_reference_errors_are_the_reference_exceptions():
    """A target no source owns: the reference asserts; so does the drop-in's planner."""
    RM = _ref()
    spl, tpl = CASES["cfg1"]["config"].layouts()
    rspl, rtpl = _reference_layout(RM, spl), _reference_layout(RM, tpl)
    name = next(iter(rtpl.layout[0]))
    for r in rspl.layout:
        rspl.layout[r].pop(name, None)
    with pytest.raises(AssertionError):
        RM.schedule_param_transfer(rspl, rtpl)
    with pytest.raises(AssertionError):
        M.Plan(rspl, rtpl)


def _functions_calling(tree, callee):
    import ast
    out = {}
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef):
            calls = [c for c in ast.walk(node) if isinstance(c, ast.Call) and isinstance(c.func, ast.Name) and c.func.id == callee]
            if calls:
                out[node.name] = calls
    return out


def test_public_api_reaches_the_drop_in_through_module_globals():
    """migration_save and migration_load (Suika/migration.py:1357,1546) call
    schedule_and_execute_param_transfer, and the IPC hand-off functions, by their module-level
    names, so rebinding those globals (the switch INTEGRATION.md describes) reroutes both paths;
    and every keyword they pass is a parameter of the drop-in."""
    import ast
    import inspect
    RM = _ref()
    tree = ast.parse(inspect.getsource(RM))
    callers = _functions_calling(tree, "schedule_and_execute_param_transfer")
    assert {"migration_save", "migration_load"} <= set(callers)
    params = list(inspect.signature(M.schedule_and_execute_param_transfer).parameters)
    for fn in ("migration_save", "migration_load"):
        for call in callers[fn]:
            assert {kw.arg for kw in call.keywords} <= set(params), fn
    ref_params = list(inspect.signature(RM.schedule_and_execute_param_transfer).parameters)
    assert params[:len(ref_params)] == ref_params  # the reference's parameters, in its order
    from suika_b200 import handoff as H
    for name, fn in (("interactive_IPC_state_dict_send", H.interactive_IPC_state_dict_send),
                     ("interactive_IPC_state_dict_recv", H.interactive_IPC_state_dict_recv)):
        sites = _functions_calling(tree, name)
        assert {"migration_save", "migration_load"} & set(sites), name
        ours = set(inspect.signature(fn).parameters)
        for calls in sites.values():
            for call in calls:
                assert {kw.arg for kw in call.keywords} <= ours, name
    # the rebinding takes: the reference module resolves the name at call time
    orig = RM.schedule_and_execute_param_transfer
    try:
        RM.schedule_and_execute_param_transfer = M.schedule_and_execute_param_transfer
        assert RM.__dict__["schedule_and_execute_param_transfer"] is M.schedule_and_execute_param_transfer
    finally:
        RM.schedule_and_execute_param_transfer = orig

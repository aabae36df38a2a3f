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

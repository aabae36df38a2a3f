"""The reference-shaped Python types (suika_b200.migration.TensorMeta / ParamLayout) behave as the
reference's (Suika/migration.py:29-254): TP queries, scale_to_tp, equality, ownership."""
import pytest
import torch

from oracle import restate as O
from suika_b200 import migration as M
from tests.golden.cases import CASES


def test_tensor_meta_tp_queries_and_scale():
    m = M.TensorMeta(name="w", dtype=torch.bfloat16, shape=[8, 6], tp_meta=(0, 1, 2))
    assert m.is_tp() and m.slice_dim() == 0 and m.tp_index() == 1 and m.tp_deg() == 2
    assert list(m.actual_shape()) == [4, 6] and m.numel() == 24 and m.volumn() == 48
    pieces = m.scale_to_tp(8)
    assert [p.tp_meta for p in pieces] == [(0, 4, 8), (0, 5, 8), (0, 6, 8), (0, 7, 8)]
    assert m.scale_to_tp(2) == [m] and m.scale_to_tp(1)[0] is m
    r = M.TensorMeta(name="n", dtype=torch.float32, shape=[6])
    assert not r.is_tp() and r.slice_dim() is None and r.tp_index() == 0 and r.tp_deg() == 1 and r.scale_to_tp(4) == [r]


def test_tensor_meta_equality_like_the_reference():
    a = M.TensorMeta(name="a", dtype=torch.float32, shape=[4, 4], tp_meta=(0, 0, 2))
    b = M.TensorMeta(name="b", dtype=torch.float32, shape=[4, 4], tp_meta=(0, 1, 4))  # same slice dim: equal
    c = M.TensorMeta(name="a", dtype=torch.float32, shape=[4, 4], tp_meta=(-1, 0, 2))
    d = M.TensorMeta(name="a", dtype=torch.float32, shape=[4, 4])
    assert a == b and a != c and a != d and a != "a"
    with pytest.raises(TypeError):
        hash(a)


def test_tensor_meta_from_parallel_linear_attributes():
    w = torch.empty(3, 5)
    w.slice_dim, w.tp_index, w.tp_deg = -1, 1, 4
    m = M.TensorMeta(tensor=w, name="w")
    assert m.tp_meta == (-1, 1, 4) and list(m.shape) == [3, 20]


@pytest.mark.parametrize("case", ["cfg2_mini", "cfg5_mini", "hetero_mini"])
def test_owners_match_the_oracle(case):
    spl, tpl = CASES[case]["config"].layouts()
    pl = M.ParamLayout()
    pl.layout = spl.layout
    for dst, metas in tpl.layout.items():
        for name, m in metas.items():
            want = [r for r, sm in spl.layout.items() if name in sm and O._owned(sm[name].tp_meta, m.tp_meta)]
            piece = M.TensorMeta(name=name, dtype=m.dtype, shape=m.shape, tp_meta=m.tp_meta)
            assert pl.owners(piece) == want, (dst, name)
            assert pl.is_owned(want[0], name) if want else True


def test_overlap_and_owned_statics():
    assert M.ParamLayout.is_tensor_tp_overlap((0, 1, 2), (0, 3, 4)) and not M.ParamLayout.is_tensor_tp_overlap((0, 0, 2), (0, 3, 4))
    assert M.ParamLayout.is_tensor_tp_overlap(None, (0, 3, 4))
    assert M.ParamLayout.is_tensor_tp_owned((0, 1, 2), (0, 3, 4)) and not M.ParamLayout.is_tensor_tp_owned((0, 3, 4), (0, 1, 2))
    with pytest.raises(AssertionError, match="slice dim mismatch"):
        M.ParamLayout.is_tensor_tp_overlap((0, 0, 2), (-1, 0, 2))

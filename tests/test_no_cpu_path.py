"""The product has no CPU path: every entry point that moves state refuses a non-CUDA device
loudly instead of falling back to host code (run on a CPU-only host)."""
import pytest
import torch

from suika_b200 import activation as A
from suika_b200 import migration as M
from suika_b200 import synthetic as S
from tests.golden.cases import CASES


def _case():
    spl, tpl = CASES["odd_mini"]["config"].layouts()
    states = S.host_states(spl, S.SUBFIELDS, seed=0)
    kinds = dict(S.SUBFIELDS)
    src = {r: {n: {s: S.to_torch(a, kinds[s]) for s, a in e.items()} for n, e in st.items()} for r, st in states.items()}
    return spl, tpl, src


def test_reshard_local_refuses_the_cpu():
    spl, tpl, src = _case()
    with pytest.raises(RuntimeError, match="CUDA"):
        M.reshard_local(spl, tpl, src, S.expected_sub_fields(), torch.device("cpu"))


def test_drop_in_refuses_the_cpu():
    spl, tpl, src = _case()
    with pytest.raises(RuntimeError, match="CUDA"):
        M.schedule_and_execute_param_transfer(spl, tpl, src[0], {"expected_sub_fields": S.expected_sub_fields()},
                                              "cpu", None)


def test_execute_param_transfer_refuses_the_cpu():
    spl, tpl, src = _case()
    sched = M.schedule_param_transfer(spl, tpl)
    with pytest.raises(RuntimeError, match="CUDA"):
        M.execute_param_transfer(sched, src[0], "cpu", S.expected_sub_fields(), fake_source_state_dicts=src, rank=0)


def test_activation_exchange_refuses_host_tensors():
    x = {0: torch.zeros(2, 3, 4)}
    t = {1: torch.zeros(2, 3, 4)}
    with pytest.raises(ValueError, match="CUDA tensor"):
        A.exchange_local([[0]], [[1]], [2], [2], x, t)

"""Checkpoint resume on B200 (execute_param_transfer with fake_source_state_dicts,
Suika/migration.py:1235-1244): each target rank's state is built on the GPU straight from host
source shards. Same bytes and piece order as the reference (tests/golden digests); singleton
targets keep their source's shape, as in the reference's checkpoint path (migration.py:477-482)."""
import os

import numpy as np
import pytest
import torch

from suika_b200 import migration as M
from suika_b200 import synthetic as S
from tests.golden.cases import CASES
from tests.helpers import SUBS, digest, golden_states, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("case", ["cfg1", "cfg2_mini", "cfg2_mini_noib", "cfg3_mini", "cfg4_mini", "cfg5_mini",
                                  "shrink_mini", "hetero_mini", "odd_mini", "pp_deepen_mini", "gpt_shrink_mini",
                                  "grow_dp_tp_mini", "qwen_grow_mini", "wide_mini", "wide_shrink_mini"])
def test_checkpoint_resume_matches_reference(case, monkeypatch):
    g = load_golden(case)
    if g["minimum_est_peers"] == 2:
        monkeypatch.setenv("NCCL_IB_DISABLE", "1")
    else:
        monkeypatch.delenv("NCCL_IB_DISABLE", raising=False)
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = golden_states(cfg, seed=g["seed"])
    kinds = dict(SUBS)
    fake = {r: {n: {s: S.to_torch(a, kinds[s]) for s, a in e.items()} for n, e in st.items()} for r, st in states.items()}
    sched = M.schedule_param_transfer(spl, tpl)
    for rank_s, want in g["ranks"].items():
        r = int(rank_s)
        out = M.execute_param_transfer(sched, fake.get(r, {}), DEV, S.expected_sub_fields(), fake_source_state_dicts=fake, rank=r)
        assert list(out) == want["order"]
        for name, fields in want["digests"].items():
            for sub, (shape, _dt, sha) in fields.items():
                t = out[name][sub]
                assert t.device == DEV
                h = t.detach().cpu()
                if h.dtype == torch.bfloat16:
                    h = h.view(torch.uint16)
                if sub == "step":
                    assert tuple(t.shape) == ()  # the source's own shape
                    assert digest(h.numpy()) == sha
                else:
                    assert list(t.shape) == shape
                    assert digest(h.numpy()) == sha, (rank_s, name, sub)

"""The next training step after a reshard on a B200, against the reference's own model.

Golden case `next_step`: a small Llama's training state (bf16 param, fp32 master / exp_avg /
exp_avg_sq, step) resharded TP4 -> TP2 on one GPU by the product (reshard_local, one sm_100a
launch). The full tensors are reassembled from the target shards and one training step runs on
the host (tests/next_step.py: the reference's SuikaLlama restated, torch.optim.AdamW on the fp32
master with the migrated moments and step).
  * Reference cat order: the losses must be bit-identical to those of the oracle's migrated state
    (byte-equal to the reference's), and equal, within 1e-6 relative, the losses the reference's
    own SuikaLlama + AdamW recorded (tests/golden/next_step_losses.json). The reference's order
    permutes rank 0's lm_head vocab rows here, so these losses differ from the un-migrated ones;
    a product that fixed or broke the order differently would fail.
  * Slice order: the losses must be bit-identical to the un-migrated state's.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import restate as O
from suika_b200 import migration as M
from suika_b200 import synthetic as S
from tests import next_step as NS
from tests.golden.cases import CASES
from tests.helpers import GOLDEN_DIR, SUB_META, SUBS, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REL_TOL = 1e-6


def _dev_np(t):
    t = t.detach().cpu().contiguous()
    return t.view(torch.uint16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


def _migrate_on_gpu(spl, tpl, states, order, minimum_est_peers):
    kinds = dict(SUBS)
    dev_states = {r: {n: {s: S.to_torch(a, kinds[s], DEV if kinds[s] != "meta" else None) for s, a in e.items()}
                      for n, e in st.items()} for r, st in states.items()}
    out = M.reshard_local(spl, tpl, dev_states, S.expected_sub_fields(), DEV, order=order, minimum_est_peers=minimum_est_peers)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("order", ["reference", "semantic"])
def test_next_step_after_reshard(order):
    with open(os.path.join(GOLDEN_DIR, "next_step_losses.json")) as f:
        gold = json.load(f)
    g = load_golden("next_step")
    cfg = CASES["next_step"]["config"]
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, SUBS, seed=g["seed"], distinct_steps=True)
    out = _migrate_on_gpu(spl, tpl, states, order, g["minimum_est_peers"])
    got = NS.losses(cfg.spec, NS.full_state(tpl, out, _dev_np))
    unmigrated = NS.losses(cfg.spec, NS.full_state(spl, states))
    if order == "semantic":
        assert got == unmigrated, (got, unmigrated)
        return
    ops = O.schedule(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    oracle_state = {r: O.execute_rank(ops, states, SUB_META, r, order="reference") for r in tpl.layout}
    assert got == NS.losses(cfg.spec, NS.full_state(tpl, oracle_state))
    want = (float.fromhex(gold["reference_order"]["loss"]), float.fromhex(gold["reference_order"]["loss_after"]))
    for a, b in zip(got, want):
        assert abs(a - b) <= REL_TOL * abs(b), (got, want)
    assert got != unmigrated
    assert np.isfinite(got).all() and got[1] < got[0]  # the step trains

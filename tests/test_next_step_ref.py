"""The next training step after a reshard, tied to the reference's own model and optimizer.

tests/golden/next_step_losses.json holds the losses that the reference's SuikaLlama and
torch.optim.AdamW produce from (a) the state migrated by the reference (its cat order, whose
received-first concatenation permutes rank 0's lm_head vocab rows in this TP4 -> TP2 shrink) and
(b) the un-migrated state (tests/golden/make_next_step_golden.py). Here:
  * the oracle's reference-order migration (byte-equal to the reference's, by digests) through the
    restated model of tests/next_step.py gives those losses;
  * the oracle's slice-order migration gives exactly the un-migrated losses;
  * with $SUIKA_REFERENCE set, the reference's SuikaLlama is run live and must agree bit for bit.
Tolerance against the stored losses: 1e-6 relative (the CPU's fp32 GEMMs may sum in another order
on another machine); on one machine the runs are bit-identical.
"""
import json
import os

import pytest

from oracle import restate as O
from suika_b200 import synthetic as S
from tests import next_step as NS
from tests.golden.cases import CASES
from tests.helpers import GOLDEN_DIR, SUB_META, SUBS, load_golden

REL_TOL = 1e-6

with open(os.path.join(GOLDEN_DIR, "next_step_losses.json")) as _f:
    GOLD = json.load(_f)


def _case():
    g = load_golden("next_step")
    cfg = CASES["next_step"]["config"]
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, SUBS, seed=g["seed"], distinct_steps=True)
    ops = O.schedule(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    return cfg, spl, tpl, states, ops


def _close(got, key):
    want = (float.fromhex(GOLD[key]["loss"]), float.fromhex(GOLD[key]["loss_after"]))
    for a, b in zip(got, want):
        assert abs(a - b) <= REL_TOL * abs(b), (key, got, want)


def test_reference_order_migration_gives_the_reference_models_next_step():
    cfg, spl, tpl, states, ops = _case()
    migrated = {r: O.execute_rank(ops, states, SUB_META, r, order="reference") for r in tpl.layout}
    got = NS.losses(cfg.spec, NS.full_state(tpl, migrated))
    _close(got, "reference_order")
    _close(NS.losses(cfg.spec, NS.full_state(spl, states)), "unmigrated")
    assert got != NS.losses(cfg.spec, NS.full_state(spl, states))  # the reference's cat order changes training


def test_slice_order_migration_keeps_the_unmigrated_next_step():
    cfg, spl, tpl, states, ops = _case()
    migrated = {r: O.execute_rank(ops, states, SUB_META, r, order="semantic") for r in tpl.layout}
    assert NS.losses(cfg.spec, NS.full_state(tpl, migrated)) == NS.losses(cfg.spec, NS.full_state(spl, states))


@pytest.mark.skipif(not os.environ.get("SUIKA_REFERENCE"), reason="needs the reference checkout ($SUIKA_REFERENCE)")
def test_restated_model_is_the_reference_model_bit_for_bit():
    from tests.golden.make_next_step_golden import reference_losses
    cfg, spl, tpl, states, ops = _case()
    for order in ("reference", "semantic"):
        migrated = {r: O.execute_rank(ops, states, SUB_META, r, order=order) for r in tpl.layout}
        full = NS.full_state(tpl, migrated)
        assert reference_losses(os.environ["SUIKA_REFERENCE"], cfg.spec, full) == NS.losses(cfg.spec, full), order

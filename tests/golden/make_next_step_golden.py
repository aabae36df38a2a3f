"""Record the reference model's next training step on the reference-migrated state (fixture generator).

Run where the reference checkout (read-only) is importable; $SUIKA_REFERENCE names its directory:

    SUIKA_REFERENCE=/path/to/Suika python tests/golden/make_next_step_golden.py

The state is golden case `next_step` (tests/golden/cases.py): a small Llama's training state
(bf16 param, fp32 master / exp_avg / exp_avg_sq, step) resharded TP4 -> TP2 x PP2.
  1. The migrated state in the reference's cat order is rebuilt with oracle/restate.py, and every
     target tensor is checked against the digests that the reference's own migration produced on
     gloo ranks (tests/golden/next_step.json, from make_golden.py), so it is the reference's bytes.
  2. Full tensors are reassembled from the target shards (TP shards concatenated in tp_index
     order); in this reshard the reference's cat order puts rank 0's received row pieces before
     its own, so some reassembled weights are row-permuted.
  3. The reference's own SuikaLlama (Suika/models/llama_model.py:108-157, one stage holding the
     whole model) and torch.optim.AdamW (tasks/task.py:72-73) take one step from it: loss, backward,
     AdamW on the fp32 master with the migrated exp_avg / exp_avg_sq / step, bf16 weights from the
     new master, loss again. The same is done from the un-migrated state.
  4. The restated model of tests/next_step.py must give bit-identical losses on this machine.
transformers 5.x's LlamaDecoderLayer returns a tensor where the reference's transformers pin
returned a tuple (SuikaLlamaBase.forward takes layer_outputs[0]); each block is wrapped to return
a 1-tuple, which restores what the reference's forward expects.

Output: tests/golden/next_step_losses.json (losses as float.hex).
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def reference_losses(ref_path: str, spec, full) -> tuple:
    import torch
    sys.path.insert(0, ref_path)
    from Suika.models.llama_model import SuikaLlama
    from tests import next_step as NS
    torch.manual_seed(0)
    model = SuikaLlama(NS.llama_config(spec), layer_index=0, n_layer=spec.n_layers, add_embedding_and_lm_head=True).float()
    for block in model.h:
        inner = block.forward
        block.forward = lambda *a, _f=inner, **k: (_f(*a, **k),)
    l0, l1 = NS.train_step(model, full, NS.tokens(spec))
    return float(l0), float(l1)


def main():
    ref_path = os.environ.get("SUIKA_REFERENCE")
    if not ref_path:
        raise SystemExit("set SUIKA_REFERENCE to the reference checkout")
    from oracle import restate as O
    from suika_b200 import synthetic as S
    from tests import next_step as NS
    from tests.golden.cases import CASES
    from tests.helpers import SUB_META, SUBS, digest, load_golden

    g = load_golden("next_step")
    cfg = CASES["next_step"]["config"]
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, SUBS, seed=g["seed"], distinct_steps=True)
    ops = O.schedule(spl, tpl, minimum_est_peers=g["minimum_est_peers"])
    migrated = {r: O.execute_rank(ops, states, SUB_META, r, order="reference") for r in tpl.layout}
    for rank_s, want in g["ranks"].items():  # the reference's own bytes
        for name, fields in want["digests"].items():
            for sub, (shape, _, sha) in fields.items():
                a = migrated[int(rank_s)][name][sub]
                assert list(a.shape) == shape and digest(a) == sha, (rank_s, name, sub)
    full_mig = NS.full_state(tpl, migrated)
    full_src = NS.full_state(spl, states)
    out = {"case": "next_step", "spec": cfg.spec.__dict__, "tokens": {"shape": list(NS.TOKENS_SHAPE), "seed": NS.TOKENS_SEED},
           "optimizer": {"lr": NS.LR, "betas": list(NS.BETAS), "eps": NS.EPS, "weight_decay": NS.WEIGHT_DECAY}}
    for key, full in (("reference_order", full_mig), ("unmigrated", full_src)):
        ref = reference_losses(ref_path, cfg.spec, full)
        mine = NS.losses(cfg.spec, full)
        assert ref == mine, (key, ref, mine)  # the restated model is the reference's, bit for bit
        out[key] = {"loss": ref[0].hex(), "loss_after": ref[1].hex(), "loss_f": ref[0], "loss_after_f": ref[1]}
        print(f"{key}: loss {ref[0]:.9f} -> {ref[1]:.9f} after one AdamW step", flush=True)
    assert out["reference_order"]["loss"] != out["unmigrated"]["loss"], "the cat-order quirk should change the model"
    with open(os.path.join(HERE, "next_step_losses.json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()

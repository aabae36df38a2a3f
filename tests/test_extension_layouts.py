"""Layouts the reference does not have (fused QKV split by head, GQA KV-head replication,
vocab-parallel embeddings), planned by interval intersection (rs_plan_build_rules). Their oracle
is the semantic one: gather each full tensor from the sources, re-slice it by the target rule.
Parity with the reference is not defined for them (it has no such layouts)."""
import numpy as np
import pytest

from oracle import restate as O
from suika_b200 import migration as M
from suika_b200 import synthetic as S
from suika_b200.layouts import SPECS, ReshardConfig, scaled_spec
from tests.helpers import SUB_ITEMSIZE, SUB_META, SUBS, emulate_program

SUBFIELD_SPEC = [(SUB_ITEMSIZE[s], kind == "meta") for s, kind in SUBS]
_gqa = scaled_spec(SPECS["qwen2-7b"], name="gqa-mini", hidden=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=32,
                   ffn=512, vocab=512, qkv_bias=True, fused_qkv=True, vocab_parallel_wte=True)
_mha = scaled_spec(SPECS["llama2-13b"], name="mha-fused-mini", hidden=320, n_layers=4, n_heads=8, ffn=512, vocab=512,
                   fused_qkv=True)

EXT_CASES = {
    # cfg3 with a fused QKV split by head: TP8 -> TP4 x PP2
    "cfg3_fused_mini": ReshardConfig("cfg3_fused_mini", _mha, [[list(range(8))]], [[[0, 1, 2, 3]], [[4, 5, 6, 7]]]),
    # GQA 8 Q / 2 KV heads: TP4 (each KV head on 2 shards) -> TP2 x DP2, vocab-parallel wte
    "gqa_rep_src": ReshardConfig("gqa_rep_src", _gqa, [[[0, 1, 2, 3]]], [[[0, 1], [2, 3]]]),
    # TP1 -> TP8: KV heads replicated 4x in the target
    "gqa_rep_dst": ReshardConfig("gqa_rep_dst", _gqa, [[[0]]], [[list(range(8))]]),
    # TP2 x PP2 -> TP4 x PP1 with stage reassignment
    "gqa_pp": ReshardConfig("gqa_pp", _gqa, [[[0, 1]], [[2, 3]]], [[[0, 1, 2, 3]]]),
}


def _check(cfg):
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, SUBS, seed=3, distinct_steps=True)
    plan = M.Plan(spl, tpl)
    assert plan.mode == "interval"
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        got = emulate_program(plan.program(rank, SUBFIELD_SPEC), plan.names, states, rank)
        want = O.semantic_target(states, spl, tpl, SUB_META, rank)
        assert list(got) == list(want)
        for name in want:
            for sub, meta in SUB_META:
                if meta:
                    assert float(got[name][sub].reshape(-1)[0]) == float(want[name][sub].reshape(-1)[0])
                    continue
                assert got[name][sub].shape == want[name][sub].shape, (rank, name, sub)
                assert np.array_equal(got[name][sub].view(np.uint8), want[name][sub].view(np.uint8)), (rank, name, sub)
    return plan


@pytest.mark.parametrize("case", sorted(EXT_CASES))
def test_interval_plan_equals_reslice(case):
    _check(EXT_CASES[case])


@pytest.mark.parametrize("case", ["cfg3_mini", "cfg5_mini", "hetero_mini", "shrink_mini"])
def test_interval_mode_on_reference_layouts_equals_semantic_order(case):
    from tests.golden.cases import CASES
    cfg = CASES[case]["config"]
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, SUBS, seed=0, distinct_steps=True)
    plan = M.Plan(spl, tpl, mode="interval")
    for rank, metas in tpl.layout.items():
        if not metas:
            continue
        got = emulate_program(plan.program(rank, SUBFIELD_SPEC), plan.names, states, rank)
        want = O.semantic_target(states, spl, tpl, SUB_META, rank)
        for name in want:
            for sub, meta in SUB_META:
                if not meta:
                    assert np.array_equal(got[name][sub].view(np.uint8), want[name][sub].view(np.uint8)), (rank, name, sub)


def test_replicated_kv_heads_are_read_once_per_target():
    """KV heads replicated on two source shards: each target piece is pulled from one of them."""
    plan = _check(EXT_CASES["gqa_rep_src"])
    ops = plan.op_array
    qkv = [i for i, n in enumerate(plan.names) if "qkv_proj.weight" in n]
    assert qkv
    for name_id in qkv:
        full = plan.names[name_id]
        per_shard = (4 * 32 + 2 * 32) * (256 if full.endswith("weight") else 1)  # TP2: 4 Q heads, 1 K, 1 V
        for r in (0, 1, 2, 3):
            sel = ops[(ops["dst_rank"] == r) & (ops["name_id"] == name_id)]
            assert int(sel["numel"].sum()) == per_shard  # every target row is read exactly once


def test_rules_need_interval_mode():
    spl, tpl = EXT_CASES["gqa_pp"].layouts()
    with pytest.raises(ValueError, match="interval"):
        M.Plan(spl, tpl, mode="reference")


@pytest.mark.parametrize("k", range(24))
def test_random_extension_reshards_equal_reslice(k):
    """Seeded random (TP, PP, DP) reshards of the GQA + fused-QKV + vocab-parallel model: the
    interval planner's programs equal re-slicing the full tensors. TP 4 replicates the 2 KV
    heads on one side or both."""
    from tests.test_planner_random import cases
    src, dst, _ = cases(n=24, seed=4321)[k]
    _check(ReshardConfig(f"rand_ext_{k}", _gqa, src, dst))

"""Parity cases shared by the golden generator and the tests.

Full-width benchmark shapes are too large for a CPU run of the reference, so most cases keep the
reference's tensor names, module order and slicing at reduced widths and depths; cfg1 runs at its
full size. Each case names the reshard (meshes) of the benchmark configuration it stands for.
"""
from suika_b200.layouts import CONFIGS, SPECS, ReshardConfig, scaled_spec

_llama_mini = scaled_spec(SPECS["llama2-13b"], name="llama-mini", hidden=256, n_layers=4, n_heads=8, ffn=512, vocab=512)
_gpt_mini = scaled_spec(SPECS["gpt-6.7b"], name="gpt-mini", hidden=128, n_layers=4, n_heads=4, ffn=512, vocab=256, pos_emb=64)
_qwen_mini = scaled_spec(SPECS["qwen2-7b"], name="qwen-mini", hidden=256, n_layers=4, n_heads=8, n_kv_heads=4, head_dim=32,
                         ffn=512, vocab=512)
_odd = scaled_spec(SPECS["llama-small"], name="llama-odd", hidden=24, n_layers=3, n_heads=2, ffn=40, vocab=50)
# narrow model, wide FFN: TP1 and TP2 shards of down_proj have rows above 8 KB (the rows the one-GPU
# default gives to the tensor-map kernel), TP4 fp32 shards too
_llama_wide = scaled_spec(SPECS["llama2-13b"], name="llama-wide", hidden=64, n_layers=2, n_heads=2, ffn=8704, vocab=64)
# the model of the next-training-step check (tests/golden/make_next_step_golden.py)
NEXT_STEP_SPEC = scaled_spec(SPECS["llama2-13b"], name="next-step", hidden=128, n_layers=2, n_heads=4, ffn=256, vocab=128)


def _cfg(name, spec, base=None, src=None, dst=None, note=""):
    b = CONFIGS[base] if base else None
    return ReshardConfig(name, spec, src if src is not None else b.src_mesh, dst if dst is not None else b.dst_mesh, note or (b.note if b else ""))


CASES = {
    "cfg1": {"config": CONFIGS["cfg1"], "description": "cfg1 at full size: small Llama TP1xPP2 -> TP2xPP1 (2 ranks)"},
    "cfg2_mini": {"config": _cfg("cfg2_mini", _llama_mini, "cfg2"), "description": "Llama (reduced) TP2xPP2xDP2 -> TP4xPP1xDP2 (8 ranks)"},
    "cfg2_mini_noib": {"config": _cfg("cfg2_mini_noib", _llama_mini, "cfg2"), "ib_disabled": True,
                       "description": "as cfg2_mini with NCCL_IB_DISABLE=1 (minimum_est_peers = 2)"},
    "cfg2b_mini": {"config": _cfg("cfg2b_mini", _llama_mini, "cfg2b"), "description": "Llama (reduced) TP1 -> TP2 (2 ranks)"},
    "cfg3_mini": {"config": _cfg("cfg3_mini", _llama_mini, "cfg3"), "description": "Llama (reduced) TP8xPP1 -> TP4xPP2 (8 ranks), TP shrink"},
    "cfg4_mini": {"config": _cfg("cfg4_mini", _gpt_mini, "cfg4"), "description": "GPT (reduced, wpe) TP2xPP2 on 4 -> TP2xPP2xDP2 on 8"},
    "cfg5_mini": {"config": _cfg("cfg5_mini", _qwen_mini, "cfg5"), "description": "Qwen2 (reduced, GQA, QKV bias) TP4xPP2 -> TP2xPP2xDP2"},
    "shrink_mini": {"config": _cfg("shrink_mini", _llama_mini, src=[[[0, 1, 2, 3]], [[4, 5, 6, 7]]], dst=[[[0, 1]]]),
                    "description": "Llama (reduced) TP4xPP2 on 8 -> TP2 on 2 (shrink, runs in the old world)"},
    "hetero_mini": {"config": _cfg("hetero_mini", _llama_mini, src=[[[0], [1, 2]]], dst=[[[0, 1, 2, 3]]]),
                    "description": "Llama (reduced) DP groups of unequal TP (TP1 + TP2) -> TP4"},
    "odd_mini": {"config": _cfg("odd_mini", _odd, src=[[[0]], [[1]]], dst=[[[0, 1]]]),
                 "description": "odd widths (rows not 16-byte multiples) TP1xPP2 -> TP2"},
    "pp_deepen_mini": {"config": _cfg("pp_deepen_mini", _llama_mini, src=[[[0, 1]], [[2, 3]]],
                                      dst=[[[0, 1]], [[2, 3]], [[4, 5]], [[6, 7]]]),
                       "description": "Llama (reduced) TP2xPP2 on 4 -> TP2xPP4 on 8 (stage boundaries move)"},
    "gpt_shrink_mini": {"config": _cfg("gpt_shrink_mini", _gpt_mini, src=[[[0, 1, 2, 3]]], dst=[[[0, 1]]]),
                        "description": "GPT (reduced, wpe, fused c_attn, row biases) TP4 -> TP2 (shrink)"},
    "grow_dp_tp_mini": {"config": _cfg("grow_dp_tp_mini", _llama_mini, src=[[[0]]], dst=[[[0, 1], [2, 3]]]),
                        "description": "Llama (reduced) TP1 on 1 -> TP2xDP2 on 4 (TP and DP grow from one rank)"},
    "qwen_grow_mini": {"config": _cfg("qwen_grow_mini", _qwen_mini, src=[[[0, 1]]], dst=[[[0, 1, 2, 3]]]),
                       "description": "Qwen2 (reduced, GQA 8/4 heads, QKV bias) TP2 -> TP4 (grow)"},
    "wide_mini": {"config": _cfg("wide_mini", _llama_wide, src=[[[0]]], dst=[[[0, 1]]]),
                  "description": "Llama (hidden 64, ffn 8704) TP1 -> TP2: column slices with 17408- and 8704-byte rows"},
    "wide_shrink_mini": {"config": _cfg("wide_shrink_mini", _llama_wide, src=[[[0, 1, 2, 3]]], dst=[[[0, 1]]]),
                         "description": "Llama (hidden 64, ffn 8704) TP4 -> TP2 (shrink): 8704-byte fp32 rows joined"},
    "next_step": {"config": _cfg("next_step", NEXT_STEP_SPEC, src=[[[0, 1, 2, 3]]], dst=[[[0, 1]]]), "seed": 7,
                  "description": "small Llama TP4 -> TP2 with embeddings (shrink: the reference's cat order puts rank "
                                 "0's received pieces first, lm_head's vocab rows included); the state of the "
                                 "next-training-step check"},
}

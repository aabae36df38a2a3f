"""suika_b200.layouts against the reference's own model code.

tests/golden/layouts_ref.json was recorded by tests/golden/make_layout_golden.py, which built every
source and target layout of the benchmark reshards with the reference's model wrappers
(SuikaLlama, SuikaQwen, SuikaGPT), its PlanConfig.to_PPEngine placement and get_param_tensor_meta
(Suika/migration.py:147-151). Here the same layouts come from layouts.mesh_layout, which is what
every golden digest, bench workload and parity test is built on: names, order, full shapes and
tp_meta of every rank must be the reference's. The default rank mesh and layer split of
get_uniform_plan_config (Suika/cluster/plan_config.py:477-540) are pinned the same way.
"""
import hashlib
import json
import os

import pytest

from suika_b200 import layouts as Ly
from tests.golden.make_layout_golden import canonical_json
from tests.helpers import GOLDEN_DIR

with open(os.path.join(GOLDEN_DIR, "layouts_ref.json")) as _f:
    REF = json.load(_f)

# The reference-representable form of each BASELINE model: the reference's GPT has no learned
# position embedding, and no model of the reference splits its embedding.
SPECS = {
    "llama-small": Ly.SPECS["llama-small"],
    "llama2-7b": Ly.SPECS["llama2-7b"],
    "llama2-13b": Ly.SPECS["llama2-13b"],
    "gpt-6.7b": Ly.scaled_spec(Ly.SPECS["gpt-6.7b"], pos_emb=0),
    "qwen2-7b": Ly.SPECS["qwen2-7b"],
}
LAYOUTS = sorted(k for k in REF if k != "uniform")


def _ours(layout: str):
    ent = REF[layout]
    world = len(ent["sha256"])
    lay = Ly.mesh_layout(SPECS[ent["model"]], ent["mesh"], world_size=world)
    return {str(r): [[n, list(m.shape), None if m.tp_meta is None else list(m.tp_meta)] for n, m in metas.items()]
            for r, metas in lay.layout.items()}


def test_fixture_covers_every_benchmark_layout():
    for name, cfg in Ly.CONFIGS.items():
        for side, mesh in (("src", cfg.src_mesh), ("dst", cfg.dst_mesh)):
            key = f"{name}_{side}"
            assert key in REF, key
            assert REF[key]["mesh"] == mesh, key


@pytest.mark.parametrize("layout", LAYOUTS)
def test_mesh_layout_equals_the_reference_model_layout(layout):
    ent = REF[layout]
    ours = _ours(layout)
    assert sorted(ours, key=int) == sorted(ent["sha256"], key=int)
    first, ref_first = next(iter(ent["first_rank"].items()))
    assert ours[first] == ref_first  # readable failure on the first rank
    for r, sha in ent["sha256"].items():
        assert len(ours[r]) == ent["n_tensors"][r], (layout, r)
        assert hashlib.sha256(canonical_json(ours[r]).encode()).hexdigest() == sha, (layout, r)


@pytest.mark.parametrize("layout", LAYOUTS)
def test_stage_split_equals_the_reference(layout):
    ent = REF[layout]
    spec = SPECS[ent["model"]]
    spans = Ly.stage_layers(spec.n_layers, len(ent["mesh"]))
    assert [hi - lo for lo, hi in spans] == ent["layer_partition"]


@pytest.mark.parametrize("shape", sorted(REF["uniform"]))
def test_uniform_mesh_and_layer_split_equal_the_reference(shape):
    pp, dp, tp, n = (int(x) for x in shape.split(","))
    ref = REF["uniform"][shape]
    assert Ly.uniform_mesh(pp, dp, tp) == ref["mesh"]
    assert [hi - lo for lo, hi in Ly.stage_layers(n, pp)] == ref["layer_partition"]


def test_qwen_gqa_and_bias_shapes_are_in_the_fixture():
    """The GQA K/V projections ([kv_heads * head_dim, hidden] = [512, 3584]) and their biases are
    among the pinned tensors."""
    names = dict((n, (s, tp)) for n, s, tp in next(iter(REF["cfg5_src"]["first_rank"].values())))
    assert names["h.0.self_attn.k_proj.weight"] == ([512, 3584], [0, 0, 4])
    assert names["h.0.self_attn.k_proj.bias"] == ([512], [0, 0, 4])
    assert names["h.0.self_attn.o_proj.weight"] == ([3584, 3584], [-1, 0, 4])

"""Record the reference's own per-rank parameter layouts of the benchmark reshards (fixture generator).

Run where the reference checkout (read-only) is importable; $SUIKA_REFERENCE names its directory:

    SUIKA_REFERENCE=/path/to/Suika python tests/golden/make_layout_golden.py [layout ...]

For every source and target layout of the BASELINE reshards, `world` gloo processes on the CPU each
  * build their pipeline stage with the reference's own model wrapper (SuikaLlama, SuikaQwen or
    SuikaGPT from Suika/models/*_model.py, init_on_meta=True, embeddings and head included);
  * place it with the reference's PlanConfig.to_PPEngine (Suika/cluster/plan_config.py:185-217):
    get_uniform_plan_config's layer partition (:477-540) and the layout's rank mesh; the engine
    applies parallelize_tp (Suika/tensor_parallel.py:486-606) to the TP group;
  * record get_param_tensor_meta(engine) (Suika/migration.py:147-151): every name in order, with
    its full shape and tp_meta.
transformers 5.x dropped the attention attributes that the reference divides by the TP degree
(num_heads, num_key_value_heads, hidden_size); they are set from the model config on each attention
module before the engine is built, which is what the reference's transformers pin provided.

Models are the reference-representable forms of the BASELINE models: the GPT has no learned
position embedding (the reference's SuikaGPT has none) and its vocabulary is 50304; Qwen2's
embedding is replicated (the reference does not split nn.Embedding).

Output: tests/golden/layouts_ref.json = {layout: {"model", "mesh", "layer_partition", "n_tensors": {rank: n},
"sha256": {rank: digest of the rank's [[name, full shape, tp_meta], ...] list (canonical_json)},
"first_rank": that list for the lowest rank, kept whole for readable failures}}, plus "uniform":
{"pp,dp,tp,layers": {"mesh", "layer_partition"}} from get_uniform_plan_config's default rank mesh.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
import traceback

HERE = os.path.dirname(os.path.abspath(__file__))

# (model, mesh[stage][dp][tp]) of every layout the benchmark reshards start from or end in.
MODELS = {
    "llama-small": ("llama", dict(hidden_size=1024, intermediate_size=2816, num_hidden_layers=8, num_attention_heads=16,
                                  vocab_size=32000)),
    "llama2-7b": ("llama", dict(hidden_size=4096, intermediate_size=11008, num_hidden_layers=32, num_attention_heads=32,
                                vocab_size=32000)),
    "llama2-13b": ("llama", dict(hidden_size=5120, intermediate_size=13824, num_hidden_layers=40, num_attention_heads=40,
                                 vocab_size=32000)),
    "gpt-6.7b": ("gpt", dict(n_embd=4096, n_layer=32, n_head=32, n_inner=16384, vocab_size=50304, n_positions=2048)),
    "qwen2-7b": ("qwen", dict(hidden_size=3584, intermediate_size=18944, num_hidden_layers=28, num_attention_heads=28,
                              num_key_value_heads=4, vocab_size=152064)),
}
LAYOUTS = {
    "cfg1_src": ("llama-small", [[[0]], [[1]]]),
    "cfg1_dst": ("llama-small", [[[0, 1]]]),
    "cfg2_src": ("llama2-7b", [[[0, 1], [2, 3]], [[4, 5], [6, 7]]]),
    "cfg2_dst": ("llama2-7b", [[[0, 1, 2, 3], [4, 5, 6, 7]]]),
    "cfg2b_src": ("llama2-7b", [[[0]]]),
    "cfg2b_dst": ("llama2-7b", [[[0, 1]]]),
    "cfg3_src": ("llama2-13b", [[[0, 1, 2, 3, 4, 5, 6, 7]]]),
    "cfg3_dst": ("llama2-13b", [[[0, 1, 2, 3]], [[4, 5, 6, 7]]]),
    "cfg4_src": ("gpt-6.7b", [[[0, 1]], [[2, 3]]]),
    "cfg4_dst": ("gpt-6.7b", [[[0, 1], [4, 5]], [[2, 3], [6, 7]]]),
    "cfg5_src": ("qwen2-7b", [[[0, 1, 2, 3]], [[4, 5, 6, 7]]]),
    "cfg5_dst": ("qwen2-7b", [[[0, 1], [2, 3]], [[4, 5], [6, 7]]]),
}


def canonical_json(tensors) -> str:
    """The byte string a rank's tensor list is digested as: [[name, shape, tp_meta or null], ...]."""
    return json.dumps([[n, [int(x) for x in shape], None if tp is None else [int(x) for x in tp]] for n, shape, tp in tensors],
                      separators=(",", ":"))


def compact(entry: dict) -> dict:
    import hashlib
    ranks = entry["ranks"]
    first = min(ranks, key=int)
    return {"model": entry["model"], "mesh": entry["mesh"], "layer_partition": entry["layer_partition"],
            "n_tensors": {r: len(t) for r, t in ranks.items()},
            "sha256": {r: hashlib.sha256(canonical_json(t).encode()).hexdigest() for r, t in ranks.items()},
            "first_rank": {first: ranks[first]}}


def _provider(model: str):
    family, kw = MODELS[model]
    if family == "llama":
        from Suika.models.llama_model import SuikaLlama
        from transformers.models.llama.modeling_llama import LlamaConfig
        cfg, cls = LlamaConfig(max_position_embeddings=16, **kw), SuikaLlama
    elif family == "qwen":
        from Suika.models.qwen_model import SuikaQwen
        from transformers.models.qwen2.modeling_qwen2 import Qwen2Config
        cfg, cls = Qwen2Config(max_position_embeddings=16, **kw), SuikaQwen
    else:
        from Suika.models.gpt_model import GPTConfig, SuikaGPT
        cfg, cls = GPTConfig(**kw), SuikaGPT

    def provider(layer_index, n_layer):
        m = cls(cfg, layer_index, n_layer, add_embedding_and_lm_head=True, init_on_meta=True)
        for mod in m.modules():  # the attention attributes the reference's transformers pin had
            if hasattr(mod, "div_by_tp_deg") and family != "gpt":
                mod.num_heads = cfg.num_attention_heads
                mod.num_key_value_heads = cfg.num_key_value_heads
                mod.hidden_size = cfg.hidden_size
        return m
    return provider, cfg


def _worker(rank, world, layout, port, ref_path, outdir):
    res = {"rank": rank}
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        sys.path.insert(0, ref_path)
        import torch
        import torch.distributed as dist
        from Suika.cluster.plan_config import get_uniform_plan_config
        from Suika.device_mesh import RawDeviceMesh3D
        from Suika.migration import get_param_tensor_meta
        model, mesh = LAYOUTS[layout]
        dist.init_process_group("gloo", rank=rank, world_size=world)
        pp, dp, tp = len(mesh), len(mesh[0]), len(mesh[0][0])
        provider, cfg = _provider(model)
        n_layer = getattr(cfg, "num_hidden_layers", None) or cfg.n_layer
        pc = get_uniform_plan_config("H100", (pp, dp, tp), gbs=8 * dp, n_layer=n_layer, n_mb=1)
        pc.rank_mesh = RawDeviceMesh3D(mesh)
        engine = pc.to_PPEngine(model_provider=provider, device="cpu", init_on_meta=True, enable_profiling=False)
        metas = get_param_tensor_meta(engine)
        res["tensors"] = [[n, list(m.shape), None if m.tp_meta is None else list(m.tp_meta)] for n, m in metas.items()]
        res["layer_partition"] = list(pc.layer_partition)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        res["error"] = traceback.format_exc()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


def run_layout(layout: str, port: int, ref_path: str) -> dict:
    import torch.multiprocessing as mp
    mesh = LAYOUTS[layout][1]
    world = 1 + max(r for st in mesh for g in st for r in g)
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, layout, port, ref_path, d), nprocs=world, join=True)
        results = [json.load(open(os.path.join(d, f"rank{r}.json"))) for r in range(world)]
    for r in results:
        if "error" in r:
            raise RuntimeError(f"{layout} rank {r['rank']}:\n{r['error']}")
    return {"model": LAYOUTS[layout][0], "mesh": mesh, "layer_partition": results[0]["layer_partition"],
            "ranks": {str(r["rank"]): r["tensors"] for r in results}}


# (pp, dp, tp, layers) shapes whose default rank mesh and layer split are recorded as well.
UNIFORM = [(1, 1, 8, 40), (2, 1, 4, 40), (2, 2, 2, 32), (1, 2, 4, 32), (2, 1, 2, 32), (2, 2, 2, 28), (3, 2, 1, 41),
           (4, 1, 2, 30), (8, 1, 1, 40), (1, 8, 1, 16), (2, 4, 1, 7)]


def uniform_meshes(ref_path: str) -> dict:
    """The reference's default rank mesh (PlanConfig.set_rank_mesh) and layer partition of
    get_uniform_plan_config (Suika/cluster/plan_config.py:477-540), per (pp, dp, tp, layers)."""
    sys.path.insert(0, ref_path)
    from Suika.cluster.plan_config import get_uniform_plan_config
    out = {}
    for pp, dp, tp, n in UNIFORM:
        pc = get_uniform_plan_config("H100", (pp, dp, tp), gbs=8 * dp, n_layer=n, n_mb=1)
        m3 = pc.set_rank_mesh()
        out[f"{pp},{dp},{tp},{n}"] = {"mesh": [[[int(r) for r in m1.mesh] for m1 in m2.mesh] for m2 in m3.mesh],
                                      "layer_partition": [int(x) for x in pc.layer_partition]}
    return out


def main(argv):
    ref_path = os.environ.get("SUIKA_REFERENCE")
    if not ref_path:
        raise SystemExit("set SUIKA_REFERENCE to the reference checkout")
    out_path = os.path.join(HERE, "layouts_ref.json")
    data = json.load(open(out_path)) if os.path.exists(out_path) else {}
    data["uniform"] = uniform_meshes(ref_path)
    for i, layout in enumerate(argv or sorted(LAYOUTS)):
        data[layout] = compact(run_layout(layout, 29600 + i, ref_path))
        print(f"{layout}: {len(data[layout]['sha256'])} ranks, {sum(data[layout]['n_tensors'].values())} tensors", flush=True)
    with open(out_path, "w") as f:
        json.dump(data, f, indent=0, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    main(sys.argv[1:])

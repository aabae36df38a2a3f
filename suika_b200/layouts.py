"""Shard layouts of the model families Suika reshards: which tensors exist on which rank, and how
each one is sliced across TP.

This restates, for building ParamLayouts without instantiating models, what the reference derives
from its model wrappers and parallel engine:
  * tensor names and module order: Suika/models/llama_model.py:16-35,107-138 (Llama),
    Suika/models/qwen_model.py:17-40,120-145 (Qwen2), Suika/models/gpt_model.py:13-31,95-120 and
    Suika/models/utils.py:433-459 (GPT, Conv1D replaced by an nn.Linear named `linear`); layer
    names carry the global layer index (OffsetModuleList, Suika/models/utils.py:375-422);
    per-stage extras come after the blocks: wte on the first stage, lm_head (+ norm) on the last;
  * TP slicing: ColumnParallelLinear slices weight and bias on dim 0
    (Suika/tensor_parallel.py:255-261), RowParallelLinear slices its weight on dim -1 and keeps
    the bias whole (Suika/tensor_parallel.py:435-441), everything else (embeddings, norms) is
    replicated; slicing is a contiguous chunk (Suika/tensor_parallel.py:200-204,378-381);
  * PP stage -> layer range: n // pp + (stage < n % pp) (Suika/cluster/plan_config.py:497-501);
  * rank mesh[stage][dp][tp] -> rank; the uniform mesh numbers ranks pp, dp, tp-major
    (Suika/cluster/plan_config.py:503-515).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .migration import ParamLayout, TensorMeta

SliceDim = Optional[int]  # 0, -1, or None (replicated)


@dataclass(frozen=True)
class ModelSpec:
    name: str
    family: str          # "llama" (Llama / Qwen2 blocks) or "gpt" (GPT-2 blocks)
    hidden: int
    n_layers: int
    n_heads: int
    ffn: int
    vocab: int
    n_kv_heads: int = 0  # 0: same as n_heads
    head_dim: int = 0    # 0: hidden // n_heads
    qkv_bias: bool = False
    pos_emb: int = 0     # learned position embedding rows (wpe); not present in the reference's models
    vocab_parallel_wte: bool = False  # slice wte on dim 0 (the reference replicates it)
    fused_qkv: bool = False  # one qkv_proj [(nh + 2 nkv) * hd, h], TP-split by head (not in the reference)

    @property
    def kv_heads(self) -> int:
        return self.n_kv_heads or self.n_heads

    @property
    def hd(self) -> int:
        return self.head_dim or self.hidden // self.n_heads


def layer_tensors(spec: ModelSpec, i: int) -> List[Tuple[str, Tuple[int, ...], SliceDim]]:
    """(name, full shape, slice dim) of decoder layer i, in module (named_parameters) order."""
    h, f = spec.hidden, spec.ffn
    p = f"h.{i}."
    if spec.family == "llama":
        q, kv = spec.n_heads * spec.hd, spec.kv_heads * spec.hd
        out = []
        if spec.fused_qkv:
            out.append((p + "self_attn.qkv_proj.weight", (q + 2 * kv, h), 0))
            if spec.qkv_bias:
                out.append((p + "self_attn.qkv_proj.bias", (q + 2 * kv,), 0))
        for proj, rows in (() if spec.fused_qkv else (("q_proj", q), ("k_proj", kv), ("v_proj", kv))):
            out.append((p + f"self_attn.{proj}.weight", (rows, h), 0))
            if spec.qkv_bias:
                out.append((p + f"self_attn.{proj}.bias", (rows,), 0))
        out += [
            (p + "self_attn.o_proj.weight", (h, q), -1),
            (p + "mlp.gate_proj.weight", (f, h), 0),
            (p + "mlp.up_proj.weight", (f, h), 0),
            (p + "mlp.down_proj.weight", (h, f), -1),
            (p + "input_layernorm.weight", (h,), None),
            (p + "post_attention_layernorm.weight", (h,), None),
        ]
        return out
    if spec.family == "gpt":
        return [
            (p + "ln_1.weight", (h,), None), (p + "ln_1.bias", (h,), None),
            (p + "attn.c_attn.linear.weight", (3 * h, h), 0), (p + "attn.c_attn.linear.bias", (3 * h,), 0),
            (p + "attn.c_proj.linear.weight", (h, h), -1), (p + "attn.c_proj.linear.bias", (h,), None),
            (p + "ln_2.weight", (h,), None), (p + "ln_2.bias", (h,), None),
            (p + "mlp.c_fc.linear.weight", (f, h), 0), (p + "mlp.c_fc.linear.bias", (f,), 0),
            (p + "mlp.c_proj.linear.weight", (h, f), -1), (p + "mlp.c_proj.linear.bias", (h,), None),
        ]
    raise ValueError(f"unknown family {spec.family}")


def qkv_rule(spec: ModelSpec) -> List[Tuple[int, int, int]]:
    """Slice rule of a fused QKV weight/bias split by head: groups Q, K, V along dim 0, each
    (offset, size, units=heads); KV heads are replicated when TP exceeds their count."""
    q, kv = spec.n_heads * spec.hd, spec.kv_heads * spec.hd
    return [(0, q, spec.n_heads), (q, kv, spec.kv_heads), (q + kv, kv, spec.kv_heads)]


def tensor_rule(spec: ModelSpec, name: str):
    if spec.fused_qkv and ".self_attn.qkv_proj." in name:
        return qkv_rule(spec)
    return None


def first_stage_tensors(spec: ModelSpec):
    wte_dim = 0 if spec.vocab_parallel_wte else None
    out = [("wte.weight", (spec.vocab, spec.hidden), wte_dim)]
    if spec.pos_emb:
        out.append(("wpe.weight", (spec.pos_emb, spec.hidden), None))
    return out


def last_stage_tensors(spec: ModelSpec):
    if spec.family == "gpt":
        return [("lm_head.weight", (spec.vocab, spec.hidden), 0), ("lm_head.bias", (spec.vocab,), 0)]
    return [("lm_head.weight", (spec.vocab, spec.hidden), 0), ("norm.weight", (spec.hidden,), None)]


def stage_layers(n_layers: int, pp: int) -> List[Tuple[int, int]]:
    """[lo, hi) layer range per stage: n // pp + (stage < n % pp) (plan_config.py:497-501)."""
    sizes = [n_layers // pp + (s < n_layers % pp) for s in range(pp)]
    out, lo = [], 0
    for s in sizes:
        out.append((lo, lo + s))
        lo += s
    return out


def stage_tensors(spec: ModelSpec, stage: int, pp: int, with_embeddings: bool = True):
    lo, hi = stage_layers(spec.n_layers, pp)[stage]
    names = [t for i in range(lo, hi) for t in layer_tensors(spec, i)]
    if with_embeddings and stage == 0:
        names += first_stage_tensors(spec)
    if with_embeddings and stage == pp - 1:
        names += last_stage_tensors(spec)
    return names


def uniform_mesh(pp: int, dp: int, tp: int, offset: int = 0) -> List[List[List[int]]]:
    """mesh[stage][dp][tp] with ranks numbered pp, dp, tp-major (plan_config.py:503-515)."""
    return [[[offset + s * dp * tp + d * tp + t for t in range(tp)] for d in range(dp)] for s in range(pp)]


def mesh_layout(spec: ModelSpec, mesh: Sequence[Sequence[Sequence[int]]], dtype: torch.dtype = torch.bfloat16,
                world_size: Optional[int] = None, with_embeddings: bool = True) -> ParamLayout:
    """ParamLayout of a model placed on a rank mesh[stage][dp][tp]; ranks of the world that hold
    nothing get an empty entry, and entries are in rank order like ParamLayout.gather's."""
    pp = len(mesh)
    per_rank: Dict[int, Dict[str, TensorMeta]] = {}
    for s, stage in enumerate(mesh):
        tensors = stage_tensors(spec, s, pp, with_embeddings)
        for group in stage:
            tp = len(group)
            for j, rank in enumerate(group):
                metas = {}
                for name, shape, sd in tensors:
                    tpm = None if sd is None else (sd, j, tp)
                    metas[name] = TensorMeta(name=name, dtype=dtype, shape=shape, tp_meta=tpm)
                    rule = tensor_rule(spec, name)
                    if rule is not None and tpm is not None:
                        metas[name].tp_rule = rule
                if rank in per_rank:
                    raise ValueError(f"rank {rank} appears twice in the mesh")
                per_rank[rank] = metas
    n = (max(per_rank) + 1) if world_size is None else world_size
    lay = ParamLayout()
    for r in range(n):
        lay.layout[r] = per_rank.get(r, {})
    return lay


# Model specs named by the reshard configurations (sizes from their published configs).
SPECS: Dict[str, ModelSpec] = {
    "llama-small": ModelSpec("llama-small", "llama", hidden=1024, n_layers=8, n_heads=16, ffn=2816, vocab=32000),
    "llama2-7b": ModelSpec("llama2-7b", "llama", hidden=4096, n_layers=32, n_heads=32, ffn=11008, vocab=32000),
    "llama2-13b": ModelSpec("llama2-13b", "llama", hidden=5120, n_layers=40, n_heads=40, ffn=13824, vocab=32000),
    "gpt-6.7b": ModelSpec("gpt-6.7b", "gpt", hidden=4096, n_layers=32, n_heads=32, ffn=16384, vocab=50304, pos_emb=2048),
    "qwen2-7b": ModelSpec("qwen2-7b", "llama", hidden=3584, n_layers=28, n_heads=28, n_kv_heads=4, head_dim=128,
                          ffn=18944, vocab=152064, qkv_bias=True),
}


@dataclass(frozen=True)
class ReshardConfig:
    """A named reshard: a model, its source mesh and its target mesh."""
    name: str
    spec: ModelSpec
    src_mesh: List[List[List[int]]]
    dst_mesh: List[List[List[int]]]
    note: str = ""

    @property
    def src_world(self) -> int:
        return 1 + max(r for st in self.src_mesh for g in st for r in g)

    @property
    def dst_world(self) -> int:
        return 1 + max(r for st in self.dst_mesh for g in st for r in g)

    @property
    def world_size(self) -> int:
        """Ranks that take part: the larger of the two worlds (grow runs in the new world, shrink
        in the old one, migration.py:1441-1481,1595-1666)."""
        return max(self.src_world, self.dst_world)

    def layouts(self, dtype: torch.dtype = torch.bfloat16, with_embeddings: bool = True):
        """(source, target) ParamLayouts, each over its own world as ParamLayout.gather builds them."""
        return (mesh_layout(self.spec, self.src_mesh, dtype, self.src_world, with_embeddings),
                mesh_layout(self.spec, self.dst_mesh, dtype, self.dst_world, with_embeddings))


def _m(*stages):
    return [[list(g) for g in st] for st in stages]


CONFIGS: Dict[str, ReshardConfig] = {
    "cfg1": ReshardConfig("cfg1", SPECS["llama-small"], _m([[0]], [[1]]), _m([[0, 1]]),
                          "small Llama TP1xPP2 -> TP2xPP1"),
    "cfg2": ReshardConfig("cfg2", SPECS["llama2-7b"], _m([[0, 1], [2, 3]], [[4, 5], [6, 7]]),
                          _m([[0, 1, 2, 3], [4, 5, 6, 7]]), "Llama2-7B TP2xPP2xDP2 -> TP4xPP1xDP2"),
    "cfg2b": ReshardConfig("cfg2b", SPECS["llama2-7b"], _m([[0]]), _m([[0, 1]]),
                           "Llama2-7B TP1 -> TP2 on one GPU (both target ranks emulated on one device)"),
    "cfg3": ReshardConfig("cfg3", SPECS["llama2-13b"], _m([list(range(8))]), _m([[0, 1, 2, 3]], [[4, 5, 6, 7]]),
                          "Llama2-13B TP8xPP1 -> TP4xPP2"),
    "cfg4": ReshardConfig("cfg4", SPECS["gpt-6.7b"], _m([[0, 1]], [[2, 3]]), _m([[0, 1], [4, 5]], [[2, 3], [6, 7]]),
                          "GPT-6.7B TP2xPP2xDP1 (4 GPUs) -> TP2xPP2xDP2 (8 GPUs), replica-preserving mesh"),
    "cfg5": ReshardConfig("cfg5", SPECS["qwen2-7b"], _m([[0, 1, 2, 3]], [[4, 5, 6, 7]]),
                          _m([[0, 1], [2, 3]], [[4, 5], [6, 7]]), "Qwen2-7B TP4xPP2 -> TP2xPP2xDP2"),
}



def shard_spans(full_shape: Sequence[int], tp_meta, rule=None) -> List[Tuple[int, int]]:
    """[lo, hi) intervals of the slice dim a shard holds, in storage order: the contiguous chunk
    of the reference, or, with a rule, each group's units (see rs_slice_rule in the C header)."""
    if tp_meta is None:
        return []
    d, i, g = tp_meta
    F = int(full_shape[d])
    if not rule:
        return [(i * F // g, (i + 1) * F // g)]
    out = []
    for off, size, units in rule:
        usz = size // units
        if units >= g:
            nu = units // g
            u0 = i * nu
        else:
            nu, u0 = 1, i * units // g
        out.append((off + u0 * usz, off + (u0 + nu) * usz))
    return out


def actual_shape(m) -> Tuple[int, ...]:
    """Shape of the shard a meta describes (TensorMeta.actual_shape, extended to slice rules)."""
    shape = [int(s) for s in m.shape]
    if m.tp_meta is not None:
        d = m.tp_meta[0]
        spans = shard_spans(shape, m.tp_meta, getattr(m, "tp_rule", None))
        shape[d] = sum(hi - lo for lo, hi in spans)
    return tuple(shape)


def scaled_spec(spec: ModelSpec, **overrides) -> ModelSpec:
    """A copy of spec with some fields replaced (reduced-size parity cases keep names and slicing)."""
    d = dict(spec.__dict__)
    d.update(overrides)
    return ModelSpec(**d)


# Reshards beyond the benchmark's list, for paths its configurations do not exercise.
EXTRA_CONFIGS: Dict[str, ReshardConfig] = {
    # DP grow from one GPU to eight: every target needs the whole state, which one GPU holds.
    # Half of Llama2-7B's layers keep source plus target of rank 0 within one GPU's memory.
    "dpgrow8": ReshardConfig("dpgrow8", scaled_spec(SPECS["llama2-7b"], name="llama2-7b-16L", n_layers=16), _m([[0]]),
                             _m([[i] for i in range(8)]),
                             "Llama2-7B-shaped 16 layers TP1xDP1 (1 GPU) -> TP1xDP8 (8 GPUs), the DP-replica fan-out case"),
}

"""One training step on a migrated training state (test infrastructure).

The model is the reference's Llama stage, SuikaLlama (Suika/models/llama_model.py:108-157), restated
from the same transformers building blocks it wraps: decoder layers (LlamaDecoderLayer) fed the
rotary position embeddings of positions 0..T-1 and no attention mask (SuikaLlamaBase.forward,
:70-104), the embedding first and the final norm plus lm_head last (:140-157), with the reference's
parameter names. The optimizer is torch.optim.AdamW, as the reference's worker builds it
(tasks/task.py:72-73), applied to the fp32 master weights with the migrated exp_avg, exp_avg_sq and
step; the bf16 params are the model's weights. tests/golden/make_next_step_golden.py runs the
reference's own SuikaLlama on the same inputs and records its losses; the tests compare against
them.

Everything runs in fp32 on the host, so two runs on byte-identical states give identical losses.
"""
from __future__ import annotations

from typing import Dict

import numpy as np
import torch
from transformers.models.llama.modeling_llama import LlamaConfig, LlamaDecoderLayer, LlamaRMSNorm, LlamaRotaryEmbedding

LR, BETAS, EPS, WEIGHT_DECAY = 1e-3, (0.9, 0.95), 1e-8, 0.1
TOKENS_SHAPE, TOKENS_SEED = (2, 16), 0


def llama_config(spec) -> LlamaConfig:
    return LlamaConfig(hidden_size=spec.hidden, intermediate_size=spec.ffn, num_hidden_layers=spec.n_layers,
                       num_attention_heads=spec.n_heads, num_key_value_heads=spec.kv_heads, vocab_size=spec.vocab,
                       max_position_embeddings=64, attn_implementation="eager")


def tokens(spec) -> torch.Tensor:
    return torch.randint(0, spec.vocab, TOKENS_SHAPE, generator=torch.Generator().manual_seed(TOKENS_SEED))


class LlamaStage(torch.nn.Module):
    """A whole Llama as one pipeline stage, parameter for parameter like SuikaLlama."""

    def __init__(self, config: LlamaConfig):
        super().__init__()
        self.h = torch.nn.ModuleList([LlamaDecoderLayer(config, layer_idx=i) for i in range(config.num_hidden_layers)])
        self.rotary_emb = LlamaRotaryEmbedding(config=config)
        self.wte = torch.nn.Embedding(config.vocab_size, config.hidden_size)
        self.lm_head = torch.nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.norm = LlamaRMSNorm(config.hidden_size, config.rms_norm_eps)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        x = self.wte(ids)
        positions = torch.arange(ids.shape[1], device=ids.device).unsqueeze(0)
        rope = self.rotary_emb(x, positions)
        for block in self.h:
            x = block(x, attention_mask=None, position_embeddings=rope)
        return self.lm_head(self.norm(x))


def loss_of(model: torch.nn.Module, ids: torch.Tensor) -> torch.Tensor:
    logits = model(ids)
    return torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))


def _f32(a: np.ndarray, kind: str) -> torch.Tensor:
    """A new fp32 tensor (never a view of the array: AdamW updates its tensors in place)."""
    t = torch.from_numpy(np.array(a, copy=True))
    return t.view(torch.bfloat16).float() if kind == "bf16" else t.float()


def train_step(model: torch.nn.Module, full: Dict[str, Dict[str, np.ndarray]], ids: torch.Tensor):
    """(loss, loss after one AdamW step) of `model` on a full state {name: {sub-field: array}}:
    weights = bf16 param; AdamW on the fp32 master with the state's exp_avg, exp_avg_sq, step;
    then weights = the new master rounded to bf16."""
    with torch.no_grad():
        model.load_state_dict({n: _f32(e["param"], "bf16") for n, e in full.items()}, strict=True)
    model.zero_grad(set_to_none=True)
    loss = loss_of(model, ids)
    loss.backward()
    grads = dict(model.named_parameters())
    masters = {n: torch.nn.Parameter(_f32(e["master"], "f32")) for n, e in full.items()}
    opt = torch.optim.AdamW(list(masters.values()), lr=LR, betas=BETAS, eps=EPS, weight_decay=WEIGHT_DECAY,
                            foreach=False, fused=False)
    for n, p in masters.items():
        e = full[n]
        p.grad = grads[n].grad.detach().clone()
        opt.state[p] = {"step": torch.tensor(float(np.asarray(e["step"]).reshape(-1)[0]), dtype=torch.float32),
                        "exp_avg": _f32(e["exp_avg"], "f32"), "exp_avg_sq": _f32(e["exp_avg_sq"], "f32")}
    opt.step()
    with torch.no_grad():
        model.load_state_dict({n: p.detach().to(torch.bfloat16).float() for n, p in masters.items()}, strict=True)
        after = loss_of(model, ids)
    return loss.detach(), after.detach()


def full_state(layout, states, to_np=np.asarray) -> Dict[str, Dict[str, np.ndarray]]:
    """{name: {sub-field: full array}} of a layout's shards, concatenating TP shards in tp_index
    order along the slice dim (one DP replica); a singleton step is taken from the first shard."""
    pieces: Dict[str, Dict[int, tuple]] = {}
    for rank, metas in layout.layout.items():
        for name, m in metas.items():
            tp = m.tp_meta
            key = 0 if tp is None else tp[1]
            pieces.setdefault(name, {}).setdefault(key, (tp, {s: to_np(a) for s, a in states[rank][name].items()}))
    out = {}
    for name, by_idx in pieces.items():
        tp0 = next(iter(by_idx.values()))[0]
        ent = {}
        for sub in next(iter(by_idx.values()))[1]:
            parts = [by_idx[i][1][sub] for i in sorted(by_idx)]
            if sub == "step":
                ent[sub] = np.asarray(parts[0]).reshape(-1)[:1]
            elif tp0 is None:
                ent[sub] = parts[0]
            else:
                ent[sub] = np.concatenate(parts, axis=tp0[0])
        out[name] = ent
    return out


def losses(spec, full) -> tuple:
    """(loss, loss after the step) as Python floats, with the restated model."""
    torch.manual_seed(0)  # the weights are all overwritten; this only fixes the throwaway init
    model = LlamaStage(llama_config(spec)).float()
    l0, l1 = train_step(model, full, tokens(spec))
    return float(l0), float(l1)

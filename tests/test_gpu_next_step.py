"""The next training step after a reshard: a small Llama's full training state is resharded on a
B200 (TP4 -> TP2 x PP2, slice order), the full tensors are reassembled from the target shards,
and one training step runs from each side: loss, backward, AdamW on the fp32 master with the
migrated m, v and step, and the loss after the step. Both losses must be bit-identical to the
ones computed from the un-migrated state. The step runs in fp32 on the host, so the comparison is
deterministic."""
import numpy as np
import pytest
import torch

from suika_b200 import migration as M
from suika_b200 import synthetic as S
from suika_b200.layouts import SPECS, ReshardConfig, scaled_spec

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SPEC = scaled_spec(SPECS["llama2-13b"], name="next-step", hidden=128, n_layers=2, n_heads=4, ffn=256, vocab=128)


def _full(layout, states, to_np):
    """name -> {sub: full array}, concatenating TP shards in tp_index order (one DP replica)."""
    pieces = {}
    for rank, metas in layout.items():
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
            if tp0 is None or sub == "step":
                ent[sub] = parts[0].reshape(-1)[:1] if sub == "step" else parts[0]
            else:
                ent[sub] = np.concatenate(parts, axis=tp0[0])
        out[name] = ent
    return out


def _t(a, kind):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.view(torch.bfloat16).float() if kind == "bf16" else t.float()


def _rms(x, w):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w


def _loss(P, tokens):
    s = SPEC
    B, T = tokens.shape
    x = P["wte.weight"][tokens]
    mask = torch.full((T, T), float("-inf")).triu(1)
    for i in range(s.n_layers):
        p = f"h.{i}."
        h = _rms(x, P[p + "input_layernorm.weight"])
        q, k, v = (h @ P[p + f"self_attn.{n}_proj.weight"].T for n in ("q", "k", "v"))
        q, k, v = (y.view(B, T, s.n_heads, s.hd).transpose(1, 2) for y in (q, k, v))
        a = torch.softmax(q @ k.transpose(-1, -2) / s.hd ** 0.5 + mask, -1) @ v
        x = x + a.transpose(1, 2).reshape(B, T, -1) @ P[p + "self_attn.o_proj.weight"].T
        h = _rms(x, P[p + "post_attention_layernorm.weight"])
        x = x + (torch.nn.functional.silu(h @ P[p + "mlp.gate_proj.weight"].T) * (h @ P[p + "mlp.up_proj.weight"].T)) @ P[p + "mlp.down_proj.weight"].T
    logits = _rms(x, P["norm.weight"]) @ P["lm_head.weight"].T
    return torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, s.vocab), tokens[:, 1:].reshape(-1))


def _train_step(full, tokens, lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.1):
    """Loss, AdamW on the fp32 master (torch.optim.AdamW's update, written out), bf16 params from
    the new master, loss again."""
    P = {n: _t(e["param"], "bf16").requires_grad_(True) for n, e in full.items()}
    loss = _loss(P, tokens)
    loss.backward()
    new = {}
    for n, e in full.items():
        g = P[n].grad
        step = float(e["step"].reshape(-1)[0]) + 1
        master, m, v = (_t(e[k], "f32") for k in ("master", "exp_avg", "exp_avg_sq"))
        master = master * (1 - lr * wd)
        m = b1 * m + (1 - b1) * g
        v = b2 * v + (1 - b2) * g * g
        master = master - lr * (m / (1 - b1 ** step)) / ((v / (1 - b2 ** step)).sqrt() + eps)
        new[n] = master.to(torch.bfloat16).float()
    with torch.no_grad():
        after = _loss(new, tokens)
    return loss.detach(), after


def test_next_step_loss_identical_after_reshard():
    cfg = ReshardConfig("next-step", SPEC, [[list(range(4))]], [[[0, 1]], [[2, 3]]])  # TP4 -> TP2 x PP2
    spl, tpl = cfg.layouts()
    states = S.host_states(spl, S.SUBFIELDS, seed=7, distinct_steps=False)
    kinds = dict(S.SUBFIELDS)
    dev_states = {r: {n: {s: S.to_torch(a, kinds[s], DEV if kinds[s] != "meta" else None) for s, a in e.items()}
                      for n, e in st.items()} for r, st in states.items()}
    out = M.reshard_local(spl, tpl, dev_states, S.expected_sub_fields(), DEV, order="semantic", minimum_est_peers=1)
    torch.cuda.synchronize()

    def dev_np(t):
        t = t.detach().cpu().contiguous()
        return t.view(torch.uint16).numpy() if t.dtype == torch.bfloat16 else t.numpy()

    before = _full(spl.layout, states, np.asarray)
    after = _full(tpl.layout, out, dev_np)
    assert set(before) == set(after)
    for n in before:
        for sub in before[n]:
            assert np.array_equal(before[n][sub].reshape(-1).view(np.uint8), after[n][sub].reshape(-1).view(np.uint8)), (n, sub)
    tokens = torch.randint(0, SPEC.vocab, (2, 16), generator=torch.Generator().manual_seed(0))
    l0_src, l1_src = _train_step(before, tokens)
    l0_dst, l1_dst = _train_step(after, tokens)
    assert torch.equal(l0_src, l0_dst) and torch.equal(l1_src, l1_dst), (l0_src, l0_dst, l1_src, l1_dst)
    assert l1_src < l0_src  # the step trains

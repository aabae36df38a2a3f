"""Seeded synthetic training state for reshard parity tests and benchmarks.

State per tensor (the benchmark's sub-fields, in this order):
    param       bf16   = round-to-nearest-even of master
    step        fp32   singleton (Adam step; a "meta" sub-field, migration.py:702-709)
    master      fp32   weights and biases ~ N(0, 0.02); norm weights 1.0, norm biases 0.0
    exp_avg     fp32   ~ N(0, 1e-3)
    exp_avg_sq  fp32   ~ |N(0, 1e-6)|

Two generators with the same distributions:
  * host (numpy PCG64): the FULL tensor of every (name, sub-field) is drawn from a seed derived
    from (seed, name, sub-field), then sliced into shards with the reference's contiguous chunk
    (Suika/tensor_parallel.py:200-204,378-381). Platform independent, so golden digests made on
    one machine hold on another; used for parity cases small enough for a CPU.
  * device (torch on CUDA): every SOURCE shard is drawn on the GPU from a seed derived from
    (seed, name, sub-field, tp index, tp degree), so replicas are byte-identical; used for the
    full-size benchmark state, which is checked by size-independent properties.
bf16 arrays are held on the host as uint16 bit patterns.
"""
from __future__ import annotations

import zlib
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

SUBFIELDS: List[Tuple[str, str]] = [("param", "bf16"), ("step", "meta"), ("master", "f32"),
                                   ("exp_avg", "f32"), ("exp_avg_sq", "f32")]
NP_DTYPE = {"bf16": np.uint16, "f32": np.float32, "meta": np.float32}
TORCH_DTYPE = {"bf16": torch.bfloat16, "f32": torch.float32, "meta": torch.float32}


def is_norm(name: str) -> bool:
    module = name.rsplit(".", 1)[0].rsplit(".", 1)[-1]
    return "norm" in module or module.startswith("ln_")


def _seed(seed: int, *parts) -> np.random.SeedSequence:
    return np.random.SeedSequence([seed] + [zlib.crc32(str(p).encode()) for p in parts])


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((b + (((b >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def step_value(name: str, distinct_steps: bool) -> float:
    return float(1 + zlib.crc32(name.encode()) % 97) if distinct_steps else 1.0


def host_full(name: str, sub: str, shape: Sequence[int], seed: int = 0, distinct_steps: bool = False) -> np.ndarray:
    """The full (unsharded) host tensor of one (name, sub-field)."""
    shape = tuple(int(s) for s in shape)
    if sub == "step":
        return np.array(step_value(name, distinct_steps), dtype=np.float32)
    rng = np.random.Generator(np.random.PCG64(_seed(seed, name, "master" if sub == "param" else sub)))
    if sub in ("param", "master"):
        if is_norm(name):
            m = np.full(shape, 0.0 if name.endswith(".bias") else 1.0, dtype=np.float32)
        else:
            m = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        return bf16_bits(m) if sub == "param" else m
    if sub == "exp_avg":
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(1e-3)).astype(np.float32)
    if sub == "exp_avg_sq":
        return np.abs(rng.standard_normal(shape, dtype=np.float32) * np.float32(1e-6)).astype(np.float32)
    raise KeyError(sub)


def _contig(a: np.ndarray) -> np.ndarray:
    """C-contiguous copy-if-needed that keeps 0-dim arrays 0-dim (np.ascontiguousarray does not)."""
    return a if a.flags.c_contiguous else np.ascontiguousarray(a)


def host_shard(full: np.ndarray, tp_meta, rule=None) -> np.ndarray:
    """The shard of a full tensor: the reference's contiguous chunk, or the spans of a slice rule."""
    if tp_meta is None or full.ndim == 0:
        return _contig(full)
    d, i, g = tp_meta
    if not rule:
        return np.ascontiguousarray(np.split(full, g, axis=d)[i])
    from .layouts import shard_spans
    parts = [np.take(full, np.arange(lo, hi), axis=d) for lo, hi in shard_spans(full.shape, tp_meta, rule)]
    return np.ascontiguousarray(np.concatenate(parts, axis=d))


def host_states(layout, subfields=SUBFIELDS, seed: int = 0, distinct_steps: bool = False,
                ranks: Optional[Sequence[int]] = None, threads: int = 0) -> Dict[int, Dict[str, Dict[str, np.ndarray]]]:
    """rank -> name -> sub-field -> host array for every tensor of a ParamLayout (only `ranks` if
    given). Full tensors are drawn on a thread pool (`threads`, default: all cores); `param` is
    rounded from the `master` draw when both are asked for (the same values host_full gives)."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    wanted: Dict[Tuple[str, str], Tuple[int, ...]] = {}
    subs = [sub for sub, _ in subfields]
    kind_of = dict(subfields)
    for rank, metas in layout.layout.items():
        if ranks is not None and rank not in ranks:
            continue
        for name, m in metas.items():
            for sub in subs:
                wanted.setdefault((name, sub), tuple(int(x) for x in m.shape))

    def draw(key):
        name, sub = key
        if sub == "param" and (name, "master") in wanted:
            return None  # rounded from the master draw below
        v = host_full(name, sub, wanted[key], seed, distinct_steps)
        if kind_of[sub] == "bf16" and sub != "param":
            v = bf16_bits(v)  # bf16 optimizer state (the reference's worker keeps m and v in bf16)
        return v

    keys = list(wanted)
    n = threads or (os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=max(1, n)) as ex:
        cache = dict(zip(keys, ex.map(draw, keys)))
    for (name, sub), v in list(cache.items()):
        if v is None:
            cache[(name, sub)] = bf16_bits(cache[(name, "master")])
    out: Dict[int, Dict[str, Dict[str, np.ndarray]]] = {}
    for rank, metas in layout.layout.items():
        if ranks is not None and rank not in ranks:
            continue
        rs = {}
        for name, m in metas.items():
            ent = {}
            for sub in subs:
                full = cache[(name, sub)]
                ent[sub] = full if sub == "step" else host_shard(full, m.tp_meta, getattr(m, "tp_rule", None))
            rs[name] = ent
        out[rank] = rs
    return out


def to_torch(arr: np.ndarray, kind: str, device=None) -> torch.Tensor:
    t = torch.from_numpy(_contig(np.asarray(arr)))
    if kind == "bf16":
        t = t.view(torch.bfloat16)
    return t.to(device) if device is not None else t


def expected_sub_fields(subfields=SUBFIELDS):
    """other_context_dict["expected_sub_fields"] as merge_model_and_optimizer_state_dict builds it
    (migration.py:702-709): ("name", "normal") or ("name", TensorMeta of the singleton)."""
    from .migration import TensorMeta
    out = []
    for sub, kind in subfields:
        if kind == "meta":
            out.append((sub, TensorMeta(tensor=torch.tensor(1.0, dtype=TORCH_DTYPE[kind]))))
        else:
            out.append((sub, "normal"))
    return out


# ---------------------------------------------------------------------------------------------
# Device generator for full-size state.
# ---------------------------------------------------------------------------------------------
def _torch_seed(seed: int, *parts) -> int:
    return int(_seed(seed, *parts).generate_state(1, dtype=np.uint64)[0] & 0x7FFFFFFFFFFFFFFF)


def fill_device_shard(out: torch.Tensor, name: str, sub: str, tp_meta, seed: int = 0, rule=None, full_shape=None) -> None:
    """Fill one source shard on its device (same distributions as the host generator). Shards of
    a slice rule are filled span by span, seeded by the span, so replicated units agree."""
    if sub == "step":
        out.fill_(1.0)
        return
    if rule and tp_meta is not None:
        from .layouts import shard_spans
        d, at = tp_meta[0], 0
        for lo, hi in shard_spans(full_shape, tp_meta, rule):
            _fill(out.narrow(d, at, hi - lo), name, sub, seed, ("span", lo, hi))
            at += hi - lo
        return
    idx, deg = (0, 1) if tp_meta is None else (tp_meta[1], tp_meta[2])
    _fill(out, name, sub, seed, (idx, deg))


def _fill(out: torch.Tensor, name: str, sub: str, seed: int, key) -> None:
    g = torch.Generator(device=out.device)
    g.manual_seed(_torch_seed(seed, name, "master" if sub == "param" else sub, *key))
    if sub in ("param", "master"):
        if is_norm(name):
            out.fill_(0.0 if name.endswith(".bias") else 1.0)
            return
        tmp = torch.empty(out.shape, dtype=torch.float32, device=out.device)
        tmp.normal_(0.0, 0.02, generator=g)
        out.copy_(tmp)  # bf16 param: round-to-nearest-even of the fp32 master draw
        return
    if not out.is_contiguous():  # a span of a rule shard
        tmp = torch.empty(out.shape, dtype=out.dtype, device=out.device)
        _fill(tmp, name, sub, seed, key)
        out.copy_(tmp)
        return
    if sub == "exp_avg":
        out.normal_(0.0, 1e-3, generator=g)
        return
    if sub == "exp_avg_sq":
        out.normal_(0.0, 1e-6, generator=g).abs_()
        return
    raise KeyError(sub)


class DeviceState:
    """A rank's source state in ONE device arena per sub-field dtype (views per tensor), the
    layout a B200-native engine keeps its state in; one CUDA IPC export covers a whole arena."""

    def __init__(self, metas: Dict[str, object], device, subfields=SUBFIELDS, seed: int = 0, fill: bool = True):
        self.device = torch.device(device)
        self.arenas: Dict[str, torch.Tensor] = {}
        self.state: Dict[str, Dict[str, torch.Tensor]] = {}
        sizes: Dict[str, int] = {}
        offs: Dict[Tuple[str, str], int] = {}
        for name, m in metas.items():
            shape = _actual_shape(m)
            numel = int(np.prod(shape)) if len(shape) else 1
            for sub, kind in subfields:
                if kind == "meta":
                    continue
                align = 256 // TORCH_DTYPE[kind].itemsize  # 256-byte aligned views
                o = (sizes.get(kind, 0) + align - 1) // align * align
                offs[(name, sub)] = o
                sizes[kind] = o + numel
        for kind, n in sizes.items():
            self.arenas[kind] = torch.empty(max(n, 1), dtype=TORCH_DTYPE[kind], device=self.device)
        kind_of = dict(subfields)
        for name, m in metas.items():
            shape = _actual_shape(m)
            numel = int(np.prod(shape)) if len(shape) else 1
            ent = {}
            for sub, kind in subfields:
                if kind == "meta":
                    ent[sub] = torch.tensor(1.0, dtype=TORCH_DTYPE[kind])  # AdamW keeps step on the host
                    continue
                o = offs[(name, sub)]
                ent[sub] = self.arenas[kind][o:o + numel].view(shape)
                if fill:
                    fill_device_shard(ent[sub], name, sub, m.tp_meta, seed, getattr(m, "tp_rule", None), m.shape)
            self.state[name] = ent
        self.kind_of = kind_of

    def nbytes(self) -> int:
        return sum(a.numel() * a.element_size() for a in self.arenas.values())


def _actual_shape(m) -> Tuple[int, ...]:
    from .layouts import actual_shape
    return actual_shape(m)

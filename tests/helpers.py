"""Shared test helpers: golden fixtures, digests, and a numpy executor of a rank's copy program
(used to check the C planner's segments on a CPU; the product has no CPU executor)."""
from __future__ import annotations

import hashlib
import json
import os
from typing import Dict

import numpy as np

from suika_b200 import synthetic as S

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SUBS = S.SUBFIELDS
SUB_META = [(s, kind == "meta") for s, kind in SUBS]
SUB_ITEMSIZE = {s: np.dtype(S.NP_DTYPE[kind]).itemsize for s, kind in SUBS}


def load_golden(case: str) -> dict:
    with open(os.path.join(GOLDEN_DIR, f"{case}.json")) as f:
        return json.load(f)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).reshape(-1).view(np.uint8).tobytes()).hexdigest()


_STATE_CACHE = {}


def golden_states(case_cfg, seed=0):
    """Source states (numpy) of a golden case, as make_golden.py feeds the reference (cached)."""
    key = (case_cfg.name, seed)
    if key not in _STATE_CACHE:
        spl, _ = case_cfg.layouts()
        _STATE_CACHE.clear()  # keep at most one case resident
        _STATE_CACHE[key] = S.host_states(spl, SUBS, seed=seed, distinct_steps=True)
    return _STATE_CACHE[key]


def schedule_as_lists(ops):
    return [[o.name, o.src, o.dst, list(o.src_tp) if o.src_tp else None, list(o.dst_tp) if o.dst_tp else None] for o in ops]


def copy_rect(dst: np.ndarray, do: int, dpitch: int, src: np.ndarray, so: int, spitch: int, rows: int, rb: int) -> None:
    """rows x rb bytes from src[so + r * spitch] to dst[do + r * dpitch] (uint8 arrays), in one numpy
    strided copy; both extents are checked first."""
    if rows <= 0 or rb <= 0:
        return
    span_s, span_d = (rows - 1) * spitch + rb, (rows - 1) * dpitch + rb
    assert so + span_s <= src.size and do + span_d <= dst.size, "rectangle leaves its buffer"
    s = np.lib.stride_tricks.as_strided(src[so:so + span_s], shape=(rows, rb), strides=(spitch, 1))
    d = np.lib.stride_tricks.as_strided(dst[do:do + span_d], shape=(rows, rb), strides=(dpitch, 1), writeable=True)
    d[...] = s


def emulate_program(prog, names, states, rank, subs=None) -> Dict[str, Dict[str, np.ndarray]]:
    """Apply a Program's slots and segments with numpy; returns {name: {sub: array}}. subs: the
    (name, kind) sub-field list the program was built for (default: the benchmark's)."""
    SUBS = subs or globals()["SUBS"]
    src_buf = []
    for ss in prog.src_slots:
        name = names[ss["name_id"]]
        sub = SUBS[ss["subfield"]][0]
        a = np.ascontiguousarray(states[int(ss["src_rank"])][name][sub])
        b = a.reshape(-1).view(np.uint8)
        assert b.nbytes == ss["nbytes"], (name, sub, b.nbytes, ss["nbytes"])
        src_buf.append(b)
    dst_buf = [np.zeros(int(ds["nbytes"]), dtype=np.uint8) for ds in prog.dst_slots]
    for sg in prog.segments:
        copy_rect(dst_buf[sg["dst_slot"]], int(sg["dst_offset"]), int(sg["dst_pitch"]),
                  src_buf[sg["src_slot"]], int(sg["src_offset"]), int(sg["src_pitch"]), int(sg["rows"]), int(sg["row_bytes"]))
    out: Dict[str, Dict[str, np.ndarray]] = {}
    for ds, buf in zip(prog.dst_slots, dst_buf):
        name = names[ds["name_id"]]
        sub, kind = SUBS[ds["subfield"]]
        shape = tuple(int(x) for x in ds["shape"][: ds["ndim"]])
        out.setdefault(name, {})[sub] = buf.view(S.NP_DTYPE[kind]).reshape(shape)
    for ms in prog.meta_slots:
        name = names[ms["name_id"]]
        sub = SUBS[ms["subfield"]][0]
        v = np.array(states[int(ms["src_rank"])][name][sub], copy=True)
        out.setdefault(name, {})[sub] = v if ms["first_is_self"] else v.reshape(1)
    # sub-fields in expected order
    return {n: {s: ent[s] for s, _ in SUBS if s in ent} for n, ent in out.items()}


class Memory:
    """Flat emulated address space: named buffers at fixed, non-overlapping base addresses."""

    def __init__(self):
        self.bufs = []  # (base, bytearray-like numpy uint8)
        self.next = 1 << 20

    def add(self, arr: np.ndarray) -> int:
        base = self.next
        self.bufs.append((base, arr))
        self.next += (arr.nbytes + (1 << 12)) // 256 * 256 + 256
        return base

    def view(self, addr, n):
        for base, a in self.bufs:
            if base <= addr and addr + n <= base + a.nbytes:
                return a[addr - base: addr - base + n]
        raise AssertionError(f"address {addr:#x}+{n} outside every buffer")

    def apply(self, descs: np.ndarray) -> None:
        """Run COPY_DESC entries against this memory."""
        for d in descs:
            rows, rb = int(d["rows"]), int(d["row_bytes"])
            if rows <= 0 or rb <= 0:
                continue
            sp, dp = int(d["src_pitch"]), int(d["dst_pitch"])
            s = self.view(int(d["src_dev"]), (rows - 1) * sp + rb)
            t = self.view(int(d["dst_dev"]), (rows - 1) * dp + rb)
            copy_rect(t, 0, dp, s, 0, sp, rows, rb)


def rank_device(rank: int, world: int):
    """(device, process-group backend) of one rank of a multi-process GPU test. With a GPU per rank:
    cuda:rank and NCCL. With fewer GPUs than ranks every rank shares cuda:0 and the process group
    is gloo (NCCL refuses two ranks on one device). CUDA IPC between processes works on one device
    too, and no kernel of this package waits on another rank, so the ranks' kernels may run in any
    order on the shared GPU."""
    import torch
    if torch.cuda.device_count() >= world:
        return torch.device("cuda", rank), "nccl"
    return torch.device("cuda", 0), "gloo"

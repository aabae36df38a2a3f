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


def emulate_program(prog, names, states, rank) -> Dict[str, Dict[str, np.ndarray]]:
    """Apply a Program's slots and segments with numpy; returns {name: {sub: array}}."""
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
        s, d = src_buf[sg["src_slot"]], dst_buf[sg["dst_slot"]]
        rows, rb = int(sg["rows"]), int(sg["row_bytes"])
        for r in range(rows):
            so, do = int(sg["src_offset"]) + r * int(sg["src_pitch"]), int(sg["dst_offset"]) + r * int(sg["dst_pitch"])
            d[do:do + rb] = s[so:so + rb]
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

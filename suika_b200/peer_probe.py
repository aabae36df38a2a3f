"""Peer-bandwidth probe between GPU 0 and GPU 1 for the reshard copy kernel.

    python -m suika_b200.peer_probe [--gib 2]

For each launch shape (SUIKA_RS_VARIANT) and each piece shape (one contiguous run; 1280-byte rows
at a 2560-byte pitch, like a TP8 -> TP4 row-parallel piece) it times, per direction:
  pull:  the kernel on GPU a reads GPU b's memory;    push: it writes GPU b's memory;
  1-way: one GPU copies;  2-way: both copy at once in opposite directions;
  +local: the same table also holds an equal local copy (remote entries are interleaved with it).
These are the patterns a reshard is made of; they decide direction and phasing (see DESIGN).
"""
from __future__ import annotations

import argparse
import ctypes
import glob
import os

import numpy as np
import torch

from . import _lib as L
from . import migration as M


def _enable_peer_access() -> None:
    libs = glob.glob(os.path.join(os.path.dirname(torch.__file__), "..", "nvidia", "cuda_runtime", "lib", "libcudart.so*"))
    if not libs:
        raise RuntimeError("libcudart not found next to torch")
    rt = ctypes.CDLL(libs[0])
    for a, b in ((0, 1), (1, 0)):
        rt.cudaSetDevice(a)
        rt.cudaDeviceEnablePeerAccess(b, 0)  # an "already enabled" return is fine


def _row(src, dst, n, strided, remote):
    if strided:
        return (src, dst, n // 2560, 1280, 2560, 2560, remote)
    return (src, dst, 1, n, n, n, remote)


def _time(per_dev, reps=5):
    preps = {}
    for dev, ents in per_dev.items():
        with torch.cuda.device(dev):
            t = np.array([_row(*e) for e in ents], dtype=L.COPY_DESC_DTYPE)
            preps[dev] = M.PreparedCopies(t, torch.device("cuda", dev))
    for dev, p in preps.items():
        with torch.cuda.device(dev):
            p.launch()
    for d in (0, 1):
        torch.cuda.synchronize(d)
    ev = {}
    for dev, p in preps.items():
        with torch.cuda.device(dev):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(reps):
                p.launch()
            b.record()
            ev[dev] = (a, b)
    for d in (0, 1):
        torch.cuda.synchronize(d)
    for p in preps.values():
        p.check()
    return max(a.elapsed_time(b) for a, b in ev.values()) / reps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gib", type=float, default=2.0)
    ap.add_argument("--variants", default="2,6")
    ap.add_argument("--one", action="store_true",
                    help="one pull launch then one push launch on GPU 0 against GPU 1 (for a profiler capture)")
    args = ap.parse_args()
    if torch.cuda.device_count() < 2:
        raise SystemExit("needs two GPUs")
    _enable_peer_access()
    n = int(args.gib * (1 << 30))
    if args.one:
        d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
        a0, b0 = torch.ones(n, dtype=torch.uint8, device=d0), torch.empty(n, dtype=torch.uint8, device=d0)
        a1 = torch.full((n,), 2, dtype=torch.uint8, device=d1)
        b1 = torch.empty(n, dtype=torch.uint8, device=d1)
        for name, (s_, d_) in (("pull", (a1, b0)), ("push", (a0, b1))):
            p = M.PreparedCopies(np.array([_row(s_.data_ptr(), d_.data_ptr(), n, False, 1)], dtype=L.COPY_DESC_DTYPE), d0)
            p.launch()
            p.check()
            assert torch.equal(d_[:1024].cpu(), s_[:1024].cpu())
            print(f"{name}: {n} bytes copied", flush=True)
        return
    b = {d: [torch.empty(n, dtype=torch.uint8, device=torch.device("cuda", d)) for _ in range(4)] for d in (0, 1)}
    p = {d: [t.data_ptr() for t in b[d]] for d in (0, 1)}
    for var in args.variants.split(","):
        os.environ["SUIKA_RS_VARIANT"] = var
        for st in (False, True):
            moved = n // 2 if st else n
            pats = {
                "pull 1-way": {0: [(p[1][0], p[0][1], n, st, 1)]},
                "pull 2-way": {0: [(p[1][0], p[0][1], n, st, 1)], 1: [(p[0][0], p[1][1], n, st, 1)]},
                "push 1-way": {0: [(p[0][0], p[1][1], n, st, 1)]},
                "push 2-way": {0: [(p[0][0], p[1][1], n, st, 1)], 1: [(p[1][0], p[0][1], n, st, 1)]},
                "pull 2-way +local": {0: [(p[1][0], p[0][1], n, st, 1), (p[0][2], p[0][3], n, st, 0)],
                                      1: [(p[0][0], p[1][1], n, st, 1), (p[1][2], p[1][3], n, st, 0)]},
                "push 2-way +local": {0: [(p[0][0], p[1][1], n, st, 1), (p[0][2], p[0][3], n, st, 0)],
                                      1: [(p[1][0], p[0][1], n, st, 1), (p[1][2], p[1][3], n, st, 0)]},
            }
            for name, cfg in pats.items():
                ms = _time(cfg)
                print(f"variant {var} {'strided' if st else 'contig '} {name:18s}: {ms:7.3f} ms  "
                      f"{moved / ms / 1e6:6.0f} GB/s per direction", flush=True)


if __name__ == "__main__":
    main()

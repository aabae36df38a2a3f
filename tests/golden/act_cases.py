"""Activation-exchange cases shared by the golden generator (make_act_golden.py) and the tests.

Each case is one hand-over between adjacent pipeline stages: the sending stage's mesh (DP groups of
TP ranks) and local batch sizes, the receiving stage's, the local activation shape (the batch dim
is filled with each rank's local batch), the batch and slice dims, and the dtype. Sizes are small:
the bytes are seeded and per rank, so every block's origin is checked.
"""
from __future__ import annotations

from typing import Dict

import numpy as np

ACT_CASES = {
    # DP2 x TP2 -> TP4: each receiver takes a chunk from both source groups, then all-gathers
    "dp2tp2_to_tp4": dict(mesh_src=[[0, 1], [2, 3]], bszs_src=[2, 2], mesh_dst=[[4, 5, 6, 7]], bszs_dst=[4],
                          shape=[-1, 5, 16], batch_dim=0, slice_dim=-1, dtype="float32"),
    "tp4_to_dp2tp2": dict(mesh_src=[[0, 1, 2, 3]], bszs_src=[4], mesh_dst=[[4, 5], [6, 7]], bszs_dst=[2, 2],
                          shape=[-1, 5, 16], batch_dim=0, slice_dim=-1, dtype="float32"),
    # heterogeneous TP inside the sending stage (TP2 next to TP1), bf16
    "hetero_tp": dict(mesh_src=[[0, 1], [2]], bszs_src=[3, 1], mesh_dst=[[3, 4, 5, 6]], bszs_dst=[4],
                      shape=[-1, 6, 32], batch_dim=0, slice_dim=-1, dtype="bfloat16"),
    # uneven local batches that straddle group boundaries
    "uneven_batches": dict(mesh_src=[[0], [1], [2]], bszs_src=[1, 2, 3], mesh_dst=[[3, 4], [5]], bszs_dst=[4, 2],
                           shape=[-1, 3, 8], batch_dim=0, slice_dim=-1, dtype="float32"),
    # sequence-first activations ([seq, batch, hidden]): the batch dim is not the outermost
    "seq_first": dict(mesh_src=[[0, 1]], bszs_src=[4], mesh_dst=[[2], [3]], bszs_dst=[2, 2],
                      shape=[4, -1, 16], batch_dim=1, slice_dim=-1, dtype="float32"),
    # slice dim outside the batch dim
    "slice_outer": dict(mesh_src=[[0], [1]], bszs_src=[2, 2], mesh_dst=[[2, 3, 4, 5]], bszs_dst=[4],
                        shape=[16, -1, 3], batch_dim=1, slice_dim=0, dtype="float32"),
    # the receiving stage holds rows no sender has: they keep the receiver's zeros
    "uncovered_rows": dict(mesh_src=[[0]], bszs_src=[2], mesh_dst=[[1, 2]], bszs_dst=[3],
                           shape=[-1, 4, 8], batch_dim=0, slice_dim=-1, dtype="float32"),
    # a source DP group with an empty local batch
    "empty_group": dict(mesh_src=[[0], [1]], bszs_src=[0, 4], mesh_dst=[[2, 3]], bszs_dst=[4],
                        shape=[-1, 2, 8], batch_dim=0, slice_dim=-1, dtype="float32"),
    # TP8 -> DP4 x TP2 in bf16 (the shape of a 13B stage boundary, reduced)
    "tp8_to_dp4tp2": dict(mesh_src=[[0, 1, 2, 3, 4, 5, 6, 7]], bszs_src=[4], mesh_dst=[[8, 9], [10, 11], [12, 13], [14, 15]],
                          bszs_dst=[1, 1, 1, 1], shape=[-1, 4, 64], batch_dim=0, slice_dim=-1, dtype="bfloat16"),
    # 4-d activation, batch dim 0, slice dim 2 (inner dims after the slice dim)
    "four_dims": dict(mesh_src=[[0, 1]], bszs_src=[2], mesh_dst=[[2, 3, 4, 5]], bszs_dst=[2],
                      shape=[-1, 3, 8, 2], batch_dim=0, slice_dim=2, dtype="float32"),
    # heterogeneous TP inside the receiving stage
    "hetero_dst": dict(mesh_src=[[0, 1, 2, 3]], bszs_src=[4], mesh_dst=[[4, 5], [6]], bszs_dst=[2, 2],
                       shape=[-1, 3, 16], batch_dim=0, slice_dim=-1, dtype="float32"),
    # one sender to a TP8 group (every receiver takes its chunk, then the all-gather)
    "tp1_to_tp8": dict(mesh_src=[[0]], bszs_src=[2], mesh_dst=[[1, 2, 3, 4, 5, 6, 7, 8]], bszs_dst=[2],
                       shape=[-1, 2, 64], batch_dim=0, slice_dim=-1, dtype="bfloat16"),
    # sequence-first with TP on both sides and DP on the sending side
    "seq_first_tp_both": dict(mesh_src=[[0, 1], [2, 3]], bszs_src=[2, 2], mesh_dst=[[4, 5, 6, 7]], bszs_dst=[4],
                              shape=[3, -1, 16], batch_dim=1, slice_dim=2, dtype="float32"),
}


def local_shape(case: dict, bsz: int):
    shape = list(case["shape"])
    shape[case["batch_dim"] % len(shape)] = bsz
    return shape


def rank_bsz(mesh, bszs) -> Dict[int, int]:
    return {r: int(b) for group, b in zip(mesh, bszs) for r in group}


def source_arrays(case: dict, seed: int = 0) -> Dict[int, np.ndarray]:
    """Each sender's activation: seeded per rank. bf16 as uint16 bit patterns (the upper halves of
    fp32 normals, so every pattern is a finite value)."""
    out = {}
    for r, b in rank_bsz(case["mesh_src"], case["bszs_src"]).items():
        rng = np.random.default_rng([seed, r])
        x = rng.standard_normal(local_shape(case, b)).astype(np.float32)
        out[r] = (x.view(np.uint32) >> 16).astype(np.uint16) if case["dtype"] == "bfloat16" else x
    return out


def zero_targets(case: dict) -> Dict[int, np.ndarray]:
    dt = np.uint16 if case["dtype"] == "bfloat16" else np.float32
    return {r: np.zeros(local_shape(case, b), dtype=dt) for r, b in rank_bsz(case["mesh_dst"], case["bszs_dst"]).items()}

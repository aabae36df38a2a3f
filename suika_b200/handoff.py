"""Old-process -> new-process hand-off of migration state without per-tensor round trips.

Drop-in for Suika's interactive_IPC_state_dict_send / interactive_IPC_state_dict_recv
(Suika/utils.py:325-406), which migration_save / migration_load use (Suika/migration.py:1424-1439,
1469-1475, 1618-1623, 1677-1682). The reference sends one CUDA tensor per queue message, waits for
an ack per tensor, and the receiver clones every tensor (a full HBM copy, and one Python round trip
per tensor). Here:

  * the template and ALL CUDA tensors travel in two queue messages. The sender first packs the
    tensors into one arena (one launch of the reshard copy kernel), so the receiver opens one CUDA
    IPC handle instead of one per allocation (about a millisecond each); without room for the
    arena the tensors are shared one storage each;
  * a received *source* state (the grow path: "source_state_dict", migration.py:1427-1432) is not
    cloned: the new process reads the old process's memory in place, and the reshard's own kernel
    reads it locally (direction "push"). The dict is a ReleasableDict; suika_b200's
    schedule_and_execute_param_transfer calls its release() when the reshard is done, which sends
    the single ack that lets the old process free its memory;
  * any other state (the shrink path's "target_state_dict", which the model keeps after the old
    process exits) is copied on receipt, as the reference does, and acknowledged at once: one copy
    of the whole arena, the received tensors being views of it.

Both processes must use these two functions (rebind them in Suika.migration).
"""
from __future__ import annotations

import gc
from typing import Any, Dict, List, Tuple

import torch


class TensorPlaceholder:
    """Marks where a CUDA tensor goes in the template (the role of Suika/utils.py:266)."""


class ReleasableDict(dict):
    """A received source state whose tensors live in the sending process. release() tells the
    sender that they are no longer read (once); until then the sender keeps them alive."""

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self._ack_queue = None

    def release(self) -> None:
        q, self._ack_queue = self._ack_queue, None
        if q is not None:
            q.put(None, block=True)


def _template(value):
    if isinstance(value, dict):
        return {k: _template(v) for k, v in value.items()}
    if isinstance(value, list):
        return [_template(v) for v in value]
    if isinstance(value, torch.Tensor) and value.device.type == "cuda":
        return TensorPlaceholder()
    return value


def _cuda_tensors(value, out: List[torch.Tensor]) -> None:
    """CUDA tensors in the template's traversal order."""
    if isinstance(value, dict):
        for v in value.values():
            _cuda_tensors(v, out)
    elif isinstance(value, list):
        for v in value:
            _cuda_tensors(v, out)
    elif isinstance(value, torch.Tensor) and value.device.type == "cuda":
        out.append(value)


def _free(tensors: List[torch.Tensor]) -> None:
    """forcefully_free_tensor (Suika/utils.py:255-260) on every storage once."""
    seen = set()
    for t in tensors:
        st = t.untyped_storage()
        key = st.data_ptr()
        if key in seen:
            continue
        seen.add(key)
        if st.resizable():
            st.resize_(0)
        else:
            t.data = torch.empty(0, device="meta")


def _cuda_gc() -> None:
    """Suika/utils.py:248-253."""
    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
        torch.cuda.synchronize()
        torch.cuda.ipc_collect()


def _pack(tensors: List[torch.Tensor]):
    """Copy the tensors of one device into one arena with a single launch of the reshard copy
    kernel; returns (arena, [(offset, shape, dtype name)]) or None when the arena does not fit.
    One allocation is one CUDA IPC handle to open in the receiver instead of one per tensor."""
    import numpy as np
    from . import _lib as L
    from .migration import launch_copies
    dev = tensors[0].device
    if any(t.device != dev for t in tensors):
        return None
    ts = [t if t.is_contiguous() else t.contiguous() for t in tensors]
    nb = [t.numel() * t.element_size() for t in ts]
    off, o = [], 0
    for n in nb:
        off.append(o)
        o += (n + 255) // 256 * 256
    try:
        arena = torch.empty(max(o, 1), dtype=torch.uint8, device=dev)
    except torch.OutOfMemoryError:
        return None
    table = np.array([(t.data_ptr(), arena.data_ptr() + a, 1, n, n, n, 0) for t, a, n in zip(ts, off, nb) if n],
                     dtype=L.COPY_DESC_DTYPE)
    with torch.cuda.device(dev):
        launch_copies(table, dev)
        torch.cuda.synchronize(dev)
    meta = [(a, tuple(t.shape), str(t.dtype).replace("torch.", "")) for t, a in zip(ts, off)]
    return arena, meta


def interactive_IPC_state_dict_send(IPC_queues: Tuple[Any, Any], state_dict: Dict, gc_size_MB: int = 1024,
                                    pack: bool = True) -> None:
    """Send a state dict to the new process: the template, then every CUDA tensor in one message
    (packed into one arena when it fits), then wait for the single ack and free the memory.
    gc_size_MB is accepted for compatibility."""
    IPC_queues[0].put(_template(state_dict))
    tensors: List[torch.Tensor] = []
    _cuda_tensors(state_dict, tensors)
    if not tensors:
        return
    packed = _pack(tensors) if pack else None
    if packed is not None:
        arena, meta = packed
        _free(tensors)  # the arena holds every byte now; the old tensors are not read again
        del tensors
        IPC_queues[0].put(("packed", arena, meta), block=True)
        IPC_queues[1].get(block=True)
        _free([arena])
        del arena
    else:
        torch.cuda.synchronize()  # the receiver may read the tensors as soon as they arrive
        IPC_queues[0].put(("tensors", tensors), block=True)
        IPC_queues[1].get(block=True)  # receiver cloned them, or finished reading them in place
        _free(tensors)
        del tensors
    _cuda_gc()


def _unpack(msg) -> List[torch.Tensor]:
    if msg[0] == "tensors":
        return msg[1]
    _, arena, meta = msg
    out = []
    for off, shape, dt in meta:
        dtype = getattr(torch, dt)
        n = dtype.itemsize
        for d in shape:
            n *= d
        out.append(arena[off:off + n].view(dtype).view(shape))
    return out


def _fill(value, tensors, pos, clone: bool):
    if isinstance(value, dict):
        for k in list(value.keys()):
            value[k], pos = _fill(value[k], tensors, pos, clone)
        return value, pos
    if isinstance(value, list):
        for i in range(len(value)):
            value[i], pos = _fill(value[i], tensors, pos, clone)
        return value, pos
    if isinstance(value, TensorPlaceholder):
        t = tensors[pos]
        return (t.clone() if clone else t), pos + 1
    return value, pos


def interactive_IPC_state_dict_recv(IPC_queues: Tuple[Any, Any]) -> Dict:
    """Receive a state dict from the old process. A "source_state_dict" entry stays in the old
    process's memory (zero copy) and is returned as a ReleasableDict; everything else is cloned
    and acknowledged at once."""
    state = IPC_queues[0].get(block=True)
    holders: List[Any] = []
    _collect_placeholders(state, holders)
    if not holders:
        return state
    msg = IPC_queues[0].get(block=True)
    tensors = _unpack(msg)
    zero_copy = isinstance(state, dict) and "source_state_dict" in state and len(state) >= 1
    if zero_copy:
        src = state["source_state_dict"]
        # tensors appear in traversal order; the source dict's come where it sits in the template
        state, _ = _fill(state, tensors, 0, clone=False)
        rel = ReleasableDict(state["source_state_dict"])
        rel._ack_queue = IPC_queues[1]
        state["source_state_dict"] = rel
        del src
    else:
        if msg[0] == "packed":
            # one copy of the whole arena; the targets are views of the copy (one storage)
            copy = msg[1].clone()
            msg = ("packed", copy, msg[2])
            state, _ = _fill(state, _unpack(msg), 0, clone=False)
        else:
            state, _ = _fill(state, tensors, 0, clone=True)
        torch.cuda.synchronize()
        del tensors, msg
        IPC_queues[1].put(None, block=True)
    return state


def _collect_placeholders(value, out):
    if isinstance(value, dict):
        for v in value.values():
            _collect_placeholders(v, out)
    elif isinstance(value, list):
        for v in value:
            _collect_placeholders(v, out)
    elif isinstance(value, TensorPlaceholder):
        out.append(value)

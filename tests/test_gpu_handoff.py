"""Old -> new process hand-off (suika_b200.handoff) on one GPU: the new process reads the old
process's source state in place (no clone), reshards it, and releases it with one ack; a target
state (shrink path) is cloned on receipt. Byte equality is checked against the old process's
own checksums."""
import hashlib
import json
import os
import tempfile
import time
import traceback

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _digest(t):
    h = t.detach().cpu().contiguous()
    if h.dtype == torch.bfloat16:
        h = h.view(torch.uint16)
    return hashlib.sha256(h.numpy().reshape(-1).view(np.uint8).tobytes()).hexdigest()


def _layouts():
    from suika_b200.layouts import SPECS, ReshardConfig, scaled_spec
    spec = scaled_spec(SPECS["llama2-13b"], hidden=256, n_layers=2, n_heads=4, ffn=512, vocab=256)
    # one rank in both worlds: the new process relayouts PP2-on-one-rank style state in place
    return ReshardConfig("handoff", spec, [[[0]]], [[[0]]]).layouts()


def _old(queues, outdir, key):
    res = {}
    try:
        from suika_b200 import handoff, synthetic as S
        torch.cuda.set_device(0)
        spl, _ = _layouts()
        st = S.host_states(spl, S.SUBFIELDS, seed=5, distinct_steps=True)[0]
        kinds = dict(S.SUBFIELDS)
        sd = {n: {s: S.to_torch(a, kinds[s], None if kinds[s] == "meta" else "cuda:0").clone() for s, a in e.items()}
              for n, e in st.items()}
        res["digests"] = {n: {s: _digest(t) for s, t in e.items() if t.is_cuda} for n, e in sd.items()}
        payload = {"source_param_layout": "layout", key: sd, "other_context_dict": {"expected_sub_fields": "x"}}
        t0 = time.perf_counter()
        handoff.interactive_IPC_state_dict_send(queues, payload)
        res["send_s"] = time.perf_counter() - t0
        res["freed"] = all(t.untyped_storage().size() == 0 for e in sd.values() for t in e.values() if t.is_cuda)
    except Exception:
        res["error"] = traceback.format_exc()
    json.dump(res, open(os.path.join(outdir, "old.json"), "w"))


def _new(queues, outdir, key):
    res = {}
    try:
        import torch.distributed as dist
        from suika_b200 import handoff, migration as M, synthetic as S
        torch.cuda.set_device(0)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT="29930")
        t0 = time.perf_counter()
        state = handoff.interactive_IPC_state_dict_recv(queues)
        res["recv_s"] = time.perf_counter() - t0
        sd = state[key]
        res["releasable"] = isinstance(sd, handoff.ReleasableDict)
        if key == "source_state_dict":
            dist.init_process_group("gloo", rank=0, world_size=1)
            spl, tpl = _layouts()
            t1 = time.perf_counter()
            out = M.schedule_and_execute_param_transfer(spl, tpl, sd, {"expected_sub_fields": S.expected_sub_fields()},
                                                        torch.device("cuda", 0), None)
            res["reshard_s"] = time.perf_counter() - t1
            res["cleared"] = len(sd) == 0
            dist.destroy_process_group()
        else:
            out = sd
        res["digests"] = {n: {s: _digest(t) for s, t in e.items() if t.is_cuda and s != "step"} for n, e in out.items()}
    except Exception:
        res["error"] = traceback.format_exc()
    json.dump(res, open(os.path.join(outdir, "new.json"), "w"))


@pytest.mark.parametrize("key", ["source_state_dict", "target_state_dict"])
def test_handoff_between_processes(key):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queues = (ctx.Queue(), ctx.Queue())
    with tempfile.TemporaryDirectory() as d:
        po = ctx.Process(target=_old, args=(queues, d, key))
        pn = ctx.Process(target=_new, args=(queues, d, key))
        po.start()
        pn.start()
        pn.join(300)
        po.join(300)
        assert po.exitcode == 0 and pn.exitcode == 0
        old = json.load(open(os.path.join(d, "old.json")))
        new = json.load(open(os.path.join(d, "new.json")))
    assert "error" not in old, old.get("error")
    assert "error" not in new, new.get("error")
    assert new["releasable"] == (key == "source_state_dict")
    assert new["digests"] == old["digests"]  # identity layout: every target equals its source
    assert old["freed"]
    if key == "source_state_dict":
        assert new["cleared"]

"""Hand-off protocol logic on the CPU (no CUDA tensors: the template path and the release hook)."""
import queue

from suika_b200 import handoff as H


class Q:
    def __init__(self):
        self.q = queue.Queue()

    def put(self, v, block=True):
        self.q.put(v)

    def get(self, block=True):
        return self.q.get()


def test_state_without_cuda_tensors_is_one_message():
    qs = (Q(), Q())
    state = {"source_param_layout": None, "source_state_dict": {"w": {"step": 3}}, "other_context_dict": {"a": 1}}
    H.interactive_IPC_state_dict_send(qs, state)
    got = H.interactive_IPC_state_dict_recv(qs)
    assert got == state
    assert qs[0].q.empty() and qs[1].q.empty()  # no tensor message, no ack


def test_release_acks_once():
    ack = Q()
    d = H.ReleasableDict({"w": 1})
    d._ack_queue = ack
    d.clear()
    d.release()
    d.release()
    assert ack.q.qsize() == 1


def test_template_and_fill_keep_traversal_order():
    tmpl = {"a": H.TensorPlaceholder(), "b": [1, H.TensorPlaceholder()], "c": {"d": H.TensorPlaceholder()}}
    filled, n = H._fill(tmpl, ["x", "y", "z"], 0, clone=False)
    assert n == 3 and filled == {"a": "x", "b": [1, "y"], "c": {"d": "z"}}

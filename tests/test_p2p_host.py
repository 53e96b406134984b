"""Host-side rules of the fused peer exchange (xrgpu_b200.p2p.PeerAllGather), on CPU.

The fused form splits an exchange in two enqueues: ``send`` (the decode GEMV writes its columns to
the other ranks) and ``recv`` / ``recv_many`` (a kernel takes the other ranks' columns). The device
protocol relies on the host keeping these rules, checked here against a fake C library and fake
streams (no GPU):
  * a group takes one send at a time: a second send, or a separate all-gather, before the receive
    is refused, and a receive needs a send;
  * a send or all-gather issued on another stream than the group's last receive waits for that
    stream -- but only inside the same CUDA graph capture (or when neither is capturing), since a
    wait across captures is illegal;
  * ``joined(seq)`` drops that ordering only if no later receive happened on the group.
"""
import ctypes

import pytest
import torch

from xrgpu_b200 import _native
from xrgpu_b200 import p2p as P


class FakeStream:
    def __init__(self, name, capture=0):
        self.name, self.capture, self.waited_on = name, capture, []
        self.cuda_stream = id(self)

    def wait_stream(self, other):
        self.waited_on.append(other.name)


class FakeLib:
    """The few C entry points PeerAllGather calls, recording their calls."""

    def __init__(self, streams):
        self.calls = []
        self.by_handle = {}
        for s in streams:
            self.by_handle[s.cuda_stream] = s

    def xrgpu_p2p_forward_send(self, g, problem, shard_cols, out, stream):
        self.calls.append(("send", g))
        return 0

    def xrgpu_p2p_forward_recv_many(self, n, groups, shard_cols, outs, valid, stream):
        self.calls.append(("recv_many", n))
        return 0

    def xrgpu_p2p_allgather(self, *args):
        self.calls.append(("allgather",))
        return 0

    def xrgpu_stream_capture_id(self, stream, out):
        out._obj.value = self.by_handle[stream.value].capture
        return 0


@pytest.fixture
def env(monkeypatch):
    streams = {"a": FakeStream("a"), "b": FakeStream("b")}
    lib = FakeLib(streams.values())
    state = {"cur": streams["a"]}
    monkeypatch.setattr(P._native, "load", lambda: lib)
    monkeypatch.setattr(P.torch.cuda, "current_stream", lambda device=None: state["cur"])

    def group(handle):
        g = object.__new__(P.PeerAllGather)
        g._g, g.broken, g.device = handle, False, torch.device("cpu")
        g._recv_done, g._sent, g._recv_seq = None, False, 0
        return g

    return streams, lib, state, group


def _send(g, out):
    g.send(_native.Problem_(), 8, out)


def test_one_send_at_a_time(env):
    streams, lib, state, group = env
    g = group(1)
    out = torch.zeros(16, dtype=torch.float16)
    _send(g, out)
    with pytest.raises(RuntimeError, match="no receive yet"):
        _send(g, out)
    with pytest.raises(RuntimeError, match="waiting for its receive"):
        g.all_gather(torch.zeros((1, 8), dtype=torch.float16), torch.zeros((1, 16), dtype=torch.float16), 16)
    g.recv(8, out, 16)
    _send(g, out)  # allowed again after the receive
    assert [c[0] for c in lib.calls] == ["send", "recv_many", "send"]


def test_receive_needs_a_send(env):
    streams, lib, state, group = env
    g = group(1)
    with pytest.raises(RuntimeError, match="without a preceding fused send"):
        g.recv(8, torch.zeros(16, dtype=torch.float16), 16)
    assert lib.calls == []


def test_receives_of_several_groups_in_one_call(env):
    streams, lib, state, group = env
    g1, g2 = group(1), group(2)
    out = torch.zeros(16, dtype=torch.float16)
    _send(g1, out)
    _send(g2, out)
    P.PeerAllGather.recv_many([(g1, 8, out, 16), (g2, 8, out, 16)])
    assert lib.calls[-1] == ("recv_many", 2)
    assert not g1._sent and not g2._sent and g1.recv_seq == 1 and g2.recv_seq == 1


def test_send_on_another_stream_waits_for_the_last_receive(env):
    streams, lib, state, group = env
    g = group(1)
    out = torch.zeros(16, dtype=torch.float16)
    _send(g, out)
    g.recv(8, out, 16)                     # on stream a
    state["cur"] = streams["b"]
    _send(g, out)                          # on stream b: waits for a
    assert streams["b"].waited_on == ["a"]
    g.recv(8, out, 16)                     # on stream b
    _send(g, out)                          # same stream: no wait
    assert streams["b"].waited_on == ["a"]


def test_no_wait_across_graph_captures(env):
    streams, lib, state, group = env
    g = group(1)
    out = torch.zeros(16, dtype=torch.float16)
    streams["a"].capture = 7
    _send(g, out)
    g.recv(8, out, 16)                     # captured in capture 7 on stream a
    streams["b"].capture = 9
    state["cur"] = streams["b"]
    _send(g, out)                          # another capture: waiting on a would be illegal
    assert streams["b"].waited_on == []
    g.recv(8, out, 16)
    streams["a"].capture = 9               # stream a joins capture 9
    state["cur"] = streams["a"]
    _send(g, out)                          # same capture, other stream: waits
    assert streams["a"].waited_on == ["b"]


def test_join_clears_only_the_latest_receive(env):
    streams, lib, state, group = env
    g = group(1)
    out = torch.zeros(16, dtype=torch.float16)
    _send(g, out)
    g.recv(8, out, 16)
    first = g.recv_seq
    _send(g, out)
    g.recv(8, out, 16)
    g.joined(first)                        # a later receive exists: ordering kept
    assert g._recv_done is not None
    g.joined(g.recv_seq)
    assert g._recv_done is None

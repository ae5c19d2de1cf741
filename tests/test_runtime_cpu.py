"""Host-side behaviour of the stage runtime's loop (hetero_infer_b200.runtime)
that needs no device: control frames pass through a middle stage in order,
and a peer that goes away ends the loop with ConnectionError (the reference
surfaces a lost peer the same way, hetero/transport.py:80-81,148-150)."""
import threading

import pytest

from hetero_infer_b200 import runtime


class _Spec:
    def __init__(self, embed, head):
        self.start, self.end, self.embed, self.head = 0, 1, embed, head


class _Stage:
    layers = [object()]


class _Backend:
    name, weight_expansion = "fake", 1.0

    def new_caches(self, n):
        return [None] * n


def _runner(head=False):
    return runtime.StageRunner(_Stage(), _Spec(False, head), 1, backend=_Backend(), name="mid")


def test_middle_stage_forwards_control_frames():
    r = _runner()
    inbound, feed = runtime.LocalChannel.pair()
    outbound, sink = runtime.LocalChannel.pair()
    frames = [{"t": "codec", "codec": "int8"}, {"t": "free", "req": "x"}, {"t": "statq"}, {"t": "reset"},
              {"t": "shape", "rtt_ms": 1.0}, {"t": "stop"}]
    r.cache_for("x")
    for h in frames:
        feed.send(dict(h))
    r.serve(inbound, outbound)
    got = [sink.recv(timeout=1)[0]["t"] for _ in range(6)]
    assert got == ["codec", "free", "statq", "reset", "shape", "stop"]
    assert r.codec == "int8" and "x" not in r.caches


def test_lost_peer_ends_serve_with_connection_error():
    r = _runner(head=True)
    inbound, feed = runtime.LocalChannel.pair()
    outbound, _ = runtime.LocalChannel.pair()
    err = []

    def loop():
        try:
            r.serve(inbound, outbound)
        except ConnectionError as e:
            err.append(e)

    t = threading.Thread(target=loop)
    t.start()
    feed.close()  # the upstream peer goes away while serve waits for a frame
    t.join(timeout=5)
    assert not t.is_alive() and len(err) == 1


def test_build_stage_refuses_over_budget(tmp_path):
    from hetero_infer_b200 import checkpoint, planner, synth
    cfg = synth.small_config(layers=2)
    synth.write_snapshot(str(tmp_path), cfg, 3, files=1)
    idx = checkpoint.WeightIndex(str(tmp_path))
    spec = planner.ShardSpec(0, 2, True, True)
    need = runtime.resident_bytes(idx, spec)
    assert need == idx.shard_bytes(spec)
    with pytest.raises(MemoryError):
        runtime.build_stage(str(tmp_path), spec, index=idx, budget_bytes=need - 1, backend=_Backend())

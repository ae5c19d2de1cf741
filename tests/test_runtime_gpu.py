"""The device stage runtime (hetero_infer_b200.runtime) against frames the
reference's own runtime produced (tests/golden/runtime_frames.npz, written by
tests/golden/make_runtime_golden.py from hetero/engine.py's StageRunner and
NumpyBackend on a synthetic MLX-format snapshot).

The stages are loaded through the reference's loading path on the device
backend: runtime.build_stage -> CudaBackend.load_stage -> checkpoint
WeightIndex / load_shard.  Headers must be equal; stage A's payloads must
decode to the reference's values within the wire's own rounding (fp16: one
unit in the last place; int8: one quantisation step); stage B reads the
reference's bytes and must return the reference's token frames, greedy and
sampled (temperature 0.7, top-p 0.9, the same seeded generator)."""
import json
import os

import numpy as np
import pytest

from hetero_infer_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "runtime_frames.npz")


def _gold():
    g = np.load(GOLDEN)
    return g, json.loads(g["meta"].tobytes())


def _ref_decode(header, payload):
    from oracle import codec
    shape = tuple(header["shape"])
    if header["codec"] == "fp16":
        return np.frombuffer(payload, dtype=np.float16).reshape(shape).astype(np.float32)
    return codec.decode_i8(payload, shape).astype(np.float32)


def _f16_ulps(a, b):
    """Distance in fp16 units in the last place between two fp16 arrays."""
    def key(x):
        i = np.asarray(x, np.float16).view(np.int16).astype(np.int32)
        return np.where(i < 0, -(i & 0x7FFF), i)
    return np.abs(key(a) - key(b))


def _stages(tmp_path, meta, codec, sampler=None):
    from hetero_infer_b200 import cuda_model, planner, runtime
    cfg = synth.small_config(**meta["cfg"])
    synth.write_snapshot(str(tmp_path), cfg, meta["seed"], files=2, tied=False)
    be = cuda_model.CudaBackend(max_ctx=64)
    spec_a, spec_b = planner.ShardSpec(*meta["spec_a"]), planner.ShardSpec(*meta["spec_b"])
    sa, _, idx = runtime.build_stage(str(tmp_path), spec_a, backend=be)
    sb, nb, _ = runtime.build_stage(str(tmp_path), spec_b, index=idx, backend=be)
    ra = runtime.StageRunner(sa, spec_a, 3, codec=codec, name="a", backend=be)
    rb = runtime.StageRunner(sb, spec_b, 3, codec=codec, sampler=sampler or runtime.Sampler(), name="b",
                             backend=be)
    return ra, rb, nb


@pytest.mark.gpu
@pytest.mark.parametrize("codec", ["fp16", "int8"])
def test_stage_runner_frames_match_reference(cuda, tmp_path, codec):
    from hetero_infer_b200 import runtime
    g, meta = _gold()
    run = meta["runs"][codec]
    ra, rb, nb = _stages(tmp_path, meta, codec)
    assert nb == run["b_shard_bytes"]
    for i, ev in enumerate(run["events"]):
        ha, pa = ra.run_frame(dict(ev["in"]), b"")
        assert ha == ev["a_out"], f"frame {i}: header"
        ref_p = g[ev["a_payload"]].tobytes()
        assert len(pa) == len(ref_p)
        ours, ref = _ref_decode(ha, pa), _ref_decode(ev["a_out"], ref_p)
        if codec == "fp16":
            # the same fp32 state up to summation order: at most one fp16 ulp
            # apart, or (near zero, where cancellation leaves fp32 sums a few
            # 1e-7 of the row's scale apart) within 1e-5 of the row's largest value
            near = np.abs(ours - ref) <= 1e-5 * np.abs(ref).max(axis=-1, keepdims=True)
            assert np.all((_f16_ulps(ours, ref) <= 1) | near), f"frame {i}"
            # 1-3% of elements sit on a rounding edge (prompt frames go through the
            # multi-token kernel, whose fp32 sums run in another order)
            assert np.mean(ours != ref) < 0.05, f"frame {i}"
        else:
            step = np.abs(ref).max(axis=-1, keepdims=True) / 127.0
            assert np.all(np.abs(ours - ref) <= 1.01 * step + 1e-6), f"frame {i}"
            assert np.mean(ours != ref) < 0.01, f"frame {i}"
        # the runtime's own decode of the reference bytes is the reference's decode
        x = runtime.decode(ev["a_out"], ref_p, "cuda").cpu().numpy()
        assert np.array_equal(x, ref)
        hb, _ = rb.run_frame(dict(ev["a_out"]), ref_p)
        assert hb == ev["b_out"], f"frame {i}: {hb} vs {ev['b_out']}"
    assert sorted(ra.caches) == sorted(rb.caches) == ["r0", "r1"]
    assert rb.stats.tokens == sum(ev["b_out"] is not None for ev in run["events"])


@pytest.mark.gpu
def test_stage_runner_sampling_matches_reference(cuda, tmp_path):
    from hetero_infer_b200 import runtime
    g, meta = _gold()
    run = meta["runs"]["fp16"]
    _, rs, _ = _stages(tmp_path, meta, "fp16", sampler=runtime.Sampler(**meta["sampler"]))
    got = []
    for ev in run["events"]:
        if ev["in"]["req"] != "r0":
            continue
        hb, _ = rs.run_frame(dict(ev["a_out"], req="s0"), g[ev["a_payload"]].tobytes())
        got.append(None if hb is None else hb["tok"])
    assert got == run["sampled_r0_frames"]


@pytest.mark.gpu
def test_stage_runner_serve_control_frames(cuda, tmp_path):
    """serve() on the head stage: forward frames become token frames; statq
    collects this stage's counters; free drops the request's cache; reset
    clears the counters; ping is answered; stop ends the loop (none of the
    control frames travels past the head stage, as in engine.py:104-147)."""
    from hetero_infer_b200 import runtime
    g, meta = _gold()
    run = meta["runs"]["fp16"]
    _, rb, _ = _stages(tmp_path, meta, "fp16")
    inbound, feed = runtime.LocalChannel.pair()
    outbound, sink = runtime.LocalChannel.pair()
    evs = run["events"][:3]
    for ev in evs:
        feed.send(dict(ev["a_out"]), g[ev["a_payload"]].tobytes())
    for h in ({"t": "statq"}, {"t": "free", "req": "r0"}, {"t": "ping"}, {"t": "reset"}, {"t": "stop"}):
        feed.send(h)
    rb.serve(inbound, outbound)
    got = []
    while True:
        try:
            got.append(sink.recv(timeout=0.1)[0])
        except TimeoutError:
            break
    toks = [h for h in got if h.get("t") == "tok"]
    assert toks == [ev["b_out"] for ev in evs if ev["b_out"] is not None]
    stat = [h for h in got if h.get("t") == "statq"][0]
    assert stat["stats"][0]["name"] == "b" and stat["stats"][0]["frames"] == 3
    assert {"t": "ack"} in got
    assert not any(h.get("t") in ("free", "stop", "reset") for h in got)
    assert "r0" not in rb.caches and "r1" in rb.caches
    assert rb.stats.frames == 0

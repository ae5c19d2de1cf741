"""Golden frames of the reference's stage runtime (hetero/engine.py:38-173).

Writes the synthetic MLX-format snapshot of tests/golden/checkpoint_index.json
(synth.write_snapshot) into a temporary directory, loads two stages from it
with the reference's own build_stage and NumpyBackend (imported unmodified
from the reference tree; its kernel is the reference's kernel/q4gemv.c built
from source by oracle/Makefile, in its portable fp32 build -- the AVX2 build
rounds x to int16 per call, ~5e-5 relative, which moves about one fp16
wire element in twenty by an ulp), and runs frames through the reference's
StageRunner.run_frame: stage A = layers [0, 2) with the embedding, stage B =
layer [2, 3) with the head, for both wire codecs.  Two requests are
interleaved: one prefilled in two chunks (the first without logits), one in a
single frame, then greedy decode frames; a third request on B samples with
temperature and top-p.  Records every frame in and out (headers as JSON,
payloads as bytes) in runtime_frames.npz.  The device runtime
(hetero_infer_b200.runtime) must reproduce them (tests/test_runtime_gpu.py).

  python tests/golden/make_runtime_golden.py [REFERENCE_ROOT]
"""
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CFG = dict(layers=3, hidden=256, heads=4, kv_heads=2, inter=512, vocab=1000)
SEED = 9
SPEC_A = (0, 2, True, False)
SPEC_B = (2, 3, False, True)
DECODE_STEPS = 4
SAMPLER = dict(temperature=0.7, top_p=0.9, seed=5)


def script():
    """The forward frames stage A receives, in order (headers only)."""
    from hetero_infer_b200 import synth
    p0 = synth.prompt_ids(31, 7, CFG["vocab"]).tolist()
    p1 = synth.prompt_ids(32, 5, CFG["vocab"]).tolist()
    return [
        {"t": "fwd", "req": "r0", "ids": [p0[0][:4]], "step": 0, "logits": False, "last": False},
        {"t": "fwd", "req": "r0", "ids": [p0[0][4:]], "step": 0, "logits": True, "last": True},
        {"t": "fwd", "req": "r1", "ids": p1, "step": 0, "logits": True, "last": True},
    ]


def main():
    if len(sys.argv) > 1:
        os.environ["HETERO_REF_ROOT"] = sys.argv[1]
    from oracle import refmodel
    refmodel.load_cpu_model("float")  # binds the reference kernel built from source
    from hetero import backends, engine, shard
    from hetero_infer_b200 import synth
    cfg = synth.small_config(**CFG)
    out = {}
    meta = {"kernel": "kernel/q4gemv.c, portable fp32 build", "cfg": CFG, "seed": SEED, "spec_a": SPEC_A,
            "spec_b": SPEC_B, "decode_steps": DECODE_STEPS, "sampler": SAMPLER, "runs": {}}
    with tempfile.TemporaryDirectory() as d:
        synth.write_snapshot(d, cfg, SEED, files=2, tied=False)
        be = backends.NumpyBackend()
        assert be.fused, "reference kernel not bound"
        for codec in ("fp16", "int8"):
            sa, _, idx = engine.build_stage(d, shard.ShardSpec(*SPEC_A), backend=be)
            sb, nb, _ = engine.build_stage(d, shard.ShardSpec(*SPEC_B), index=idx, backend=be)
            ra = engine.StageRunner(sa, shard.ShardSpec(*SPEC_A), 3, codec=codec, name="a", backend=be)
            rb = engine.StageRunner(sb, shard.ShardSpec(*SPEC_B), 3, codec=codec, sampler=engine.Sampler(),
                                    name="b", backend=be)
            events = []
            frames = script()
            last_tok = {}
            k = 0
            while frames:
                hin = frames.pop(0)
                ha, pa = ra.run_frame(dict(hin), b"")
                hb, _ = rb.run_frame(dict(ha), pa)
                key = f"{codec}.{k}"
                out[key] = np.frombuffer(pa, dtype=np.uint8)
                events.append({"in": hin, "a_out": ha, "a_payload": key, "b_out": hb})
                k += 1
                if hb is not None:
                    last_tok[hb["req"]] = hb["tok"]
                    step = hin["step"] + 1
                    if step <= DECODE_STEPS:
                        frames.append({"t": "fwd", "req": hb["req"], "ids": [[hb["tok"]]], "step": step,
                                       "logits": True, "last": True})
            # temperature / top-p on B, fed the same A frames of request r0
            rs = engine.StageRunner(sb, shard.ShardSpec(*SPEC_B), 3, codec=codec,
                                    sampler=engine.Sampler(**SAMPLER), name="b-sampled", backend=be)
            sampled = []
            for ev in events:
                if ev["in"]["req"] != "r0":
                    continue
                hb, _ = rs.run_frame(dict(ev["a_out"], req="s0"), out[ev["a_payload"]].tobytes())
                sampled.append(None if hb is None else hb["tok"])
            meta["runs"][codec] = {"events": events, "sampled_r0_frames": sampled, "b_shard_bytes": nb}
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "runtime_frames.npz"), **out)
    print("wrote runtime_frames.npz:", {c: len(r["events"]) for c, r in meta["runs"].items()})


if __name__ == "__main__":
    main()

"""Golden index of the reference's weight index (hetero/shard.py:72-158) over
the synthetic MLX-format snapshots of synth.write_snapshot.

Writes the snapshots into a temporary directory, indexes them with the
reference's own WeightIndex (imported unmodified; build container only) and
records its byte accounting and per-stage ownership.  The tests rebuild the
same snapshots and compare hetero_infer_b200.checkpoint against it.

  python tests/golden/make_checkpoint_golden.py [REFERENCE_ROOT]
"""
import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CFG = dict(layers=3, hidden=256, heads=4, kv_heads=2, inter=512, vocab=1000)
SEED = 9
SPECS = [(0, 3, True, True), (0, 1, True, False), (1, 3, False, True), (1, 2, False, False), (2, 3, False, True)]


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.sep, "root", "reference")
    sys.path.insert(0, ref_root)
    from hetero import shard
    from hetero_infer_b200 import synth
    cfg = synth.small_config(**CFG)
    out = {"cfg": CFG, "seed": SEED, "specs": SPECS, "snapshots": {}}
    for tied in (False, True):
        with tempfile.TemporaryDirectory() as d:
            synth.write_snapshot(d, cfg, SEED, files=2, tied=tied)
            idx = shard.WeightIndex(d)
            rec = {"layer_bytes": idx.layer_bytes(), "embed_bytes": idx.embed_bytes(),
                   "head_bytes": idx.head_bytes(), "total_bytes": idx.total_bytes(),
                   "entries": {n: [os.path.basename(p), dt, shape, nb] for n, (p, dt, shape, nb) in
                               sorted(idx.entries.items())},
                   "shards": []}
            for s in SPECS:
                spec = shard.ShardSpec(*s)
                rec["shards"].append({"bytes": idx.shard_bytes(spec),
                                      "names": sorted(n for n in idx.names() if idx.owns(n, spec))})
            out["snapshots"]["tied" if tied else "untied"] = rec
    with open(os.path.join(HERE, "checkpoint_index.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote checkpoint_index.json")


if __name__ == "__main__":
    main()

"""MLX-format safetensors snapshots (hetero/shard.py:72-158 WeightIndex).

The index and per-stage ownership are compared with what the reference's own
WeightIndex recorded on the same synthetic snapshots (tests/golden/
checkpoint_index.json, written by make_checkpoint_golden.py); a stage's
tensors must come back exactly as written; on the GPU a stage built from the
snapshot decodes the oracle's tokens."""
import json
import os

import numpy as np
import pytest

from hetero_infer_b200 import checkpoint, planner, synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "checkpoint_index.json")


def _gold():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.fixture(scope="module", params=["untied", "tied"])
def snap(request, tmp_path_factory):
    g = _gold()
    cfg = synth.small_config(**g["cfg"])
    d = str(tmp_path_factory.mktemp(request.param))
    w = synth.write_snapshot(d, cfg, g["seed"], files=2, tied=request.param == "tied")
    return request.param, d, w, cfg, g


def test_index_matches_reference(snap):
    kind, d, w, cfg, g = snap
    ref = g["snapshots"][kind]
    idx = checkpoint.WeightIndex(d)
    assert idx.layer_bytes() == ref["layer_bytes"]
    assert idx.embed_bytes() == ref["embed_bytes"]
    assert idx.head_bytes() == ref["head_bytes"]
    assert idx.total_bytes() == ref["total_bytes"]
    got = {n: [os.path.basename(p), dt, shape, nb] for n, (p, dt, shape, nb) in idx.entries.items()}
    assert got == ref["entries"]
    for s, r in zip(g["specs"], ref["shards"]):
        spec = planner.ShardSpec(*s)
        assert idx.shard_bytes(spec) == r["bytes"]
        assert sorted(n for n in idx.names() if idx.owns(n, spec)) == r["names"]


def test_load_shard_reads_exactly_the_stage_tensors(snap):
    kind, d, w, cfg, g = snap
    idx = checkpoint.WeightIndex(d)
    for s, r in zip(g["specs"], g["snapshots"][kind]["shards"]):
        got = idx.load_shard(planner.ShardSpec(*s))
        assert sorted(got) == r["names"]
        for n, a in got.items():
            assert a.dtype == w[n].dtype and a.shape == w[n].shape and np.array_equal(a, w[n]), n


def test_unclassified_tensor_is_an_error(tmp_path):
    from safetensors.numpy import save_file
    cfg = synth.small_config(layers=1)
    synth.write_snapshot(str(tmp_path), cfg, 1, files=1)
    save_file({"vision_tower.weight": np.zeros(4, np.float16)}, str(tmp_path / "extra.safetensors"))
    idx = checkpoint.WeightIndex(str(tmp_path))
    with pytest.raises(KeyError):
        idx.shard_bytes(planner.ShardSpec(0, 1, True, True))


@pytest.mark.gpu
@pytest.mark.parametrize("tied", [False, True])
def test_stage_from_snapshot_decodes_oracle_tokens(cuda, tmp_path, tied):
    """The whole model (embedding, layers, head; tied or not) loaded from a
    snapshot onto the device: greedy tokens equal the oracle stage's on the
    same tensors (the quantized embedding rows dequantized as the reference's
    Stage.embed does)."""
    import torch
    from oracle import q4
    from oracle import stage as ost
    g = _gold()
    cfg = synth.small_config(**g["cfg"])
    w = synth.write_snapshot(str(tmp_path), cfg, g["seed"], files=2, tied=tied)
    L = cfg["num_hidden_layers"]
    spec = planner.ShardSpec(0, L, True, True)
    st = checkpoint.stage_from_snapshot(str(tmp_path), spec, device="cuda", max_ctx=64)
    orc = q4.Oracle()
    gs = cfg["quantization"]["group_size"]
    ew, es, eb = w["model.embed_tokens.weight"], w["model.embed_tokens.scales"], w["model.embed_tokens.biases"]
    rows = lambda ids: np.stack([orc.dequant(ew[i:i + 1], es[i:i + 1], eb[i:i + 1], 0, 1, gs)[0] for i in ids])
    ow = dict(w)
    if tied:
        ow["lm_head.weight"], ow["lm_head.scales"], ow["lm_head.biases"] = ew, es, eb
    ref = ost.OracleStage(dict(cfg, tie_word_embeddings=tied), ow, 0, L, True, True, embed_rows=rows)
    ids = synth.prompt_ids(5, 6, cfg["vocab_size"])
    caches_d, caches_o = st.new_caches(), ref.new_caches()
    x_d, x_o = ids, ids
    for step in range(5):
        zd = st(x_d, caches_d, apply_head=True)
        zo = ref(x_o, caches_o, apply_head=True, last_only=True)
        td = int(np.asarray(torch.as_tensor(zd).float().cpu()).reshape(-1, cfg["vocab_size"])[-1].argmax())
        to = int(np.asarray(zo)[0, -1].argmax())
        assert td == to, f"step {step}"
        x_d = x_o = np.array([[to]])

"""Pin the stage oracle (oracle/stage.py): bit for bit against the reference's
own cpu_model.Stage (float kernel build) when the reference tree is present,
and against the committed golden fixture the reference produced
(tests/golden/golden_small.npz) everywhere."""
import os

import numpy as np
import pytest

from hetero_infer_b200 import synth
from oracle import refmodel, q4
from oracle import stage as ost

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "golden_small.npz")
SMALL = dict(layers=2, hidden=256, heads=4, kv_heads=2, inter=512, vocab=1024)
SEED = 7


def oracle_greedy(cfg, w, prompt, n, seed):
    st = ost.OracleStage(cfg, w, 0, cfg["num_hidden_layers"], True, True,
                         embed_rows=lambda ids: synth.embed_rows(seed, ids, cfg["hidden_size"]))
    caches = st.new_caches()
    x, toks, logits = prompt, [], []
    for _ in range(n):
        z = st(x, caches, apply_head=True, last_only=True)[0, -1]
        logits.append(z)
        toks.append(int(z.argmax()))
        x = np.array([[toks[-1]]])
    return np.array(toks), np.stack(logits)


def test_oracle_stage_matches_golden_reference_run():
    g = np.load(GOLDEN)
    cfg = synth.small_config(**SMALL)
    w = synth.model_weights(cfg, SEED)
    toks, logits = oracle_greedy(cfg, w, g["prompt"], len(g["tokens_float"]), SEED)
    assert np.array_equal(toks, g["tokens_float"])
    assert np.array_equal(logits, g["logits_float"]), "oracle stage must equal the reference (float kernel)"
    # the reference's x86 kernel quantises x to int16: same tokens, logits close
    assert np.array_equal(toks, g["tokens_avx2"])
    rel = np.linalg.norm(logits - g["logits_avx2"]) / np.linalg.norm(g["logits_avx2"])
    assert rel < 1e-3


def test_golden_prompt_is_regenerable():
    g = np.load(GOLDEN)
    assert np.array_equal(g["prompt"], synth.prompt_ids(SEED, g["prompt"].shape[1], SMALL["vocab"]))


@pytest.mark.skipif(not refmodel.available() or "float" not in q4.available_ref_variants(),
                    reason="reference tree not mounted (golden fixture covers this)")
def test_oracle_stage_bit_exact_vs_live_reference_prefill_and_decode():
    cfg = synth.small_config(layers=2, hidden=256, heads=4, kv_heads=1, inter=384, vocab=700, gs=128)
    w = synth.model_weights(cfg, 4)
    cm = refmodel.load_cpu_model("float")
    ref = refmodel.build_stage(cm, cfg, w, 0, 2, True, True)
    orc = ost.OracleStage(cfg, w, 0, 2, True, True, embed_rows=lambda ids: synth.embed_rows(4, ids, 256))
    prompt = synth.prompt_ids(2, 19, cfg["vocab_size"])      # > 16 rows: dequant + matmul path
    rc, oc = [cm.KVCache() for _ in ref.layers], orc.new_caches()
    a = ref(prompt, rc, apply_head=True, last_only=False)
    b = orc(prompt, oc, apply_head=True, last_only=False)
    assert np.array_equal(a, b)
    x = np.array([[int(a[0, -1].argmax())]])
    for _ in range(4):
        a = ref(x, rc, apply_head=True, last_only=True)
        b = orc(x, oc, apply_head=True, last_only=True)
        assert np.array_equal(a, b)
        x = np.array([[int(a[0, -1].argmax())]])

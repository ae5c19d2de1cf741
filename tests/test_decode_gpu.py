"""Persistent decode (hq4_decode_plan_*): every layer of a decode step in one
cooperative launch against the same step as five launches per layer.

Both run the same device arithmetic (the streaming GEMV's consumer steps and
the attention row), so the bar is bit equality: the greedy tokens, the last
logits, the hidden row and every layer's KV cache.  The per-launch path is
itself tested against the stage oracle and the reference's golden logits
(tests/test_stage_gpu.py), and the 7B-shape decode through the persistent plan
against the reference's tokens (test_7b_greedy_decode_token_identical_to_reference).
"""
import numpy as np
import pytest

from hetero_infer_b200 import synth


class Spec:
    def __init__(self, start, end, embed, head):
        self.start, self.end, self.embed, self.head = start, end, embed, head


CONFIGS = [
    # gs 64; 32 strips per projection: most CTAs own none
    dict(layers=3, hidden=512, heads=4, kv_heads=2, inter=1024, vocab=1000),
    # gs 128, grouped-query 4:1
    dict(layers=2, hidden=1024, heads=8, kv_heads=2, inter=2048, vocab=2048, gs=128),
    # gs 256; gate|up 512 strips: up to 4 per CTA (the shared-memory strip slots)
    dict(layers=2, hidden=2048, heads=16, kv_heads=4, inter=4096, vocab=512, gs=256),
]


def _stage(cfg, seed, max_ctx=256):
    from hetero_infer_b200 import cuda_model
    w = synth.model_weights(cfg, seed)
    return cuda_model.Stage(cfg, Spec(0, cfg["num_hidden_layers"], True, True), w, max_ctx=max_ctx)


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(len(CONFIGS)))
def test_persistent_decode_bit_identical_to_layer_launches(cuda, ci):
    import torch
    from hetero_infer_b200 import _lib, cuda_model
    cfg = synth.small_config(**CONFIGS[ci])
    stage = _stage(cfg, seed=60 + ci)
    prompt = synth.prompt_ids(ci, 9, cfg["vocab_size"])
    lib = _lib.load()
    lib.hq4_device_status(1)
    ref = cuda_model.GreedyDecoder(stage, persistent=False)
    dec = cuda_model.GreedyDecoder(stage, persistent=True)
    info = dec.plan.info()
    assert info["phases"] == 5 * cfg["num_hidden_layers"] and info["ring"] >= 2
    n = 14
    ta = ref.generate(prompt, n)
    tb = dec.generate(prompt, n)
    torch.cuda.synchronize()
    assert lib.hq4_device_status(0) == 0
    assert ta == tb
    assert torch.equal(ref.logits, dec.logits)
    assert torch.equal(ref.h, dec.h)
    for i in range(cfg["num_hidden_layers"]):
        assert torch.equal(ref.cache.k[i], dec.cache.k[i]), f"k cache of layer {i}"
        assert torch.equal(ref.cache.v[i], dec.cache.v[i]), f"v cache of layer {i}"


@pytest.mark.gpu
def test_persistent_decode_eager_steps_and_repeat(cuda):
    """Eager plan runs (no graph) step after step: the barrier words reset at
    every exit, so consecutive launches agree with the per-launch path."""
    import torch
    from hetero_infer_b200 import _lib, cuda_model
    cfg = synth.small_config(**CONFIGS[0])
    stage = _stage(cfg, seed=5)
    lib = _lib.load()
    lib.hq4_device_status(1)
    a = cuda_model.GreedyDecoder(stage, persistent=False)
    b = cuda_model.GreedyDecoder(stage, persistent=True)
    prompt = synth.prompt_ids(3, 5, cfg["vocab_size"])
    for d in (a, b):
        d.prefill(prompt)
        with torch.cuda.stream(d.stream):
            for _ in range(30):
                d._step()
                d.cache.offset += 1
    torch.cuda.synchronize()
    assert lib.hq4_device_status(0) == 0
    assert torch.equal(a.history, b.history)
    assert torch.equal(a.h, b.h)


@pytest.mark.gpu
def test_persistent_decode_rejects_unfit_shapes(cuda):
    from hetero_infer_b200 import cuda_model
    cfg = synth.small_config(layers=1, hidden=256, heads=4, kv_heads=2, inter=512, vocab=300)  # n_in/gs = 4
    stage = _stage(cfg, seed=1)
    assert cuda_model.GreedyDecoder(stage, persistent="auto").plan is None  # falls back to per-layer launches
    assert cuda_model.GreedyDecoder(stage).plan is None  # the default: per-layer launches
    with pytest.raises(ValueError):
        cuda_model.GreedyDecoder(stage, persistent=True)


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(len(CONFIGS)))
def test_persistent_decode_logits_match_stage_oracle(cuda, ci):
    """Every step's logits of the persistent plan against the NumPy stage
    oracle (oracle/stage.py, pinned bit for bit to the reference's
    cpu_model.Stage): relative L2 <= 5e-5 and the same greedy token.  (The
    per-layer path gives the same bits; over ten steps of these three-layer
    models the fp32 summation-order differences reach ~3e-5 at one step.)"""
    import torch
    from hetero_infer_b200 import cuda_model
    from oracle import stage as ost
    from tests.test_stage_gpu import LOGIT_TOL, _decode_top5, rel_l2
    cfg = synth.small_config(**CONFIGS[ci])
    seed = 80 + ci
    w = synth.model_weights(cfg, seed)
    stage = cuda_model.Stage(cfg, Spec(0, cfg["num_hidden_layers"], True, True), w, max_ctx=256)
    orc = ost.OracleStage(cfg, w, 0, cfg["num_hidden_layers"], True, True,
                          embed_rows=lambda ids: synth.embed_rows(seed, ids, cfg["hidden_size"]))
    dec = cuda_model.GreedyDecoder(stage, persistent=True)
    prompt = synth.prompt_ids(40 + ci, 6, cfg["vocab_size"])
    n = 10
    toks, rows = _decode_top5(dec, prompt, n)
    oc = orc.new_caches()
    x = prompt
    for i in range(n):
        b = orc(x, oc, apply_head=True, last_only=True)[0, -1]
        assert rel_l2(rows[i], b) <= 2.5 * LOGIT_TOL, f"step {i}: {rel_l2(rows[i], b):.2e}"
        assert toks[i] == int(b.argmax()), f"step {i}: token {toks[i]} vs {int(b.argmax())}"
        x = np.array([[toks[i]]])
    dec.graph = None
    dec.plan.close()
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_persistent_decode_barrier_timeout_reports_and_recovers(cuda):
    """Failure path of the plan's grid barrier, without faulting the GPU: one
    CTA withholds its arrival at the first barrier (hq4_decode_plan_fault),
    so every CTA's bounded wait (20 ms here) runs out.  The launch returns,
    status bit 0 reports it, and the barrier words are reset: after the hook
    is cleared, a full decode through the same plan is bit-identical to the
    per-layer launches."""
    import time
    import torch
    from hetero_infer_b200 import _lib, cuda_model
    cfg = synth.small_config(**CONFIGS[0])
    stage = _stage(cfg, seed=17)
    lib = _lib.load()
    prompt = synth.prompt_ids(8, 5, cfg["vocab_size"])
    ref = cuda_model.GreedyDecoder(stage, persistent=False)
    dec = cuda_model.GreedyDecoder(stage, persistent=True)
    dec.prefill(prompt)
    torch.cuda.synchronize()
    lib.hq4_device_status(1)
    dec.plan.inject_fault(skip_cta=3, barrier_ns=20_000_000)
    t0 = time.perf_counter()
    with torch.cuda.stream(dec.stream):
        dec.plan.run()
    torch.cuda.synchronize()
    took = time.perf_counter() - t0
    assert lib.hq4_device_status(1) & 1, "the barrier timeout was not reported"
    assert took < 10.0
    dec.plan.inject_fault(-1, 0)
    # a fresh decode in the same buffers: position back to 0
    dec.cache.pos.zero_()
    dec.cache.offset = 0
    n = 12
    tb = dec.generate(prompt, n)
    ta = ref.generate(prompt, n)
    torch.cuda.synchronize()
    assert lib.hq4_device_status(0) == 0
    assert ta == tb
    assert torch.equal(ref.h, dec.h)
    assert torch.equal(ref.logits, dec.logits)

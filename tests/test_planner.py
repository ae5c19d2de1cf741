"""The GPU pipeline planner keeps the reference's DP (hetero/planner.py): on the
same inputs it must choose the same cuts, head placement and predicted time as
the reference's own plan_pipeline (run here when the reference tree is
mounted), and it must give balanced cuts for identical GPUs with a sharded head."""
import sys

import pytest

from hetero_infer_b200 import planner, synth
from oracle import refmodel


def _ref_planner():
    if refmodel.REF_ROOT not in sys.path:
        sys.path.insert(0, refmodel.REF_ROOT)
    import importlib
    return importlib.import_module("hetero.planner")


CASES = [
    # (per-node (mem GiB, s/layer, head_s)), objective
    ([(160, 60e-6, 50e-6)] * 2, "throughput"),
    ([(160, 60e-6, 50e-6)] * 4, "throughput"),
    ([(160, 60e-6, 50e-6)] * 8, "latency"),
    ([(5.0, 60e-6, 50e-6), (160, 120e-6, 500e-6), (3.0, 30e-6, 10e-6)], "throughput"),
    ([(2.4, 400e-6, 2e-3), (2.4, 7e-3, 0.85)], "latency"),     # infeasible on both
    ([(3.0, 400e-6, 2e-3), (3.0, 7e-3, 0.85)], "latency"),
    ([(4.0, 400e-6, 2e-3), (2.0, 2e-3, 0.2), (1.5, 1e-3, 0.01)], "throughput"),
]


@pytest.mark.skipif(not refmodel.available(), reason="reference tree not mounted")
@pytest.mark.parametrize("case", range(len(CASES)))
def test_same_plan_as_reference_planner(case):
    rp = _ref_planner()
    specs, objective = CASES[case]
    cfg = dict(synth.QWEN2_7B)
    index = planner.ModelIndex(cfg)
    mine = [planner.NodeProfile(f"n{i}", mem_bytes=int(m * 2**30), decode_s_per_layer=s, head_s=h)
            for i, (m, s, h) in enumerate(specs)]
    theirs = [rp.NodeProfile(f"n{i}", mem_bytes=int(m * 2**30), decode_s_per_layer=s, head_s=h)
              for i, (m, s, h) in enumerate(specs)]
    link_m = planner.LinkSpec(bandwidth_mbps=1000.0, rtt_ms=0.3)
    link_t = rp.LinkSpec(bandwidth_mbps=1000.0, rtt_ms=0.3)
    try:
        b = rp.plan_pipeline(index, theirs, link_t, objective, max_ctx=4096)
    except MemoryError:
        with pytest.raises(MemoryError):
            planner.plan_pipeline(index, mine, link_m, objective, max_ctx=4096)
        return
    a = planner.plan_pipeline(index, mine, link_m, objective, max_ctx=4096)
    assert a.cuts == b.cuts
    assert a.head_node == b.head_node
    assert abs(a.predicted_decode_s - b.predicted_decode_s) <= 1e-15 + 1e-12 * b.predicted_decode_s


@pytest.mark.parametrize("n,cuts", [(2, [0, 14, 28]), (4, [0, 7, 14, 21, 28])])
def test_sharded_head_balances_identical_gpus(n, cuts):
    p = planner.plan_gpu_pipeline(synth.QWEN2_7B, n, layer_s=60e-6, head_s=50e-6)
    assert p.cuts == cuts
    assert p.head_node == -1 and not any(s.head for s in p.specs)
    assert p.specs[0].embed and not any(s.embed for s in p.specs[1:])


def test_eight_gpus_split_28_layers_4_and_3():
    p = planner.plan_gpu_pipeline(synth.QWEN2_7B, 8, layer_s=60e-6, head_s=50e-6)
    sizes = [s.n_layers for s in p.specs]
    assert sum(sizes) == 28 and max(sizes) == 4 and min(sizes) == 3


def test_memory_is_a_hard_constraint():
    with pytest.raises(MemoryError):
        planner.plan_gpu_pipeline(synth.QWEN2_7B, 2, layer_s=60e-6, mem_bytes=2 * 2**30)


def test_sharded_head_costs_every_stage_its_share_and_the_collectives():
    cfg = dict(synth.QWEN2_7B)
    link = planner.LinkSpec()
    for n in (2, 4, 8):
        p = planner.plan_gpu_pipeline(cfg, n, layer_s=45e-6, head_s=50e-6, link=link)
        coll = link.seconds_for(cfg["hidden_size"] * 4) + link.seconds_for(8 * n)
        for spec, t in zip(p.specs, p.stage_compute_s):
            assert abs(t - (spec.n_layers * 45e-6 + 50e-6 / n + coll)) < 1e-12


def test_int8_wire_sends_fewer_bytes():
    cfg = dict(synth.QWEN2_7B)
    assert planner.hidden_bytes(cfg, codec="int8") == cfg["hidden_size"] + 4
    # over NVLink the hand-off is latency-bound: the codec does not move a cut
    n16 = planner.plan_gpu_pipeline(cfg, 4, layer_s=45e-6, head_s=50e-6, codec="fp16")
    n8 = planner.plan_gpu_pipeline(cfg, 4, layer_s=45e-6, head_s=50e-6, codec="int8")
    assert n8.cuts == n16.cuts == [0, 7, 14, 21, 28]
    # over a link slow enough to matter, halving the bytes lowers every send
    # and the predicted tick, and the cuts shift back toward balance
    slow = planner.LinkSpec(bandwidth_mbps=80.0, rtt_ms=0.0)
    p16 = planner.plan_gpu_pipeline(cfg, 4, layer_s=45e-6, head_s=50e-6, link=slow, codec="fp16")
    p8 = planner.plan_gpu_pipeline(cfg, 4, layer_s=45e-6, head_s=50e-6, link=slow, codec="int8")
    assert p8.predicted_decode_s < p16.predicted_decode_s
    assert all(a < b for a, b in zip(p8.stage_comm_s[:-1], p16.stage_comm_s[:-1]))
    assert p8.cuts[-2] - p8.cuts[1] > p16.cuts[-2] - p16.cuts[1]


def test_plan_from_snapshot_index(tmp_path):
    """The byte accounting can come from a checkpoint's own index: the plan is
    balanced and its memory per stage adds up to the snapshot's bytes."""
    from hetero_infer_b200 import checkpoint
    cfg = synth.small_config(layers=8, hidden=256, heads=4, kv_heads=2, inter=512, vocab=1000)
    synth.write_snapshot(str(tmp_path), cfg, 3, files=2)
    idx = checkpoint.WeightIndex(str(tmp_path))
    p = planner.plan_gpu_pipeline(idx.config, 4, layer_s=45e-6, head_s=50e-6, index=idx, max_ctx=16)
    assert p.cuts == [0, 2, 4, 6, 8]
    weights = sum(idx.shard_bytes(s) for s in p.specs) - 3 * (idx.head_bytes() - idx.head_bytes() // 4)
    assert weights > 0

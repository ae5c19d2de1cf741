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

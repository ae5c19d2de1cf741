"""The pipelined decode on GPUs over NCCL (one process per GPU).

* small model, 2 GPUs: every microbatch's tokens equal a single-process run of
  the same stage slices joined by the reference's fp16 wire (the stage oracle,
  pinned to the reference), with the vocabulary projection row-sharded;
* the benchmark's 7B-shape model at the planner's 2/4/8-GPU cuts with the
  reference's fp16 wire: the tokens the reference's own stages, wire
  conversion and sampler produced (tests/golden/golden_7b_pipe.json);
* the 7B-shape model on 2 GPUs with an fp32 wire: the 128 tokens of the
  reference's unsplit NumPy backend (tests/golden/golden_7b.json).

Each case needs as many GPUs as it has stages and skips otherwise."""
import json
import os
import socket

import numpy as np
import pytest

from tests.test_pipeline_cpu import CFG, N_MICRO, PROMPT, SEED, STEPS, reference_tokens
from hetero_infer_b200 import pipeline, synth

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, case, q):
    import datetime
    import torch
    import torch.distributed as dist
    from hetero_infer_b200.planner import ShardSpec
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        cuts = case["cuts"]
        cfg = dict(synth.QWEN2_7B) if case["model"] == "7b" else synth.small_config(**CFG)
        a, b = cuts[rank], cuts[rank + 1]
        w = synth.model_weights(cfg, case["seed"], layers=range(a, b), embed=(rank == 0), head=True)
        comp = pipeline.DeviceCompute(cfg, ShardSpec(a, b, rank == 0, False), w,
                                      pipeline.head_rows(cfg["vocab_size"], world, rank), dev,
                                      max_ctx=256, wire=case["wire"])
        del w
        prompts = [synth.prompt_ids(s, case["prompt_len"], cfg["vocab_size"]) for s in case["prompt_seeds"]]
        pr = pipeline.PipelineRank(pipeline.Comm(rank, world, dev), comp, len(prompts))
        pr.prefill(prompts)
        pr.decode(case["steps"])
        torch.cuda.synchronize()
        pr.close()  # its graphs hold NCCL calls: release them before the process group goes
        q.put((rank, pr.tokens))
    finally:
        dist.destroy_process_group()


def _run(world, case):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(1, world):
        assert got[r] == got[0], f"rank {r} disagrees with rank 0"
    return got[0]


@pytest.mark.gpu
@pytest.mark.parametrize("wire", ["float16", "int8"])
def test_nccl_pipeline_two_gpus_matches_single_process(wire):
    """The device codec (hq4_act_encode_i8 / decode, bit-identical to the
    reference's NumPy codec) on the NCCL wire gives the tokens of the oracle
    stages joined by the reference's codec."""
    cuts = [0, 2, 3]
    got = _run(2, dict(model="small", cuts=cuts, seed=SEED, wire=wire, prompt_len=PROMPT,
                       prompt_seeds=[100 + m for m in range(N_MICRO)], steps=STEPS))
    assert got == reference_tokens(cuts, wire)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [2, 4, 8])
def test_7b_pipeline_fp16_wire_matches_reference_stages(n):
    """The specified random model overflows fp16 at every cut (its residual
    stream reaches ~1e5), so the reference's wire produces inf, its next
    stage's RMSNorm NaN and its sampler the first NaN index: the golden file
    records that, and the device pipeline must produce the same tokens."""
    import torch
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    gold = json.load(open(os.path.join(GOLDEN_DIR, "golden_7b_pipe.json")))
    ref = gold["variants"]["avx2"][str(n)]
    assert ref == gold["variants"]["float"][str(n)]
    got = _run(n, dict(model="7b", cuts=ref["cuts"], seed=gold["seed"], wire="float16",
                       prompt_len=gold["prompt_tokens"], prompt_seeds=[r["prompt_seed"] for r in ref["runs"]],
                       steps=gold["generated"] - 1))
    assert got == [r["tokens"] for r in ref["runs"]]


@pytest.mark.gpu
def test_7b_pipeline_fp32_wire_matches_unsplit_reference():
    """With the hidden state sent in fp32 the two-stage pipeline computes the
    unsplit model: 128 greedy tokens identical to the reference's NumPy
    backend (both kernel builds), two identical streams interleaved."""
    gold = json.load(open(os.path.join(GOLDEN_DIR, "golden_7b.json")))
    prompt = synth.prompt_ids(gold["seed"], gold["prompt_tokens"], synth.QWEN2_7B["vocab_size"])
    assert [int(i) for i in prompt.reshape(-1)] == gold["prompt"]
    got = _run(2, dict(model="7b", cuts=[0, 14, 28], seed=gold["seed"], wire="float32",
                       prompt_len=gold["prompt_tokens"], prompt_seeds=[gold["seed"]] * 2,
                       steps=gold["generated"] - 1))
    for v in ("avx2", "float"):
        ref = [s["token"] for s in gold["variants"][v]["steps"]]
        assert got[0] == ref and got[1] == ref, v

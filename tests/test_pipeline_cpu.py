"""The pipelined decode (hetero_infer_b200/pipeline.py) on CPU ranks over gloo,
with the NumPy stage oracle as the compute: the schedule, the grouped
send/recv of the wire, the broadcast + row-sharded head + all-gather must
give every microbatch the tokens of a single-process run of the same stages
joined by the reference's fp16 wire (hetero/backends.py:100-104) or its int8
codec (hetero/transport.py:198-225)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from hetero_infer_b200 import pipeline, synth
from tests._oracle_compute import OracleCompute

CFG = dict(layers=3, hidden=256, heads=4, kv_heads=2, inter=512, vocab=1000)
SEED, N_MICRO, PROMPT, STEPS = 4, 3, 5, 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def reference_tokens(cuts, wire="float16"):
    """Single process: stage slices joined by the wire (the reference's fp16
    conversion, or its int8 codec), full head."""
    from oracle import codec
    from oracle import stage as ost
    cfg = synth.small_config(**CFG)
    w = synth.model_weights(cfg, SEED)
    rows = lambda ids: synth.embed_rows(SEED, ids, cfg["hidden_size"])
    stages = [ost.OracleStage(cfg, w, a, b, i == 0, i == len(cuts) - 2, embed_rows=rows)
              for i, (a, b) in enumerate(zip(cuts[:-1], cuts[1:]))]
    out = []
    for m in range(N_MICRO):
        caches = [s.new_caches() for s in stages]
        x = synth.prompt_ids(100 + m, PROMPT, cfg["vocab_size"])
        toks = []
        for _ in range(STEPS + 1):
            h = x
            for i, s in enumerate(stages):
                h = s(h, caches[i], apply_head=True, last_only=True)
                if i < len(stages) - 1 and wire == "int8":
                    # engine.py:97: transport.encode(backend.to_wire(y), "int8")
                    h = np.asarray(h, np.float16).astype(np.float32)
                    h = codec.decode_i8(codec.encode_i8(h), h.shape).astype(np.float32)
                elif i < len(stages) - 1:
                    h = np.asarray(h, np.float16).astype(np.float32)
            toks.append(int(np.asarray(h)[0, -1].argmax()))
            x = np.array([[toks[-1]]])
        out.append(toks)
    return out


def _rank_main(rank, world, port, cuts, q, wire="float16"):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = synth.small_config(**CFG)
        a, b = cuts[rank], cuts[rank + 1]
        w = synth.model_weights(cfg, SEED, layers=range(a, b), embed=(rank == 0), head=True)
        comp = OracleCompute(cfg, a, b, w, pipeline.head_rows(cfg["vocab_size"], world, rank),
                             embed_rows=lambda ids: synth.embed_rows(SEED, ids, cfg["hidden_size"]),
                             wire=wire)
        pr = pipeline.PipelineRank(pipeline.Comm(rank, world, torch.device("cpu")), comp, N_MICRO)
        pr.prefill([synth.prompt_ids(100 + m, PROMPT, cfg["vocab_size"]) for m in range(N_MICRO)])
        pr.decode(STEPS)
        q.put((rank, pr.tokens))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cuts,wire", [([0, 2, 3], "float16"), ([0, 1, 2, 3], "float16"), ([0, 1, 2, 3], "int8")])
def test_gloo_pipeline_matches_single_process(cuts, wire):
    world = len(cuts) - 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, cuts, q, wire)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = reference_tokens(cuts, wire)
    for r in range(world):
        assert got[r] == ref, f"rank {r}"


def _rank_leaves_main(rank, world, port, q):
    """Every rank prefills; then the last rank leaves (between steps, with
    nothing of its own in flight) and the others start decoding.  Each
    survivor reports the exception its next collective raised and how long
    that took; the process group's timeout is the outer bound."""
    import datetime
    import time
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    cfg = synth.small_config(**CFG)
    cuts = [0, 1, 2, 3]
    a, b = cuts[rank], cuts[rank + 1]
    w = synth.model_weights(cfg, SEED, layers=range(a, b), embed=(rank == 0), head=True)
    comp = OracleCompute(cfg, a, b, w, pipeline.head_rows(cfg["vocab_size"], world, rank),
                         embed_rows=lambda ids: synth.embed_rows(SEED, ids, cfg["hidden_size"]))
    pr = pipeline.PipelineRank(pipeline.Comm(rank, world, torch.device("cpu")), comp, N_MICRO)
    pr.prefill([synth.prompt_ids(100 + m, PROMPT, cfg["vocab_size"]) for m in range(N_MICRO)])
    dist.barrier()
    if rank == world - 1:
        q.put((rank, "left", 0.0))
    else:
        t0 = time.perf_counter()
        try:
            pr.decode(STEPS)
            q.put((rank, "no error", time.perf_counter() - t0))
        except Exception as e:  # noqa: BLE001 -- the test checks which
            q.put((rank, type(e).__name__, time.perf_counter() - t0))
    q.close()
    q.join_thread()
    os._exit(0)  # no teardown handshake with a group that lost a member


def test_gloo_pipeline_rank_leaving_raises_on_survivors():
    """A stage that goes away is reported to the others as an error from their
    next collective, within the process group's timeout, not as a hang (the
    reference's transport surfaces a lost peer as ConnectionError,
    hetero/transport.py:80-81,148-150)."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_leaves_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, what, dt = q.get(timeout=240)
        got[r] = (what, dt)
    for p in procs:
        p.join(timeout=60)
    assert got[world - 1][0] == "left"
    for r in range(world - 1):
        what, dt = got[r]
        assert what not in ("no error",), f"rank {r} finished decoding without its peer"
        assert dt < 60.0, f"rank {r} took {dt:.1f} s to notice"


@pytest.mark.parametrize("micro,steps,stages", [(4, 5, 2), (4, 3, 8), (8, 4, 8), (1, 3, 4), (3, 1, 2)])
def test_admission_schedule(micro, steps, stages):
    adm = pipeline.admission_schedule(micro, steps, stages)
    assert sum(1 for m in adm if m >= 0) == micro * steps
    last = {}
    for t, m in enumerate(adm):
        if m >= 0:
            assert m not in last or t - last[m] >= stages   # previous token known
            last[m] = t
    if micro >= stages:
        assert all(m >= 0 for m in adm)                     # pipeline stays full


def test_pick_token_tie_rule():
    import torch
    pairs = torch.tensor([[3.0, 700.0], [5.0, 12.0], [5.0, 3.0], [1.0, 0.0]], dtype=torch.float64)
    assert pipeline.pick_token(pairs) == 3


def test_pick_token_is_numpy_argmax_over_shards():
    """Per-shard (numpy argmax value, global index) pairs reduce to numpy's
    argmax over the concatenated vocabulary, NaN and -inf included."""
    import torch
    rng = np.random.default_rng(11)
    for trial in range(300):
        n = int(rng.integers(2, 40))
        z = np.round(rng.standard_normal(n) * 2).astype(np.float32)
        kind = trial % 5
        if kind == 1:
            z[rng.integers(0, n, size=int(rng.integers(1, 3)))] = np.nan
        elif kind == 2:
            z[:] = -np.inf
        elif kind == 3:
            z[:] = np.nan
        elif kind == 4:
            z[rng.integers(0, n)] = np.inf
        world = int(rng.integers(1, min(n, 8) + 1))
        rows = []
        for r in range(world):
            lo, hi = pipeline.head_rows(n, world, r)
            i = int(z[lo:hi].argmax())
            rows.append([float(z[lo + i]), float(lo + i)])
        assert pipeline.pick_token(torch.tensor(rows, dtype=torch.float64)) == int(z.argmax()), (z, world)

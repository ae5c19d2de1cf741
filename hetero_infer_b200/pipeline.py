"""Pipelined decode across the GPUs of one box (one process per GPU).

The reference pipelines a model over machines: each node runs a contiguous
slice of layers, hidden states travel to the next node as fp16 frames over
TCP, and several requests in flight keep every stage busy
(hetero/engine.py:68-147, hetero/transport.py:86-225,
hetero/coordinator.py:294-325).  Here the nodes are GPUs of one NVSwitch box
and the transport is NCCL over NVLink:

* stage i holds layers [cuts[i], cuts[i+1]) of the plan (planner.py); stage 0
  also embeds;
* per tick, one grouped NCCL send/recv moves the fp16 hidden state
  (hetero/backends.py:100-104 wire format, 7168 B per token for the 7B shape)
  from every stage to the next -- grouped, so no rank waits on a send whose
  receiver is still busy with a collective;
* the vocabulary projection is row-sharded over all stages: the last stage's
  fp32 hidden state is broadcast, every rank computes V/N logits and their
  (max, first index), and an 8-byte-per-rank all-gather picks the token with
  numpy's argmax rule (largest value, lowest index).  On GPUs these run on a
  side stream over a second communicator, so the collectives join the ranks
  off the layers' critical path: the next tick's send/recv and layers go
  ahead, and only rank 0, when it feeds a stream's token back in (one tick
  later at the earliest), waits for that stream's head;
* microbatches are independent requests with their own KV caches.  Rank 0
  admits, each tick, the next microbatch (round robin) whose previous token is
  known; stage i works on what rank 0 admitted i ticks earlier.  The schedule
  is a pure function of (microbatches, steps, stages), so every rank computes
  it and the send/recv pairs match without any control messages.

The runner is written against a small compute interface so the same schedule
and communication run on GPUs (NCCL, device stage) and in CPU tests (gloo,
the NumPy stage oracle).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist


def admission_schedule(n_micro: int, n_steps: int, n_stages: int) -> List[int]:
    """Microbatch rank 0 admits at each tick (-1: none) for `n_steps` decode
    steps per microbatch.  A microbatch admitted at tick t has its next token
    at the end of tick t + n_stages - 1, so it is admissible again at
    t + n_stages."""
    ready = [0] * n_micro
    left = [n_steps] * n_micro
    out: List[int] = []
    nxt, t = 0, 0
    while any(left):
        pick = -1
        for j in range(n_micro):
            m = (nxt + j) % n_micro
            if left[m] > 0 and ready[m] <= t:
                pick = m
                break
        out.append(pick)
        if pick >= 0:
            left[pick] -= 1
            ready[pick] = t + n_stages
            nxt = (pick + 1) % n_micro
        t += 1
    return out


_SIDE_GROUPS: Dict[int, object] = {}


class Comm:
    """The few torch.distributed operations the pipeline uses."""

    def __init__(self, rank: int, world: int, device: torch.device, group=None):
        self.rank, self.world, self.device, self.group = rank, world, device, group

    def side(self) -> "Comm":
        """The same ranks over a second communicator (created once per base
        group, on every rank in the same order), for collectives issued on
        another CUDA stream: NCCL orders the operations of one communicator,
        so two streams must not share one."""
        key = id(self.group)
        if key not in _SIDE_GROUPS:
            _SIDE_GROUPS[key] = dist.new_group(list(range(self.world)))
        return Comm(self.rank, self.world, self.device, group=_SIDE_GROUPS[key])

    def exchange(self, send: Optional[torch.Tensor], recv: Optional[torch.Tensor]) -> None:
        """Send to rank+1 and/or receive from rank-1 as one group."""
        ops = []
        if send is not None:
            ops.append(dist.P2POp(dist.isend, send, self.rank + 1, group=self.group))
        if recv is not None:
            ops.append(dist.P2POp(dist.irecv, recv, self.rank - 1, group=self.group))
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()

    def broadcast(self, t: torch.Tensor, src: int) -> None:
        dist.broadcast(t, src, group=self.group)

    def all_gather_into(self, out: torch.Tensor, t: torch.Tensor) -> None:
        """all_gather into a caller buffer [world, *t.shape] (NCCL)."""
        dist.all_gather_into_tensor(out, t, group=self.group)

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        if dist.get_backend(self.group) == "nccl":
            out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(out, t, group=self.group)
            return out
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t, group=self.group)
        return torch.stack(parts)


def pick_token(pairs: torch.Tensor) -> int:
    """Global argmax from per-shard (value, global index) rows, each the numpy
    argmax of its contiguous shard: numpy argmax over the whole vocabulary,
    i.e. the first NaN if any shard holds one, else the largest value, lowest
    index among equals."""
    p = pairs.double().cpu().numpy()
    vals, idx = p[:, 0], p[:, 1]
    nan = np.isnan(vals)
    if nan.any():
        return int(idx[nan].min())
    return int(idx[vals == vals.max()].min())


class PipelineRank:
    """One rank's side of the pipelined decode.

    compute: object with
      hidden_dim, wire_empty(rows) -> receive buffer of the wire format on the
      comm device (fp16 is the reference's format; fp32 and the reference's
      int8 codec are the others),
      new_cache(), embed_forward(ids, cache) -> h, forward(h, cache) -> h,
      to_wire(h) -> wire tensor on the comm device, from_wire(t) -> h,
      to_comm32(h_last) -> fp32 [H] tensor on the comm device,
      head(h32) -> (max value, global index) of this rank's vocabulary shard.
    """

    def __init__(self, comm: Comm, compute, n_micro: int, max_tokens: int = 4096, graphs: bool = True):
        self.comm, self.c, self.n_micro = comm, compute, n_micro
        self.caches = [compute.new_cache() for _ in range(n_micro)]
        self.ticks = 0
        # Device compute keeps the sampled tokens on the device (a history per
        # microbatch, read back once by `tokens`); no host sync per tick.
        self.on_device = getattr(compute, "device_tokens", False)
        if self.on_device:
            self.hist = torch.zeros((n_micro, max_tokens), dtype=torch.int32, device=comm.device)
            self.count = [0] * n_micro
        else:
            self._tokens: List[List[int]] = [[] for _ in range(n_micro)]
        # device compute over several GPUs: the head on a side stream and
        # communicator; tok_ev[m] marks stream m's latest token in the history
        self.async_head = self.on_device and comm.world > 1
        if self.async_head:
            dev = comm.device
            self.hcomm = comm.side()
            self.hstream = torch.cuda.Stream(dev)
            self.hbuf = torch.empty((n_micro, compute.hidden_dim), dtype=torch.float32, device=dev)
            self.tok_ev: List[Optional[torch.cuda.Event]] = [None] * n_micro
            # the token of stream m goes to tokdst[m] (on rank 0 the input
            # buffer of m's step) and to hist[m][cnt[m]] (device counter)
            self.cnt = torch.zeros(n_micro, dtype=torch.int32, device=dev)
            self.gat = torch.empty((comm.world, 2), dtype=torch.int32, device=dev)
            self.tokdst = ([compute.statics(m, True, self.last)[0] for m in range(n_micro)] if self.first else
                           [t for t in torch.zeros((n_micro, 1), dtype=torch.int32, device=dev)])
        # decode ticks replayed from CUDA graphs (device compute, several GPUs)
        self.graphs = graphs and self.async_head
        self._tick_g: Dict[tuple, torch.cuda.CUDAGraph] = {}
        self._head_g: Dict[int, torch.cuda.CUDAGraph] = {}

    @property
    def tokens(self) -> List[List[int]]:
        if self.on_device:
            if self.async_head:
                torch.cuda.current_stream(self.comm.device).wait_stream(self.hstream)
            h = self.hist.cpu().numpy()
            return [[int(v) for v in h[m, :self.count[m]]] for m in range(self.n_micro)]
        return self._tokens

    def _record(self, m: int, tok) -> None:
        if self.on_device:
            self.count[m] += 1
        else:
            self._tokens[m].append(tok)

    def _last_token(self, m: int):
        if self.on_device:
            return self.hist[m, self.count[m] - 1:self.count[m]].view(1, 1)
        return np.array([[self._tokens[m][-1]]])

    @property
    def first(self) -> bool:
        return self.comm.rank == 0

    @property
    def last(self) -> bool:
        return self.comm.rank == self.comm.world - 1

    def _head(self, h_last, m: int):
        """Broadcast the last stage's final hidden state, row-sharded head,
        all-gather of (max, index) -> the token of microbatch m (identical on
        every rank).  Device compute: the token goes straight into the device
        history; host compute: returned as an int."""
        if self.async_head:
            return self._head_side(h_last, m)
        H = self.c.hidden_dim
        buf = self.c.to_comm32(h_last) if self.last else torch.empty(H, dtype=torch.float32,
                                                                        device=self.comm.device)
        self.comm.broadcast(buf, self.comm.world - 1)
        if self.on_device:
            pairs = self.comm.all_gather(self.c.head_pair(buf))
            self.c.pick_into(pairs, self.comm.world, self.hist[m], self.count[m])
            return None
        val, idx = self.c.head(buf)
        pair = torch.tensor([val, float(idx)], dtype=torch.float64, device=self.comm.device)
        return pick_token(self.comm.all_gather(pair))

    def close(self) -> None:
        """Drop the CUDA graphs that hold NCCL calls (before the process group
        is destroyed, which would otherwise wait for them)."""
        self._tick_g = {}
        self._head_g = {}

    def _head_ops(self, m: int, h_last=None) -> None:
        """The head of stream m on the current (side) stream: the final row
        into hbuf[m] (last rank), broadcast, this rank's shard and its pick,
        all-gather, the global pick into tokdst[m] and hist[m][cnt[m]]."""
        buf = self.hbuf[m]
        if self.last:
            src = h_last if h_last is not None else self.c.statics(m, self.first, True)[2]
            buf.copy_(self.c.to_comm32(src))
        self.hcomm.broadcast(buf, self.comm.world - 1)
        self.hcomm.all_gather_into(self.gat, self.c.head_pair(buf))
        self.c.pick_next(self.gat, self.comm.world, self.tokdst[m], self.hist[m], self.cnt[m:m + 1])

    def _head_side(self, h_last, m: int) -> None:
        """_head on the side stream: after this rank's work so far on the main
        stream (the last stage's final hidden row), the head of stream m;
        tok_ev[m] records its completion.  hbuf[m] is stream m's own buffer and
        the side stream runs the heads in order, so no head overwrites what an
        earlier one still reads.  Within graph-replayed decode the head is a
        graph of its own per stream, captured on its first use."""
        main = torch.cuda.current_stream(self.comm.device)
        ready = torch.cuda.Event()
        ready.record(main)
        with torch.cuda.stream(self.hstream):
            self.hstream.wait_event(ready)
            if h_last is None and self.graphs:
                g = self._head_g.get(m)
                if g is None:
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=self.hstream, capture_error_mode="thread_local"):
                        self._head_ops(m)
                    self._head_g[m] = g
                g.replay()
            else:
                self._head_ops(m, h_last)
            done = torch.cuda.Event()
            done.record(self.hstream)
        self.tok_ev[m] = done
        return None

    def _tick_ops(self, send: int, mine: int) -> None:
        """One tick of this rank on the current stream: send stream `send`'s
        wire output to rank+1 and receive stream `mine`'s input from rank-1 (one
        group), then `mine`'s step."""
        c, r = self.c, self.comm.rank
        ops = []
        if send >= 0:
            ops.append(dist.P2POp(dist.isend, c.statics(send, self.first, self.last)[1], r + 1,
                                  group=self.comm.group))
        if mine >= 0 and r > 0:
            ops.append(dist.P2POp(dist.irecv, c.statics(mine, self.first, self.last)[0], r - 1,
                                  group=self.comm.group))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        if mine >= 0:
            c.record_step(mine, self.caches[mine], self.first, self.last)

    def _decode_graphed(self, n_steps: int) -> None:
        """decode() with every tick one CUDA-graph replay per rank (its
        send/recv and step, captured the first time each (send, receive)
        pair occurs) and each finished stream's head one more on the side
        stream: the host issues a few graph launches per tick instead of the
        tick's dozens of launches and NCCL calls.  Rank 0 waits for a
        stream's head (its token is written into the step's input buffer)
        before that stream's next step."""
        W, r = self.comm.world, self.comm.rank
        main = torch.cuda.current_stream(self.comm.device)
        adm = admission_schedule(self.n_micro, n_steps, W)
        n_ticks = len(adm) + W - 1
        prev = -1
        for t in range(n_ticks):
            mine = adm[t - r] if 0 <= t - r < len(adm) else -1
            send = -1 if self.last else prev
            if mine >= 0:
                cache = self.caches[mine]
                if cache.offset + 1 > cache.max_ctx:
                    raise ValueError(f"context {cache.offset + 1} exceeds max_ctx {cache.max_ctx}")
                if self.first and self.tok_ev[mine] is not None:
                    main.wait_event(self.tok_ev[mine])
            if mine >= 0 or send >= 0:
                key = (send, mine)
                g = self._tick_g.get(key)
                if g is None:  # captured on a side stream (the default stream cannot capture)
                    cap = torch.cuda.Stream(self.comm.device)
                    cap.wait_stream(main)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=cap, capture_error_mode="thread_local"):
                        self._tick_ops(send, mine)
                    main.wait_stream(cap)
                    self._tick_g[key] = g
                g.replay()
                if mine >= 0:
                    self.caches[mine].offset += 1  # the graph advanced the device position
            done = adm[t - (W - 1)] if 0 <= t - (W - 1) < len(adm) else -1
            if done >= 0:
                self._head_side(None, done)
                self._record(done, None)
            prev = mine
        self.ticks += n_ticks

    def prefill(self, prompts: Sequence[np.ndarray]) -> None:
        """Each prompt [1, P] through the stages one after another; the first
        generated token of every microbatch comes from the sharded head."""
        W, r = self.comm.world, self.comm.rank
        for m, prompt in enumerate(prompts):
            P = int(np.asarray(prompt).shape[-1])
            h = None
            for s in range(W):   # stage s computes at sub-tick s
                if r == s:
                    if self.first:
                        h = self.c.embed_forward(np.asarray(prompt).reshape(1, P), self.caches[m])
                    else:
                        h = self.c.forward(self.c.from_wire(wire_in), self.caches[m])
                    if not self.last:
                        self.comm.exchange(self.c.to_wire(h), None)
                elif r == s + 1:
                    wire_in = self.c.wire_empty(P)
                    self.comm.exchange(None, wire_in)
            self._record(m, self._head(h if self.last else None, m))

    def decode(self, n_steps: int) -> None:
        """n_steps more tokens for every microbatch, pipelined."""
        if self.graphs:
            return self._decode_graphed(n_steps)
        W, r = self.comm.world, self.comm.rank
        adm = admission_schedule(self.n_micro, n_steps, W)
        n_ticks = len(adm) + W - 1
        H = self.c.hidden_dim
        out_prev = None       # this rank's wire output of the previous tick
        for t in range(n_ticks):
            # this rank works on what rank 0 admitted r ticks ago -- which is
            # also what rank r-1 worked on (and sends now) one tick ago
            mine = adm[t - r] if 0 <= t - r < len(adm) else -1
            recv = None
            if r > 0 and mine >= 0:
                recv = self.c.wire_empty(1)
            self.comm.exchange(out_prev if (not self.last and out_prev is not None) else None, recv)
            out_prev = None
            h = None
            if mine >= 0:
                if self.first and self.async_head and self.tok_ev[mine] is not None:
                    torch.cuda.current_stream(self.comm.device).wait_event(self.tok_ev[mine])
                src = self._last_token(mine) if self.first else recv
                wire, h = self.c.decode_tick(mine, self.caches[mine], src, self.first, self.last)
                if not self.last:
                    out_prev = wire
            # head of the microbatch the last stage finished this tick
            done = adm[t - (W - 1)] if 0 <= t - (W - 1) < len(adm) else -1
            if done >= 0:
                self._record(done, self._head(h if self.last else None, done))
        self.ticks += n_ticks


# ---------------------------------------------------------------------------
# compute adapters
# ---------------------------------------------------------------------------

class DeviceCompute:
    """Stage slice on this rank's GPU plus its row shard of the vocabulary
    projection (libhq4 kernels: the stage forward, the norm-fused head GEMV,
    argmax with value).

    wire: "float16" is the reference's hand-off (backends.py:100-104; values
    beyond fp16 range become inf there and here alike); "int8" is the
    reference's int8 codec (transport.py:198-225: per-row fp32 scale + int8,
    half the bytes) applied, as its engine applies it (engine.py:97), to the
    fp16 wire array; encoded and decoded on the device, bit-identical to the
    NumPy codec; "float32" sends the fp32 hidden state unchanged, so the
    pipelined model computes exactly what one unsplit stage computes (not a
    reference format)."""

    def __init__(self, cfg: dict, spec, weights: Dict[str, np.ndarray], head_rows: tuple,
                 device: torch.device, max_ctx: int = 1024, wire: str = "float16"):
        from . import _lib, cuda_model
        if wire not in ("float16", "float32", "int8"):
            raise ValueError(f"wire must be float16, float32 or int8, not {wire!r}")
        self.wire = wire
        self.wire_dtype = torch.uint8 if wire == "int8" else getattr(torch, wire)
        self.cfg, self.device = cfg, device
        self.hidden_dim = cfg["hidden_size"]
        self.stage = cuda_model.Stage(cfg, spec, weights, device=device, max_ctx=max_ctx)
        lo, hi = head_rows
        self.lo, self.hi = lo, hi
        gs = cfg["quantization"]["group_size"]
        self.gs = gs
        self.lm_w = cuda_model._dev_array(weights["lm_head.weight"][lo:hi], device=device)
        self.lm_s = cuda_model._dev_array(weights["lm_head.scales"][lo:hi], torch.float16, device)
        self.lm_b = cuda_model._dev_array(weights["lm_head.biases"][lo:hi], torch.float16, device)
        self.norm_w = cuda_model._dev_array(np.asarray(weights["model.norm.weight"], np.float32),
                                            torch.float32, device)
        self.logits = torch.empty(hi - lo, dtype=torch.float32, device=device)
        self.idx = torch.empty(1, dtype=torch.int32, device=device)
        self.val = torch.empty(1, dtype=torch.float32, device=device)
        self.pair = torch.empty(2, dtype=torch.int32, device=device)
        self.tok = torch.empty(1, dtype=torch.int32, device=device)
        self._graphs = {}
        self._static = {}
        self.lib = _lib.load()
        self._check = _lib.check

    def new_cache(self):
        return self.stage.new_caches()

    def release_graphs(self) -> None:
        """Drop the per-microbatch decode graphs and their buffers (they are
        bound to the caches of the runner that captured them); a new runner
        captures its own."""
        self._graphs = {}
        self._static = {}

    def statics(self, m, first: bool, last: bool):
        """Microbatch m's fixed step buffers on this stage, created once: the
        input (a token id on the first stage, else a wire frame), the wire
        output (none on the last stage) and the final hidden row."""
        sb = self._static.get(m)
        if sb is None:
            static_in = (torch.zeros((1, 1), dtype=torch.int32, device=self.device) if first
                         else self.wire_empty(1).zero_())
            static_wire = None if last else self.wire_empty(1)
            static_h = torch.empty((1, 1, self.hidden_dim), dtype=torch.float32, device=self.device)
            sb = self._static[m] = (static_in, static_wire, static_h)
        return sb

    def record_step(self, m, cache, first: bool, last: bool) -> None:
        """Microbatch m's decode step on the current stream, from its input
        buffer to its wire output and final row (eagerly or into a capture):
        embedding or wire decode, the stage's layers, the position advance."""
        st = self.stage
        H = self.hidden_dim
        static_in, static_wire, static_h = self.statics(m, first, last)
        h = st.embed(static_in) if first else self.from_wire(static_in)
        h = h.reshape(1, H).contiguous()
        for i in range(len(st.layers)):
            st.layer_forward(i, h, cache, 1)
        if len(st.layers):
            st._check(st.lib.hq4_advance_position(cache.pos.data_ptr(), 1, st._stream()), "hq4_advance_position")
        if static_wire is not None:
            self._encode_into(h, static_wire)
        static_h.copy_(h.view(1, 1, H))

    def embed_forward(self, ids, cache):
        return self.stage(ids, cache, apply_head=False)

    def forward(self, h, cache):
        return self.stage(h, cache, apply_head=False)

    def decode_tick(self, m, cache, src, first: bool, last: bool):
        """One decode token of microbatch m through this stage: token id (first
        stage) or wire hidden state in, wire hidden state (or, on the last
        stage, the final hidden row) out.  The first tick of a microbatch runs
        eagerly and records the step as a CUDA graph (its KV cache and device
        position are fixed per microbatch); later ticks copy the input into the
        graph's buffer and replay it -- one launch instead of five per layer."""
        g = self._graphs.get(m)
        if g is None:
            h = self.embed_forward(src, cache) if first else self.forward(self.from_wire(src), cache)
            self._graphs[m] = self._capture(m, cache, first, last)
            return (None if last else self.to_wire(h)), h
        static_in, static_wire, static_h, graph = g
        if cache.offset + 1 > cache.max_ctx:
            raise ValueError(f"context {cache.offset + 1} exceeds max_ctx {cache.max_ctx}")
        static_in.copy_(src.reshape(static_in.shape))
        graph.replay()
        cache.offset += 1  # the graph advanced the device position
        return static_wire, static_h

    def _capture(self, m, cache, first: bool, last: bool):
        static_in, static_wire, static_h = self.statics(m, first, last)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side, capture_error_mode="thread_local"):
            self.record_step(m, cache, first, last)
        torch.cuda.current_stream(self.device).wait_stream(side)
        return static_in, static_wire, static_h, graph

    def wire_empty(self, rows: int) -> torch.Tensor:
        H = self.hidden_dim
        if self.wire == "int8":
            return torch.empty(rows * (4 + H), dtype=torch.uint8, device=self.device)
        return torch.empty((1, rows, H), dtype=self.wire_dtype, device=self.device)

    def _encode_into(self, h, dst):
        if self.wire == "int8":
            from . import ops
            ops.act_encode_i8(h.reshape(-1, self.hidden_dim), payload=dst, wire=True)
        else:
            dst.copy_(h.view(dst.shape).to(self.wire_dtype))

    def to_wire(self, h):
        rows = h.numel() // self.hidden_dim
        t = self.wire_empty(rows)
        self._encode_into(h.contiguous(), t)
        return t

    def from_wire(self, t):
        H = self.hidden_dim
        if self.wire == "int8":
            from . import ops
            rows = t.numel() // (4 + H)
            return ops.act_decode_i8(t, rows, H, dtype=torch.float32).view(1, rows, H)
        return t.to(torch.float32)

    def to_comm32(self, h):
        return h.reshape(-1, self.hidden_dim)[-1].contiguous()

    device_tokens = True

    def head_pair(self, h32):
        """This rank's shard of the vocabulary projection and its greedy pick as
        an (value bits, global index) int32 pair on the device."""
        st = torch.cuda.current_stream(self.device).cuda_stream
        self._check(self.lib.hq4_gemv_norm(self.lm_w.data_ptr(), self.lm_s.data_ptr(), self.lm_b.data_ptr(),
                                           h32.data_ptr(), self.logits.data_ptr(), self.hi - self.lo,
                                           self.hidden_dim, self.gs, 1, self.norm_w.data_ptr(),
                                           float(self.cfg["rms_norm_eps"]), 0, None, None, st), "head")
        self._check(self.lib.hq4_argmax_pair(self.logits.data_ptr(), self.hi - self.lo, self.lo,
                                             self.pair.data_ptr(), st), "argmax_pair")
        return self.pair

    def pick_next(self, pairs, world: int, tok, history_row, count) -> None:
        """Global token from the gathered pairs into tok[0] and
        history_row[count[0]]; count[0] advances (device counter)."""
        st = torch.cuda.current_stream(self.device).cuda_stream
        self._check(self.lib.hq4_pick_token_next(pairs.data_ptr(), world, tok.data_ptr(), history_row.data_ptr(),
                                                 count.data_ptr(), history_row.numel(), st), "pick_token_next")

    def pick_into(self, pairs, world: int, history_row, slot: int):
        """Global token from the gathered pairs, written to history_row[slot]."""
        st = torch.cuda.current_stream(self.device).cuda_stream
        self._check(self.lib.hq4_pick_token(pairs.data_ptr(), world, self.tok.data_ptr(), history_row.data_ptr(),
                                            slot, st), "pick_token")

    def head(self, h32):
        from ._lib import expect
        expect(h32, self.hidden_dim * 4, "head x", 16)
        expect(self.logits, (self.hi - self.lo) * 4, "shard logits")
        expect(self.lm_w, (self.hi - self.lo) * self.hidden_dim // 2, "lm shard w", 32)
        st = torch.cuda.current_stream(self.device).cuda_stream
        self._check(self.lib.hq4_gemv_norm(self.lm_w.data_ptr(), self.lm_s.data_ptr(), self.lm_b.data_ptr(),
                                           h32.data_ptr(), self.logits.data_ptr(), self.hi - self.lo,
                                           self.hidden_dim, self.gs, 1, self.norm_w.data_ptr(),
                                           float(self.cfg["rms_norm_eps"]), 0, None, None, st), "head")
        self._check(self.lib.hq4_argmax(self.logits.data_ptr(), self.hi - self.lo, self.idx.data_ptr(), None, 0,
                                        None, self.val.data_ptr(), st), "argmax")
        return float(self.val.item()), self.lo + int(self.idx.item())


def head_rows(vocab: int, world: int, rank: int) -> tuple:
    """Row range of the vocabulary projection on `rank` (contiguous, balanced)."""
    return (vocab * rank // world, vocab * (rank + 1) // world)

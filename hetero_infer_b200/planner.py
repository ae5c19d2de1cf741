"""Where to cut the model across the GPUs of one box.

The reference cuts a model into contiguous layer slices over heterogeneous
machines with a dynamic programme over (node, cut) (hetero/planner.py:118-217):
objective `latency` sums stage times plus link crossings, `throughput` takes the
max over stages of compute plus outgoing communication, memory is a hard
constraint, and ties go to the split with the most memory headroom.  This
module keeps that procedure (restated; the cost model and tie-break are the
reference's, so plans agree with it on the same inputs -- tests/test_planner.py
checks that against the reference's own planner) and changes only its inputs
for one 8xB200 box:

* nodes are GPUs with measured per-layer decode time and an HBM budget;
* weight bytes come from the packed layout of a config (``ModelIndex``), not
  from safetensors headers -- it offers the part of WeightIndex's interface the
  planner reads (shard.py:72-134);
* the link is NVLink through NVSwitch (uniform to every peer);
* ``plan_gpu_pipeline`` can row-shard the vocabulary projection across all
  stages (its cost then lands on every stage as head_s / N) instead of placing
  it on one end of the ring.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import List, Optional


@dataclass(frozen=True)
class ShardSpec:
    """Layers [start, end) plus ownership of the embedding and the head
    (the reference's ShardSpec, hetero/shard.py:25-46)."""
    start: int
    end: int
    embed: bool
    head: bool

    @property
    def n_layers(self) -> int:
        return self.end - self.start

    def to_json(self) -> dict:
        return asdict(self)


@dataclass
class NodeProfile:
    """What one device brings (the reference's NodeProfile, planner.py:26-45)."""
    name: str
    mem_bytes: int = 0
    decode_s_per_layer: float = 0.0
    prefill_s_per_layer_token: float = 0.0
    embed_s: float = 0.0
    head_s: float = 0.0
    backend: str = "cuda"
    weight_expansion: float = 1.0


@dataclass
class LinkSpec:
    bandwidth_mbps: float = 7.2e6   # 900 GB/s NVLink 5 per direction
    rtt_ms: float = 0.02            # ~10 us one way for a small NCCL send

    def seconds_for(self, nbytes: int) -> float:
        return self.rtt_ms / 2000.0 + (nbytes * 8.0) / (self.bandwidth_mbps * 1e6)


@dataclass
class Plan:
    cuts: List[int]
    nodes: List[NodeProfile]
    head_node: int = -1             # -1: head row-sharded over every stage
    specs: List[ShardSpec] = field(default_factory=list)
    objective: str = "throughput"
    predicted_decode_s: float = 0.0
    stage_compute_s: List[float] = field(default_factory=list)
    stage_comm_s: List[float] = field(default_factory=list)
    stage_mem_bytes: List[int] = field(default_factory=list)

    def describe(self) -> str:
        lines = [f"plan[{self.objective}, head {'sharded' if self.head_node < 0 else self.head_node}] "
                 f"predicted {self.predicted_decode_s * 1e3:.3f} ms/token"]
        for i, (n, s) in enumerate(zip(self.nodes, self.specs)):
            lines.append(f"  stage {i} {n.name:<8} layers {s.start:>2}-{s.end - 1:<2} ({s.n_layers:>2}) "
                         f"mem {self.stage_mem_bytes[i] / 2**30:6.2f} GiB compute "
                         f"{self.stage_compute_s[i] * 1e6:8.1f} us")
        return "\n".join(lines)


def q4_bytes(n_out: int, n_in: int, gs: int, bias: bool = False) -> int:
    """Bytes of one packed int4 linear: words + fp16 scales + fp16 biases (+ bias)."""
    return n_out * n_in // 2 + 2 * n_out * (n_in // gs) * 2 + (2 * n_out if bias else 0)


class ModelIndex:
    """Weight bytes of a quantised qwen2 config, with the slice of the
    reference WeightIndex interface the planner uses."""

    def __init__(self, cfg: dict, qkv_bias: bool = True, embed_fp16: bool = True):
        self.config = cfg
        H, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
        hd = H // cfg["num_attention_heads"]
        kv = cfg["num_key_value_heads"] * hd
        gs = cfg["quantization"]["group_size"]
        self._layer = (q4_bytes(H, H, gs, qkv_bias) + 2 * q4_bytes(kv, H, gs, qkv_bias) + q4_bytes(H, H, gs)
                       + 2 * q4_bytes(I, H, gs) + q4_bytes(H, I, gs) + 2 * 2 * H)
        self._embed = V * H * 2 if embed_fp16 else q4_bytes(V, H, gs)
        self._head = q4_bytes(V, H, gs) + 2 * H

    @property
    def tied(self) -> bool:
        return bool(self.config.get("tie_word_embeddings", False))

    def layer_bytes(self) -> List[int]:
        return [self._layer] * int(self.config["num_hidden_layers"])

    def embed_bytes(self) -> int:
        return self._embed

    def head_bytes(self) -> int:
        return self._head

    def shard_bytes(self, spec) -> int:
        b = sum(self.layer_bytes()[spec.start:spec.end])
        if spec.embed:
            b += self._embed
        if spec.head:
            b += self._head
        return b

    def total_bytes(self) -> int:
        return sum(self.layer_bytes()) + self._embed + self._head


def kv_bytes_per_layer(cfg: dict, max_ctx: int, batch: int = 1, dtype_bytes: int = 4) -> int:
    """KV cache of one layer (fp32 on the device, as the reference's NumPy cache)."""
    n_kv = cfg.get("num_key_value_heads", cfg["num_attention_heads"])
    head_dim = cfg.get("head_dim", cfg["hidden_size"] // cfg["num_attention_heads"])
    return 2 * batch * n_kv * head_dim * max_ctx * dtype_bytes


def hidden_bytes(cfg: dict, tokens: int = 1, batch: int = 1, codec: str = "fp16") -> int:
    d = cfg["hidden_size"]
    if codec == "int8":
        return batch * tokens * (d + 4)
    return batch * tokens * d * 2


def _resident(index, spec, expansion: float) -> int:
    layer = sum(index.layer_bytes()[spec.start:spec.end])
    return int(layer * expansion + index.shard_bytes(spec) - layer)


def _stage_time(node: NodeProfile, spec: ShardSpec, head_share: float = 0.0) -> float:
    t = spec.n_layers * node.decode_s_per_layer
    if spec.embed:
        t += node.embed_s
    if spec.head:
        t += node.head_s
    return t + head_share


def plan_pipeline(index, nodes: List[NodeProfile], link: LinkSpec, objective: str = "throughput",
                  max_ctx: int = 4096, batch: int = 1, codec: str = "fp16",
                  kv_dtype_bytes: int = 2) -> Plan:
    """Head on stage N-1 or 0, whichever predicts faster (planner.py:118-140)."""
    best, best_cost, err = None, float("inf"), None
    for head_at in ({len(nodes) - 1, 0} if len(nodes) > 1 else {len(nodes) - 1}):
        try:
            p = _plan(index, nodes, link, head_at, objective, max_ctx, batch, codec, kv_dtype_bytes)
        except MemoryError as e:
            err = e
            continue
        if p.predicted_decode_s < best_cost:
            best, best_cost = p, p.predicted_decode_s
    if best is None:
        raise err
    return best


def _plan(index, nodes, link, head_at, objective, max_ctx, batch, codec, kv_dtype_bytes,
          sharded_head: bool = False) -> Plan:
    """The DP over cut points for one head placement (planner.py:143-217).

    head_at = -1 with sharded_head: no stage owns the whole head; every stage
    pays head_s / N and holds 1/N of its bytes."""
    cfg = index.config
    L = int(cfg["num_hidden_layers"])
    N = len(nodes)
    if N < 2:
        raise ValueError("need at least two nodes to split a model")
    kv = kv_bytes_per_layer(cfg, max_ctx, batch, kv_dtype_bytes)
    act = hidden_bytes(cfg, tokens=1, batch=batch, codec=codec)
    comm = link.seconds_for(act + 96)
    ret_comm = link.seconds_for(96)
    head_share_bytes = index.head_bytes() // N if sharded_head else 0
    INF = float("inf")
    best = [[INF] * (L + 1) for _ in range(N + 1)]
    # secondary key for the sharded-head GPU plan: sum of squared stage times,
    # so that among splits with the same slowest stage the balanced one wins
    # (identical GPUs tie on the throughput objective alone)
    sq = [[INF] * (L + 1) for _ in range(N + 1)]
    choice = [[-1] * (L + 1) for _ in range(N + 1)]
    best[N][L] = 0.0
    sq[N][L] = 0.0

    def combine(a, b):
        return max(a, b) if objective == "throughput" else a + b

    def mem(i, spec):
        return _resident(index, spec, nodes[i].weight_expansion) + spec.n_layers * kv + head_share_bytes

    # a row-sharded head costs every stage, every token, its share of the
    # head GEMV plus the two collectives that join the shards: the broadcast
    # of the last stage's fp32 hidden state and the all-gather of the N
    # (value, index) pairs
    head_coll = (link.seconds_for(int(cfg["hidden_size"]) * 4) + link.seconds_for(8 * N)) if sharded_head else 0.0

    def share(i):
        return nodes[i].head_s / N + head_coll if sharded_head else 0.0

    for i in range(N - 1, -1, -1):
        node = nodes[i]
        for c in range(L + 1):
            for c2 in range(c, L + 1):
                if best[i + 1][c2] == INF:
                    continue
                spec = ShardSpec(c, c2, i == 0, i == head_at)
                m = mem(i, spec)
                if m > node.mem_bytes:
                    continue
                out = (comm if head_at == 0 else ret_comm) if i == N - 1 else comm
                t = _stage_time(node, spec, share(i)) + out
                cost = combine(t, best[i + 1][c2])
                cost += 1e-12 * (m / node.mem_bytes) ** 8
                if sharded_head:
                    s2 = sq[i + 1][c2] + t * t
                    close = abs(cost - best[i][c]) <= 1e-9 * max(cost, 1e-30)
                    if cost < best[i][c] and not close or (close and s2 < sq[i][c]):
                        best[i][c], sq[i][c], choice[i][c] = cost, s2, c2
                elif cost < best[i][c]:
                    best[i][c] = cost
                    choice[i][c] = c2
    if best[0][0] == INF:
        raise MemoryError(f"no feasible split of {index.total_bytes() / 2**30:.2f} GiB over {N} nodes")
    cuts, c = [0], 0
    for i in range(N):
        c = choice[i][c]
        cuts.append(c)
    specs = [ShardSpec(cuts[i], cuts[i + 1], i == 0, i == head_at) for i in range(N)]
    plan = Plan(cuts=cuts, nodes=nodes, specs=specs, objective=objective, head_node=head_at)
    plan.stage_compute_s = [_stage_time(n, s, share(i)) for i, (n, s) in enumerate(zip(nodes, specs))]
    plan.stage_comm_s = [(comm if head_at == 0 else ret_comm) if i == N - 1 else comm for i in range(N)]
    plan.stage_mem_bytes = [mem(i, s) for i, s in enumerate(specs)]
    if objective == "throughput":
        plan.predicted_decode_s = max(a + b for a, b in zip(plan.stage_compute_s, plan.stage_comm_s))
    else:
        plan.predicted_decode_s = sum(plan.stage_compute_s) + sum(plan.stage_comm_s)
    return plan


def plan_gpu_pipeline(cfg: dict, n_gpus: int, layer_s: float, head_s: float = 0.0,
                      embed_s: float = 0.0, mem_bytes: int = 160 * 2**30,
                      objective: str = "throughput", max_ctx: int = 2048,
                      sharded_head: bool = True, link: Optional[LinkSpec] = None,
                      index=None, codec: str = "fp16") -> Plan:
    """Cut `cfg` over `n_gpus` identical GPUs of one box.  With sharded_head the
    vocabulary projection is row-sharded across every stage (each computes
    V/N logits and a local argmax, reduced by an all-gather; every stage pays
    its share and the two collectives per token).  `index` gives the weight
    bytes (a checkpoint.WeightIndex of a snapshot; by default they follow
    from the config); `codec` is the wire format ("fp16" or "int8")."""
    nodes = [NodeProfile(f"gpu{i}", mem_bytes=mem_bytes, decode_s_per_layer=layer_s, embed_s=embed_s,
                         head_s=head_s) for i in range(n_gpus)]
    index = index if index is not None else ModelIndex(cfg)
    link = link or LinkSpec()
    if n_gpus == 1:
        spec = ShardSpec(0, int(cfg["num_hidden_layers"]), True, True)
        return Plan(cuts=[0, spec.end], nodes=nodes, specs=[spec], objective=objective, head_node=0,
                    predicted_decode_s=_stage_time(nodes[0], spec), stage_compute_s=[_stage_time(nodes[0], spec)],
                    stage_comm_s=[0.0], stage_mem_bytes=[index.total_bytes()])
    if sharded_head:
        return _plan(index, nodes, link, -1, objective, max_ctx, 1, codec, 4, sharded_head=True)
    return plan_pipeline(index, nodes, link, objective, max_ctx, 1, codec, 4)

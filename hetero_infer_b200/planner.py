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
    """Head on the last stage or on stage 0, whichever predicts faster
    (planner.py:118-140); the placements are tried in the reference's order
    and the first of two equal predictions is kept."""
    best, err = None, None
    for head_at in _head_placements(len(nodes)):
        try:
            p = _plan(index, nodes, link, head_at, objective, max_ctx, batch, codec, kv_dtype_bytes)
        except MemoryError as e:
            err = e
            continue
        if best is None or p.predicted_decode_s < best.predicted_decode_s:
            best = p
    if best is None:
        raise err
    return best


def _head_placements(n: int) -> List[int]:
    # the reference iterates the set {n - 1, 0}; keep its iteration order
    return list({n - 1, 0}) if n > 1 else [n - 1]


class _StageCosts:
    """Every per-stage term of one head placement, shared by the cut search
    and by the finished plan: head_at is the stage owning the vocabulary
    projection, or -1 when it is row-sharded over all N stages (each then
    pays head_s / N, holds 1/N of its bytes and joins two collectives per
    token: the broadcast of the last stage's fp32 hidden state and the
    all-gather of the N (value, index) pairs)."""

    def __init__(self, index, nodes, link, head_at, max_ctx, batch, codec, kv_dtype_bytes, sharded):
        cfg = index.config
        self.index, self.nodes, self.head_at, self.sharded = index, nodes, head_at, sharded
        self.n = len(nodes)
        self.kv = kv_bytes_per_layer(cfg, max_ctx, batch, kv_dtype_bytes)
        self.hand_off = link.seconds_for(hidden_bytes(cfg, tokens=1, batch=batch, codec=codec) + 96)
        self.token_back = link.seconds_for(96)
        self.head_part = index.head_bytes() // self.n if sharded else 0
        self.head_coll = (link.seconds_for(int(cfg["hidden_size"]) * 4) + link.seconds_for(8 * self.n)
                          if sharded else 0.0)

    def spec(self, i: int, start: int, end: int) -> ShardSpec:
        return ShardSpec(start, end, i == 0, i == self.head_at)

    def mem(self, i: int, spec: ShardSpec) -> int:
        return _resident(self.index, spec, self.nodes[i].weight_expansion) + spec.n_layers * self.kv + self.head_part

    def compute(self, i: int, spec: ShardSpec) -> float:
        share = self.nodes[i].head_s / self.n + self.head_coll if self.sharded else 0.0
        return _stage_time(self.nodes[i], spec, share)

    def send(self, i: int) -> float:
        """What stage i ships on: a hidden state to the next stage; the last
        stage returns a token id, or a hidden state when stage 0 owns the head."""
        if i < self.n - 1 or self.head_at == 0:
            return self.hand_off
        return self.token_back


def _cut_search(costs: _StageCosts, n_layers: int, objective: str) -> List[int]:
    """Cut points [0, c1, ..., L] of the cheapest feasible split.

    A backward pass over the stages keeps, for every first layer c of the
    stages i.., the best (cost, sum of squared stage times, next cut).  A
    stage's cost is its time plus what it sends, combined with the rest by max
    (throughput) or sum (latency), plus 1e-12 (mem / budget)^8 so that equal
    costs go to the split with the most memory headroom; the first cut
    reaching the minimum wins, as in the reference (planner.py:180-205).  With
    a sharded head a near-tie is broken by the smaller sum of squared stage
    times, so identical GPUs get balanced stages."""
    join = max if objective == "throughput" else (lambda a, b: a + b)
    INF = float("inf")
    rest = {n_layers: (0.0, 0.0, None)}  # nothing left for the stages after the last
    tables = []
    for i in range(costs.n - 1, -1, -1):
        budget = costs.nodes[i].mem_bytes
        here = {}
        for c in range(n_layers + 1):
            cost_b, sq_b, cut_b = INF, INF, -1
            for c2 in range(c, n_layers + 1):
                after = rest.get(c2)
                if after is None:
                    continue
                spec = costs.spec(i, c, c2)
                m = costs.mem(i, spec)
                if m > budget:
                    continue
                t = costs.compute(i, spec) + costs.send(i)
                cost = join(t, after[0])
                cost += 1e-12 * (m / budget) ** 8
                if costs.sharded:
                    sq = after[1] + t * t
                    near = abs(cost - cost_b) <= 1e-9 * max(cost, 1e-30)
                    take = (cost < cost_b and not near) or (near and sq < sq_b)
                else:
                    sq, take = 0.0, cost < cost_b
                if take:
                    cost_b, sq_b, cut_b = cost, sq, c2
            if cut_b >= 0:
                here[c] = (cost_b, sq_b, cut_b)
        tables.append(here)
        rest = here
    if 0 not in rest:
        raise MemoryError(f"no feasible split of {costs.index.total_bytes() / 2**30:.2f} GiB over {costs.n} nodes")
    cuts = [0]
    for here in reversed(tables):  # stage 0 first
        cuts.append(here[cuts[-1]][2])
    return cuts


def _plan(index, nodes, link, head_at, objective, max_ctx, batch, codec, kv_dtype_bytes,
          sharded_head: bool = False) -> Plan:
    """The cut search for one head placement (planner.py:143-217).

    head_at = -1 with sharded_head: no stage owns the whole head; every stage
    pays head_s / N and holds 1/N of its bytes."""
    if len(nodes) < 2:
        raise ValueError("need at least two nodes to split a model")
    costs = _StageCosts(index, nodes, link, head_at, max_ctx, batch, codec, kv_dtype_bytes, sharded_head)
    cuts = _cut_search(costs, int(index.config["num_hidden_layers"]), objective)
    specs = [costs.spec(i, cuts[i], cuts[i + 1]) for i in range(len(nodes))]
    plan = Plan(cuts=cuts, nodes=nodes, specs=specs, objective=objective, head_node=head_at)
    plan.stage_compute_s = [costs.compute(i, s) for i, s in enumerate(specs)]
    plan.stage_comm_s = [costs.send(i) for i in range(len(nodes))]
    plan.stage_mem_bytes = [costs.mem(i, s) for i, s in enumerate(specs)]
    totals = [a + b for a, b in zip(plan.stage_compute_s, plan.stage_comm_s)]
    plan.predicted_decode_s = max(totals) if objective == "throughput" else (
        sum(plan.stage_compute_s) + sum(plan.stage_comm_s))
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

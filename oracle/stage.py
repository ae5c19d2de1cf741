"""CPU oracle of the qwen2 stage forward -- TEST INFRASTRUCTURE ONLY.

A restatement, in NumPy, of the reference's NumPy stage
(hetero/cpu_model.py:164-368) used as the checker for the device stage on the
GPU box, where the reference tree is absent.  The quantised products go
through the C oracle (oracle/q4_oracle.c, float path), dispatched as the
reference's QLinear dispatches them (cpu_model.py:145-158): up to 16 rows one
GEMV per row, more rows by an fp32 expansion and a float32 matmul.  In the
build container tests/test_stage_oracle.py pins this file against the
reference's own cpu_model.Stage run with the reference kernel built from
source.  Only tests/, __graft_entry__.smoke() and bench.py's CPU leg use it.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np

from .q4 import Oracle

GEMV_ROWS_MAX = 16          # cpu_model.py:30


class OLinear:
    """Quantised linear as the reference dispatches it (cpu_model.py:84-158)."""

    def __init__(self, orc: Oracle, w, s, b, bias, gs):
        self.orc, self.w, self.s, self.b, self.gs = orc, np.ascontiguousarray(w), s, b, gs
        self.bias = None if bias is None else np.asarray(bias, dtype=np.float32)
        self.n_out, self.n_in = w.shape[0], w.shape[1] * 8

    def __call__(self, x: np.ndarray) -> np.ndarray:
        flat = np.asarray(x, dtype=np.float32).reshape(-1, self.n_in)
        if flat.shape[0] <= GEMV_ROWS_MAX:
            out = self.orc.gemv_f32(self.w, self.s, self.b, flat, self.gs)
        else:
            W = self.orc.dequant(self.w, self.s, self.b, 0, self.n_out, self.gs)
            out = flat @ W.T
        if self.bias is not None:
            out = out + self.bias
        return out.reshape(*np.shape(x)[:-1], self.n_out)


def rms_norm(x, w, eps):
    x = x.astype(np.float32)
    r = np.float32(1.0) / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return x * r * w


def silu(x):
    return x / (np.float32(1.0) + np.exp(-x, dtype=np.float32))


class Rope:
    """Half-split rotary embedding with a float32 cos/sin table."""

    def __init__(self, head_dim: int, base: float):
        self.half = head_dim // 2
        self.inv = base ** (-np.arange(0, self.half, dtype=np.float32) * 2.0 / head_dim)

    def __call__(self, x, offset: int):
        n = x.shape[2]
        ang = np.arange(offset, offset + n, dtype=np.float32)[:, None] * self.inv[None, :]
        c, s = np.cos(ang), np.sin(ang)
        a, b = x[..., :self.half], x[..., self.half:]
        out = np.empty_like(x)
        out[..., :self.half] = a * c - b * s
        out[..., self.half:] = a * s + b * c
        return out


class Cache:
    def __init__(self):
        self.k = self.v = None
        self.offset = 0

    def append(self, k, v):
        self.k = k if self.k is None else np.concatenate([self.k, k], axis=2)
        self.v = v if self.v is None else np.concatenate([self.v, v], axis=2)
        self.offset += k.shape[2]
        return self.k, self.v


def attention(q, k, v, scale):
    """Grouped-query attention, causal when several queries."""
    B, Hq, L, D = q.shape
    Hk, S = k.shape[1], k.shape[2]
    g = Hq // Hk
    qg = q.reshape(B, Hk, g, L, D)
    sc = np.einsum("bkgld,bksd->bkgls", qg, k) * np.float32(scale)
    if L > 1:
        allowed = np.arange(S)[None, :] <= (np.arange(L)[:, None] + (S - L))
        sc = np.where(allowed, sc, -np.inf)
    sc = sc - sc.max(-1, keepdims=True)
    e = np.exp(sc)
    e = e / e.sum(-1, keepdims=True)
    return np.einsum("bkgls,bksd->bkgld", e, v).reshape(B, Hq, L, D).astype(np.float32)


class OracleStage:
    """Embedding (fp16 table rows), layers [start, end), optional head."""

    def __init__(self, cfg: dict, w: Dict[str, np.ndarray], start: int, end: int, embed: bool,
                 head: bool, embed_rows=None, orc: Optional[Oracle] = None):
        self.orc = orc or Oracle()
        self.cfg, self.embed_on, self.head_on = cfg, embed, head
        self.embed_rows = embed_rows
        H, nh, nkv = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
        self.H, self.nh, self.nkv, self.hd = H, nh, nkv, H // nh
        self.eps = cfg["rms_norm_eps"]
        gs = cfg["quantization"]["group_size"]
        self.scale = self.hd ** -0.5
        self.rope = Rope(self.hd, cfg["rope_theta"])
        self.layers = []
        for i in range(start, end):
            p = f"model.layers.{i}"
            lin = lambda name: OLinear(self.orc, w[f"{p}.{name}.weight"], w[f"{p}.{name}.scales"],
                                       w[f"{p}.{name}.biases"], w.get(f"{p}.{name}.bias"), gs)
            self.layers.append({
                "q": lin("self_attn.q_proj"), "k": lin("self_attn.k_proj"), "v": lin("self_attn.v_proj"),
                "o": lin("self_attn.o_proj"), "gate": lin("mlp.gate_proj"), "up": lin("mlp.up_proj"),
                "down": lin("mlp.down_proj"),
                "in_w": np.asarray(w[f"{p}.input_layernorm.weight"], np.float32),
                "post_w": np.asarray(w[f"{p}.post_attention_layernorm.weight"], np.float32)})
        if head:
            self.norm_w = np.asarray(w["model.norm.weight"], np.float32)
            self.lm = OLinear(self.orc, w["lm_head.weight"], w["lm_head.scales"], w["lm_head.biases"],
                              w.get("lm_head.bias"), gs)

    def new_caches(self) -> List[Cache]:
        return [Cache() for _ in self.layers]

    def _layer(self, L, x, cache):
        B, T, _ = x.shape
        hx = rms_norm(x, L["in_w"], self.eps)
        q = L["q"](hx).reshape(B, T, self.nh, -1).transpose(0, 2, 1, 3)
        k = L["k"](hx).reshape(B, T, self.nkv, -1).transpose(0, 2, 1, 3)
        v = L["v"](hx).reshape(B, T, self.nkv, -1).transpose(0, 2, 1, 3)
        off = cache.offset if cache is not None else 0
        q, k = self.rope(q, off), self.rope(k, off)
        if cache is not None:
            k, v = cache.append(k, v)
        o = attention(q, k, v, self.scale)
        x = x + L["o"](o.transpose(0, 2, 1, 3).reshape(B, T, -1))
        hm = rms_norm(x, L["post_w"], self.eps)
        return x + L["down"](silu(L["gate"](hm)) * L["up"](hm))

    def __call__(self, x, caches=None, apply_head=True, last_only=False):
        if self.embed_on:
            ids = np.asarray(x)
            x = self.embed_rows(ids.reshape(-1)).astype(np.float32).reshape(*ids.shape, -1)
        x = np.asarray(x, dtype=np.float32)
        for i, L in enumerate(self.layers):
            x = self._layer(L, x, None if caches is None else caches[i])
        if self.head_on and apply_head:
            if last_only:
                x = x[:, -1:, :]
            x = self.lm(rms_norm(x, self.norm_w, self.eps))
        return x

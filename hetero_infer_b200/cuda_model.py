"""The qwen2 stage on the GPU: the device-side counterpart of the reference's
NumPy model (hetero/cpu_model.py).

This module starts with the quantised linear layer, ``QLinear``, whose
constructor and call signature are the reference's
(``hetero/cpu_model.py:84-158``): packed MLX-layout weights in, activations in,
activations out.  Weights are uploaded once to HBM; every product runs in
``libhq4.so``.  Host (NumPy) inputs are staged through pinned memory and come
back as NumPy arrays, so code written against the reference's QLinear runs
unchanged; CUDA tensors in give CUDA tensors out, which is what the device
stage uses.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib, ops


def _dev_array(a, dtype=None, device="cuda"):
    """NumPy (or torch) array -> contiguous CUDA tensor; uint32 travels as int32."""
    if isinstance(a, torch.Tensor):
        t = a
    else:
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint32:
            a = a.view(np.int32)
        t = torch.from_numpy(a)
    if dtype is not None:
        t = t.to(dtype)
    return t.to(device).contiguous()


def _raw_stream(idx: int) -> int:
    """Handle of the current CUDA stream of device idx (without building a
    Stream object on every call)."""
    get = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return get(idx) if get is not None else torch.cuda.current_stream(idx).cuda_stream


class _Pinned:
    """Grow-only pinned host buffers keyed by name (host<->device staging)."""

    def __init__(self):
        self.bufs = {}

    def get(self, name: str, shape, dtype) -> torch.Tensor:
        n = int(np.prod(shape))
        b = self.bufs.get(name)
        if b is None or b.numel() < n or b.dtype != dtype:
            b = torch.empty(max(n, 1), dtype=dtype, pin_memory=True)
            self.bufs[name] = b
        return b[:n].view(*shape)


class QLinear:
    """Weights stay 4-bit in HBM; the fused int4 GEMV reads them once per token.

    Same constructor as ``hetero/cpu_model.py:96``.  ``bits`` must be 4 (the
    only width the device kernels read); the reference falls back to an fp32
    expansion for other widths, this class raises instead."""

    def __init__(self, w, scales, biases, bias, group_size, bits, device="cuda"):
        if bits != 4:
            raise NotImplementedError("device QLinear reads 4-bit packed weights only")
        self.group_size, self.bits = int(group_size), int(bits)
        self.n_out, self.n_in = int(w.shape[0]), int(w.shape[1]) * (32 // bits)
        self.device = torch.device(device)
        self.w = _dev_array(w, device=self.device)
        self.scales = _dev_array(scales, torch.float16, self.device)
        self.biases = _dev_array(biases, torch.float16, self.device)
        self.bias = None if bias is None else _dev_array(bias, torch.float32, self.device)
        self._pinned = _Pinned()
        self._ptrs = (self.w.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr(),
                      None if self.bias is None else self.bias.data_ptr())
        self._stage = None  # (rows, pinned x, pinned y, device x, device y, x view, y view)
        self._calls = {}    # rows -> (pinned x view, pinned y view, C-call arguments)
        self._dev_idx = None
        self._host_fn = _lib.load().hq4_gemv_host

    def forward_device(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                       residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """CUDA fp32 [..., n_in] -> CUDA fp32 [..., n_out] (+ bias, + residual)."""
        return ops.q4_gemv_fused(self.w, self.scales, self.biases, x.contiguous(),
                                 self.group_size, self.bias, residual, out)

    def _staging(self, m: int):
        """Pinned host and device staging for m rows (grow-only)."""
        st = self._stage
        if st is None or st[0] < m:
            hx = torch.empty((m, self.n_in), dtype=torch.float32, pin_memory=True)
            hy = torch.empty((m, self.n_out), dtype=torch.float32, pin_memory=True)
            dx = torch.empty((m, self.n_in), dtype=torch.float32, device=self.device)
            dy = torch.empty((m, self.n_out), dtype=torch.float32, device=self.device)
            st = self._stage = (m, hx, hy, dx, dy, hx.numpy(), hy.numpy(),
                                (hx.data_ptr(), hy.data_ptr(), dx.data_ptr(), dy.data_ptr()))
        return st

    def __call__(self, x):
        if isinstance(x, torch.Tensor) and x.is_cuda:
            return self.forward_device(x)
        # host path: NumPy in, NumPy out (the reference's calling convention);
        # one C call copies x in, runs the GEMV (whose epilogue writes the
        # pinned output directly) and waits -- q4_gemv's own synchronous
        # host-buffer contract
        xa = np.asarray(x, dtype=np.float32)
        lead = xa.shape[:-1]
        flat = xa if xa.ndim == 2 else xa.reshape(-1, self.n_in)
        if flat.shape[-1] != self.n_in:
            raise ValueError(f"x has {flat.shape[-1]} features, the layer takes {self.n_in}")
        m = flat.shape[0]
        call = self._calls.get(m)
        if call is None:
            call = self._host_call(m)
        hx, hy, args = call
        np.copyto(hx, flat)
        idx = self._dev_idx
        if idx is None:
            idx = self._dev_idx = (self.device.index if self.device.index is not None
                                   else torch.cuda.current_device())
        if torch.cuda.current_device() != idx:
            with torch.cuda.device(idx):
                return self.__call__(x)
        rc = self._host_fn(*args, _raw_stream(idx))
        if rc:
            _lib.check(rc, "hq4_gemv_host")
        y = hy.copy()
        return y if len(lead) == 1 else y.reshape(*lead, self.n_out)

    def _host_call(self, m: int):
        """(pinned x view, pinned y view, hq4_gemv_host arguments but the
        stream) for m rows, kept per row count."""
        before = self._stage
        *_, hxn, hyn, (hxp, hyp, dxp, dyp) = self._staging(m)
        if self._stage is not before:
            self._calls.clear()  # the staging grew: calls cached on the old buffers are stale
        w, s, b, bias = self._ptrs
        call = (hxn[:m], hyn[:m], (w, s, b, bias, hxp, hyp, self.n_out, self.n_in, self.group_size, m, dxp, dyp))
        self._calls[m] = call
        return call


# ---------------------------------------------------------------------------
# The qwen2 stage (hetero/cpu_model.py:164-368) on the device
# ---------------------------------------------------------------------------

def rope_tables(head_dim: int, base: float, n: int):
    """cos/sin tables [n][head_dim/2], computed on the host with the same NumPy
    float32 expression as the reference's RoPE (hetero/cpu_model.py:181-193),
    so the rotation is bit-identical to it."""
    half = head_dim // 2
    inv = base ** (-np.arange(0, half, dtype=np.float32) * 2.0 / head_dim)
    ang = np.arange(n, dtype=np.float32)[:, None] * inv[None, :]
    return np.cos(ang), np.sin(ang)


def rope_pair_rows(n_heads: int, head_dim: int) -> np.ndarray:
    """Row order for q or k that puts the rotation pair (d, d + hd/2) of every
    head on rows g and g+8 of one 16-row strip (the layout hq4_qkv_rope reads)."""
    half = head_dim // 2
    rows = []
    for h in range(n_heads):
        for jb in range(0, half, 8):
            base = h * head_dim + jb
            rows.extend(range(base, base + 8))
            rows.extend(range(base + half, base + half + 8))
    return np.asarray(rows, dtype=np.int64)


def interleave_gate_up(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """Rows of the fused gate|up matrix: per 16-row strip, gate rows 8s..8s+7
    then up rows 8s..8s+7 (the layout the silu*up epilogue reads)."""
    n = gate.shape[0]
    if n % 8:
        raise ValueError("intermediate size must be a multiple of 8")
    g = gate.reshape(n // 8, 8, *gate.shape[1:])
    u = up.reshape(n // 8, 8, *up.shape[1:])
    return np.concatenate([g, u], axis=1).reshape(2 * n, *gate.shape[1:])


class _Packed:
    """A packed int4 matrix on the device (w int32 view, fp16 scales/biases)."""

    def __init__(self, w, s, b, device):
        self.w = _dev_array(w, device=device)
        self.s = _dev_array(s, torch.float16, device)
        self.b = _dev_array(b, torch.float16, device)
        self.n_out, self.n_in = int(w.shape[0]), int(w.shape[1]) * 8


class DeviceKVCache:
    """Per-request KV cache of a whole stage: fp32 k, v [layers][n_kv][max_ctx][hd]
    and the device position the kernels read (the reference keeps one growing
    cache per layer, hetero/cpu_model.py:207-230; here the capacity is
    preallocated and `offset` mirrors the position on the host)."""

    def __init__(self, n_layers: int):
        self.n_layers = n_layers
        self.k = self.v = self.pos = None
        self.offset = 0

    def __len__(self):
        return self.n_layers

    def __getitem__(self, i):
        return self  # per-layer views are taken by the stage

    def allocate(self, n_kv, head_dim, max_ctx, device):
        if self.k is None:
            shape = (self.n_layers, n_kv, max_ctx, head_dim)
            self.k = torch.zeros(shape, dtype=torch.float32, device=device)
            self.v = torch.zeros(shape, dtype=torch.float32, device=device)
            self.pos = torch.zeros(1, dtype=torch.int32, device=device)
            self.max_ctx = max_ctx


class _Layer:
    def __init__(self, cfg, w, idx, device):
        from . import _lib
        p = f"model.layers.{idx}"
        H = cfg["hidden_size"]
        nh, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
        hd = H // nh
        gs = cfg["quantization"]["group_size"]
        get = lambda proj, part: w[f"{p}.{proj}.{part}"]
        pq, pk = rope_pair_rows(nh, hd), rope_pair_rows(nkv, hd)
        parts = []
        for part in ("weight", "scales", "biases"):
            q = get("self_attn.q_proj", part)[pq]
            k = get("self_attn.k_proj", part)[pk]
            v = get("self_attn.v_proj", part)
            parts.append(np.concatenate([q, k, v], axis=0))
        self.qkv = _Packed(*parts, device)
        bias = []
        for proj, perm, n in (("q_proj", pq, nh * hd), ("k_proj", pk, nkv * hd), ("v_proj", None, nkv * hd)):
            b = w.get(f"{p}.self_attn.{proj}.bias")
            b = np.zeros(n, np.float32) if b is None else np.asarray(b, np.float32)
            bias.append(b[perm] if perm is not None else b)
        self.qkv_bias = _dev_array(np.concatenate(bias), torch.float32, device)
        self.o = _Packed(get("self_attn.o_proj", "weight"), get("self_attn.o_proj", "scales"),
                         get("self_attn.o_proj", "biases"), device)
        if w.get(f"{p}.self_attn.o_proj.bias") is not None:
            raise NotImplementedError("o_proj bias")
        gu = [interleave_gate_up(get("mlp.gate_proj", part), get("mlp.up_proj", part))
              for part in ("weight", "scales", "biases")]
        self.gate_up = _Packed(*gu, device)
        self.down = _Packed(get("mlp.down_proj", "weight"), get("mlp.down_proj", "scales"),
                            get("mlp.down_proj", "biases"), device)
        self.in_w = _dev_array(np.asarray(w[f"{p}.input_layernorm.weight"], np.float32), torch.float32, device)
        self.post_w = _dev_array(np.asarray(w[f"{p}.post_attention_layernorm.weight"], np.float32),
                                 torch.float32, device)
        self.gs, self.H, self.nh, self.nkv, self.hd = gs, H, nh, nkv, hd
        self.I = cfg["intermediate_size"]
        self._lib = _lib.load()


class Stage:
    """The device counterpart of ``hetero/cpu_model.py:Stage`` (same constructor
    and call signature).  Hidden states, KV cache and softmax are fp32 as in
    the reference; every product is a libhq4 kernel.

    Per layer, five launches: q|k|v GEMV (RMSNorm prologue, bias + RoPE +
    cache append epilogue), attention, o GEMV (+ residual), gate|up GEMV
    (RMSNorm prologue, silu*up epilogue), down GEMV (+ residual)."""

    def __init__(self, cfg: dict, spec, w: dict, device="cuda", max_ctx: int = 2048):
        from . import _lib, synth
        if cfg.get("model_type") != "qwen2" or "quantization" not in cfg:
            raise NotImplementedError("device backend handles quantised qwen2 only")
        if cfg["quantization"]["bits"] != 4:
            raise NotImplementedError("device backend reads 4-bit weights only")
        self.cfg, self.spec = cfg, spec
        self.device = torch.device(device)
        self.lib = _lib.load()
        self.max_ctx = int(max_ctx)
        self.eps = float(cfg["rms_norm_eps"])
        H = cfg["hidden_size"]
        self.H, self.nh, self.nkv = H, cfg["num_attention_heads"], cfg["num_key_value_heads"]
        self.hd = H // self.nh
        self.gs = cfg["quantization"]["group_size"]
        self.I = cfg["intermediate_size"]
        self.V = cfg["vocab_size"]
        # the reference scales scores by head_dim ** -0.5 as a float32 multiply
        self.scale = float(np.float32(self.hd ** -0.5))
        self.layers = [_Layer(cfg, w, i, self.device) for i in range(spec.start, spec.end)]
        self.embed_table = None
        self.embed_q = None
        if spec.embed:
            if synth.EMBED_SYNTH_KEY in w:
                t = torch.empty((self.V, H), dtype=torch.float16, device=self.device)
                rc = self.lib.hq4_synth_embed_f16(int(w[synth.EMBED_SYNTH_KEY]), self.V, H, 0.02,
                                                  t.data_ptr(), self._stream())
                _lib.check(rc, "hq4_synth_embed_f16")
                self.embed_table = t
            elif "model.embed_tokens.table" in w:
                self.embed_table = _dev_array(w["model.embed_tokens.table"], torch.float16, self.device)
            else:  # quantised table, dequantised row by row (cpu_model.py:334-338)
                self.embed_q = _Packed(w["model.embed_tokens.weight"], w["model.embed_tokens.scales"],
                                       w["model.embed_tokens.biases"], self.device)
        if spec.head:
            self.norm_w = _dev_array(np.asarray(w["model.norm.weight"], np.float32), torch.float32, self.device)
            if cfg.get("tie_word_embeddings", False):
                self.lm_head = _Packed(w["model.embed_tokens.weight"], w["model.embed_tokens.scales"],
                                       w["model.embed_tokens.biases"], self.device)
                self.lm_bias = None
            else:
                self.lm_head = _Packed(w["lm_head.weight"], w["lm_head.scales"], w["lm_head.biases"],
                                       self.device)
                lb = w.get("lm_head.bias")
                self.lm_bias = None if lb is None else _dev_array(np.asarray(lb, np.float32), torch.float32,
                                                                  self.device)
        cos, sin = rope_tables(self.hd, float(cfg["rope_theta"]), self.max_ctx)
        self.rope_cos = _dev_array(cos, torch.float32, self.device)
        self.rope_sin = _dev_array(sin, torch.float32, self.device)

    # -- plumbing ----------------------------------------------------------
    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def _check(self, rc, what):
        from . import _lib
        _lib.check(rc, what)

    def new_caches(self) -> DeviceKVCache:
        c = DeviceKVCache(len(self.layers))
        c.allocate(self.nkv, self.hd, self.max_ctx, self.device)
        return c

    # -- pieces ------------------------------------------------------------
    def embed(self, ids) -> torch.Tensor:
        if isinstance(ids, torch.Tensor) and ids.is_cuda:
            # token ids already on the device (a sampled token): no host round
            # trip; the kernel zeroes rows of out-of-range ids and flags them
            if self.embed_table is None:
                raise NotImplementedError("device token ids need the fp16 embedding table")
            d_ids = ids.reshape(-1).to(torch.int32).contiguous()
            n = d_ids.numel()
            out = torch.empty((n, self.H), dtype=torch.float32, device=self.device)
            self._check(self.lib.hq4_embed_f16(self.embed_table.data_ptr(), d_ids.data_ptr(), n, self.H,
                                               self.embed_table.shape[0], out.data_ptr(), self._stream()),
                        "hq4_embed_f16")
            return out.view(*ids.shape, self.H)
        ids_np = np.asarray(ids).reshape(-1).astype(np.int32)
        n = ids_np.size
        out = torch.empty((n, self.H), dtype=torch.float32, device=self.device)
        if ids_np.size and (ids_np.min() < 0 or ids_np.max() >= self.V):
            raise ValueError(f"token id out of range [0, {self.V})")
        if self.embed_table is not None:
            d_ids = torch.from_numpy(ids_np).to(self.device)
            self._check(self.lib.hq4_embed_f16(self.embed_table.data_ptr(), d_ids.data_ptr(), n, self.H,
                                               self.embed_table.shape[0], out.data_ptr(), self._stream()), "hq4_embed_f16")
        else:
            e = self.embed_q
            for i, t in enumerate(ids_np):
                self._check(self.lib.hq4_dequant(e.w.data_ptr(), e.s.data_ptr(), e.b.data_ptr(),
                                                 out[i].data_ptr(), int(t), int(t) + 1, self.H, self.gs,
                                                 self._stream()), "hq4_dequant")
        return out.view(*np.asarray(ids).shape, self.H)

    def layer_forward(self, i: int, h: torch.Tensor, cache: DeviceKVCache, L: int, bufs=None):
        """One decoder layer on L tokens, in place on h [L, H]."""
        from ._lib import expect
        lay, lib, st = self.layers[i], self.lib, self._stream()
        q = bufs["q"] if bufs else torch.empty((L, self.nh * self.hd), dtype=torch.float32, device=self.device)
        a = bufs["a"] if bufs else torch.empty((L, self.nh * self.hd), dtype=torch.float32, device=self.device)
        m = bufs["m"] if bufs else torch.empty((L, self.I), dtype=torch.float32, device=self.device)
        kc, vc = cache.k[i], cache.v[i]
        f4 = 4
        expect(h, L * self.H * f4, "h", 16)
        expect(q, L * self.nh * self.hd * f4, "q", 16)
        expect(a, L * self.nh * self.hd * f4, "a", 16)
        expect(m, L * self.I * f4, "m", 16)
        expect(kc, self.nkv * cache.max_ctx * self.hd * f4, "k_cache")
        expect(vc, self.nkv * cache.max_ctx * self.hd * f4, "v_cache")
        expect(cache.pos, 4, "pos")
        for t, nb, nm in ((lay.qkv.w, lay.qkv.n_out * self.H // 2, "qkv.w"), (lay.o.w, self.H * self.H // 2, "o.w"),
                          (lay.gate_up.w, 2 * self.I * self.H // 2, "gu.w"), (lay.down.w, self.H * self.I // 2, "down.w"),
                          (self.rope_cos, cache.max_ctx * self.hd // 2 * f4, "cos")):
            expect(t, nb, nm, 32 if nm.endswith(".w") else 4)
        if cache.max_ctx > self.max_ctx:
            raise RuntimeError("cache larger than the stage's rope table")
        self._check(lib.hq4_qkv_rope(lay.qkv.w.data_ptr(), lay.qkv.s.data_ptr(), lay.qkv.b.data_ptr(),
                                     h.data_ptr(), self.nh, self.nkv, self.hd, self.H, self.gs, L,
                                     lay.in_w.data_ptr(), self.eps, lay.qkv_bias.data_ptr(),
                                     cache.pos.data_ptr(), self.rope_cos.data_ptr(),
                                     self.rope_sin.data_ptr(), cache.max_ctx, q.data_ptr(), kc.data_ptr(),
                                     vc.data_ptr(), st), "hq4_qkv_rope")
        self._check(lib.hq4_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), a.data_ptr(), self.nh,
                                      self.nkv, self.hd, cache.max_ctx, cache.pos.data_ptr(), L, self.scale,
                                      st), "hq4_attention")
        self._check(lib.hq4_gemv_fused(lay.o.w.data_ptr(), lay.o.s.data_ptr(), lay.o.b.data_ptr(),
                                       a.data_ptr(), h.data_ptr(), self.H, self.H, self.gs, L, None,
                                       h.data_ptr(), st), "hq4_gemv_fused(o)")
        self._check(lib.hq4_gemv_norm(lay.gate_up.w.data_ptr(), lay.gate_up.s.data_ptr(),
                                      lay.gate_up.b.data_ptr(), h.data_ptr(), m.data_ptr(), 2 * self.I,
                                      self.H, self.gs, L, lay.post_w.data_ptr(), self.eps, 1, None, None,
                                      st), "hq4_gemv_norm(gate_up)")
        self._check(lib.hq4_gemv_fused(lay.down.w.data_ptr(), lay.down.s.data_ptr(), lay.down.b.data_ptr(),
                                       m.data_ptr(), h.data_ptr(), self.H, self.I, self.gs, L, None,
                                       h.data_ptr(), st), "hq4_gemv_fused(down)")

    def head_logits(self, h: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """RMSNorm + vocabulary projection of rows h [R, H] -> [R, V]."""
        from ._lib import expect
        R = h.shape[0]
        if out is None:
            out = torch.empty((R, self.V), dtype=torch.float32, device=self.device)
        expect(h, R * self.H * 4, "head h", 16)
        expect(out, R * self.V * 4, "logits")
        lm = self.lm_head
        self._check(self.lib.hq4_gemv_norm(lm.w.data_ptr(), lm.s.data_ptr(), lm.b.data_ptr(), h.data_ptr(),
                                           out.data_ptr(), self.V, self.H, self.gs, R, self.norm_w.data_ptr(),
                                           self.eps, 0,
                                           self.lm_bias.data_ptr() if self.lm_bias is not None else None,
                                           None, self._stream()), "hq4_gemv_norm(lm_head)")
        return out

    def _advance(self, cache: DeviceKVCache, L: int):
        self._check(self.lib.hq4_advance_position(cache.pos.data_ptr(), L, self._stream()),
                    "hq4_advance_position")
        cache.offset += L

    # -- the reference's surface ---------------------------------------------
    def body(self, x, caches=None, mask=None):
        """Embedding (if owned) plus this stage's layers; no head."""
        return self._run(x, caches, apply_head=False, last_only=False)

    def head_forward(self, x, last_only: bool = True):
        h = self._as_hidden(x)
        if last_only:
            h = h[:, -1:, :]
        B, L, H = h.shape
        return self.head_logits(h.reshape(B * L, H).contiguous()).view(B, L, self.V)

    def __call__(self, x, caches=None, mask=None, apply_head=True, last_only=False):
        return self._run(x, caches, apply_head, last_only)

    def _as_hidden(self, x) -> torch.Tensor:
        if isinstance(x, torch.Tensor):
            return x.to(self.device, torch.float32)
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(self.device)

    def _run(self, x, caches, apply_head, last_only):
        if self.spec.embed:
            h = self.embed(x)
        else:
            h = self._as_hidden(x)
        if h.dim() != 3 or h.shape[0] != 1:
            raise NotImplementedError("device stage runs batch 1 (as the reference's decode)")
        L = h.shape[1]
        h = h.reshape(L, self.H).contiguous()
        cache = caches
        if cache is None or isinstance(cache, list):
            cache = DeviceKVCache(len(self.layers))  # no cache: a scratch one (positions 0..L-1)
        cache.allocate(self.nkv, self.hd, self.max_ctx, self.device)
        if cache.offset + L > cache.max_ctx:
            raise ValueError(f"context {cache.offset + L} exceeds max_ctx {cache.max_ctx}")
        for i in range(len(self.layers)):
            self.layer_forward(i, h, cache, L)
        if len(self.layers):
            self._advance(cache, L)
        if self.spec.head and apply_head:
            rows = h[-1:] if last_only else h
            return self.head_logits(rows.contiguous()).view(1, rows.shape[0], self.V)
        return h.view(1, L, self.H)


class CudaBackend:
    """The reference's backend surface (hetero/backends.py:70-130) on B200."""

    name = "cuda+q4"
    weight_expansion = 1.0

    def __init__(self, device="cuda", max_ctx: int = 2048):
        self.device = torch.device(device)
        self.max_ctx = max_ctx

    def load_stage(self, model_dir, spec, index=None):
        """The stage owning `spec` from an MLX-format snapshot, and the bytes
        it holds (hetero/backends.py:83-85 -> cpu_model.load_stage,
        hetero/cpu_model.py:371-375): `index` is a checkpoint.WeightIndex of
        model_dir, built here when not given."""
        from . import checkpoint
        idx = index if index is not None else checkpoint.WeightIndex(model_dir)
        stage = Stage(idx.config, spec, idx.load_shard(spec), self.device, self.max_ctx)
        return stage, idx.shard_bytes(spec)

    def build_stage(self, cfg, spec, weights):
        return Stage(cfg, spec, weights, self.device, self.max_ctx)

    def new_caches(self, n: int):
        return DeviceKVCache(n)

    def array(self, data):
        return np.asarray(data)

    def eval(self, *xs):
        torch.cuda.current_stream(self.device).synchronize()

    def hidden(self, shape):
        return torch.zeros(shape, dtype=torch.float32, device=self.device)

    def to_wire(self, x) -> np.ndarray:
        if isinstance(x, torch.Tensor):
            return x.to(torch.float16).cpu().numpy()
        return np.asarray(x, dtype=np.float16)

    def from_wire(self, a: np.ndarray):
        return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(self.device)

    def sample(self, logits, temperature: float, top_p: float, rng) -> int:
        """NumpyBackend.sample (hetero/backends.py:106-120) on the device:
        numpy's argmax at temperature 0 (hq4_argmax), else the temperature /
        top-p draw (hq4_sample) with the uniform variate taken from `rng` --
        one rng.random(), the variate rng.choice itself consumes -- so a seeded
        generator advances exactly as the reference's does."""
        from . import _lib
        if isinstance(logits, torch.Tensor):
            z = logits.reshape(-1).to(self.device, torch.float32).contiguous()
        else:
            z = torch.from_numpy(np.ascontiguousarray(np.asarray(logits, dtype=np.float32).reshape(-1))).to(
                self.device)
        lib = _lib.load()
        out = torch.empty(1, dtype=torch.int32, device=z.device)
        st = torch.cuda.current_stream(z.device).cuda_stream
        if temperature <= 0:
            _lib.check(lib.hq4_argmax(z.data_ptr(), z.numel(), out.data_ptr(), None, 0, None, None, st),
                       "hq4_argmax")
        else:
            u = float(rng.random())
            _lib.check(lib.hq4_sample(z.data_ptr(), z.numel(), float(temperature), float(top_p), u,
                                      out.data_ptr(), st), "hq4_sample")
        return int(out.item())

    def peak_bytes(self) -> int:
        return int(torch.cuda.max_memory_allocated(self.device))

    def reset_peak(self):
        torch.cuda.reset_peak_memory_stats(self.device)

    def clear_cache(self):
        torch.cuda.empty_cache()


def get(name: str = "auto"):
    """`cuda` selects this backend (the reference's get() chooses mlx/numpy)."""
    if name in ("auto", "cuda", "gpu"):
        return CudaBackend()
    raise ValueError(f"unknown backend {name}")


class _DecodeLayer(ctypes.Structure):
    """include/hq4.h hq4_decode_layer: one layer's device pointers."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "qkv_w", "qkv_s", "qkv_b", "qkv_bias", "input_norm", "o_w", "o_s", "o_b", "post_norm",
        "gate_up_w", "gate_up_s", "gate_up_b", "down_w", "down_s", "down_b", "k_cache", "v_cache")]


class DecodePlan:
    """Every layer of a stage for one decode token as ONE persistent launch
    (hq4_decode_plan_*): the same five steps per layer as
    ``Stage.layer_forward`` with the same bits, without the kernel boundaries.
    Bound to the hidden row h [1, H], the KV cache and the step buffers;
    ``run`` is capturable in a CUDA graph.

    ``DecodePlan.build`` returns None when a shape does not fit the kernel
    (-1 from the library); any other failure raises."""

    def __init__(self, handle, stage, keep):
        self.handle, self.stage, self._keep = handle, stage, keep

    @classmethod
    def build(cls, stage: "Stage", h: torch.Tensor, cache: "DeviceKVCache", bufs: dict):
        from ._lib import expect
        lib = stage.lib
        n = len(stage.layers)
        if n == 0:
            return None
        arr = (_DecodeLayer * n)()
        for i, lay in enumerate(stage.layers):
            e = arr[i]
            e.qkv_w, e.qkv_s, e.qkv_b = lay.qkv.w.data_ptr(), lay.qkv.s.data_ptr(), lay.qkv.b.data_ptr()
            e.qkv_bias, e.input_norm = lay.qkv_bias.data_ptr(), lay.in_w.data_ptr()
            e.o_w, e.o_s, e.o_b = lay.o.w.data_ptr(), lay.o.s.data_ptr(), lay.o.b.data_ptr()
            e.post_norm = lay.post_w.data_ptr()
            e.gate_up_w, e.gate_up_s, e.gate_up_b = (lay.gate_up.w.data_ptr(), lay.gate_up.s.data_ptr(),
                                                     lay.gate_up.b.data_ptr())
            e.down_w, e.down_s, e.down_b = lay.down.w.data_ptr(), lay.down.s.data_ptr(), lay.down.b.data_ptr()
            e.k_cache, e.v_cache = cache.k[i].data_ptr(), cache.v[i].data_ptr()
        expect(h, stage.H * 4, "h", 16)
        if cache.max_ctx > stage.max_ctx:
            raise RuntimeError("cache larger than the stage's rope table")
        handle = ctypes.c_void_p()
        rc = lib.hq4_decode_plan_create(arr, n, stage.H, stage.nh, stage.nkv, stage.hd, stage.I, stage.gs,
                                        stage.eps, stage.scale, stage.rope_cos.data_ptr(),
                                        stage.rope_sin.data_ptr(), cache.max_ctx, h.data_ptr(),
                                        cache.pos.data_ptr(), bufs["q"].data_ptr(), bufs["a"].data_ptr(),
                                        bufs["m"].data_ptr(), ctypes.byref(handle))
        if rc == -1:
            return None
        _lib.check(rc, "hq4_decode_plan_create")
        return cls(handle, stage, (h, cache, bufs))

    def run(self) -> None:
        self.stage._check(self.stage.lib.hq4_decode_plan_run(self.handle, self.stage._stream()),
                          "hq4_decode_plan_run")

    def inject_fault(self, skip_cta: int = -1, barrier_ns: int = 0) -> None:
        """Failure-path testing: CTA skip_cta withholds its first grid-barrier
        arrival on later runs, whose waits then end after barrier_ns with
        status bit 0 set (hq4_decode_plan_fault); (-1, 0) restores normal runs."""
        _lib.check(self.stage.lib.hq4_decode_plan_fault(self.handle, int(skip_cta), int(barrier_ns)),
                   "hq4_decode_plan_fault")

    def info(self) -> dict:
        out = (ctypes.c_int * 4)()
        _lib.check(self.stage.lib.hq4_decode_plan_info(self.handle, out), "hq4_decode_plan_info")
        return {"grid": out[0], "ring": out[1], "smem": out[2], "phases": out[3]}

    def close(self) -> None:
        if self.handle:
            self.stage.lib.hq4_decode_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GreedyDecoder:
    """Batch-1 greedy generation on one device stage that owns the embedding
    and the head (the single-node decode loop of hetero/coordinator.py:266-292).

    The prompt is prefilled eagerly; after that one CUDA graph holds a whole
    decode step -- embedding of the previous token, every layer, the head,
    argmax, position advance -- and is replayed once per token.  The token, the
    position and the history of generated tokens stay on the device, so there
    is no host round trip between steps; `generate` reads the history once.

    persistent: the layers of a decode step run as one persistent launch
    (DecodePlan) -- True requires it, "auto" takes the plan when the shapes
    fit it, False (the default, the faster path on B200 as measured) keeps one
    launch per layer step."""

    def __init__(self, stage: Stage, cache: Optional[DeviceKVCache] = None, persistent=False):
        if not (stage.spec.embed and stage.spec.head):
            raise ValueError("GreedyDecoder needs a stage with both embedding and head")
        self.stage = stage
        self.cache = cache if cache is not None else stage.new_caches()
        # a caller's cache may not be allocated yet (DeviceKVCache(n) allocates lazily)
        self.cache.allocate(stage.nkv, stage.hd, stage.max_ctx, stage.device)
        dev = stage.device
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.history = torch.zeros(stage.max_ctx, dtype=torch.int32, device=dev)
        self.h = torch.empty((1, stage.H), dtype=torch.float32, device=dev)
        self.logits = torch.empty((1, stage.V), dtype=torch.float32, device=dev)
        self.bufs = {"q": torch.empty((1, stage.nh * stage.hd), dtype=torch.float32, device=dev),
                     "a": torch.empty((1, stage.nh * stage.hd), dtype=torch.float32, device=dev),
                     "m": torch.empty((1, stage.I), dtype=torch.float32, device=dev)}
        self.graph = None
        self.stream = torch.cuda.Stream(dev)
        self.plan = None
        if persistent:
            self.plan = DecodePlan.build(stage, self.h, self.cache, self.bufs)
            if self.plan is None and persistent is True:
                raise ValueError("the stage's shapes do not fit the persistent decode kernel")

    def _argmax(self):
        s = self.stage
        s._check(s.lib.hq4_argmax(self.logits.data_ptr(), s.V, self.tok.data_ptr(), self.history.data_ptr(),
                                  s.max_ctx, self.cache.pos.data_ptr(), None, s._stream()), "hq4_argmax")

    def _step(self):
        s = self.stage
        s._check(s.lib.hq4_embed_f16(s.embed_table.data_ptr(), self.tok.data_ptr(), 1, s.H, s.embed_table.shape[0],
                                     self.h.data_ptr(), s._stream()), "hq4_embed_f16")
        if self.plan is not None:
            self.plan.run()
        else:
            for i in range(len(s.layers)):
                s.layer_forward(i, self.h, self.cache, 1, self.bufs)
        s._check(s.lib.hq4_advance_position(self.cache.pos.data_ptr(), 1, s._stream()), "advance")
        s.head_logits(self.h, self.logits)
        self._argmax()

    def prefill(self, prompt) -> None:
        """Prompt [1, P] through the stage (causal), first token sampled on device."""
        s = self.stage
        if s.embed_table is None:
            raise NotImplementedError("graph decode needs an fp16 embedding table")
        with torch.cuda.stream(self.stream):
            logits = s(prompt, self.cache, apply_head=True, last_only=True)
            self.logits.copy_(logits.view(1, s.V))
            self._argmax()
        self.start = self.cache.offset

    def capture(self) -> None:
        """Record one decode step as a CUDA graph (after one eager step, which
        is a real step: its token goes to the history like any other)."""
        with torch.cuda.stream(self.stream):
            self._step()
            self.cache.offset += 1
            torch.cuda.current_stream().synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._step()
        self.graph = g

    def steps(self, n: int) -> None:
        """Replay n decode steps (asynchronously on the decoder's stream)."""
        if self.cache.offset + n > self.stage.max_ctx:
            raise ValueError("context would exceed max_ctx")
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                self.graph.replay()
        self.cache.offset += n

    def tokens(self):
        """Generated tokens so far (first from the prefill)."""
        torch.cuda.current_stream().wait_stream(self.stream)
        return self.history[self.start:self.cache.offset + 1].cpu().tolist()

    def generate(self, prompt, n_tokens: int):
        """Prefill + n_tokens-1 decode steps -> list of n_tokens token ids."""
        self.prefill(prompt)
        if n_tokens > 1:
            self.capture()
            if n_tokens > 2:
                self.steps(n_tokens - 2)
        toks = self.tokens()
        return toks[:n_tokens]

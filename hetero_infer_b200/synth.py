"""Seeded synthetic weights in the reference's packed int4 layout.

There is no checkpoint on the GPU box and no network, so every benchmark and
parity case runs on random weights with the shapes and value distributions the
benchmark configurations name:

* linear weights: uniform random nibbles 0-15, eight per little-endian uint32
  along K, low nibble first (MLX affine layout, ``kernel/q4gemv.c:7-11``);
* per group of ``gs`` along K: an fp16 scale ``|N(0,1)| * 0.01`` and an fp16
  bias equal to ``-8 * scale`` (exact in fp16);
* embeddings fp16 ``N(0, 0.02)``, RMSNorm weights ones, q/k/v biases fp16
  ``N(0, 0.02)`` (qwen2 has them; ``hetero/cpu_model.py:266`` reads them with
  ``w.get``).

The embedding table (152064 x 3584 for the 7B shape) is the one tensor too
large to generate on the host for every run, and only the rows looked up
matter.  It uses a counter-based generator instead: element (r, c) is
0.02 * (sum of 12 uniform 24-bit integers - 6 * 2^24) / 2^24 -- an
Irwin-Hall(12) approximation of N(0, 1) -- with the integers drawn from
splitmix64 of (seed, r, c, i), summed exactly in integers, converted to fp32
once, scaled, and rounded to fp16.  ``embed_rows`` evaluates any rows on the
host; the device kernel ``hq4_synth_embed_f16`` fills the full table with the
same bits.

Every tensor draws from its own ``numpy.random.default_rng([seed, crc32(name)])``
stream, so one tensor (or one layer) can be regenerated alone and the values do
not depend on which other tensors were generated before it.
"""
from __future__ import annotations

import zlib
from typing import Dict, Iterable, Optional

import numpy as np

QWEN2_7B = {
    "model_type": "qwen2",
    "hidden_size": 3584,
    "num_hidden_layers": 28,
    "num_attention_heads": 28,
    "num_key_value_heads": 4,
    "intermediate_size": 18944,
    "vocab_size": 152064,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1e6,
    "tie_word_embeddings": False,
    "quantization": {"group_size": 64, "bits": 4},
}

# The seven int4 projections of one decoder layer: (name, n_out, n_in) as
# functions of the config (hetero/cpu_model.py:263-289).
PROJ_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def small_config(layers: int = 2, hidden: int = 256, heads: int = 4, kv_heads: int = 2,
                 inter: int = 512, vocab: int = 1024, gs: int = 64) -> dict:
    """A qwen2 config with the same structure at test-friendly sizes."""
    cfg = dict(QWEN2_7B)
    cfg.update(hidden_size=hidden, num_hidden_layers=layers, num_attention_heads=heads,
               num_key_value_heads=kv_heads, intermediate_size=inter, vocab_size=vocab,
               quantization={"group_size": gs, "bits": 4})
    return cfg


def proj_shapes(cfg: dict) -> Dict[str, tuple]:
    h = cfg["hidden_size"]
    hd = h // cfg["num_attention_heads"]
    kv = cfg["num_key_value_heads"] * hd
    i = cfg["intermediate_size"]
    return {"q_proj": (h, h), "k_proj": (kv, h), "v_proj": (kv, h), "o_proj": (h, h),
            "gate_proj": (i, h), "up_proj": (i, h), "down_proj": (h, i)}


def rng_for(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([int(seed), zlib.crc32(name.encode())])


def q4_tensor(rng: np.random.Generator, n_out: int, n_in: int, gs: int = 64):
    """(w uint32 [n_out, n_in/8], scales fp16 [n_out, n_in/gs], biases fp16)."""
    if n_in % gs or n_in % 8:
        raise ValueError(f"n_in={n_in} must be a multiple of gs={gs} and of 8")
    n_words = n_out * (n_in // 8)
    if n_words % 2 == 0:
        # raw 64-bit draws split into two words: uniform bits, ~20x faster than
        # Generator.integers for the ~1e9 words of the 7B-shape model
        w = rng.bit_generator.random_raw(n_words // 2).view("<u4").reshape(n_out, n_in // 8)
        w = w.astype(np.uint32, copy=False)
    else:
        w = rng.integers(0, 2 ** 32, size=(n_out, n_in // 8), dtype=np.uint32)
    s = (np.abs(rng.standard_normal((n_out, n_in // gs), dtype=np.float32)) * 0.01)
    s = s.astype(np.float16)
    b = (s.astype(np.float32) * -8.0).astype(np.float16)
    return w, s, b


def q4_linear(seed: int, name: str, n_out: int, n_in: int, gs: int = 64):
    return q4_tensor(rng_for(seed, name), n_out, n_in, gs)


def fp16_normal(seed: int, name: str, shape, std: float = 0.02) -> np.ndarray:
    r = rng_for(seed, name)
    return (r.standard_normal(shape, dtype=np.float32) * std).astype(np.float16)


def _splitmix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def embed_rows(seed: int, ids, hidden: int, std: float = 0.02) -> np.ndarray:
    """Rows `ids` of the counter-based synthetic embedding table, fp16."""
    ids = np.asarray(ids, dtype=np.uint64).reshape(-1)
    col = np.arange(hidden, dtype=np.uint64)
    with np.errstate(over="ignore"):
        key = (np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15)
               + ids[:, None] * np.uint64(hidden) + col[None, :])
        acc = np.zeros(key.shape, dtype=np.int64)
        for i in range(12):
            z = _splitmix64(key * np.uint64(12) + np.uint64(i))
            acc += (z >> np.uint64(40)).astype(np.int64)
    acc -= 6 * (1 << 24)
    v = acc.astype(np.float32) * np.float32(1.0 / (1 << 24))
    return (v * np.float32(std)).astype(np.float16)


EMBED_SYNTH_KEY = "model.embed_tokens.synth_seed"


def activation(seed: int, name: str, shape, dtype=np.float32) -> np.ndarray:
    return rng_for(seed, name).standard_normal(shape, dtype=np.float32).astype(dtype)


def layer_weights(cfg: dict, seed: int, idx: int, qkv_bias: bool = True) -> Dict[str, np.ndarray]:
    """Tensors of decoder layer ``idx`` under their checkpoint names."""
    gs = cfg["quantization"]["group_size"]
    p = f"model.layers.{idx}"
    out: Dict[str, np.ndarray] = {}
    for proj, (n_out, n_in) in proj_shapes(cfg).items():
        sub = "self_attn" if proj in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
        name = f"{p}.{sub}.{proj}"
        w, s, b = q4_linear(seed, name, n_out, n_in, gs)
        out[f"{name}.weight"], out[f"{name}.scales"], out[f"{name}.biases"] = w, s, b
        if qkv_bias and proj in ("q_proj", "k_proj", "v_proj"):
            out[f"{name}.bias"] = fp16_normal(seed, f"{name}.bias", (n_out,))
    h = cfg["hidden_size"]
    out[f"{p}.input_layernorm.weight"] = np.ones(h, np.float16)
    out[f"{p}.post_attention_layernorm.weight"] = np.ones(h, np.float16)
    return out


def model_weights(cfg: dict, seed: int, layers: Optional[Iterable[int]] = None,
                  embed: bool = True, head: bool = True,
                  qkv_bias: bool = True) -> Dict[str, np.ndarray]:
    """All tensors a stage owning ``layers`` (and optionally embed/head) needs.

    The embedding is the counter-based fp16 table described above (the
    benchmark configuration asks for fp16 N(0, 0.02) embeddings rather than a
    quantised table); it is represented by its seed under EMBED_SYNTH_KEY and
    materialised by whoever needs it (``embed_rows`` on the host, the device
    kernel on the GPU)."""
    if layers is None:
        layers = range(cfg["num_hidden_layers"])
    out: Dict[str, np.ndarray] = {}
    if embed:
        out[EMBED_SYNTH_KEY] = np.array(int(seed) & 0x7FFFFFFF, dtype=np.int64)
    for i in layers:
        out.update(layer_weights(cfg, seed, i, qkv_bias))
    if head:
        gs = cfg["quantization"]["group_size"]
        w, s, b = q4_linear(seed, "lm_head", cfg["vocab_size"], cfg["hidden_size"], gs)
        out["lm_head.weight"], out["lm_head.scales"], out["lm_head.biases"] = w, s, b
        out["model.norm.weight"] = np.ones(cfg["hidden_size"], np.float16)
    return out


def prompt_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    """Uniform-random prompt token ids, shape [1, n]."""
    return rng_for(seed, "prompt").integers(0, vocab, size=(1, n)).astype(np.int64)


def snapshot_weights(cfg: dict, seed: int, tied: bool = False) -> Dict[str, np.ndarray]:
    """Every tensor of the model as an MLX-format checkpoint holds it: the
    quantized layers and head of ``model_weights`` plus a quantized embedding
    table (model.embed_tokens.{weight,scales,biases}); a tied model has no
    lm_head tensors (its head is the embedding)."""
    gs = cfg["quantization"]["group_size"]
    out = model_weights(cfg, seed, embed=False, head=True)
    w, s, b = q4_linear(seed, "model.embed_tokens", cfg["vocab_size"], cfg["hidden_size"], gs)
    out["model.embed_tokens.weight"], out["model.embed_tokens.scales"], out["model.embed_tokens.biases"] = w, s, b
    if tied:
        for k in ("lm_head.weight", "lm_head.scales", "lm_head.biases"):
            out.pop(k)
    return out


def write_snapshot(model_dir: str, cfg: dict, seed: int, files: int = 2, tied: bool = False) -> Dict[str, np.ndarray]:
    """An MLX-format safetensors snapshot of the synthetic model: config.json
    and `files` .safetensors files (tensors spread over them by sorted name).
    Returns the tensors written."""
    import json
    import os
    from safetensors.numpy import save_file
    os.makedirs(model_dir, exist_ok=True)
    w = snapshot_weights(cfg, seed, tied)
    names = sorted(w)
    for f in range(files):
        part = {n: np.ascontiguousarray(w[n]) for i, n in enumerate(names) if i % files == f}
        save_file(part, os.path.join(model_dir, f"model-{f + 1:05d}-of-{files:05d}.safetensors"))
    conf = dict(cfg, tie_word_embeddings=bool(tied))
    with open(os.path.join(model_dir, "config.json"), "w") as fh:
        json.dump(conf, fh, indent=1, sort_keys=True)
    return w

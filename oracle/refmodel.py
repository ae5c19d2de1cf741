"""Drive the reference's own NumPy backend -- TEST INFRASTRUCTURE ONLY.

Used in the build container (where the reference tree is mounted) to produce
golden fixtures and to pin ``oracle/stage.py``.  It imports the reference's
``hetero.cpu_model`` from its own tree, unmodified, and points its ctypes
kernel loader (``hetero/cpu_model.py:33-45``) at the reference kernel built
from source in ``oracle/_ref/`` instead of the prebuilt binary that ships in
the reference tree (that binary is never loaded).  Nothing on the GPU box
imports this module: the reference tree does not exist there.
"""
from __future__ import annotations

import ctypes
import importlib
import os
import sys
from typing import Dict, List, Optional

import numpy as np

from .q4 import REF_DIR, REF_VARIANTS

# The reference checkout: $HETERO_REF_ROOT, else a directory named
# `reference` beside this repository.
REF_ROOT = os.environ.get("HETERO_REF_ROOT") or os.path.abspath(
    os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "reference"))


def available() -> bool:
    return os.path.exists(os.path.join(REF_ROOT, "hetero", "cpu_model.py"))


def load_cpu_model(variant: str = "avx2", threads: Optional[int] = None):
    """Import the reference ``hetero.cpu_model`` with the kernel variant given."""
    if not available():
        raise FileNotFoundError(f"reference tree not found at {REF_ROOT}")
    threads = threads or os.cpu_count() or 1
    # The reference kernel pool defaults to 4 threads and clamps every call to
    # it (kernel/q4gemv.c:219-222,274-275): set it to the core count.
    os.environ.setdefault("HETERO_KERNEL_THREADS", str(min(threads, 16)))
    os.environ.setdefault("HETERO_THREADS", str(threads))
    built = os.path.join(REF_DIR, REF_VARIANTS[variant])
    if not os.path.exists(built):
        raise FileNotFoundError(f"{built} missing: run make -C oracle ref")
    shipped = os.path.join(REF_ROOT, "kernel", "libq4gemv.so")
    real_cdll = ctypes.CDLL

    def redirect(name, *a, **k):
        if os.path.abspath(str(name)) == os.path.abspath(shipped):
            name = built
        return real_cdll(name, *a, **k)

    if REF_ROOT not in sys.path:
        sys.path.insert(0, REF_ROOT)
    ctypes.CDLL = redirect
    try:
        if "hetero.cpu_model" in sys.modules:
            cm = importlib.reload(sys.modules["hetero.cpu_model"])
        else:
            cm = importlib.import_module("hetero.cpu_model")
    finally:
        ctypes.CDLL = real_cdll
    if cm.KERNEL is None or os.path.abspath(cm.KERNEL._name) != os.path.abspath(built):
        raise RuntimeError("reference cpu_model did not bind the kernel built from source")
    return cm


def build_stage(cm, cfg: dict, weights: Dict[str, np.ndarray], start: int, end: int,
                embed: bool, head: bool):
    """A reference ``Stage`` over in-memory weights (hetero/cpu_model.py:309-333).

    The benchmark model has an fp16 embedding table rather than a quantised one;
    the stage's ``embed`` is replaced by a plain fp16->fp32 row lookup, which is
    what the device stage does too.  A synthetic table (hetero_infer_b200.synth)
    is evaluated row by row on demand."""
    from hetero.shard import ShardSpec
    from hetero_infer_b200 import synth
    w = dict(weights)
    table = w.pop("model.embed_tokens.table", None)
    seed = w.pop(synth.EMBED_SYNTH_KEY, None)
    hidden = cfg["hidden_size"]
    if table is None and seed is not None:
        s_ = int(seed)
        table_rows = lambda ids: synth.embed_rows(s_, ids, hidden)
    elif table is not None:
        table_rows = lambda ids: table[np.asarray(ids).reshape(-1)]
    else:
        table_rows = None
    if embed:
        # Stage.__init__ insists on quantised embedding tensors when it owns the
        # embedding; give it placeholders and swap in the fp16 lookup below.
        w["model.embed_tokens.weight"] = np.zeros((1, 1), np.uint32)
        w["model.embed_tokens.scales"] = np.zeros((1, 1), np.float16)
        w["model.embed_tokens.biases"] = np.zeros((1, 1), np.float16)
    stage = cm.Stage(cfg, ShardSpec(start, end, embed, head), w)
    if embed:
        if table_rows is None:
            raise KeyError("embedding table")
        stage.embed = lambda ids: table_rows(np.asarray(ids).reshape(-1)).astype(np.float32).reshape(
            *np.asarray(ids).shape, -1)
    return stage


def greedy_decode(cm, stage, prompt: np.ndarray, n_tokens: int):
    """Prefill then greedy steps, as Coordinator.generate drives one stage
    (hetero/coordinator.py:266-292, engine.py:68-93): returns tokens, and per
    step the top-1/top-2 logit margin and the logits' L2 norm."""
    caches = [cm.KVCache() for _ in stage.layers]
    toks: List[int] = []
    margins: List[float] = []
    norms: List[float] = []
    x = np.asarray(prompt)
    for _ in range(n_tokens):
        y = stage(x, caches, apply_head=True, last_only=True)
        z = np.asarray(y[:, -1, :], dtype=np.float32).reshape(-1)
        t = int(z.argmax())
        top2 = np.partition(z, -2)[-2:]
        margins.append(float(top2[1] - top2[0]))
        norms.append(float(np.linalg.norm(z)))
        toks.append(t)
        x = np.array([[t]])
    return toks, margins, norms

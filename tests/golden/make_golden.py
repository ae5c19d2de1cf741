"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference's own NumPy stage (hetero/cpu_model.py, imported unmodified
from the reference tree, with its kernel/q4gemv.c compiled from source into
oracle/_ref/ by oracle/Makefile) on the seeded synthetic models of
hetero_infer_b200/synth.py, and records what it produces.  Needs the reference
tree (build container only); the GPU tests read the fixtures it writes.

  python tests/golden/make_golden.py [--small] [--big]

golden_small.npz  2-layer qwen2 (hidden 256): prompt, 8 greedy tokens and the
                  per-step last-position logits, for the reference's float and
                  AVX2 kernel builds.
golden_7b.json    the benchmark's Qwen2-7B-shape random model (seed 0): 32-token
                  prompt, 128 greedy tokens, per-step top-1/top-2 margin, logits
                  L2 norm and top-5 (index, value), for both kernel builds.
golden_7b_pipe.json  the same model split at the planner's 2/4/8-GPU cuts, the
                  stages joined by the reference backend's own wire conversion
                  (NumpyBackend.to_wire / from_wire, fp16) and greedy sampling
                  (NumpyBackend.sample): per cut set and prompt, the tokens, how
                  many wire elements overflowed fp16, and whether the logits
                  were finite.
"""
import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

SMALL = dict(layers=2, hidden=256, heads=4, kv_heads=2, inter=512, vocab=1024)
SMALL_SEED, SMALL_PROMPT, SMALL_TOKENS = 7, 6, 8
BIG_SEED, BIG_PROMPT, BIG_TOKENS = 0, 32, 128
PIPE_CUTS = {2: [0, 14, 28], 4: [0, 7, 14, 21, 28], 8: [0, 3, 6, 9, 12, 16, 20, 24, 28]}
PIPE_PROMPT_SEEDS, PIPE_TOKENS = (1000, 1001), 6


def run_small(variant):
    from hetero_infer_b200 import synth
    from oracle import refmodel
    cfg = synth.small_config(**SMALL)
    w = synth.model_weights(cfg, SMALL_SEED)
    cm = refmodel.load_cpu_model(variant)
    st = refmodel.build_stage(cm, cfg, w, 0, cfg["num_hidden_layers"], True, True)
    prompt = synth.prompt_ids(SMALL_SEED, SMALL_PROMPT, cfg["vocab_size"])
    caches = [cm.KVCache() for _ in st.layers]
    x, toks, logits = prompt, [], []
    for _ in range(SMALL_TOKENS):
        y = st(x, caches, apply_head=True, last_only=True)
        z = np.asarray(y[0, -1], np.float32)
        logits.append(z)
        toks.append(int(z.argmax()))
        x = np.array([[toks[-1]]])
    return prompt, np.array(toks, np.int64), np.stack(logits)


def run_big(variant):
    from hetero_infer_b200 import synth
    from oracle import refmodel
    cfg = dict(synth.QWEN2_7B)
    t0 = time.time()
    w = synth.model_weights(cfg, BIG_SEED)
    cm = refmodel.load_cpu_model(variant)
    st = refmodel.build_stage(cm, cfg, w, 0, cfg["num_hidden_layers"], True, True)
    prompt = synth.prompt_ids(BIG_SEED, BIG_PROMPT, cfg["vocab_size"])
    caches = [cm.KVCache() for _ in st.layers]
    x, steps = prompt, []
    for _ in range(BIG_TOKENS):
        y = st(x, caches, apply_head=True, last_only=True)
        z = np.asarray(y[0, -1], np.float32)
        top = np.argsort(-z, kind="stable")[:5]
        srt = np.sort(z)
        steps.append({"token": int(z.argmax()), "margin": float(srt[-1] - srt[-2]),
                      "norm": float(np.linalg.norm(z)), "top5_idx": [int(i) for i in top],
                      "top5_val": [float(z[i]) for i in top]})
        x = np.array([[steps[-1]["token"]]])
    return prompt, steps, time.time() - t0


def run_pipe(variant):
    import importlib
    from hetero_infer_b200 import synth
    from oracle import refmodel
    cfg = dict(synth.QWEN2_7B)
    L = cfg["num_hidden_layers"]
    w = synth.model_weights(cfg, BIG_SEED)
    cm = refmodel.load_cpu_model(variant)
    be = importlib.import_module("hetero.backends").NumpyBackend()
    out = {}
    for n, cuts in PIPE_CUTS.items():
        stages = [refmodel.build_stage(cm, cfg, w, a, b, a == 0, b == L) for a, b in zip(cuts, cuts[1:])]
        runs = []
        for ps in PIPE_PROMPT_SEEDS:
            prompt = synth.prompt_ids(ps, BIG_PROMPT, cfg["vocab_size"])
            caches = [[cm.KVCache() for _ in st.layers] for st in stages]
            x, toks, overflow, finite = prompt, [], 0, []
            for _ in range(PIPE_TOKENS):
                h = x
                for i, st in enumerate(stages):
                    last = i == len(stages) - 1
                    y = st(h, caches[i], apply_head=last, last_only=last)
                    if not last:
                        wire = be.to_wire(y)
                        overflow += int(np.isinf(wire).sum())
                        h = be.from_wire(wire)
                z = np.asarray(y[0, -1], np.float32)
                finite.append(bool(np.isfinite(z).all()))
                toks.append(be.sample(z, 0.0, 1.0, None))
                x = np.array([[toks[-1]]])
            runs.append({"prompt_seed": ps, "tokens": toks, "wire_inf_elements": overflow,
                         "logits_finite": finite})
            print(variant, n, ps, toks, overflow, finite, flush=True)
        out[str(n)] = {"cuts": cuts, "runs": runs}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--small", action="store_true")
    ap.add_argument("--big", action="store_true")
    ap.add_argument("--pipe", action="store_true")
    a = ap.parse_args()
    if not (a.small or a.big or a.pipe):
        a.small = a.big = a.pipe = True
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "all"], check=True, capture_output=True)
    if a.small:
        out = {}
        for v in ("float", "avx2"):
            # each variant in its own process: the reference module binds one kernel
            code = ("import sys, numpy as np; sys.path.insert(0, %r); sys.path.insert(0, %r); "
                    "import make_golden as m; p, t, l = m.run_small(%r); "
                    "np.savez(%r, prompt=p, tokens=t, logits=l)") % (
                ROOT, HERE, v, os.path.join(HERE, f"_tmp_{v}.npz"))
            subprocess.run([sys.executable, "-c", code], check=True)
            d = np.load(os.path.join(HERE, f"_tmp_{v}.npz"))
            out["prompt"] = d["prompt"]
            out[f"tokens_{v}"], out[f"logits_{v}"] = d["tokens"], d["logits"]
            os.remove(os.path.join(HERE, f"_tmp_{v}.npz"))
        np.savez_compressed(os.path.join(HERE, "golden_small.npz"), **out)
        print("golden_small.npz", {k: v.shape for k, v in out.items()})
    if a.big:
        res = {"config": "QWEN2_7B", "seed": BIG_SEED, "prompt_tokens": BIG_PROMPT,
               "generated": BIG_TOKENS, "variants": {}}
        for v in ("avx2", "float"):
            code = ("import sys, json; sys.path.insert(0, %r); sys.path.insert(0, %r); "
                    "import make_golden as m; p, s, dt = m.run_big(%r); "
                    "json.dump({'prompt': [int(i) for i in p.reshape(-1)], 'steps': s, 'seconds': dt}, "
                    "open(%r, 'w'))") % (ROOT, HERE, v, os.path.join(HERE, f"_tmp_{v}.json"))
            subprocess.run([sys.executable, "-c", code], check=True)
            d = json.load(open(os.path.join(HERE, f"_tmp_{v}.json")))
            os.remove(os.path.join(HERE, f"_tmp_{v}.json"))
            res["prompt"] = d["prompt"]
            res["variants"][v] = {"steps": d["steps"], "seconds": round(d["seconds"], 1),
                                  "kernel": "kernel/q4gemv.c built " +
                                            ("-O3 -mavx2 -mfma -mf16c" if v == "avx2" else "-O3 (portable fp32 path)")}
            print(v, "tokens", [s["token"] for s in d["steps"]][:16], "...", round(d["seconds"], 1), "s")
        with open(os.path.join(HERE, "golden_7b.json"), "w") as f:
            json.dump(res, f)
    if a.pipe:
        res = {"config": "QWEN2_7B", "seed": BIG_SEED, "prompt_tokens": BIG_PROMPT, "generated": PIPE_TOKENS,
               "wire": "NumpyBackend.to_wire (fp16)", "variants": {}}
        for v in ("avx2", "float"):
            tmp = os.path.join(HERE, f"_tmp_pipe_{v}.json")
            code = ("import sys, json; sys.path.insert(0, %r); sys.path.insert(0, %r); "
                    "import make_golden as m; json.dump(m.run_pipe(%r), open(%r, 'w'))") % (ROOT, HERE, v, tmp)
            subprocess.run([sys.executable, "-c", code], check=True)
            res["variants"][v] = json.load(open(tmp))
            os.remove(tmp)
        with open(os.path.join(HERE, "golden_7b_pipe.json"), "w") as f:
            json.dump(res, f)


if __name__ == "__main__":
    main()

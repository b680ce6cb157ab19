#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ by running the UNMODIFIED reference forward.

The reference's whole-model CPU oracle is ``tools/reference_qwen2.py`` (pure numpy). This script
writes seeded random-init Qwen2 GGUFs (``muyo_llm_b200.gguf``), runs that file as a subprocess,
and stores what it prints or dumps:

* ``qwen2_tiny.npz``  a 2-layer model of the same architecture, 8 prompt ids: the per-step argmax
  and top-5 the reference prints, its step-0 intermediates (``REF_DUMP``,
  ``tools/reference_qwen2.py:116-165``) and the last step's logits.
* ``qwen2_05b_greedy.json``  the Qwen2.5-0.5B-architecture config (24 layers, vocab 151936):
  32 seeded prompt ids and 256 greedy ids. The reference only teacher-forces the ids it is given
  (``tools/reference_qwen2.py:101-168``), so a candidate greedy sequence is produced by the C
  oracle, fed back through the reference once, and accepted only where the reference's argmax at
  every step equals the next id. On a disagreement the reference's id is taken, the oracle
  regenerates the tail from there, and the check repeats.

Run from the repository root, in the container where the reference is mounted:
    python tests/golden/make_golden.py [--tiny] [--full] [--ref PATH]
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from muyo_llm_b200 import gguf, synth  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
TINY_SEED = 1234
FULL_SEED = 20261201
FULL_PROMPT = 32
FULL_PREDICT = 256

_STEP = re.compile(r"\[ref\] step (\d+) argmax (\d+) top5 \[(.*)\]")
_PAIR = re.compile(r"\((\d+), (-?[\d.e+-]+)\)")

def dump_lengths(cfg) -> dict[str, int]:
    """Element count of each step-0 dump (``tools/reference_qwen2.py:116-165``). Under NumPy 2 the
    division by ``np.sqrt(head_dim)`` (line 135) promotes the scores to float64, and everything
    downstream of them stays float64, so the element size is read off the file size."""
    h, q, kv, f = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.ffn
    return {"embedding": h, "b0.xn": h, "b0.q": q, "b0.kvec": kv, "b0.qr": q, "b0.vvec": kv,
            "b0.scores": cfg.heads, "b0.probs": cfg.heads, "b0.attn_out": q, "b0.o": h, "b0.x1": h,
            "b0.gate": f, "b0.up": f, "b0.act": f, "b0.mlp_out": h, "b0.out": h, "final_norm": h,
            "logits": cfg.vocab}


def read_dump(path: str, n: int) -> np.ndarray:
    size = os.path.getsize(path)
    dtype = {4 * n: np.float32, 8 * n: np.float64}[size]
    return np.fromfile(path, dtype)


def run_reference(ref: str, gguf_path: str, ids, dump_dir: str | None = None, out: str | None = None):
    """Run reference_qwen2.py unmodified; return [(step, argmax, [(id, logit)...])]."""
    env = dict(os.environ)
    if dump_dir:
        env["REF_DUMP"] = dump_dir
    cmd = [sys.executable, ref, gguf_path, ",".join(str(int(i)) for i in ids)] + ([out] if out else [])
    t0 = time.time()
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, check=True)
    steps = []
    for line in proc.stderr.splitlines():
        m = _STEP.match(line)
        if m:
            top = [(int(a), float(b)) for a, b in _PAIR.findall(m.group(3))]
            steps.append((int(m.group(1)), int(m.group(2)), top))
    print(f"[golden] reference ran {len(ids)} steps in {time.time() - t0:.1f}s", file=sys.stderr)
    return steps


def make_tiny(ref: str) -> None:
    cfg = synth.QWEN2_TINY
    ids = synth.prompt_ids(TINY_SEED, 8, cfg.vocab)
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "tiny.gguf")
        gguf.write_synthetic_qwen2(path, cfg, TINY_SEED)
        dump_dir = os.path.join(tmp, "dump")
        os.mkdir(dump_dir)
        logits_path = os.path.join(tmp, "last_logits.bin")
        steps = run_reference(ref, path, ids, dump_dir=dump_dir, out=logits_path)
        arrays = {}
        for name, n in dump_lengths(cfg).items():
            arrays["dump_" + name.replace(".", "_")] = read_dump(os.path.join(dump_dir, name + ".bin"), n)
        raw = np.fromfile(logits_path, np.uint8)
        vocab = int(raw[:4].view(np.int32)[0])
        arrays["last_logits"] = raw[4:].view(np.float32)[:vocab].copy()
    arrays["ids"] = ids
    arrays["seed"] = np.int64(TINY_SEED)
    arrays["argmax"] = np.array([s[1] for s in steps], np.int32)
    arrays["top5_ids"] = np.array([[t[0] for t in s[2]] for s in steps], np.int32)
    np.savez_compressed(os.path.join(HERE, "qwen2_tiny.npz"), **arrays)
    print("[golden] wrote qwen2_tiny.npz", file=sys.stderr)


def make_full(ref: str) -> None:
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # the C restatement: only proposes candidates, the reference decides

    cfg = synth.QWEN2_05B
    prompt = synth.prompt_ids(FULL_SEED, FULL_PROMPT, cfg.vocab)
    model = synth.make_model(cfg, FULL_SEED)
    forced = list(int(i) for i in prompt)
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "qwen2_05b.gguf")
        gguf.write_synthetic_qwen2(path, cfg, FULL_SEED)
        for attempt in range(8):
            seq, margins = oracle.qwen2_greedy(cfg, model, forced, FULL_PROMPT + FULL_PREDICT, kv_f16=False)
            steps = run_reference(ref, path, seq[:-1])
            mismatch = None
            for step, arg, _top in steps:
                if step >= FULL_PROMPT - 1 and arg != seq[step + 1]:
                    mismatch = step
                    break
            if mismatch is None:
                break
            print(f"[golden] reference disagrees at step {mismatch}: oracle {seq[mismatch + 1]} "
                  f"reference {steps[mismatch][1]} (oracle margin {margins[mismatch]:.3g})", file=sys.stderr)
            forced = seq[:mismatch + 1] + [steps[mismatch][1]]
        else:
            raise SystemExit("[golden] no agreement after 8 attempts")
    top5 = {str(s): [[i, v] for i, v in t] for s, _a, t in steps[:4]}
    doc = {
        "config": {k: getattr(cfg, k) for k in ("layers", "hidden", "ffn", "heads", "kv_heads", "vocab",
                                                 "rms_eps", "rope_base", "max_seq")},
        "seed": FULL_SEED,
        "n_prompt": FULL_PROMPT,
        "n_predict": FULL_PREDICT,
        "prompt": [int(i) for i in prompt],
        "generated": [int(i) for i in seq[FULL_PROMPT:]],
        "reference_argmax": [int(a) for _s, a, _t in steps],
        "oracle_top2_margin": [float(m) for m in margins],
        "reference_top5_first_steps": top5,
        "kv_cache": "f32 (as tools/reference_qwen2.py:127-130)",
        "made_by": "tests/golden/make_golden.py running tools/reference_qwen2.py unmodified",
    }
    with open(os.path.join(HERE, "qwen2_05b_greedy.json"), "w") as f:
        json.dump(doc, f, indent=1)
    print("[golden] wrote qwen2_05b_greedy.json", file=sys.stderr)


def make_full_f16() -> None:
    """Adds the oracle's greedy ids with the F16 KV cache BASELINE names (keys after RoPE and values
    rounded to F16 at append) to the 0.5B fixture. The reference forward keeps an F32 cache
    (tools/reference_qwen2.py:127-130), so this sequence is the oracle's, pinned by the F32 run above."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    path = os.path.join(HERE, "qwen2_05b_greedy.json")
    doc = json.load(open(path))
    cfg = synth.QWEN2_05B
    model = synth.make_model(cfg, doc["seed"])
    seq, margins = oracle.qwen2_greedy(cfg, model, doc["prompt"], doc["n_prompt"] + doc["n_predict"], kv_f16=True)
    doc["oracle_kv_f16_generated"] = [int(i) for i in seq[doc["n_prompt"]:]]
    doc["oracle_kv_f16_top2_margin"] = [float(m) for m in margins]
    with open(path, "w") as f:
        json.dump(doc, f, indent=1)
    print("[golden] added the F16-cache oracle ids to qwen2_05b_greedy.json", file=sys.stderr)


def main() -> None:
    ap = argparse.ArgumentParser()
    ref_tree = os.environ.get("MUYO_REFERENCE")
    ap.add_argument("--ref", default=os.path.join(ref_tree, "tools", "reference_qwen2.py") if ref_tree else None,
                    help="the reference's tools/reference_qwen2.py (default: under $MUYO_REFERENCE)")
    ap.add_argument("--tiny", action="store_true")
    ap.add_argument("--full", action="store_true")
    ap.add_argument("--full-f16", action="store_true")
    a = ap.parse_args()
    if (a.tiny or a.full or not a.full_f16) and not a.ref:
        ap.error("give --ref or set MUYO_REFERENCE to the muyo-llm source tree")
    if not (a.tiny or a.full or a.full_f16):
        a.tiny = a.full = a.full_f16 = True
    if a.tiny:
        make_tiny(a.ref)
    if a.full:
        make_full(a.ref)
    if a.full_f16:
        make_full_f16()


if __name__ == "__main__":
    main()

"""Writes tests/golden/sampler_cases.json: the draws of the REFERENCE's own Sampler (src/Sampler.cpp,
compiled unmodified into oracle/_ref/libsampler_ref.so by oracle/Makefile) on seeded inputs, so that
the sampler restatement (oracle_sample) is pinned to it where the reference tree is absent.

Per case (penalty, temperature, top-k, top-p, window, engine seed): 40 consecutive draws over a
151936-entry vocabulary. Step s draws from (numpy default_rng(1000 + case)) standard-normal logits
scaled by 3, with a history of 20 seeded ids plus the first 5 again, extended by every drawn id.
Recorded: each drawn id and the SHA-256 of the logits the Sampler leaves behind (it modifies them in
place: penalty, temperature), so a restatement must match them bit for bit. Run from the repo root
in the build container, with MUYO_REFERENCE naming the reference tree:
    MUYO_REFERENCE=<tree> python tests/golden/make_sampler_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

CASES = [
    dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1, repeat_last_n=64, seed=7),
    dict(temperature=1.0, top_k=0, top_p=0.9, repeat_penalty=1.0, repeat_last_n=64, seed=123),
    dict(temperature=0.5, top_k=1, top_p=0.95, repeat_penalty=1.3, repeat_last_n=-1, seed=5),
    dict(temperature=1.2, top_k=200, top_p=1.0, repeat_penalty=0.9, repeat_last_n=8, seed=2**63 + 11),
    dict(temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.2, repeat_last_n=16, seed=1),
]
VOCAB = 151936
STEPS = 40


def inputs(case: int):
    """The history and a generator of the per-step logits of case `case` (shared with the test)."""
    rng = np.random.default_rng(1000 + case)
    history = [int(i) for i in rng.integers(0, VOCAB, 20)]
    history += history[:5]

    def next_logits():
        return (rng.standard_normal(VOCAB) * 3).astype(np.float32)

    return history, next_logits


def main() -> None:
    import oracle

    if oracle.build_ref() is None:
        sys.exit("the reference tree is needed: set MUYO_REFERENCE")
    out = {"vocab": VOCAB, "steps": STEPS, "made_by": "tests/golden/make_sampler_golden.py with the reference's "
           "src/Sampler.cpp compiled unmodified (oracle/_ref/libsampler_ref.so)", "cases": []}
    for c, kw in enumerate(CASES):
        ref = oracle.RefSampler(**kw)
        history, next_logits = inputs(c)
        tokens, digests = [], []
        for _ in range(STEPS):
            logits = next_logits()
            t = ref.sample(logits, history)
            tokens.append(t)
            digests.append(hashlib.sha256(logits.tobytes()).hexdigest())
            history.append(t)
        out["cases"].append({"params": {k: (str(v) if k == "seed" else v) for k, v in kw.items()},
                             "tokens": tokens, "logits_sha256": digests})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler_cases.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print(f"wrote {path}", file=sys.stderr)


if __name__ == "__main__":
    main()

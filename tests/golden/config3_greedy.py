"""Selects the BASELINE config-3 prompt for the bf16 greedy-identity test and writes its fixture,
tests/golden/config3_greedy.npz.

The bf16 path must give the CPU reference's greedy tokens for 64 steps. A step can only be held to that where the
reference's top-2 margin exceeds the bf16 path's logit error (a smaller margin can flip in any bf16 implementation),
so the prompt is chosen the way the reference chooses its own greedy prompts (tools/goldens/tiny_model.py:67-70: the
first candidate whose top-2 margin is at least MIN_MARGIN at every one of the 64 steps), with MIN_MARGIN = 2 x the
worst bf16 logit error measured at config 3 (0.0202, teacher forced over 128 steps).

    python tests/golden/config3_greedy.py screen [candidates] [out.json]   # on a GPU: the bf16 engine
    python tests/golden/config3_greedy.py confirm SEED [out.npz]            # on the CPU: the oracle

`screen` runs every candidate prompt (512 uniform-random ids, random_prompt(vocab, 512, seed=s,
stream="config3-greedy"), s = 0, 1, ...) through the engine's free-running greedy schedule, 64 at a time, and lists
the candidates whose engine margin is at least 2 x MIN_MARGIN at all 64 steps (so the reference's margins clear
MIN_MARGIN whatever the sign of the errors), with how many distinct ids their 64 tokens hold. Random-weight models
mostly settle into repeating one token; of the passing candidates the one with the most distinct ids (lowest seed on
ties) is taken, so the test covers a trajectory whose tokens change.

`confirm` runs the oracle (fp32, the reference's schedule) on that prompt, checks that its margin is at least
MIN_MARGIN at every step, and stores the seed, the oracle's 64 ids and margins and, per step, the logits at 2,048
fixed columns (every 8th of tests/golden/make_config45.py's sample) plus the top 64.
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

PROMPT, STEPS = 512, 64
BF16_WORST_ERR = 0.0202
MIN_MARGIN = 2 * BF16_WORST_ERR


def config():
    from rosylnalive_b200 import synthetic as S

    return dataclasses.replace(S.QWEN3_0_6B, max_pos=PROMPT + STEPS + 16)


def prompt(seed: int) -> np.ndarray:
    from rosylnalive_b200 import synthetic as S

    return S.random_prompt(S.QWEN3_0_6B.vocab, PROMPT, seed=seed, stream="config3-greedy")


def screen(candidates: int, out: str) -> None:
    import torch

    from rosylnalive_b200 import qwen as Qw
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S

    cfg = config()
    B = 64
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    passing = []
    t0 = time.time()
    with Qw.QwenEngine(cfg, weights, cos, sin, max_seqs=B, max_tokens=B * PROMPT, max_batch=B) as eng:
        for b0 in range(0, candidates, B):
            seeds = list(range(b0, min(candidates, b0 + B)))
            ids, logits = eng.greedy([prompt(s) for s in seeds], STEPS, want_logits=True)
            top2 = torch.from_numpy(logits.reshape(-1, cfg.vocab)).topk(2, dim=1).values
            margins = (top2[:, 0] - top2[:, 1]).numpy().reshape(len(seeds), STEPS)
            for i, s in enumerate(seeds):
                if margins[i].min() >= 2 * MIN_MARGIN:
                    passing.append({"seed": s, "distinct": int(len(set(ids[i].tolist()))),
                                    "min_margin": float(margins[i].min()), "ids": ids[i].tolist()})
    passing.sort(key=lambda r: (-r["distinct"], r["seed"]))
    with open(out, "w") as f:
        json.dump({"candidates": candidates, "threshold": 2 * MIN_MARGIN, "passing": passing}, f)
    print(f"{candidates} candidates in {time.time() - t0:.0f} s; {len(passing)} pass; best "
          f"{[(r['seed'], r['distinct'], round(r['min_margin'], 3)) for r in passing[:10]]}")


def confirm(seed: int, out: str) -> None:
    from oracle import oracle as O
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S
    from tests.golden.make_config45 import columns, row_summary

    cfg = config()
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    oc = O.Config(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab, cfg.eps,
                  cfg.max_pos)
    t0 = time.time()
    ids, logits = O.greedy(O.Model.from_hf(oc, weights, cos, sin), prompt(seed), STEPS, "f32", return_logits=True)
    cols = columns(cfg.vocab)[::8]  # 2,048 of make_config45's sampled columns: 64 rows stay a small fixture
    rows = [row_summary(lg, cols) for lg in logits]
    margins = np.array([r["margin"] for r in rows])
    print(f"oracle greedy in {time.time() - t0:.0f} s: ids {ids.tolist()}; min margin {margins.min():.4f}")
    if margins.min() < MIN_MARGIN:
        raise SystemExit(f"seed {seed}: the oracle's margin falls to {margins.min():.4f} < {MIN_MARGIN}")
    res = {"seed": np.int64(seed), "ids": ids.astype(np.int64), "min_margin": np.float64(MIN_MARGIN),
           "columns": cols}
    for k in rows[0]:
        res[k] = np.stack([np.asarray(r[k]) for r in rows])
    np.savez_compressed(out, **res)
    with open(out, "rb") as f:
        print(f"wrote {out}: sha256 {hashlib.sha256(f.read()).hexdigest()}")


if __name__ == "__main__":
    if len(sys.argv) >= 2 and sys.argv[1] == "screen":
        screen(int(sys.argv[2]) if len(sys.argv) > 2 else 4096,
               sys.argv[3] if len(sys.argv) > 3 else "config3_screen.json")
    elif len(sys.argv) >= 3 and sys.argv[1] == "confirm":
        confirm(int(sys.argv[2]), sys.argv[3] if len(sys.argv) > 3 else os.path.join(HERE, "config3_greedy.npz"))
    else:
        raise SystemExit(__doc__)

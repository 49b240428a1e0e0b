"""Generates tests/golden/config45.npz: the CPU reference's (the oracle's, fp32) outputs for BASELINE configs 4 and 5
at their own sizes, so the GPU tests can check the bench's own shapes without running a multi-minute oracle on the
GPU host.

    python tests/golden/make_config45.py [out.npz]        (about 15 minutes on 8 cores)

Model: the Qwen3-0.6B architecture with the seeded random weights every full-size test and the bench use
(rosylnalive_b200.synthetic.random_weights(QWEN3_0_6B, seed=0)), RoPE T_spec from the pinned inverse frequencies.
The composition is the reference's forward and greedy schedule (tests/Lrm.Tensor.Tests/TinyModel.fs:144-236) as
oracle/oracle.py restates it, in fp32.

  * config 5: one 4096-token prompt (random_prompt(vocab, 4096, seed=5, stream="config5-parity")), its prefill and
    8 greedy decode steps; for each of the 9 logits rows (prefill last row, then each step) the oracle's argmax,
    top-2 margin, full-row L2 norm, its 64 largest logits (index, value) and the values at 16,384 fixed columns
    (a seeded sample of the vocabulary, the same for every row); the 8 fed tokens; and the final residual stream
    (the last layer's output, before the final norm) of the rows ROWS5 of the prompt.
  * config 4: one 2048-token prompt (seed=4, stream="config4-parity"), its prefill: the last row's logits as above
    and the final residual of the rows ROWS4.

Logits are stored as the column sample plus the top 64 rather than whole rows (151,936 floats each) to keep the
fixture small; the GPU tests compare on those columns and the argmax/margin of the whole row.
"""

from __future__ import annotations

import dataclasses
import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from rosylnalive_b200 import rope as R  # noqa: E402
from rosylnalive_b200 import synthetic as S  # noqa: E402

STEPS5 = 8
LEN5, LEN4 = 4096, 2048
ROWS5 = (0, 1, 15, 16, 127, 128, 2047, 4094, 4095)
ROWS4 = (0, 1, 15, 16, 127, 128, 1000, 2046, 2047)
NCOLS, TOPK = 16384, 64


def columns(vocab: int) -> np.ndarray:
    return np.sort(np.random.default_rng(12345).choice(vocab, NCOLS, replace=False)).astype(np.int64)


def prompt5(vocab):
    return S.random_prompt(vocab, LEN5, seed=5, stream="config5-parity")


def prompt4(vocab):
    return S.random_prompt(vocab, LEN4, seed=4, stream="config4-parity")


class _Keep(dict):
    """A taps dict that keeps only the named intermediates (the rest of a 4096-token forward is gigabytes)."""

    def __init__(self, names):
        super().__init__()
        self.names = set(names)

    def __setitem__(self, k, v):
        if k in self.names:
            super().__setitem__(k, np.array(v, copy=True))


def row_summary(logits: np.ndarray, cols: np.ndarray) -> dict:
    lg = np.asarray(logits, np.float32)
    top = np.argsort(-lg, kind="stable")[:TOPK]
    part = np.partition(lg, -2)
    return {"argmax": int(O.argmax_rows(lg[None], "f32")[0]), "margin": float(part[-1] - part[-2]),
            "norm": float(np.linalg.norm(lg.astype(np.float64))), "top_idx": top.astype(np.int64),
            "top_val": lg[top], "cols_val": lg[cols]}


def main(out: str) -> None:
    t0 = time.time()
    cfg = dataclasses.replace(S.QWEN3_0_6B, max_pos=LEN5 + STEPS5 + 16)
    weights = S.random_weights(cfg, seed=0)
    cos, sin = R.t_spec(R.torch_inv_freq_bits(cfg.rope_theta, cfg.head_dim), cfg.max_pos)
    oc = O.Config(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab, cfg.eps,
                  cfg.max_pos)
    m = O.Model.from_hf(oc, weights, cos, sin)
    cols = columns(cfg.vocab)
    last = f"L{cfg.layers - 1}.out"
    res = {"columns": cols, "rows5": np.array(ROWS5, np.int64), "rows4": np.array(ROWS4, np.int64)}

    # config 4: one 2048-token prefill
    p4 = prompt4(cfg.vocab)
    keep = _Keep([last])
    cache = O.Cache.new(oc, "f32")
    lg = O.forward(m, cache, 0, p4, "f32", taps=keep, logits_rows="last")
    s = row_summary(lg[-1], cols)
    for k, v in s.items():
        res[f"c4_{k}"] = np.asarray(v)
    res["c4_hidden"] = keep[last][list(ROWS4)].astype(np.float32)
    res["c4_prompt"] = p4
    print(f"config 4 prefill done at {time.time() - t0:.0f} s; argmax {s['argmax']} margin {s['margin']:.4f}",
          flush=True)
    del cache, keep

    # config 5: a 4096-token prefill, then 8 greedy decode steps
    p5 = prompt5(cfg.vocab)
    keep = _Keep([last])
    cache = O.Cache.new(oc, "f32")
    lg = O.forward(m, cache, 0, p5, "f32", taps=keep, logits_rows="last")
    res["c5_hidden"] = keep[last][list(ROWS5)].astype(np.float32)
    rows = [row_summary(lg[-1], cols)]
    fed = []
    print(f"config 5 prefill done at {time.time() - t0:.0f} s", flush=True)
    for step in range(STEPS5):
        tok = rows[-1]["argmax"]
        fed.append(tok)
        lg = O.forward(m, cache, LEN5 + step, [tok], "f32", logits_rows="last")
        rows.append(row_summary(lg[-1], cols))
    for k in rows[0]:
        res[f"c5_{k}"] = np.stack([np.asarray(r[k]) for r in rows])
    res["c5_fed"] = np.array(fed, np.uint32)
    res["c5_prompt"] = p5
    print(f"config 5 decode done at {time.time() - t0:.0f} s; ids {[r['argmax'] for r in rows]}; margins "
          f"{[round(r['margin'], 4) for r in rows]}", flush=True)
    np.savez_compressed(out, **res)
    with open(out, "rb") as f:
        print(f"wrote {out}: sha256 {hashlib.sha256(f.read()).hexdigest()}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "config45.npz"))

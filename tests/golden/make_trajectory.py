"""Generates the small-LM loss-trajectory fixture from the CPU oracle.

The small decoder LM (6 layers, d_model 512, 8 heads, FFN 2048, vocab 8192,
seq 512, batch 16 = 8,192 tokens per step), N(0, 0.02) weights from a seed,
50 AdamW steps (lr 1e-3, beta 0.9 / 0.999, eps 1e-8, weight decay 0.01,
constant schedule, no clipping) on seeded uniform token batches.  The oracle
restates the reference's per-op arithmetic in its own order (serial f32
sums, glibc libm), and its composition follows the M3 schedule order with
RoPE on Q/K; per-op it is bit-identical to the reference's C providers.

Written to tests/golden/small_lm_trajectory.json:
  * the loss of every step (f32 bit patterns),
  * the final weights at 8,192 seeded indices, with the initial values, so a
    test can bound each sampled element against the update size,
  * the final per-tensor sum of squares (f64).

It takes about an hour and a half on 8 host cores; the GPU tests only read
the JSON.  Usage: python tests/golden/make_trajectory.py
"""
from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle import oracle as orc  # noqa: E402

SHAPE = dict(layers=6, d_model=512, heads=8, ffn=2048, vocabulary=8192, seq_len=512, batch=16)
STEPS = 50
INIT_SEED = 20260503
BATCH_SEED0 = 7000
SAMPLE_SEED = 31337
SAMPLE = 8192
ADAMW = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01)


def batch_seed(step: int) -> int:
    return BATCH_SEED0 + step


def main() -> None:
    s = SHAPE
    om = orc.LanguageModel(s["layers"], s["d_model"], s["heads"], s["ffn"], s["vocabulary"],
                           s["seq_len"], s["batch"])
    params = om.init(INIT_SEED)
    initial = params.copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    opts = orc.adamw_options(ADAMW["lr"], ADAMW["beta1"], ADAMW["beta2"], ADAMW["eps"],
                             ADAMW["weight_decay"])
    losses = []
    t0 = time.time()
    for step in range(1, STEPS + 1):
        ids, targets = orc.synthetic_batch(batch_seed(step), s["batch"], s["seq_len"],
                                           s["vocabulary"])
        loss, grads = om.forward_backward(params, ids, targets)
        assert om.adamw(params, grads, m, v, opts, step) == 0
        losses.append(loss)
        print(f"step {step} loss {loss:.7f} ({time.time() - t0:.0f} s)", flush=True)
    rng = np.random.default_rng(SAMPLE_SEED)
    idx = np.sort(rng.choice(params.size, SAMPLE, replace=False)).astype(np.int64)
    out = {
        "generator": "tests/golden/make_trajectory.py (CPU oracle, liboracle.so)",
        "shape": s, "steps": STEPS, "init_seed": INIT_SEED, "batch_seed0": BATCH_SEED0,
        "adamw": ADAMW,
        "loss_bits": [f"{orc.bits(x):08x}" for x in losses],
        "sample_index": idx.tolist(),
        "sample_initial_bits": [f"{b:08x}" for b in initial[idx].view(np.uint32).tolist()],
        "sample_final_bits": [f"{b:08x}" for b in params[idx].view(np.uint32).tolist()],
        "tensor_sumsq": [float(np.sum(t.astype(np.float64) ** 2)) for t in om.split(params)],
    }
    (HERE / "small_lm_trajectory.json").write_text(json.dumps(out, indent=0) + "\n")


if __name__ == "__main__":
    main()

"""The small LM's 50-step training trajectory against the oracle's.

Small decoder LM (6 layers, d_model 512, 8 heads, FFN 2048, vocab 8192,
seq 512, batch 16), seeded N(0, 0.02) weights, AdamW (lr 1e-3, beta 0.9 /
0.999, eps 1e-8, weight decay 0.01) over 50 seeded batches.  The oracle's
trajectory (serial f32 in the reference's order) is the committed fixture
tests/golden/small_lm_trajectory.json, written on the CPU by
tests/golden/make_trajectory.py.

Bars, in both f32-grade contraction modes:

* loss of step s within LOSS_TOL(s) relative.  Step 1 sees identical weights,
  so its bar is the reference's TR3 loss tolerance, 2e-5.  Later steps start
  from weights that already differ: AdamW moves every weight by about lr per
  step whatever the gradient's size, so a weight whose gradient is close to
  zero can move either way, and the losses drift apart slowly; the bar widens
  linearly, 2e-5 (1 + (s - 1) / 10), i.e. 1.2e-4 at step 50.
* sampled final weights (8,192 seeded indices), against the oracle's after the
  same 50 updates: median distance at most WEIGHT_MEDIAN lr, 99th percentile
  at most WEIGHT_P99 lr, every element within WEIGHT_MAX lr (one update moves
  a weight by up to about lr, so these bound the drift at 1/1000, 1/100 and
  1/20 of a single update).
"""
import json

import numpy as np
import pytest

import eshkol_transformer_b200 as etb
from helpers import GOLDEN
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

WEIGHT_MEDIAN = 1e-3
WEIGHT_P99 = 1e-2
WEIGHT_MAX = 5e-2


def loss_tol(step: int) -> float:
    return 2e-5 * (1.0 + (step - 1) / 10.0)


@pytest.fixture(scope="module")
def fixture():
    return json.loads((GOLDEN / "small_lm_trajectory.json").read_text())


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3])
def test_small_lm_50_step_trajectory(lib, cuda, fixture, precision):
    s = fixture["shape"]
    shape = etb.ModelShape(s["layers"], s["d_model"], s["heads"], s["ffn"], s["vocabulary"],
                           s["seq_len"], s["batch"])
    a = fixture["adamw"]
    model = etb.LanguageModel(shape, precision=precision, lr=a["lr"], beta1=a["beta1"],
                              beta2=a["beta2"], eps=a["eps"], weight_decay=a["weight_decay"])
    model.init(fixture["init_seed"])
    idx = np.array(fixture["sample_index"], np.int64)
    initial = np.array([int(h, 16) for h in fixture["sample_initial_bits"]], np.uint32).view(
        np.float32)
    assert np.array_equal(model.read(0)[idx].view(np.uint32), initial.view(np.uint32))
    want = np.array([int(h, 16) for h in fixture["loss_bits"]], np.uint32).view(np.float32)
    worst = []
    for step in range(1, fixture["steps"] + 1):
        ids, targets = orc.synthetic_batch(fixture["batch_seed0"] + step, shape.batch,
                                           shape.seq_len, shape.vocabulary)
        loss = model.step(ids, targets)
        rel = abs(loss - float(want[step - 1])) / abs(float(want[step - 1]))
        worst.append(rel / loss_tol(step))
        assert rel <= loss_tol(step), (step, loss, float(want[step - 1]), rel)
    final = np.array([int(h, 16) for h in fixture["sample_final_bits"]], np.uint32).view(
        np.float32)
    got = model.read(0)[idx]
    assert model.update_counts() == (fixture["steps"], 0)
    model.close()
    lr = a["lr"]
    diff = np.abs(got.astype(np.float64) - final)
    print(f"precision {precision}: worst loss / bar {max(worst):.2f}; weight diff median "
          f"{np.median(diff) / lr:.2e} lr, p99 {np.percentile(diff, 99) / lr:.2e} lr, max "
          f"{diff.max() / lr:.2e} lr")
    assert np.median(diff) <= WEIGHT_MEDIAN * lr
    assert np.percentile(diff, 99) <= WEIGHT_P99 * lr
    assert diff.max() <= WEIGHT_MAX * lr

"""Parity at the medium LM's widths (the throughput benchmark's shapes).

One layer of the medium decoder LM (d_model 1024, 16 heads, FFN 4096, vocab
32,768, seq 1024) on 4 sequences = 4,096 tokens, in both f32-grade contraction
modes: the weight-gradient GEMMs run split-K over K = 4,096 tokens, the tied
head contracts V = 32,768, attention runs 8 query tiles per (sequence, head),
and in split-f16 mode every operand is a binary16 pair with its tensor's
measured scale.  Gradients are compared tensor by tensor with the oracle
(serial f32 in the reference's order) under the same normwise bound as the
tiny LM, and the per-row error is reported beside it: split-f16 scales are per
tensor, so a row far below its tensor's maximum keeps an absolute error of
about 2^-35 of that maximum per operand element.  PER_ROW_FLOOR states the
per-row bound that follows: |err_row| <= tol * max|row| + floor * max|tensor|.
"""
import numpy as np
import pytest

import eshkol_transformer_b200 as etb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

SHAPE = etb.ModelShape(1, 1024, 16, 4096, 32768, 1024, 4)
SEED, BATCH_SEED = 2027, 314
GRAD_TOL = 5e-5
PER_ROW_FLOOR = 1e-6


@pytest.fixture(scope="module")
def reference():
    s = SHAPE
    om = orc.LanguageModel(s.layers, s.d_model, s.heads, s.ffn, s.vocabulary, s.seq_len, s.batch)
    params = om.init(SEED)
    ids, targets = orc.synthetic_batch(BATCH_SEED, s.batch, s.seq_len, s.vocabulary)
    loss, grads = om.forward_backward(params, ids, targets)
    return om, ids, targets, loss, grads


def _rows(t: np.ndarray, size: int, shapes: dict) -> np.ndarray:
    return t.reshape(shapes.get(size, (1, size)))


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3])
def test_medium_width_gradients_vs_oracle(lib, cuda, reference, precision):
    om, ids, targets, loss_ref, grads_ref = reference
    s = SHAPE
    model = etb.LanguageModel(s, precision=precision)
    model.init(SEED)
    loss = model.forward_backward(ids, targets)
    if precision == etb.PRECISION_F16X3:
        loss = model.forward_backward(ids, targets)  # the binary16-pair pass
    grads = model.read(1)
    model.close()
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (loss, loss_ref)
    d, F, V = s.d_model, s.ffn, s.vocabulary
    shapes = {V * d: (V, d), 3 * d * d: (3 * d, d), d * d: (d, d), F * d: (F, d)}
    report, failures = [], []
    for t, (g, r) in enumerate(zip(om.split(grads), om.split(grads_ref))):
        r64 = r.astype(np.float64)
        scale = max(np.abs(r64).max(), 1e-30)
        err = np.abs(g.astype(np.float64) - r64)
        ge, re = _rows(err, g.size, shapes), _rows(np.abs(r64), g.size, shapes)
        rowmax = re.max(axis=1)
        worst_row = float(np.max(ge.max(axis=1) / np.maximum(rowmax, 1e-30)))
        report.append((t, float(err.max() / scale), worst_row, float(rowmax.min() / scale)))
        if err.max() > GRAD_TOL * scale:
            failures.append((t, "normwise", float(err.max() / scale)))
        if not np.all(ge.max(axis=1) <= GRAD_TOL * rowmax + PER_ROW_FLOOR * scale):
            failures.append((t, "per-row", worst_row))
    for t, norm_err, row_err, spread in report:
        print(f"tensor {t}: normwise {norm_err:.2e}, worst row {row_err:.2e} "
              f"(smallest row max / tensor max {spread:.1e})")
    assert not failures, failures

"""Parity at the medium LM's widths (the throughput benchmark's shapes).

One layer of the medium decoder LM (d_model 1024, 16 heads, FFN 4096, vocab
32,768, seq 1024) on 4 sequences = 4,096 tokens, in both f32-grade contraction
modes: the weight-gradient GEMMs contract K = 4,096 tokens (split-K), the tied
head's dX contracts V = 32,768, attention runs 8 query tiles per (sequence,
head), and in split-f16 mode every operand is a binary16 pair with its
tensor's measured scale.

Three results are compared per tensor: ours, the oracle (serial f32 in the
reference's order) and a float64 evaluation of the same step (tests/lm_f64.py,
torch autograd), the ground truth for both.  The bars:

* ours vs the oracle: max |err| <= GRAD_TOL * max |oracle| (the LM gradient
  bar of the tiny model);
* ours vs float64: no more than F64_FACTOR times the oracle's own distance from
  float64, plus F64_FLOOR, tensor-wise (relative to the tensor's max) and for
  the worst row (each row relative to its own max), so small rows are held to
  the same standard as the reference's.

The oracle itself sits 2-5e-6 from float64 at these widths.  The tensor pipe's
f32 accumulation truncates, so a single accumulator over a long K drifts
(about 5e-4 relative at K = 65,536); the GEMM sums K in chunks of 1,024
(binary16 pairs) or 512 (TF32 pairs) and adds the chunks in f32, which keeps
each contraction within about 4e-6 -- without the chunks this test fails by an
order of magnitude.  Contractions of K <= 1,024 (the fused-epilogue GEMMs,
attention over 1,024 keys) keep one accumulator.
"""
import numpy as np
import pytest

import eshkol_transformer_b200 as etb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

SHAPE = etb.ModelShape(1, 1024, 16, 4096, 32768, 1024, 4)
SEED, BATCH_SEED = 2027, 314
GRAD_TOL = 5e-5
F64_FACTOR = 6.0
F64_FLOOR = 2e-6


@pytest.fixture(scope="module")
def reference(cuda):
    import lm_f64
    s = SHAPE
    om = orc.LanguageModel(s.layers, s.d_model, s.heads, s.ffn, s.vocabulary, s.seq_len, s.batch)
    params = om.init(SEED)
    ids, targets = orc.synthetic_batch(BATCH_SEED, s.batch, s.seq_len, s.vocabulary)
    loss, grads = om.forward_backward(params, ids, targets)
    loss64, grads64 = lm_f64.forward_backward(params, om.tensor_sizes, s, ids, targets)
    return om, ids, targets, loss, grads, loss64, grads64


def _rows(t: np.ndarray, size: int, shapes: dict) -> np.ndarray:
    return t.reshape(shapes.get(size, (1, size)))


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3])
def test_medium_width_gradients_vs_oracle(lib, cuda, reference, precision):
    om, ids, targets, loss_ref, grads_ref, loss64, grads64 = reference
    s = SHAPE
    model = etb.LanguageModel(s, precision=precision)
    model.init(SEED)
    loss = model.forward_backward(ids, targets)
    if precision == etb.PRECISION_F16X3:
        loss = model.forward_backward(ids, targets)  # the binary16-pair pass
    grads = model.read(1)
    model.close()
    print(f"loss ours {loss:.8f} oracle {loss_ref:.8f} f64 {loss64:.8f}")
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (loss, loss_ref)
    d, F, V = s.d_model, s.ffn, s.vocabulary
    shapes = {V * d: (V, d), 3 * d * d: (3 * d, d), d * d: (d, d), F * d: (F, d)}
    failures = []
    for t, (g, r, x) in enumerate(zip(om.split(grads), om.split(grads_ref), om.split(grads64))):
        scale = max(np.abs(x).max(), 1e-30)
        e_ours = np.abs(g.astype(np.float64) - x)
        e_orc = np.abs(r.astype(np.float64) - x)
        cross = np.abs(g.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30)
        rows_x = np.maximum(_rows(np.abs(x), g.size, shapes).max(axis=1), 1e-30)
        row_ours = _rows(e_ours, g.size, shapes).max(axis=1) / rows_x
        row_orc = _rows(e_orc, g.size, shapes).max(axis=1) / rows_x
        print(f"tensor {t}: vs f64 ours {e_ours.max() / scale:.2e} oracle {e_orc.max() / scale:.2e}"
              f" | ours vs oracle {cross:.2e} | worst row vs f64 ours {row_ours.max():.2e} "
              f"oracle {row_orc.max():.2e} (smallest row max / tensor max "
              f"{rows_x.min() / scale:.1e})")
        if cross > GRAD_TOL:
            failures.append((t, "vs oracle", float(cross)))
        if e_ours.max() / scale > F64_FACTOR * e_orc.max() / scale + F64_FLOOR:
            failures.append((t, "vs f64", float(e_ours.max() / scale), float(e_orc.max() / scale)))
        if row_ours.max() > F64_FACTOR * row_orc.max() + F64_FLOOR:
            failures.append((t, "per row vs f64", float(row_ours.max()), float(row_orc.max())))
    assert not failures, failures

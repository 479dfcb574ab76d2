"""The masked objective in the fused training step (L3S loss mask, D2
planes) against the oracle.

The tiny LM (2 layers, d 128, 4 heads, FFN 512, vocab 1024, seq 64, batch 8;
512 tokens, so the numerator seed carries 2^-9).  With a loss mask the
device gradients hold the mask-weighted numerators 2^-9 (the oracle's
forward_backward_masked with upstream scale 2^-9) and AdamW divides by the
weight sum(mask) 2^-9, the reference's O2 division (o2_optimizer.c:1738).
Bars as the unmasked step's: per-tensor gradients within GRAD_TOL normwise,
loss within 2e-5 relative (TR3), weights after several steps as in the
unmasked trajectory test."""
import numpy as np
import pytest
import torch

import eshkol_transformer_b200 as etb
from helpers import bits_equal
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TINY = etb.TINY
SEED_SCALE = 2.0 ** -9  # 2^-ceil(log2(512 tokens))
GRAD_TOL = 5e-5
MODES = [etb.PRECISION_TF32X3, etb.PRECISION_F16X3]


def _oracle_model():
    s = TINY
    return orc.LanguageModel(s.layers, s.d_model, s.heads, s.ffn, s.vocabulary, s.seq_len, s.batch)


def _mask(seed: int) -> np.ndarray:
    R = TINY.batch * TINY.seq_len
    m = (orc.fill_tokens(seed, 7, R, 10) < 7).astype(np.uint8)  # about 70 % kept
    m[TINY.seq_len:2 * TINY.seq_len] = 0                        # one sequence fully masked
    return m


@pytest.mark.parametrize("precision", MODES)
def test_masked_gradients_vs_oracle(lib, cuda, precision):
    s = TINY
    om = _oracle_model()
    params = om.init(4321)
    ids, targets = orc.synthetic_batch(78, s.batch, s.seq_len, s.vocabulary)
    mask = _mask(1)
    loss_ref, grads_ref = om.forward_backward_masked(params, ids, targets, mask, SEED_SCALE)
    model = etb.LanguageModel(s, precision=precision)
    model.init(4321)
    model.set_loss_mask(mask)
    loss = model.forward_backward(ids, targets)
    if precision == etb.PRECISION_F16X3:  # the second pass runs on binary16 pairs
        loss = model.forward_backward(ids, targets)
    grads = model.read(1)
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (loss, loss_ref)
    for t, (g, r) in enumerate(zip(om.split(grads), om.split(grads_ref))):
        err = np.abs(g.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30)
        assert err <= GRAD_TOL, (t, err)
    model.close()


@pytest.mark.parametrize("precision", MODES)
def test_masked_training_vs_oracle(lib, cuda, precision):
    """Four AdamW steps, a different mask each: the loss per step and the
    final weights (median distance 1e-3 lr, 99th percentile 1e-2 lr, every
    element within 1 lr of the oracle's)."""
    s = TINY
    om = _oracle_model()
    params = om.init(77)
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    opts = orc.adamw_options(1e-3, 0.9, 0.999, 1e-8, 0.01)
    model = etb.LanguageModel(s, precision=precision)
    model.init(77)
    for step in range(1, 5):
        ids, targets = orc.synthetic_batch(2000 + step, s.batch, s.seq_len, s.vocabulary)
        mask = _mask(10 + step)
        loss_ref, num = om.forward_backward_masked(params, ids, targets, mask, SEED_SCALE)
        weight = float(np.float32(mask.sum()) * np.float32(SEED_SCALE))
        assert orc.adamw_step(params, num, m, v, opts, step, weight=weight) == 0
        model.set_loss_mask(mask)
        loss = model.step(ids, targets)
        assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (step, loss, loss_ref)
    assert model.update_counts() == (4, 0)
    w = model.read(0)
    diff = np.abs(w.astype(np.float64) - params)
    lr = 1e-3  # bars in units of one update, as the tiny-LM trajectory test states them
    print(f"weights vs oracle: median {np.median(diff) / lr:.2e} lr, p99 "
          f"{np.percentile(diff, 99) / lr:.2e} lr, max {diff.max() / lr:.2e} lr")
    assert np.median(diff) <= 1e-3 * lr
    assert np.percentile(diff, 99) <= 1e-2 * lr
    assert diff.max() <= 1.0 * lr
    model.close()


def test_all_ones_mask_is_the_unmasked_step(lib, cuda):
    """All ones: the seed 2^-9 equals the unmasked 1/N and AdamW's weight is
    512 2^-9 = 1, so two steps give bit-identical losses, gradients and
    weights."""
    s = TINY
    R = s.batch * s.seq_len
    a = etb.LanguageModel(s, precision=etb.PRECISION_TF32X3)
    b = etb.LanguageModel(s, precision=etb.PRECISION_TF32X3)
    a.init(8)
    b.init(8)
    b.set_loss_mask(np.ones(R, np.uint8))
    for step in range(2):
        ids, targets = orc.synthetic_batch(300 + step, s.batch, s.seq_len, s.vocabulary)
        assert a.step(ids, targets) == b.step(ids, targets)
        assert bits_equal(a.read(1), b.read(1))
    assert bits_equal(a.read(0), b.read(0))
    a.close()
    b.close()


def test_invalid_and_empty_masks_update_nothing(lib, cuda):
    s = TINY
    R = s.batch * s.seq_len
    model = etb.LanguageModel(s, precision=etb.PRECISION_TF32X3)
    model.init(12)
    ids, targets = orc.synthetic_batch(400, s.batch, s.seq_len, s.vocabulary)
    model.set_loss_mask(_mask(3))
    model.step(ids, targets)
    before = [model.read(i) for i in (0, 2, 3)]
    # a host byte other than 0 / 1 is rejected by the setter
    bad = _mask(4)
    bad[5] = 2
    with pytest.raises(etb.B200Error):
        model.set_loss_mask(bad)
    # the same byte in device memory voids the step
    dev = torch.from_numpy(bad).cuda()
    model.set_loss_mask(device_ptr=dev.data_ptr())
    with pytest.raises(etb.B200Error, match="loss mask byte"):
        model.step(ids, targets)
    # a mask that selects no token
    model.set_loss_mask(np.zeros(R, np.uint8))
    with pytest.raises(etb.B200Error, match="selects no token"):
        model.step(ids, targets)
    for i, b in zip((0, 2, 3), before):
        assert bits_equal(model.read(i), b)
    assert model.update_counts() == (1, 0)
    # a valid mask trains again
    model.set_loss_mask(_mask(5))
    model.step(ids, targets)
    assert model.update_counts() == (2, 0)
    model.close()


def test_d2_planes_feed_the_step(lib, cuda):
    """Batch planes cut from a token stream by the D2 row rule (the last row
    of the batch partly filled, so its tail is masked) train like the
    oracle's masked step on the same planes."""
    s = TINY
    length = (s.batch - 1) * s.seq_len + s.seq_len // 2
    stream = orc.fill_tokens(31, 1, length, s.vocabulary)
    ids, targets, mask = etb.d2_rows(stream, s.seq_len, 0, s.batch)
    assert mask.sum() == length - 1 and not mask[-1, -1]
    om = _oracle_model()
    params = om.init(55)
    loss_ref, grads_ref = om.forward_backward_masked(params, ids, targets, mask.ravel(),
                                                     SEED_SCALE)
    model = etb.LanguageModel(s, precision=etb.PRECISION_TF32X3)
    model.init(55)
    model.set_loss_mask(mask)
    loss = model.forward_backward(ids, targets)
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref)
    for t, (g, r) in enumerate(zip(om.split(model.read(1)), om.split(grads_ref))):
        err = np.abs(g.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30)
        assert err <= GRAD_TOL, (t, err)
    model.close()

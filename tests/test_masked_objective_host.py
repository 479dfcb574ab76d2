"""The masked objective's host side (no GPU): the oracle's masked mean loss
pinned to the reference's own L3S provider, the oracle's masked LM step
against its unmasked one, and the D2 batch planes against a plain-Python
restatement of the reference's row rule."""
import numpy as np
import pytest

import eshkol_transformer_b200 as etb
from eshkol_transformer_b200 import k1
from helpers import bits_equal
from oracle import oracle as orc


@pytest.mark.skipif(orc.ref() is None, reason="oracle/_ref/libref.so is not built")
@pytest.mark.parametrize("ce,mask", [((0.7, 2.5), (1, 1)), ((0.7, 2.5), (0, 1)),
                                     ((3.25, 1e-3), (1, 0)), ((0.1, 0.2), (1, 1))])
def test_masked_mean_matches_reference_l3s_reduce(ce, mask):
    """l3s.masked-objective.reduce.bool at its exact [1, 2] profile
    (native/l3s_masked_objective_provider.c:125-175): numerator, weight and
    mean against the oracle's masked mean, bit for bit."""
    l3s = k1.provider(orc.ref(), "et_l3s_kernel_provider_v1")
    c = np.array([ce], np.float32)
    m = np.array([mask], np.uint8)
    n, w, mean = (np.zeros((), np.float32) for _ in range(3))
    rc, err = k1.dispatch(l3s, k1.KernelCall("l3s.masked-objective",
                                             "l3s.masked-objective.reduce.bool", (1, 2),
                                             [c, m], [n, w, mean]))
    assert rc == 0, str(err)
    assert float(w) == float(sum(mask))
    got = orc.masked_mean_loss(c.ravel(), m.ravel())
    assert bits_equal(np.float32(got), mean), (got, float(mean))


@pytest.mark.skipif(orc.ref() is None, reason="oracle/_ref/libref.so is not built")
def test_numerator_seed_is_the_mask():
    """l3s.masked-objective.numerator-seed.bool: the CE upstream of each token
    is its mask value (the seed the fused step scales by 2^-k)."""
    l3s = k1.provider(orc.ref(), "et_l3s_kernel_provider_v1")
    m = np.array([[1, 0]], np.uint8)
    seed = np.zeros((1, 2), np.float32)
    rc, err = k1.dispatch(l3s, k1.KernelCall("l3s.masked-objective",
                                             "l3s.masked-objective.numerator-seed.bool", (1, 2),
                                             [m], [seed]))
    assert rc == 0, str(err)
    assert seed.tolist() == [[1.0, 0.0]]


MICRO = dict(layers=1, d_model=32, heads=2, ffn=64, vocabulary=64, seq_len=16, batch=2)


def test_oracle_all_ones_mask_is_the_unmasked_objective():
    om = orc.LanguageModel(**MICRO)
    params = om.init(5)
    ids, targets = orc.synthetic_batch(9, MICRO["batch"], MICRO["seq_len"], MICRO["vocabulary"])
    R = MICRO["batch"] * MICRO["seq_len"]
    loss_a, ga = om.forward_backward(params, ids, targets)
    loss_b, gb = om.forward_backward_masked(params, ids, targets, np.ones(R, np.uint8), 1.0 / R)
    assert loss_a == loss_b and bits_equal(ga, gb)


def test_oracle_masked_gradient_is_the_kept_tokens_numerator():
    """Masking tokens out equals training on the kept tokens alone: the
    gradient numerator of a mask is the sum of the per-token gradients of the
    kept tokens (checked with one kept token at a time against the full
    mask, the numerators summed in f64)."""
    om = orc.LanguageModel(**MICRO)
    params = om.init(6)
    ids, targets = orc.synthetic_batch(10, MICRO["batch"], MICRO["seq_len"], MICRO["vocabulary"])
    R = MICRO["batch"] * MICRO["seq_len"]
    mask = np.zeros(R, np.uint8)
    kept = [0, 5, 17, 30]
    mask[kept] = 1
    loss, g = om.forward_backward_masked(params, ids, targets, mask, 1.0)
    total = np.zeros_like(g, np.float64)
    per = []
    for r in kept:
        one = np.zeros(R, np.uint8)
        one[r] = 1
        l1, g1 = om.forward_backward_masked(params, ids, targets, one, 1.0)
        total += g1
        per.append(l1)
    assert abs(loss - np.mean(per)) <= 1e-6 * abs(loss)
    assert np.abs(g - total).max() <= 1e-5 * np.abs(total).max()


@pytest.mark.parametrize("length,seq_len,first_row,rows", [
    (1, 4, 0, 2), (5, 4, 0, 1), (6, 4, 0, 3), (17, 4, 1, 3), (100, 7, 3, 5), (9, 8, 0, 1),
    (10, 8, 0, 2)])
def test_d2_planes_match_the_row_rule(length, seq_len, first_row, rows):
    toks = orc.fill_tokens(3, length, length, 50) + 1  # nonzero, so padding is visible
    count = 0 if length < 2 else 1 + (length - 2) // seq_len
    assert etb.d2_row_count(length, seq_len) == count
    if first_row >= count:
        with pytest.raises(etb.B200Error):
            etb.d2_rows(toks, seq_len, first_row, rows)
        return
    got = etb.d2_rows(toks, seq_len, first_row, rows)
    want = orc.d2_rows(toks, seq_len, first_row, rows)
    for a, b in zip(got, want):
        assert np.array_equal(a, b)
    ids, targets, mask = got
    assert mask.any()
    # shifted pairs: every kept target is the next input of the stream
    flat = np.asarray(toks)
    for r in range(rows):
        for t in range(seq_len):
            if mask[r, t]:
                s = (first_row + r) * seq_len + t
                assert ids[r, t] == flat[s] and targets[r, t] == flat[s + 1]
            else:
                assert ids[r, t] == 0 and targets[r, t] == 0

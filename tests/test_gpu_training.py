"""The fused training step and the device AdamW against the oracle.

* O2 AdamW on device: parameters and moments bit-identical to the
  reference's per-element arithmetic when clipping is inactive (oracle pinned
  by the adamw fixtures), within stated bounds when it is active; updates are
  all or nothing.
* The tiny decoder LM (2 layers, d 128, 4 heads, FFN 512, vocab 1024, seq 64,
  batch 8): seeded initial weights bit-identical; per-tensor gradients within
  a stated normwise tolerance; updated weights; the loss over several steps.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import eshkol_transformer_b200 as etb
from helpers import assert_close, assert_close_norm, bits_equal
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


# Clipped updates: the device norm is an f64 sum of squares rounded once; the
# reference's is a scaled f32 recurrence in parameter order
# (o2_optimizer.c:1548-1618).  The two norms differ by delta (relative, below
# NORM_RTOL here), which scales every clipped gradient by the same (1 + delta):
# the moments move by at most that relative amount and the parameter update
# m_hat / (sqrt(v_hat) + eps), nearly invariant to a common gradient scale,
# by a small multiple of delta * lr.  Unclipped updates stay bit-identical.
NORM_RTOL = 1e-5
CLIP_MOMENT_RTOL = 4 * NORM_RTOL
CLIP_PARAM_ATOL_PER_LR = 1e-3


@pytest.mark.parametrize("clip,schedule", [(0.0, 0), (0.5, 0), (0.0, 1), (1e9, 1)])
def test_o2_device_adamw_vs_reference_order(lib, cuda, clip, schedule):
    """Four updates of four tensors against the oracle run with the
    reference's own norm (its scaled f32 recurrence), not the device's:
    bit-identical parameters and moments whenever clipping is inactive, and
    within the stated bounds when it is active."""
    sizes = [1000, 37, 4096, 1]
    opts = [(1e-3, 0.9, 0.999, 1e-8, 0.01), (5e-3, 0.8, 0.95, 1e-6, 0.0),
            (2e-2, 0.9, 0.999, 1e-8, 0.1), (1e-3, 0.5, 0.9, 1e-5, 0.2)]
    params = [orc.fill_normal(3, i, n) for i, n in enumerate(sizes)]
    p_dev = [torch.from_numpy(p.copy()).cuda() for p in params]
    g_dev = [torch.zeros(n, device="cuda") for n in sizes]
    entries = [(p_dev[i].data_ptr(), g_dev[i].data_ptr(), n, *opts[i]) for i, n in enumerate(sizes)]
    warm, total, minimum = (2, 6, 0.1) if schedule else (0, 0, 0.0)
    opt = etb.Optimizer(entries, clip_kind=1 if clip else 0, clip_max=clip,
                        schedule_kind=schedule, warmup=warm, total=total, minimum_ratio=minimum)
    ref_p = [p.copy() for p in params]
    ref_m = [np.zeros(n, np.float32) for n in sizes]
    ref_v = [np.zeros(n, np.float32) for n in sizes]
    weight = 3.0
    clipped = False
    for step in range(1, 5):
        grads = [orc.fill_normal(100 + step, i, n, 0.0, 2.0) for i, n in enumerate(sizes)]
        for gd, g in zip(g_dev, grads):
            gd.copy_(torch.from_numpy(g))
        norm = opt.step(weight)
        ref_norm = orc.global_norm(grads, weight)
        assert abs(norm - ref_norm) <= NORM_RTOL * ref_norm, (norm, ref_norm)
        clip_f = np.float32(1.0)
        if clip and ref_norm > clip:
            clip_f = np.float32(np.float32(clip) / np.float32(ref_norm))
            clipped = True
        sched = orc.schedule_factor(schedule, warm, total, orc.bits(minimum) if schedule else 0,
                                    step)
        for i in range(len(sizes)):
            assert orc.adamw_step(ref_p[i], grads[i], ref_m[i], ref_v[i],
                                  orc.adamw_options(*opts[i]), step, weight, sched,
                                  float(clip_f)) == 0
        torch.cuda.synchronize()
        for i in range(len(sizes)):
            m_ptr, v_ptr = opt.moments(i)
            m = device_view(m_ptr, sizes[i]).cpu().numpy()
            v = device_view(v_ptr, sizes[i]).cpu().numpy()
            p = p_dev[i].cpu().numpy()
            if not clipped:
                assert bits_equal(p, ref_p[i]), (step, i, "parameter")
                assert bits_equal(m, ref_m[i]), (step, i, "exp_avg")
                assert bits_equal(v, ref_v[i]), (step, i, "exp_avg_sq")
                continue
            lr = opts[i][0]
            ulp = np.spacing(np.abs(ref_p[i]).astype(np.float32))
            assert np.all(np.abs(p.astype(np.float64) - ref_p[i]) <=
                          CLIP_PARAM_ATOL_PER_LR * lr + ulp), (step, i, "parameter")
            assert_close(m, ref_m[i], CLIP_MOMENT_RTOL * np.abs(ref_m[i]).max(),
                         CLIP_MOMENT_RTOL, f"exp_avg {step} {i}")
            assert_close(v, ref_v[i], CLIP_MOMENT_RTOL * np.abs(ref_v[i]).max(),
                         CLIP_MOMENT_RTOL, f"exp_avg_sq {step} {i}")
    assert clipped == (clip == 0.5)
    opt.close()


def test_o2_device_adamw_all_or_nothing(lib, cuda):
    """The reference validates every tensor before it commits any
    (o2_optimizer.c:1813-1926).  A nonfinite parameter in one tensor, or a
    finite gradient whose square overflows in another, must leave every
    parameter, moment and the update counter unchanged and return the
    reference's message; the next finite step applies normally."""
    sizes = [4096, 1000]
    params = [orc.fill_normal(5, i, n) for i, n in enumerate(sizes)]
    p_dev = [torch.from_numpy(p.copy()).cuda() for p in params]
    g_dev = [torch.from_numpy(orc.fill_normal(6, i, n)).cuda() for i, n in enumerate(sizes)]
    opt = etb.Optimizer([(p_dev[i].data_ptr(), g_dev[i].data_ptr(), n, 1e-3, 0.9, 0.999, 1e-8,
                          0.01) for i, n in enumerate(sizes)])
    opt.step(1.0)  # one good update so the moments are nonzero

    def snapshot():
        out = [p.clone() for p in p_dev]
        for i, n in enumerate(sizes):
            m_ptr, v_ptr = opt.moments(i)
            out += [device_view(m_ptr, n).clone(), device_view(v_ptr, n).clone()]
        return out

    def updates():
        c = C.c_uint64()
        lib.et_b200_o2_optimizer_completed_updates_v1(opt.handle, C.byref(c))
        return c.value

    for inject, message in ((lambda: p_dev[1].__setitem__(7, float("inf")),
                             "parameter, gradient, or moment is nonfinite"),
                            (lambda: g_dev[0].__setitem__(4000, 1e20),
                             "AdamW produced a nonfinite value")):
        before_p = [p.clone() for p in p_dev]
        inject()
        before = snapshot()
        with pytest.raises(etb.B200Error) as info:
            opt.step(1.0)
        assert message in str(info.value)
        after = snapshot()
        assert all(torch.equal(a.view(torch.int32), b.view(torch.int32))
                   for a, b in zip(before, after)), message
        assert updates() == 1
        for p, b in zip(p_dev, before_p):
            p.copy_(b)
        g_dev[0][4000] = 0.25
    opt.step(1.0)
    assert updates() == 2
    opt.close()


class _DeviceArray:
    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3}


def device_view(ptr: int, n: int) -> torch.Tensor:
    """Zero-copy torch view of an f32 device buffer the library owns."""
    return torch.as_tensor(_DeviceArray(ptr, n), device="cuda")


TINY = etb.TINY


def _oracle_model():
    s = TINY
    return orc.LanguageModel(s.layers, s.d_model, s.heads, s.ffn, s.vocabulary, s.seq_len, s.batch)


# Per-tensor gradient tolerance (max |err| <= tol * max |ref|) of one step of
# the tiny LM against the serial-f32 oracle: the GEMMs, attention, LN and CE
# reductions all sum in a different order from the reference.
GRAD_TOL = {etb.PRECISION_TF32X3: 5e-5, etb.PRECISION_F16X3: 5e-5, etb.PRECISION_F32: 5e-5,
            etb.PRECISION_TF32: 5e-3}


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3,
                                       etb.PRECISION_F32, etb.PRECISION_TF32])
def test_tiny_lm_gradients_vs_oracle(lib, cuda, precision):
    """One forward/backward against the oracle.  Split-f16 measures its
    operand scales in a first (3xTF32) pass; the second pass, on the same
    weights, is the split-f16 one compared here."""
    s = TINY
    om = _oracle_model()
    params = om.init(1234)
    ids, targets = orc.synthetic_batch(77, s.batch, s.seq_len, s.vocabulary)
    loss_ref, grads_ref = om.forward_backward(params, ids, targets)
    model = etb.LanguageModel(s, precision=precision)
    model.init(1234)
    assert bits_equal(model.read(0), params)  # seeded init is bit-identical
    loss = model.forward_backward(ids, targets)
    if precision == etb.PRECISION_F16X3:
        first = model.read(1)
        loss = model.forward_backward(ids, targets)
        assert not bits_equal(model.read(1), first)  # the binary16 path did run
    grads = model.read(1)
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (loss, loss_ref)
    worst = []
    for t, (g, r) in enumerate(zip(om.split(grads), om.split(grads_ref))):
        err = np.abs(g.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30)
        worst.append(err)
        assert err <= GRAD_TOL[precision], (t, err)
    print("worst per-tensor normwise gradient error", max(worst))
    model.close()


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3])
def test_tiny_lm_training_trajectory_vs_oracle(lib, cuda, precision):
    """Five AdamW steps: the loss trajectory within 2e-5 relative (the
    reference's TR3 loss tolerance) and the final weights against the
    oracle's after the same updates, in units of the learning rate (one update
    moves a weight by up to about lr): median distance at most 1e-3 lr, 99th
    percentile at most 1e-2 lr (the bulk follows the oracle to a small part
    of one update), every element within 1 lr.  AdamW's lr m / (sqrt(v) +
    eps) is close to lr sign(g), so an element whose gradient lies within the
    gradient error of zero (a few per million here) can take a step of either
    sign; the maximum is bounded by the update size, not by the gradient
    error."""
    s = TINY
    om = _oracle_model()
    params = om.init(99)
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    opts = orc.adamw_options(1e-3, 0.9, 0.999, 1e-8, 0.01)
    model = etb.LanguageModel(s, precision=precision)
    model.init(99)
    for step in range(1, 6):
        ids, targets = orc.synthetic_batch(1000 + step, s.batch, s.seq_len, s.vocabulary)
        loss_ref, grads_ref = om.forward_backward(params, ids, targets)
        assert om.adamw(params, grads_ref, m, v, opts, step) == 0
        loss = model.step(ids, targets)
        assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (step, loss, loss_ref)
    w = model.read(0)
    diff = np.abs(w.astype(np.float64) - params)
    lr = 1e-3
    print(f"weights vs oracle: median {np.median(diff) / lr:.2e} lr, p99 "
          f"{np.percentile(diff, 99) / lr:.2e} lr, max {diff.max() / lr:.2e} lr")
    assert np.median(diff) <= 1e-3 * lr
    assert np.percentile(diff, 99) <= 1e-2 * lr
    assert diff.max() <= 1.0 * lr
    model.close()


def test_split_f16_overflow_is_redone_in_3xtf32(lib, cuda, monkeypatch):
    """The operand-overflow path of split-f16, without any GPU fault: with
    the scale target at 17 every operand's max lands above binary16's largest
    finite value, so each split-f16 step overflows.  The check after the
    backward must catch it, AdamW must skip the update, and the host call must
    redo the step in 3xTF32: the loss trajectory then still follows the
    oracle (2e-5 relative) and every step after the first is counted."""
    monkeypatch.setenv("ET_B200_F16_SCALE_TARGET", "17")
    s = TINY
    om = _oracle_model()
    params = om.init(99)
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    opts = orc.adamw_options(1e-3, 0.9, 0.999, 1e-8, 0.01)
    model = etb.LanguageModel(s, precision=etb.PRECISION_F16X3)
    model.init(99)
    for step in range(1, 4):
        ids, targets = orc.synthetic_batch(1000 + step, s.batch, s.seq_len, s.vocabulary)
        loss_ref, grads_ref = om.forward_backward(params, ids, targets)
        assert om.adamw(params, grads_ref, m, v, opts, step) == 0
        loss = model.step(ids, targets)
        assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (step, loss, loss_ref)
    assert model.f16_redone_steps() == 2  # step 1 measures the scales in 3xTF32
    model.close()


def _state(model):
    return [model.read(k).copy() for k in (0, 2, 3)]


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3])
def test_step_is_all_or_nothing(lib, cuda, precision):
    """et_b200_lm_step_v1 with a target outside the vocabulary, then with a
    host-written inf weight: each call fails with INVALID_ARGUMENT and leaves
    the weights, both moments and the update counter bit-unchanged (the
    reference validates before it commits, o2_optimizer.c:1813-1926); a good
    step afterwards applies as update 2 and matches the oracle's second
    update."""
    s = TINY
    om = _oracle_model()
    params = om.init(41)
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    opts = orc.adamw_options(1e-3, 0.9, 0.999, 1e-8, 0.01)
    model = etb.LanguageModel(s, precision=precision)
    model.init(41)
    ids, targets = orc.synthetic_batch(41, s.batch, s.seq_len, s.vocabulary)
    model.step(ids, targets)
    _, grads = om.forward_backward(params, ids, targets)
    assert om.adamw(params, grads, m, v, opts, 1) == 0
    before = _state(model)
    bad = targets.copy()
    bad[1, 7] = s.vocabulary
    with pytest.raises(etb.B200Error) as info:
        model.step(ids, bad)
    assert "outside the vocabulary" in str(info.value)
    assert all(bits_equal(a, b) for a, b in zip(before, _state(model)))
    assert model.update_counts() == (1, 0)
    w = before[0].copy()
    w[123] = np.inf
    model.write(w)
    with pytest.raises(etb.B200Error) as info:
        model.step(ids, targets)
    assert "nonfinite" in str(info.value)
    after = _state(model)
    assert bits_equal(after[0], w) and bits_equal(after[1], before[1])
    assert bits_equal(after[2], before[2])
    assert model.update_counts() == (1, 0)
    model.write(before[0])
    ids2, targets2 = orc.synthetic_batch(42, s.batch, s.seq_len, s.vocabulary)
    loss = model.step(ids2, targets2)
    loss_ref, grads = om.forward_backward(params, ids2, targets2)
    assert om.adamw(params, grads, m, v, opts, 2) == 0
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref)
    assert model.update_counts() == (2, 0)
    diff = np.abs(model.read(0).astype(np.float64) - params)
    assert diff.max() <= 2 * 2 * 1e-3, diff.max()
    assert np.mean(diff <= 2e-6) >= 0.99
    model.close()


def test_device_step_skips_count_and_keep_update_numbers(lib, cuda, monkeypatch):
    """Steps enqueued with et_b200_lm_step_device_v1 that must not apply --
    here split-f16 steps whose operands all overflow (scale target 17) and one
    with an out-of-range target -- are skipped on the device and counted; the
    applied-update counter, and with it the bias corrections of later steps,
    advance only for applied steps.  After the skips a host step applies
    update 2 and the weights match the oracle's two updates."""
    monkeypatch.setenv("ET_B200_F16_SCALE_TARGET", "17")
    s = TINY
    om = _oracle_model()
    params = om.init(43)
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    opts = orc.adamw_options(1e-3, 0.9, 0.999, 1e-8, 0.01)
    model = etb.LanguageModel(s, precision=etb.PRECISION_F16X3)
    model.init(43)
    batches = [orc.synthetic_batch(500 + i, s.batch, s.seq_len, s.vocabulary) for i in range(4)]
    dev = [(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()) for a, b in batches]
    bad = dev[3][1].clone()
    bad[0, 0] = -1
    for ids, tg in (dev[0], dev[1], dev[2], (dev[3][0], bad)):
        model.step_device(ids.data_ptr(), tg.data_ptr())
    # step 1 measured the scales in 3xTF32 and applied; steps 2-3 overflowed;
    # step 4 had a bad target
    assert model.update_counts() == (1, 3)
    _, grads = om.forward_backward(params, *batches[0])
    assert om.adamw(params, grads, m, v, opts, 1) == 0
    ids, targets = orc.synthetic_batch(600, s.batch, s.seq_len, s.vocabulary)
    loss = model.step(ids, targets)  # re-measures in 3xTF32: applies
    loss_ref, grads = om.forward_backward(params, ids, targets)
    assert om.adamw(params, grads, m, v, opts, 2) == 0
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref)
    assert model.update_counts() == (2, 3)
    diff = np.abs(model.read(0).astype(np.float64) - params)
    assert diff.max() <= 2 * 2 * 1e-3, diff.max()
    assert np.mean(diff <= 2e-6) >= 0.99
    model.close()


def test_forward_backward_rejects_out_of_range_ids(lib, cuda):
    s = TINY
    model = etb.LanguageModel(s)
    model.init(5)
    ids, targets = orc.synthetic_batch(5, s.batch, s.seq_len, s.vocabulary)
    targets[0, 3] = s.vocabulary
    with pytest.raises(etb.B200Error):
        model.forward_backward(ids, targets)
    ids2, targets2 = orc.synthetic_batch(6, s.batch, s.seq_len, s.vocabulary)
    assert np.isfinite(model.forward_backward(ids2, targets2))  # recovers
    model.close()


def test_launch_counter_and_device_step(lib, cuda):
    s = TINY
    model = etb.LanguageModel(s)
    model.init(3)
    ids, targets = orc.synthetic_batch(3, s.batch, s.seq_len, s.vocabulary)
    d_ids = torch.from_numpy(ids).cuda()
    d_tg = torch.from_numpy(targets).cuda()
    loss = torch.zeros(1, device="cuda")
    before = etb.launch_count()
    model.step_device(d_ids.data_ptr(), d_tg.data_ptr(), loss.data_ptr())
    torch.cuda.synchronize()
    assert etb.launch_count() - before > 20
    assert np.isfinite(loss.item())
    model.close()


def test_long_sequence_lm_gradients_vs_oracle(lib, cuda):
    """One layer at T = 1024 and 4 sequences (4,096 rows): the weight-gradient
    GEMMs then have K = 4,096 over one or two output tiles, which takes the
    split-K path (partial sums reduced in a fixed order), and attention runs
    several query tiles per head with RoPE.  Same per-tensor normwise bound as
    the tiny model."""
    s = etb.ModelShape(1, 64, 2, 256, 512, 1024, 4)
    om = orc.LanguageModel(s.layers, s.d_model, s.heads, s.ffn, s.vocabulary, s.seq_len, s.batch)
    params = om.init(2024)
    ids, targets = orc.synthetic_batch(88, s.batch, s.seq_len, s.vocabulary)
    loss_ref, grads_ref = om.forward_backward(params, ids, targets)
    model = etb.LanguageModel(s, precision=etb.PRECISION_TF32X3)
    model.init(2024)
    loss = model.forward_backward(ids, targets)
    grads = model.read(1)
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (loss, loss_ref)
    for t, (g, r) in enumerate(zip(om.split(grads), om.split(grads_ref))):
        err = np.abs(g.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30)
        assert err <= GRAD_TOL[etb.PRECISION_TF32X3], (t, err)
    model.close()


@pytest.mark.parametrize("heads, d_model, seq_len", [(4, 256, 384), (2, 256, 256)])
def test_split_f16_lm_binary16_attention_vs_oracle(lib, cuda, heads, d_model, seq_len):
    """Split-f16 steps at head_dim 64 and 128 run the binary16 attention with
    its operand pairs written by the GEMM epilogues: the QKV projection's
    (RoPE'd Q, K and V) and dO's (with delta and the log-sum-exp), each pair
    scaled by the exponent its slot took from the previous step's maximum,
    dS's exponent from this step's maxima of V and dO.  The second pass (the
    first one measures the maxima in 3xTF32) against the oracle, with the LM
    gradient bar."""
    s = etb.ModelShape(1, d_model, heads, 4 * d_model, 1024, seq_len, 3)
    om = orc.LanguageModel(s.layers, s.d_model, s.heads, s.ffn, s.vocabulary, s.seq_len, s.batch)
    params = om.init(4321)
    ids, targets = orc.synthetic_batch(55, s.batch, s.seq_len, s.vocabulary)
    loss_ref, grads_ref = om.forward_backward(params, ids, targets)
    model = etb.LanguageModel(s, precision=etb.PRECISION_F16X3)
    model.init(4321)
    model.forward_backward(ids, targets)
    first = model.read(1)
    loss = model.forward_backward(ids, targets)
    grads = model.read(1)
    model.close()
    assert not bits_equal(grads, first)  # the binary16 pass did run
    assert abs(loss - loss_ref) <= 2e-5 * abs(loss_ref), (loss, loss_ref)
    worst = 0.0
    for t, (g, r) in enumerate(zip(om.split(grads), om.split(grads_ref))):
        err = np.abs(g.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30)
        worst = max(worst, err)
        assert err <= GRAD_TOL[etb.PRECISION_F16X3], (t, err)
    print(f"head_dim {d_model // heads}: worst per-tensor normwise gradient error {worst:.2e}")


def test_o2_device_adamw_outside_check_envelope(lib, cuda):
    """Finite values outside the check pass's envelope (a gradient of 2^40, a
    moment of 2^35, a parameter of 2^110) take its exact computation; the
    update is finite, so it applies, bit-identical to the reference's
    arithmetic."""
    n = 4096
    p = orc.fill_normal(8, 1, n)
    g = orc.fill_normal(8, 2, n)
    g[5] = np.float32(2.0 ** 40)
    p[9] = np.float32(2.0 ** 110)
    p_dev, g_dev = torch.from_numpy(p.copy()).cuda(), torch.from_numpy(g).cuda()
    opt = etb.Optimizer([(p_dev.data_ptr(), g_dev.data_ptr(), n, 1e-3, 0.9, 0.999, 1e-8, 0.01)])
    m_ptr, v_ptr = opt.moments(0)
    m0 = np.zeros(n, np.float32)
    m0[17] = np.float32(2.0 ** 35)
    device_view(m_ptr, n).copy_(torch.from_numpy(m0))
    ref_p, ref_m, ref_v = p.copy(), m0.copy(), np.zeros(n, np.float32)
    opt.step(1.0)
    assert orc.adamw_step(ref_p, g, ref_m, ref_v, orc.adamw_options(1e-3, 0.9, 0.999, 1e-8, 0.01),
                          1) == 0
    torch.cuda.synchronize()
    assert bits_equal(p_dev.cpu().numpy(), ref_p)
    assert bits_equal(device_view(m_ptr, n).cpu().numpy(), ref_m)
    assert bits_equal(device_view(v_ptr, n).cpu().numpy(), ref_v)
    opt.close()

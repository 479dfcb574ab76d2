"""Causal attention with RoPE on device tensors (et_b200_attention_*_v1)
against the oracle.

The oracle composes the reference's own order: rope.forward on Q and K,
causal-attention forward and backward (native/a2_attention_provider.c:669-790),
rope.backward on dQ and dK (:792-935).  Bars: the A2 fixture tolerances,
2e-5 (output) and 5e-5 (gradients) absolute plus relative.  Shapes cover the
tensor-core forward and backward (head_dim 32 / 64), head_dim 128 (tensor-core
forward), grouped query heads, and -- for the attention sweep's shape, batch 4,
16 heads, T = 2,048, head_dim 64 and 128 -- sampled (sequence, head) slices
checked against the oracle run on that slice alone.
"""
import numpy as np
import pytest
import torch

import eshkol_transformer_b200 as etb
from attention_f64 import attention_f64
from helpers import assert_close
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _inv_freq(dh: int) -> np.ndarray:
    return np.array([np.float32(1.0 / 10000.0 ** (2 * i / dh)) for i in range(dh // 2)],
                    np.float32)


def _run(B, Hq, Hkv, T, Dh, seed, rope=True, contraction=etb.ATTENTION_DEFAULT,
         mags=(1.0, 1.0, 1.0, 1.0)):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, Hq, T, Dh, device="cuda", generator=g) * mags[0]
    k = torch.randn(B, Hkv, T, Dh, device="cuda", generator=g) * mags[1]
    v = torch.randn(B, Hkv, T, Dh, device="cuda", generator=g) * mags[2]
    do = torch.randn(B, Hq, T, Dh, device="cuda", generator=g) * mags[3]
    pos = torch.arange(T, dtype=torch.int64, device="cuda").repeat(B, 1).contiguous()
    cos = sin = None
    if rope:
        c, s = etb.rope_tables(T, Dh)
        cos, sin = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    att = etb.Attention(B, Hq, Hkv, T, T, Dh, pos, pos, None, cos, sin, contraction=contraction)
    o = torch.empty_like(q)
    m = torch.empty(B, Hq, T, device="cuda")
    l = torch.empty(B, Hq, T, device="cuda")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    att.forward(q, k, v, o, m, l)
    att.backward(q, k, v, o, do, m, l, dq, dk, dv)
    torch.cuda.synchronize()
    host = lambda t: t.cpu().numpy()
    return [host(t) for t in (q, k, v, do, o, dq, dk, dv)]


def _oracle(q, k, v, do, rope=True):
    B, Hq, T, Dh = q.shape
    Hkv = k.shape[1]
    pos = np.tile(np.arange(T, dtype=np.int64), (B, 1))
    mask = np.ones((B, T, T), np.uint8)
    inv = _inv_freq(Dh)
    qr = orc.rope((B, Hq, T, Dh), q, pos, inv) if rope else q
    kr = orc.rope((B, Hkv, T, Dh), k, pos, inv) if rope else k
    shape = (B, Hq, Hkv, T, T, Dh)
    o = orc.attention_forward(shape, qr, kr, v, pos, pos, mask)
    dqr, dkr, dv = orc.attention_backward(shape, qr, kr, v, pos, pos, mask, do)
    dq = orc.rope((B, Hq, T, Dh), dqr, pos, inv, backward=True) if rope else dqr
    dk = orc.rope((B, Hkv, T, Dh), dkr, pos, inv, backward=True) if rope else dkr
    return o, dq, dk, dv


MODES = [etb.ATTENTION_DEFAULT, etb.ATTENTION_BWD_PAIRS16]


@pytest.mark.parametrize("contraction", MODES)
@pytest.mark.parametrize("B,Hq,Hkv,T,Dh,rope", [(2, 4, 4, 256, 64, True),
                                                (2, 4, 2, 200, 32, True),
                                                (1, 2, 2, 384, 128, True),
                                                (2, 4, 2, 330, 128, True),
                                                (2, 2, 2, 96, 64, False),
                                                # head_dim 64 just above the default's
                                                # binary16 threshold (768^2), ragged tiles
                                                (1, 2, 2, 800, 64, True)])
def test_device_attention_vs_oracle(lib, cuda, B, Hq, Hkv, T, Dh, rope, contraction):
    q, k, v, do, o, dq, dk, dv = _run(B, Hq, Hkv, T, Dh, 7 + T, rope, contraction)
    ro, rdq, rdk, rdv = _oracle(q, k, v, do, rope)
    assert_close(o, ro, 2e-5, 2e-5, "o")
    for name, got, want in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        assert_close(got, want, 5e-5, 5e-5, name)


@pytest.mark.parametrize("Dh,contraction", [(64, etb.ATTENTION_DEFAULT),
                                            (64, etb.ATTENTION_BWD_PAIRS16),
                                            (128, etb.ATTENTION_DEFAULT)])
def test_sweep_shape_sampled_heads_vs_oracle(lib, cuda, Dh, contraction):
    """B4 H16 T2048: two sampled (sequence, head) slices of the full device
    computation against the oracle on the slice alone."""
    B, H, T = 4, 16, 2048
    q, k, v, do, o, dq, dk, dv = _run(B, H, H, T, Dh, 2048 + Dh, contraction=contraction)
    for b, h in ((0, 3), (3, 14)):
        sl = lambda a: np.ascontiguousarray(a[b:b + 1, h:h + 1])
        ro, rdq, rdk, rdv = _oracle(sl(q), sl(k), sl(v), sl(do))
        assert_close(sl(o), ro, 2e-5, 2e-5, f"o[{b},{h}]")
        for name, got, want in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
            assert_close(sl(got), want, 5e-5, 5e-5, f"{name}[{b},{h}]")


def test_device_attention_rejects_bad_shapes(lib, cuda):
    pos = torch.arange(8, dtype=torch.int64, device="cuda").repeat(1, 1)
    with pytest.raises(ValueError):
        etb.Attention(1, 3, 2, 8, 8, 64, pos, pos)  # q heads not a multiple of kv heads
    with pytest.raises(ValueError):
        etb.Attention(1, 2, 2, 8, 8, 63, pos, pos)  # odd head_dim


@pytest.mark.parametrize("Dh", [64, 128])
@pytest.mark.parametrize("mags", [(30.0, 0.01, 1000.0, 1e-5), (1e-3, 1e-3, 1e-4, 300.0)])
def test_binary16_pairs_track_operand_magnitudes(lib, cuda, Dh, mags):
    """The binary16-pair backward scales each operand tensor by its own power
    of two: operands far from 1 (dO near 1e-5 as in a mean loss over many
    tokens, V near 1e3, Q / K near 1e-3) keep the f32-grade bar, normwise per
    tensor (max error <= tol max |reference|)."""
    B, H, T = 1, 2, 320
    q, k, v, do, o, dq, dk, dv = _run(B, H, H, T, Dh, 99 + Dh, True, etb.ATTENTION_BWD_PAIRS16,
                                      mags)
    ro, rdq, rdk, rdv = _oracle(q, k, v, do)
    for name, got, want in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        err = np.abs(got.astype(np.float64) - want).max()
        assert err <= 5e-5 * np.abs(want).max(), (name, err, np.abs(want).max())


def test_unknown_contraction_mode_is_rejected(lib, cuda):
    pos = torch.arange(8, dtype=torch.int64, device="cuda").repeat(1, 1)
    with pytest.raises(ValueError):
        etb.Attention(1, 2, 2, 8, 8, 64, pos, pos, contraction=7)


@pytest.mark.parametrize("Dh,contraction", [(32, etb.ATTENTION_DEFAULT),
                                            (64, etb.ATTENTION_DEFAULT),
                                            (128, etb.ATTENTION_DEFAULT)])
def test_long_sequence_slice_vs_float64(lib, cuda, Dh, contraction):
    """T = 8,192, one (sequence, head): every key tile's dK / dV sums
    thousands of query rows, across several f32 chunks of the accumulation
    (without the chunks dK / dV drifted to 1e-4 at T = 16,384): head_dim 32
    on the 3xTF32 kernels, 64 and 128 on the binary16-pair ones (their
    default at this length).  Against a float64 evaluation, element-wise
    within the A2 bar (5e-5 abs + rel)."""
    T = 8192
    q, k, v, do = (orc.fill_normal(700 + Dh, i, T * Dh).reshape(1, 1, T, Dh) for i in range(4))
    pos = torch.arange(T, dtype=torch.int64, device="cuda").reshape(1, T)
    c, s_ = etb.rope_tables(T, Dh)
    att = etb.Attention(1, 1, 1, T, T, Dh, pos, pos, None, torch.from_numpy(c).cuda(),
                        torch.from_numpy(s_).cuda(), contraction=contraction)
    tq, tk, tv, tdo = (torch.from_numpy(x).cuda() for x in (q, k, v, do))
    o = torch.empty_like(tq)
    m = torch.empty(1, 1, T, device="cuda")
    l = torch.empty_like(m)
    dq, dk, dv = torch.empty_like(tq), torch.empty_like(tk), torch.empty_like(tv)
    att.forward(tq, tk, tv, o, m, l)
    att.backward(tq, tk, tv, o, tdo, m, l, dq, dk, dv)
    torch.cuda.synchronize()
    want = attention_f64(q[0, 0], k[0, 0], v[0, 0], do[0, 0], c, s_)
    for name, got, ref in zip(("o", "dq", "dk", "dv"), (o, dq, dk, dv), want):
        g = got.cpu().numpy()[0, 0].astype(np.float64)
        bad = np.abs(g - ref) > 5e-5 + 5e-5 * np.abs(ref)
        assert not bad.any(), (name, int(bad.sum()), float(np.abs(g - ref).max()))


# TF32-grade mode: one product of operands rounded to 11 significant bits;
# the bar is the TF32 LM-gradient bar (normwise per tensor).
TF32_TOL = 5e-3


@pytest.mark.parametrize("B,Hq,Hkv,T,Dh", [(2, 4, 4, 256, 64), (2, 4, 2, 200, 32),
                                           (1, 2, 2, 384, 128), (1, 4, 2, 300, 128)])
def test_tf32_mode_vs_oracle(lib, cuda, B, Hq, Hkv, T, Dh):
    q, k, v, do, o, dq, dk, dv = _run(B, Hq, Hkv, T, Dh, 31 + T, True, etb.ATTENTION_TF32)
    ro, rdq, rdk, rdv = _oracle(q, k, v, do)
    for name, got, want in (("o", o, ro), ("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        err = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
        assert err <= TF32_TOL, (name, err)
        assert err > 1e-5, (name, err)  # one product ran: above the f32-grade ~1e-6

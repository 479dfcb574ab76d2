"""The oracle restatement is bit-identical to the reference's C providers.

tests/golden/reference_vectors.json holds outputs of eshkol-transformer's own
A2 and L2 providers (compiled unmodified by oracle/Makefile.ref) on seeded
inputs; the oracle must reproduce them bit for bit.  When oracle/_ref is built
(this container), the same comparison also runs live, including the N2
runners, at further shapes.
"""
import ctypes as C
import json

import numpy as np
import pytest

from helpers import GOLDEN, bits_equal, decode_ref_vector
from oracle import oracle as orc

VECTORS = json.loads((GOLDEN / "reference_vectors.json").read_text())


def _inputs(case):
    return {k: decode_ref_vector(v) for k, v in case["inputs"].items()}


def _outputs(case):
    return {k: decode_ref_vector(v) for k, v in case["outputs"].items()}


@pytest.mark.parametrize("case", VECTORS["cases"], ids=lambda c: f"{c['kind']}{c['shape']}")
def test_oracle_bit_identical_to_reference_vectors(case):
    x, want = _inputs(case), _outputs(case)
    shape = tuple(case["shape"])
    if case["kind"] == "attention":
        o = orc.attention_forward(shape, x["q"], x["k"], x["v"], x["pos"], x["pos"], x["mask"])
        dq, dk, dv = orc.attention_backward(shape, x["q"], x["k"], x["v"], x["pos"], x["pos"],
                                            x["mask"], x["dout"])
        got = {"o": o, "dq": dq, "dk": dk, "dv": dv}
    elif case["kind"] == "rope":
        got = {op: orc.rope(shape, x["x"], x["pos"], x["inv_freq"], backward=op == "backward")
               for op in ("forward", "backward")}
    else:
        got = {"loss": orc.ce_forward(x["logits"], x["targets"]),
               "grad": orc.ce_backward(x["logits"], x["targets"], x["upstream"])}
    for name, arr in want.items():
        assert bits_equal(got[name], arr), name


ref = orc.ref()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref (reference build) not present")


def _fp(a):
    return a.ctypes.data_as(C.c_void_p)


@needs_ref
@pytest.mark.parametrize("n,t,din,dout", [(2, 8, 16, 24), (1, 33, 40, 7), (4, 16, 64, 96)])
def test_linear_runners_bit_identical(n, t, din, dout):
    x = orc.fill_normal(7, 1, n * t * din).reshape(n, t, din)
    w = orc.fill_normal(7, 2, dout * din, 0, 0.1).reshape(dout, din)
    b = orc.fill_normal(7, 3, dout)
    dy = orc.fill_normal(7, 4, n * t * dout).reshape(n, t, dout)
    y_ref = np.empty((n, t, dout), np.float32)
    assert ref.ref_n2_linear_forward(C.c_size_t(n), C.c_size_t(t), C.c_size_t(din),
                                     C.c_size_t(dout), _fp(x), _fp(w), _fp(b), _fp(y_ref)) == 1
    assert bits_equal(orc.linear_forward(x, w, b), y_ref)
    dx_r, dw_r, db_r = np.empty_like(x), np.empty_like(w), np.empty_like(b)
    assert ref.ref_n2_linear_backward(C.c_size_t(n), C.c_size_t(t), C.c_size_t(din),
                                      C.c_size_t(dout), _fp(x), _fp(w), _fp(dy), 1, _fp(dx_r),
                                      _fp(dw_r), _fp(db_r)) == 1
    dx, dw, db = orc.linear_backward(x, w, dy)
    assert bits_equal(dx, dx_r) and bits_equal(dw, dw_r) and bits_equal(db, db_r)


@needs_ref
@pytest.mark.parametrize("n,t,d", [(2, 5, 8), (1, 17, 128), (3, 4, 33)])
def test_norm_gelu_embedding_runners_bit_identical(n, t, d):
    x = orc.fill_normal(9, 1, n * t * d, 0.5, 2.0).reshape(n, t, d)
    gamma = orc.fill_normal(9, 2, d, 1.0, 0.1)
    beta = orc.fill_normal(9, 3, d, 0.0, 0.1)
    dy = orc.fill_normal(9, 4, n * t * d).reshape(n, t, d)
    eps = np.float32(1e-5)
    y_ref = np.empty_like(x)
    assert ref.ref_n2_layer_norm_forward(C.c_size_t(n), C.c_size_t(t), C.c_size_t(d), _fp(x),
                                         _fp(gamma), _fp(beta), C.c_float(eps), _fp(y_ref)) == 1
    assert bits_equal(orc.layer_norm_forward(x, gamma, beta, float(eps)), y_ref)
    dx_r, dg_r, db_r = np.empty_like(x), np.empty_like(gamma), np.empty_like(beta)
    assert ref.ref_n2_layer_norm_backward(C.c_size_t(n), C.c_size_t(t), C.c_size_t(d), _fp(x),
                                          _fp(gamma), C.c_float(eps), _fp(dy), _fp(dx_r),
                                          _fp(dg_r), _fp(db_r)) == 1
    dx, dg, db = orc.layer_norm_backward(x, gamma, float(eps), dy)
    assert bits_equal(dx, dx_r) and bits_equal(dg, dg_r) and bits_equal(db, db_r)
    g_ref = np.empty_like(x)
    assert ref.ref_n2_gelu(C.c_size_t(n), C.c_size_t(t), C.c_size_t(d), _fp(x), None,
                           _fp(g_ref)) == 1
    assert bits_equal(orc.gelu_forward(x), g_ref)
    gb_ref = np.empty_like(x)
    assert ref.ref_n2_gelu(C.c_size_t(n), C.c_size_t(t), C.c_size_t(d), _fp(x), _fp(dy),
                           _fp(gb_ref)) == 1
    assert bits_equal(orc.gelu_backward(x, dy), gb_ref)
    V = 11
    ids = orc.fill_tokens(9, 5, n * t, V).reshape(n, t)
    w = orc.fill_normal(9, 6, V * d).reshape(V, d)
    e_ref = np.empty((n, t, d), np.float32)
    assert ref.ref_n2_embedding_forward(C.c_size_t(n), C.c_size_t(t), C.c_size_t(V),
                                        C.c_size_t(d), _fp(ids), _fp(w), _fp(e_ref)) == 1
    assert bits_equal(orc.embedding_forward(ids, w), e_ref)
    dw_r = np.empty((V, d), np.float32)
    assert ref.ref_n2_embedding_backward(C.c_size_t(n), C.c_size_t(t), C.c_size_t(V),
                                         C.c_size_t(d), _fp(ids), _fp(dy), _fp(dw_r)) == 1
    assert bits_equal(orc.embedding_backward(ids, dy, V), dw_r)


@needs_ref
def test_attention_live_against_reference_provider():
    from eshkol_transformer_b200 import k1
    a2 = k1.provider(ref, "et_a2_kernel_provider_v1")
    shape = (2, 6, 3, 20, 20, 16)
    N, Hq, Hkv, T, _, Dh = shape
    q = orc.fill_normal(11, 1, N * Hq * T * Dh).reshape(N, Hq, T, Dh)
    k = orc.fill_normal(11, 2, N * Hkv * T * Dh).reshape(N, Hkv, T, Dh)
    v = orc.fill_normal(11, 3, N * Hkv * T * Dh).reshape(N, Hkv, T, Dh)
    g = orc.fill_normal(11, 4, N * Hq * T * Dh).reshape(N, Hq, T, Dh)
    pos = np.tile(np.arange(T, dtype=np.int64) * 2 + 1, (N, 1))
    mask = (orc.fill_tokens(11, 5, N * T * T, 4) > 0).astype(np.uint8).reshape(N, T, T)
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    rc, err = k1.dispatch(a2, k1.KernelCall("kernel.causal-attention",
                                            "causal-attention.backward", shape,
                                            [q, k, v, pos, pos, mask, g], [dq, dk, dv]))
    assert rc == 0, str(err)
    oq, ok, ov = orc.attention_backward(shape, q, k, v, pos, pos, mask, g)
    assert bits_equal(oq, dq) and bits_equal(ok, dk) and bits_equal(ov, dv)

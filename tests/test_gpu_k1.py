"""Parity of the B200 K1 providers with the oracle, through the C-ABI.

Every provider call goes through the provider's validate_call/invoke_call
(the K1 two-phase contract) with device "cuda" views (device pointers) and
device "cpu" views (host pointers staged through the GPU).  References:
the reference's golden fixtures, the reference's own outputs
(tests/golden/reference_vectors.json) and the bit-pinned oracle.
Tolerances are stated per test; integer/gather work and the rounding-exact
elementwise ops are compared bit for bit.
"""
import json

import numpy as np
import pytest
import torch

import eshkol_transformer_b200 as etb
from eshkol_transformer_b200 import k1
from golden_cases import a2_cases, l2_cases, n2_cases
from helpers import GOLDEN, assert_close, assert_close_norm, bits_equal, decode_ref_vector
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

PROVIDER_FOR = {
    "kernel.causal-attention": "et_a2_kernel_provider_v1",
    "kernel.rope": "et_a2_kernel_provider_v1",
    "kernel.indexed-cross-entropy": "et_l2_indexed_cross_entropy_provider_v1",
    "n3k.linear": "et_n3k_kernel_provider_v1",
}


def provider_for(lib, capability):
    return k1.provider(lib, PROVIDER_FOR.get(capability, "et_n2_kernel_provider_v1"))


def run_call(lib, capability, operation, shape, inputs, out_shapes, device):
    """Dispatches one K1 call; returns numpy outputs (raises on an error)."""
    # np.require keeps 0-d arrays 0-d (the LayerNorm epsilon is a rank-0 view)
    inputs = [np.require(a, requirements="C") for a in inputs]
    if device == "cuda":
        ins = [torch.from_numpy(a).cuda() for a in inputs]
        outs = [torch.full(s, float("nan"), dtype=torch.float32, device="cuda") for s in out_shapes]
    else:
        ins = inputs
        outs = [np.full(s, np.nan, np.float32) for s in out_shapes]
    call = k1.KernelCall(capability, operation, tuple(shape), ins, outs, device=device)
    rc, err = k1.dispatch(provider_for(lib, capability), call)
    assert rc == 0, str(err)
    if device == "cuda":
        torch.cuda.synchronize()
        return [o.cpu().numpy() for o in outs]
    return outs


CASES = a2_cases() + n2_cases() + l2_cases()


@pytest.mark.parametrize("device", ["cuda", "cpu"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_provider_matches_reference_fixture(lib, cuda, case, device):
    lib.et_b200_k1_precision_v1(etb.PRECISION_TF32X3)
    got = run_call(lib, case.capability, case.operation, case.shape, case.inputs,
                   [e.shape for e in case.outputs], device)
    for i, (a, e) in enumerate(zip(got, case.outputs)):
        assert_close(a, e, case.atol, case.rtol, f"{case.name}[{i}]")


VECTORS = json.loads((GOLDEN / "reference_vectors.json").read_text())


@pytest.mark.parametrize("case", VECTORS["cases"], ids=lambda c: f"{c['kind']}{c['shape']}")
def test_provider_against_reference_outputs(lib, cuda, case):
    x = {k: decode_ref_vector(v) for k, v in case["inputs"].items()}
    want = {k: decode_ref_vector(v) for k, v in case["outputs"].items()}
    shape = tuple(case["shape"])
    if case["kind"] == "attention":
        N, Hq, Hkv, Tq, Tk, Dh = shape
        ins = [x["q"], x["k"], x["v"], x["pos"], x["pos"], x["mask"]]
        (o,) = run_call(lib, "kernel.causal-attention", "causal-attention.forward", shape, ins,
                        [(N, Hq, Tq, Dh)], "cuda")
        dq, dk, dv = run_call(lib, "kernel.causal-attention", "causal-attention.backward", shape,
                              ins + [x["dout"]], [(N, Hq, Tq, Dh), (N, Hkv, Tk, Dh),
                                                  (N, Hkv, Tk, Dh)], "cuda")
        # A2 fixture tolerance (tests/a2/fixtures: 2e-5 forward, 5e-5 gradients)
        assert_close(o, want["o"], 2e-5, 2e-5, "o")
        for n, a in (("dq", dq), ("dk", dk), ("dv", dv)):
            assert_close(a, want[n], 5e-5, 5e-5, n)
    elif case["kind"] == "rope":
        for op in ("forward", "backward"):
            (y,) = run_call(lib, "kernel.rope", f"rope.{op}", shape,
                            [x["x"], x["pos"], x["inv_freq"]], [shape], "cuda")
            assert bits_equal(y, want[op]), op  # host libm table: bit-exact rotation
    else:
        N, T, V = shape
        (loss,) = run_call(lib, "kernel.indexed-cross-entropy", "indexed-cross-entropy.forward",
                           shape, [x["logits"], x["targets"]], [(N, T)], "cuda")
        (grad,) = run_call(lib, "kernel.indexed-cross-entropy", "indexed-cross-entropy.backward",
                           shape, [x["logits"], x["targets"], x["upstream"]], [shape], "cuda")
        # L2 fixture tolerances (tests/q0/fixtures/indexed_cross_entropy_v1.json)
        assert_close(loss, want["loss"], 2e-6, 2e-5, "loss")
        assert_close(grad, want["grad"], 3e-6, 3e-5, "grad")


def _attention_inputs(shape, seed, masked=False):
    N, Hq, Hkv, Tq, Tk, Dh = shape
    q = orc.fill_normal(seed, 1, N * Hq * Tq * Dh).reshape(N, Hq, Tq, Dh)
    k = orc.fill_normal(seed, 2, N * Hkv * Tk * Dh).reshape(N, Hkv, Tk, Dh)
    v = orc.fill_normal(seed, 3, N * Hkv * Tk * Dh).reshape(N, Hkv, Tk, Dh)
    g = orc.fill_normal(seed, 4, N * Hq * Tq * Dh).reshape(N, Hq, Tq, Dh)
    qpos = np.tile(np.arange(Tk - Tq, Tk, dtype=np.int64), (N, 1))
    kpos = np.tile(np.arange(Tk, dtype=np.int64), (N, 1))
    mask = np.ones((N, Tq, Tk), np.uint8)
    if masked:
        mask = (orc.fill_tokens(seed, 5, N * Tq * Tk, 5) > 0).astype(np.uint8).reshape(N, Tq, Tk)
        mask[:, 0, :] = 0  # an empty row: output and gradients +0
    return q, k, v, qpos, kpos, mask, g


@pytest.mark.parametrize("shape,masked", [
    ((2, 4, 4, 128, 128, 32), False),   # the single-layer attention config (B2 H4 T128 Dh32)
    ((2, 4, 2, 100, 100, 64), True),    # GQA, ragged tiles, keep mask, empty row
    ((1, 2, 2, 37, 70, 128), False),    # Tq < Tk (cached-decode layout), Dh 128
    ((1, 3, 3, 65, 65, 8), True),
    ((1, 2, 2, 512, 512, 64), False),   # several query tiles, fully visible key blocks
    ((1, 4, 2, 300, 800, 32), False),   # Tq < Tk over several tiles, GQA
    ((1, 2, 2, 256, 256, 128), False),  # Dh 128 over several tiles
    ((2, 4, 2, 100, 100, 128), True),   # Dh 128 (binary16-pair backward): GQA, mask, empty row
    ((1, 4, 2, 1024, 1024, 64), True),  # Dh 64 at 1024^2 (binary16 pairs, 128-query blocks): GQA, mask
    ((1, 2, 2, 600, 1800, 64), False),  # Dh 64 binary16 with Tq < Tk over several tiles
])
def test_attention_vs_oracle(lib, cuda, shape, masked):
    N, Hq, Hkv, Tq, Tk, Dh = shape
    q, k, v, qpos, kpos, mask, g = _attention_inputs(shape, 123, masked)
    ins = [q, k, v, qpos, kpos, mask]
    (o,) = run_call(lib, "kernel.causal-attention", "causal-attention.forward", shape, ins,
                    [q.shape], "cuda")
    dq, dk, dv = run_call(lib, "kernel.causal-attention", "causal-attention.backward", shape,
                          ins + [g], [q.shape, k.shape, v.shape], "cuda")
    o_ref = orc.attention_forward(shape, *ins)
    dq_r, dk_r, dv_r = orc.attention_backward(shape, *ins, g)
    assert_close(o, o_ref, 5e-5, 5e-5, "o")
    assert_close(dq, dq_r, 5e-5, 5e-5, "dq")
    assert_close(dk, dk_r, 5e-5, 5e-5, "dk")
    assert_close(dv, dv_r, 5e-5, 5e-5, "dv")
    if masked:
        assert np.all(o[:, :, 0, :] == 0) and np.all(dq[:, :, 0, :] == 0)


# Normwise bounds against the serial-f32 oracle, whose own rounding error is
# ~sqrt(K) 2^-24 of the row norm: FFMA 2e-6; 3xTF32 (drops lo*lo and the
# TF32 rounding of lo: ~2^-22 per product) 1e-5; split-f16 (binary16 hi/lo
# pairs, 11 + 11 bits, lo*lo dropped: the same ~2^-22) 1e-5; single TF32
# (2^-11) 2e-3.
LINEAR_TOL = {etb.PRECISION_TF32X3: 1e-5, etb.PRECISION_F16X3: 1e-5, etb.PRECISION_TF32: 2e-3,
              etb.PRECISION_F32: 2e-6}


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3,
                                       etb.PRECISION_TF32, etb.PRECISION_F32])
@pytest.mark.parametrize("n,t,din,dout", [(2, 64, 128, 384), (1, 300, 256, 96), (3, 50, 100, 70),
                                          (8, 64, 512, 1024)])
def test_linear_all_layouts_vs_oracle(lib, cuda, precision, n, t, din, dout):
    """Forward (A, B K-major), dX (B N-major) and dW (A M-major, B N-major).
    Tolerance: max |err| <= tol * max |ref| per tensor, tol 2e-6 for the
    f32-grade modes (3xTF32, FFMA) and 2e-3 for single TF32."""
    lib.et_b200_k1_precision_v1(precision)
    x = orc.fill_normal(5, 1, n * t * din).reshape(n, t, din)
    w = orc.fill_normal(5, 2, dout * din, 0, 0.05).reshape(dout, din)
    b = orc.fill_normal(5, 3, dout)
    dy = orc.fill_normal(5, 4, n * t * dout).reshape(n, t, dout)
    shape = (n, t, din, dout)
    (y,) = run_call(lib, "kernel.matmul", "linear.forward", shape, [x, w, b], [(n, t, dout)], "cuda")
    dx, dw, db = run_call(lib, "kernel.matmul", "linear.backward", shape, [x, w, dy],
                          [(n, t, din), (dout, din), (dout,)], "cuda")
    lib.et_b200_k1_precision_v1(etb.PRECISION_TF32X3)
    tol = LINEAR_TOL[precision]
    assert_close_norm(y, orc.linear_forward(x, w, b), tol, "y")
    dx_r, dw_r, db_r = orc.linear_backward(x, w, dy)
    assert_close_norm(dx, dx_r, tol, "dx")
    assert_close_norm(dw, dw_r, tol, "dw")
    assert_close_norm(db, db_r, 2e-6, "db")


@pytest.mark.parametrize("sx,sw,sg", [(1e4, 1e-3, 1e-7), (1e-5, 30.0, 2e3)])
def test_linear_split_f16_scaled_operands(lib, cuda, sx, sw, sg):
    """Split-f16 operands far from binary16's range: each tensor's power-of-two
    scale brings it into range, and the accumulator is scaled back exactly."""
    n, t, din, dout = 2, 96, 256, 192
    x = orc.fill_normal(8, 1, n * t * din).reshape(n, t, din) * np.float32(sx)
    w = orc.fill_normal(8, 2, dout * din).reshape(dout, din) * np.float32(sw)
    b = orc.fill_normal(8, 3, dout)
    dy = orc.fill_normal(8, 4, n * t * dout).reshape(n, t, dout) * np.float32(sg)
    shape = (n, t, din, dout)
    lib.et_b200_k1_precision_v1(etb.PRECISION_F16X3)
    try:
        (y,) = run_call(lib, "kernel.matmul", "linear.forward", shape, [x, w, b], [(n, t, dout)],
                        "cuda")
        dx, dw, _ = run_call(lib, "kernel.matmul", "linear.backward", shape, [x, w, dy],
                             [(n, t, din), (dout, din), (dout,)], "cuda")
    finally:
        lib.et_b200_k1_precision_v1(etb.PRECISION_TF32X3)
    tol = LINEAR_TOL[etb.PRECISION_F16X3]
    assert_close_norm(y, orc.linear_forward(x, w, b), tol, "y")
    dx_r, dw_r, _ = orc.linear_backward(x, w, dy)
    assert_close_norm(dx, dx_r, tol, "dx")
    assert_close_norm(dw, dw_r, tol, "dw")


# Long contractions against float64 (torch on the GPU): the tensor pipe's
# accumulation truncates, so the f32-grade GEMMs sum K in chunks and add the
# chunks in f32; their error then stays flat in K.  LONG_K_TOL: max |err| <=
# tol * max |f64| for sign-mixed operands, and the same bound for all-positive
# operands, where truncation errors cannot cancel.
LONG_K_TOL = {etb.PRECISION_TF32X3: 1e-5, etb.PRECISION_F16X3: 1.5e-5}


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3])
@pytest.mark.parametrize("K", [4096, 65536])
@pytest.mark.parametrize("positive", [False, True])
def test_linear_long_k_vs_float64(lib, cuda, precision, K, positive):
    M, N = 256, 512
    g = torch.Generator(device="cuda").manual_seed(K + positive)
    x = torch.randn(1, M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g)
    if positive:
        x, w = x.abs(), w.abs()
    y = torch.full((1, M, N), float("nan"), device="cuda")
    lib.et_b200_k1_precision_v1(precision)
    try:
        call = k1.KernelCall("kernel.matmul", "linear.forward-no-bias", (1, M, K, N), [x, w], [y],
                             device="cuda")
        rc, err = k1.dispatch(provider_for(lib, "kernel.matmul"), call)
        torch.cuda.synchronize()
    finally:
        lib.et_b200_k1_precision_v1(etb.PRECISION_TF32X3)
    assert rc == 0, str(err)
    ref = x[0].double() @ w.double().T
    rel = ((y[0].double() - ref).abs().max() / ref.abs().max()).item()
    assert rel <= LONG_K_TOL[precision], rel


@pytest.mark.parametrize("precision", [etb.PRECISION_TF32X3, etb.PRECISION_F16X3])
def test_linear_dx_rows_spanning_2e20(lib, cuda, precision):
    """dY rows scaled from 1 down to 2^-20 inside one tensor: dX row by row
    against float64, besides the normwise bar.  3xTF32 pairs carry f32's
    exponent range, so every row keeps the relative bound.  Split-f16 scales
    each tensor by one power of two, so an element far below the tensor's max
    keeps an absolute representation error of at most 2^-35 max|dY| (half the
    binary16 subnormal spacing at that scale); the per-row bound adds what that
    error contributes to a dX element: 2^-35 max|dY| ||W[:, i]||_1."""
    n, t, din, dout = 1, 256, 512, 1024
    x = orc.fill_normal(9, 1, n * t * din).reshape(n, t, din)
    w = orc.fill_normal(9, 2, dout * din, 0, 0.05).reshape(dout, din)
    dy = orc.fill_normal(9, 4, n * t * dout).reshape(n, t, dout)
    row_scale = np.float32(2.0) ** -np.linspace(0, 20, t).astype(np.float32)
    dy = (dy * row_scale[None, :, None]).astype(np.float32)
    lib.et_b200_k1_precision_v1(precision)
    try:
        dx, _, _ = run_call(lib, "kernel.matmul", "linear.backward", (n, t, din, dout), [x, w, dy],
                            [(n, t, din), (dout, din), (dout,)], "cuda")
    finally:
        lib.et_b200_k1_precision_v1(etb.PRECISION_TF32X3)
    ref = dy[0].astype(np.float64) @ w.astype(np.float64)
    err = np.abs(dx[0].astype(np.float64) - ref)
    assert err.max() <= 1e-5 * np.abs(ref).max(), err.max() / np.abs(ref).max()
    floor = 0.0
    if precision == etb.PRECISION_F16X3:
        floor = 2.0 ** -35 * np.abs(dy).max() * np.abs(w.astype(np.float64)).sum(axis=0)
    rowmax = np.abs(ref).max(axis=1, keepdims=True)
    assert np.all(err <= 1e-5 * rowmax + floor), \
        float(((err - floor) / rowmax).max())
    per_row = (err / rowmax).max(axis=1)
    print(f"precision {precision}: normwise {err.max() / np.abs(ref).max():.2e}, worst row "
          f"{per_row.max():.2e} (row of max 2^-20: {per_row[-1]:.2e})")


def test_n3k_linear_no_bias(lib, cuda):
    x = orc.fill_normal(6, 1, 4 * 32 * 64).reshape(4, 32, 64)
    w = orc.fill_normal(6, 2, 48 * 64, 0, 0.1).reshape(48, 64)
    (y,) = run_call(lib, "n3k.linear", "n3k.linear.forward-no-bias", (4, 32, 64, 48), [x, w],
                    [(4, 32, 48)], "cuda")
    assert_close_norm(y, orc.linear_forward(x, w), 2e-6, "y")


@pytest.mark.parametrize("rows,d", [(512, 128), (300, 1024), (7, 33)])
def test_norm_activation_embedding_vs_oracle(lib, cuda, rows, d):
    x = orc.fill_normal(8, 1, rows * d, 0.3, 1.5).reshape(1, rows, d)
    gamma = orc.fill_normal(8, 2, d, 1.0, 0.2)
    beta = orc.fill_normal(8, 3, d, 0.0, 0.2)
    dy = orc.fill_normal(8, 4, rows * d).reshape(1, rows, d)
    eps = np.array(1e-5, np.float32)
    shape = (1, rows, d)
    (y,) = run_call(lib, "kernel.norm", "layer-norm.forward", shape, [x, gamma, beta, eps],
                    [shape], "cuda")
    assert_close_norm(y, orc.layer_norm_forward(x, gamma, beta, 1e-5), 2e-6, "ln y")
    dx, dg, db = run_call(lib, "kernel.norm", "layer-norm.backward", shape, [x, gamma, eps, dy],
                          [shape, (d,), (d,)], "cuda")
    dx_r, dg_r, db_r = orc.layer_norm_backward(x, gamma, 1e-5, dy)
    assert_close_norm(dx, dx_r, 5e-6, "ln dx")
    assert_close_norm(dg, dg_r, 5e-6, "ln dgamma")
    assert_close_norm(db, db_r, 5e-6, "ln dbeta")
    (gf,) = run_call(lib, "kernel.activation", "gelu.forward", shape, [x], [shape], "cuda")
    assert_close(gf, orc.gelu_forward(x), 1e-6, 2e-6, "gelu")
    (gb,) = run_call(lib, "kernel.activation", "gelu.backward", shape, [x, dy], [shape], "cuda")
    assert_close(gb, orc.gelu_backward(x, dy), 1e-6, 2e-6, "gelu'")
    (r,) = run_call(lib, "kernel.residual", "residual.forward", shape, [x, dy], [shape], "cuda")
    assert bits_equal(r, (x + dy).astype(np.float32))
    a, b = run_call(lib, "kernel.residual", "residual.backward", shape, [dy], [shape, shape], "cuda")
    assert bits_equal(a, dy) and bits_equal(b, dy)
    (rl,) = run_call(lib, "kernel.activation", "relu.backward", shape, [x, dy], [shape], "cuda")
    assert bits_equal(rl, np.where(x > 0, dy, np.float32(0)))
    V = 50
    ids = orc.fill_tokens(8, 5, rows, V).reshape(1, rows)
    w = orc.fill_normal(8, 6, V * d).reshape(V, d)
    (e,) = run_call(lib, "kernel.embedding-forward", "embedding.forward", (1, rows, V, d),
                    [ids, w], [(1, rows, d)], "cuda")
    assert bits_equal(e, orc.embedding_forward(ids, w))
    (dw,) = run_call(lib, "kernel.embedding-backward", "embedding.backward", (1, rows, V, d),
                     [ids, dy], [(V, d)], "cuda")
    assert bits_equal(dw, orc.embedding_backward(ids, dy, V))  # same summation order


@pytest.mark.parametrize("rows,V", [(64, 1024), (33, 32768), (5, 1001), (4, 1)])
def test_cross_entropy_vs_oracle(lib, cuda, rows, V):
    logits = (orc.fill_normal(4, 1, rows * V) * 4).astype(np.float32).reshape(1, rows, V)
    targets = orc.fill_tokens(4, 2, rows, V).reshape(1, rows)
    up = orc.fill_normal(4, 3, rows).reshape(1, rows)
    (loss,) = run_call(lib, "kernel.indexed-cross-entropy", "indexed-cross-entropy.forward",
                       (1, rows, V), [logits, targets], [(1, rows)], "cuda")
    (grad,) = run_call(lib, "kernel.indexed-cross-entropy", "indexed-cross-entropy.backward",
                       (1, rows, V), [logits, targets, up], [(1, rows, V)], "cuda")
    # Against float64 ground truth: the L2 fixture tolerances at every V.
    x64 = logits.astype(np.float64)[0]
    m = x64.max(axis=1, keepdims=True)
    e = np.exp(x64 - m)
    s = e.sum(axis=1, keepdims=True)
    t = targets[0]
    loss64 = np.log(s[:, 0]) + m[:, 0] - x64[np.arange(rows), t]
    p = e / s
    p[np.arange(rows), t] -= 1.0
    assert_close(loss[0], loss64, 2e-6, 2e-5, "loss vs f64")
    assert_close(grad[0], p * up[0][:, None], 3e-6, 3e-5, "grad vs f64")
    # Against the oracle (the reference's sequential f32 exp-sum, whose own
    # rounding error grows like sqrt(V) 2^-24): fixture bounds widened by
    # sqrt(V / 1024) above V = 1024.
    widen = max(1.0, np.sqrt(V / 1024.0))
    assert_close(loss, orc.ce_forward(logits, targets), 2e-6 * widen, 2e-5 * widen, "loss")
    assert_close(grad, orc.ce_backward(logits, targets, up), 3e-6 * widen, 3e-5 * widen, "grad")


def test_validate_rejects_and_leaves_outputs_unchanged(lib, cuda):
    shape = (1, 2, 2, 4, 4, 8)
    q, k, v, qpos, kpos, mask, g = _attention_inputs(shape, 9)
    q[0, 1, 2, 3] = np.inf
    out = torch.full(q.shape, 7.0, device="cuda")
    call = k1.KernelCall("kernel.causal-attention", "causal-attention.forward", shape,
                         [torch.from_numpy(a).cuda() for a in (q, k, v, qpos, kpos, mask)], [out])
    rc, err = k1.dispatch(provider_for(lib, "kernel.causal-attention"), call)
    assert rc == k1.ERROR_INVALID_ARGUMENT
    assert torch.all(out == 7.0)
    # noncanonical positions and masks, bad targets, Hkv < 2
    q[0, 1, 2, 3] = 0
    bad = kpos.copy()
    bad[0, 2] = bad[0, 1]
    rc, err = k1.dispatch(provider_for(lib, "kernel.causal-attention"),
                          k1.KernelCall("kernel.causal-attention", "causal-attention.forward",
                                        shape, [q, k, v, qpos, bad, mask], [np.zeros_like(q)]))
    assert rc == k1.ERROR_INVALID_ARGUMENT
    m2 = mask.copy()
    m2[0, 0, 0] = 2
    rc, _ = k1.dispatch(provider_for(lib, "kernel.causal-attention"),
                        k1.KernelCall("kernel.causal-attention", "causal-attention.forward",
                                      shape, [q, k, v, qpos, kpos, m2], [np.zeros_like(q)]))
    assert rc == k1.ERROR_INVALID_ARGUMENT
    logits = np.zeros((1, 2, 5), np.float32)
    rc, _ = k1.dispatch(provider_for(lib, "kernel.indexed-cross-entropy"),
                        k1.KernelCall("kernel.indexed-cross-entropy",
                                      "indexed-cross-entropy.forward", (1, 2, 5),
                                      [logits, np.array([[1, 5]], np.int64)],
                                      [np.zeros((1, 2), np.float32)]))
    assert rc == k1.ERROR_SHAPE_MISMATCH
    s1 = (1, 2, 1, 4, 4, 8)
    rc, _ = k1.dispatch(provider_for(lib, "kernel.causal-attention"),
                        k1.KernelCall("kernel.causal-attention", "causal-attention.forward", s1,
                                      [q, k[:, :1].copy(), v[:, :1].copy(), qpos, kpos, mask],
                                      [np.zeros_like(q)]))
    assert rc == k1.ERROR_SHAPE_MISMATCH
    # an output aliasing an input
    x = torch.zeros(1, 4, 8, device="cuda")
    rc, err = k1.dispatch(provider_for(lib, "kernel.residual"),
                          k1.KernelCall("kernel.residual", "residual.forward", (1, 4, 8),
                                        [x, x.clone()], [x]))
    assert rc == k1.ERROR_INVALID_ARGUMENT and err.code == k1.CODE_ALIASING_OUTPUT


def test_reference_k1_runtime_dispatches_b200_provider(lib, cuda):
    """The reference's K1 runtime (native/kernel_abi.c) dispatching the B200
    A2 provider on cuda views: the drop-in path a C host would take."""
    import ctypes as C
    ref = orc.ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    RESOLVER = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_char_p)
    fn = lib.et_a2_kernel_provider_v1
    fn.restype = C.c_void_p
    target = fn()
    resolver = RESOLVER(lambda ctx, sym: target)
    runtime = C.c_void_p()
    err = k1.KernelError()
    ref.et_kernel_runtime_discover.argtypes = [RESOLVER, C.c_void_p, C.POINTER(C.c_void_p),
                                               C.POINTER(k1.KernelError)]
    assert ref.et_kernel_runtime_discover(resolver, None, C.byref(runtime), C.byref(err)) == 0
    shape = (2, 4, 4, 128, 128, 32)
    q, k, v, qpos, kpos, mask, g = _attention_inputs(shape, 77)
    out = torch.zeros(q.shape, device="cuda")
    call = k1.KernelCall("kernel.causal-attention", "causal-attention.forward", shape,
                         [torch.from_numpy(a).cuda() for a in (q, k, v, qpos, kpos, mask)], [out])
    ref.et_kernel_runtime_dispatch.argtypes = [C.c_void_p, C.POINTER(k1.Call),
                                               C.POINTER(k1.KernelError)]
    rc = ref.et_kernel_runtime_dispatch(runtime, C.pointer(call.call), C.byref(err))
    assert rc == 0, str(err)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), orc.attention_forward(shape, q, k, v, qpos, kpos, mask),
                 5e-5, 5e-5, "o")
    ref.et_kernel_runtime_destroy.argtypes = [C.c_void_p]
    ref.et_kernel_runtime_destroy(runtime)


def test_reference_k1_runtime_dispatches_composite_through_k2_resolver(lib, cuda):
    """The reference's K1 runtime discovering through the fixed K2 resolver
    (et_b200_k2_resolver_v1 with its private context) gets the composite B200
    provider and dispatches attention and cross-entropy calls to it."""
    import ctypes as C
    ref = orc.ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    lib.et_b200_k2_resolver_context_v1.restype = C.c_void_p
    lib.et_b200_k2_resolver_v1.restype = C.c_void_p
    lib.et_b200_k2_resolver_v1.argtypes = [C.c_void_p, C.c_char_p]
    RESOLVER = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_char_p)
    resolver = RESOLVER(lambda c, s: lib.et_b200_k2_resolver_v1(c, s))
    runtime = C.c_void_p()
    err = k1.KernelError()
    ref.et_kernel_runtime_discover.argtypes = [RESOLVER, C.c_void_p, C.POINTER(C.c_void_p),
                                               C.POINTER(k1.KernelError)]
    assert ref.et_kernel_runtime_discover(resolver, lib.et_b200_k2_resolver_context_v1(),
                                          C.byref(runtime), C.byref(err)) == 0, str(err)
    ref.et_kernel_runtime_dispatch.argtypes = [C.c_void_p, C.POINTER(k1.Call),
                                               C.POINTER(k1.KernelError)]
    shape = (2, 4, 4, 128, 128, 32)
    q, k, v, qpos, kpos, mask, g = _attention_inputs(shape, 78)
    out = torch.zeros(q.shape, device="cuda")
    call = k1.KernelCall("kernel.causal-attention", "causal-attention.forward", shape,
                         [torch.from_numpy(a).cuda() for a in (q, k, v, qpos, kpos, mask)], [out])
    assert ref.et_kernel_runtime_dispatch(runtime, C.pointer(call.call), C.byref(err)) == 0
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), orc.attention_forward(shape, q, k, v, qpos, kpos, mask),
                 5e-5, 5e-5, "o")
    rows, V = 16, 1024
    logits = orc.fill_normal(5, 1, rows * V).reshape(1, rows, V)
    targets = orc.fill_tokens(5, 2, rows, V).reshape(1, rows)
    loss = torch.zeros(1, rows, device="cuda")
    call = k1.KernelCall("kernel.indexed-cross-entropy", "indexed-cross-entropy.forward",
                         (1, rows, V), [torch.from_numpy(logits).cuda(),
                                        torch.from_numpy(targets).cuda()], [loss])
    assert ref.et_kernel_runtime_dispatch(runtime, C.pointer(call.call), C.byref(err)) == 0
    torch.cuda.synchronize()
    assert_close(loss.cpu().numpy(), orc.ce_forward(logits, targets), 2e-6, 2e-5, "loss")
    ref.et_kernel_runtime_destroy.argtypes = [C.c_void_p]
    ref.et_kernel_runtime_destroy(runtime)

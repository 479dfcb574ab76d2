"""The O2 Eshkol bridge over the device optimizer, driven through the
extension's extern signatures (native/o2_wave2_extension.esk:4-29).

* three updates of two parameters: bit-identical to the reference's
  per-element arithmetic (oracle pinned by the adamw fixtures);
* the step's gradient checks (o2_optimizer.c:1813-1856): an absent gradient
  and inconsistent accumulation metadata are refused with O2 status 7, and
  nothing changes;
* snapshot / load (o2_optimizer.c:2052, 2173): a second optimizer loaded from
  a snapshot -- in memory, and through the atomic state file -- continues
  bit for bit like the first; a mismatched configuration is refused.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import eshkol_transformer_b200 as etb
from eshkol_transformer_b200 import k1
from helpers import bits_equal
from o2_bridge import bind
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

OPTS = (1e-3, 0.9, 0.999, 1e-8, 0.01)
SIZES = (1000, 4096)


def _param(br, value, grad):
    out = C.c_void_p()
    err = k1.KernelError()
    assert br.et_b200_parameter_create_v1(value.data_ptr(), grad.data_ptr(), value.numel(),
                                          C.byref(out), C.byref(err)) == 0, str(err)
    return out


def _optimizer(br, params, ident):
    b = br.et_o2_private_builder_create_v1(len(params), 0, 0, 0, 0, 0, 0)
    assert b
    bits = [etb.f32_bits(x) for x in OPTS]
    for i, p in enumerate(params):
        assert br.et_o2_private_builder_set_v1(b, i, p, C.addressof(ident), *bits) == 0
    opt = br.et_o2_private_builder_finish_v1(b)
    assert opt, br.et_b200_o2_bridge_last_error_message_v1()
    return opt


def _accumulate(br, params, grads_dev, grads, weight=2.0, counts=(4, 4)):
    for p, gd, g, c in zip(params, grads_dev, grads, counts):
        gd.copy_(torch.from_numpy(g))
        err = k1.KernelError()
        assert br.et_b200_parameter_set_gradient_v1(p, c, etb.f32_bits(weight), C.byref(err)) == 0


def test_bridge_steps_match_reference_arithmetic(lib, cuda):
    br = bind(lib)
    ident = C.c_int(7)
    values = [torch.from_numpy(orc.fill_normal(40, i, n)).cuda() for i, n in enumerate(SIZES)]
    grads_dev = [torch.zeros(n, device="cuda") for n in SIZES]
    params = [_param(br, v, g) for v, g in zip(values, grads_dev)]
    opt = _optimizer(br, params, ident)
    ref_p = [orc.fill_normal(40, i, n) for i, n in enumerate(SIZES)]
    ref_m = [np.zeros(n, np.float32) for n in SIZES]
    ref_v = [np.zeros(n, np.float32) for n in SIZES]
    for step in range(1, 4):
        grads = [orc.fill_normal(41 + step, i, n) for i, n in enumerate(SIZES)]
        _accumulate(br, params, grads_dev, grads)
        assert br.et_o2_private_optimizer_require_absent_gradients_v1(opt) == 7
        assert br.et_o2_private_optimizer_step_v1(opt) == 0
        for i in range(2):
            assert orc.adamw_step(ref_p[i], grads[i], ref_m[i], ref_v[i],
                                  orc.adamw_options(*OPTS), step, 2.0) == 0
            assert bits_equal(values[i].cpu().numpy(), ref_p[i]), (step, i)
        assert br.et_o2_private_optimizer_completed_updates_v1(opt) == step
        assert br.et_o2_private_optimizer_zero_grad_v1(opt) == 0
        assert all(torch.count_nonzero(g).item() == 0 for g in grads_dev)
        assert br.et_o2_private_optimizer_require_absent_gradients_v1(opt) == 0
    assert br.et_o2_private_optimizer_schedule_factor_bits_v1(opt) == 0x3f800000
    # refusals leave everything as it was
    before = [v.clone() for v in values]
    assert br.et_o2_private_optimizer_step_v1(opt) == 7  # gradients absent
    grads = [orc.fill_normal(60, i, n) for i, n in enumerate(SIZES)]
    _accumulate(br, params, grads_dev, grads, counts=(4, 5))
    assert br.et_o2_private_optimizer_step_v1(opt) == 7  # inconsistent metadata
    assert b"inconsistent" in br.et_b200_o2_bridge_last_error_message_v1()
    assert all(torch.equal(a, b) for a, b in zip(values, before))
    assert br.et_o2_private_optimizer_completed_updates_v1(opt) == 3
    h = C.c_void_p(opt)
    br.et_b200_o2_bridge_destroy_v1(C.byref(h))
    for p in params:
        br.et_b200_parameter_destroy_v1(C.byref(p))


def test_bridge_snapshot_load_and_state_file(lib, cuda, tmp_path):
    br = bind(lib)
    ident = C.c_int(8)

    def make():
        vals = [torch.from_numpy(orc.fill_normal(50, i, n)).cuda() for i, n in enumerate(SIZES)]
        gds = [torch.zeros(n, device="cuda") for n in SIZES]
        ps = [_param(br, v, g) for v, g in zip(vals, gds)]
        return vals, gds, ps, _optimizer(br, ps, ident)

    va, ga, pa, oa = make()
    for step in range(1, 3):
        _accumulate(br, pa, ga, [orc.fill_normal(70 + step, i, n) for i, n in enumerate(SIZES)])
        assert br.et_o2_private_optimizer_step_v1(oa) == 0
        assert br.et_o2_private_optimizer_zero_grad_v1(oa) == 0
    st = br.et_o2_private_optimizer_state_snapshot_v1(oa)
    assert st
    path = str(tmp_path / "o2.state").encode()
    assert br.et_b200_o2_state_write_v1(st, path) == 0
    st_file = br.et_b200_o2_state_read_v1(path)
    assert st_file
    # two fresh optimizers over copies of the current values, loaded from the
    # in-memory snapshot and from the file
    clones = []
    for state in (st, st_file):
        vb, gb, pb, ob = make()
        for a, b in zip(va, vb):
            b.copy_(a)
        assert br.et_o2_private_optimizer_load_state_v1(ob, state) == 0
        assert br.et_o2_private_optimizer_completed_updates_v1(ob) == 2
        clones.append((vb, gb, pb, ob))
    for step in range(3, 5):
        grads = [orc.fill_normal(70 + step, i, n) for i, n in enumerate(SIZES)]
        for vals, gds, ps, o in [(va, ga, pa, oa)] + clones:
            _accumulate(br, ps, gds, grads)
            assert br.et_o2_private_optimizer_step_v1(o) == 0
            assert br.et_o2_private_optimizer_zero_grad_v1(o) == 0
        for vb, _, _, _ in clones:
            assert all(bits_equal(a.cpu().numpy(), b.cpu().numpy()) for a, b in zip(va, vb))
    # a configuration that differs is refused and leaves the optimizer untouched
    b = br.et_o2_private_builder_create_v1(2, 1, etb.f32_bits(1.0), 0, 0, 0, 0)
    vc, gc, pc, _ = make()
    bits = [etb.f32_bits(x) for x in OPTS]
    for i, p in enumerate(pc):
        assert br.et_o2_private_builder_set_v1(b, i, p, C.addressof(ident), *bits) == 0
    oc = br.et_o2_private_builder_finish_v1(b)
    assert br.et_o2_private_optimizer_load_state_v1(oc, st) == 7
    assert br.et_o2_private_optimizer_completed_updates_v1(oc) == 0
    for state in (st, st_file):
        assert br.et_o2_private_optimizer_state_release_v1(state) == 0
    for o in [oa, oc] + [c[3] for c in clones]:
        h = C.c_void_p(o)
        br.et_b200_o2_bridge_destroy_v1(C.byref(h))

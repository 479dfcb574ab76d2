"""The AdamW entry point that allocates nothing (et_b200_adamw_step_noalloc_v1).

It serves callers that cannot let the library allocate device memory: hosts
that give all of HBM to their own allocator at start-up, and training loops
that keep the device footprint fixed because cudaMalloc/cudaFree can
synchronise the device mid-step.  The caller owns every tensor; the call's only
scratch is a static device array.  Its results must match the optimizer entry
point that does allocate (et_b200_o2_optimizer_step_v1) on two updates in a
row: parameters and moments bit for bit (the AdamW parity bar), the gradient
norm within 1e-6 relative (the two sum the f64 partials in different groups).

This file is collected last so that a failure here comes after every other
test has run; it also passes alone in a fresh process.
"""
import ctypes as C
import struct

import numpy as np
import pytest
import torch

import eshkol_transformer_b200 as etb
from eshkol_transformer_b200 import k1

pytestmark = pytest.mark.gpu

OPTS = (1e-3, 0.9, 0.999, 1e-8, 0.01)


def _entry(lib):
    fn = lib.et_b200_adamw_step_noalloc_v1
    fn.restype = C.c_int32
    fn.argtypes = ([C.c_void_p] * 4 + [C.c_uint64] + [C.c_uint32] * 5 +
                   [C.c_uint64, C.c_uint32, C.c_uint32, C.c_void_p, C.POINTER(C.c_uint32),
                    C.POINTER(k1.KernelError)])
    return fn


def _f32(bits: int) -> float:
    return struct.unpack("<f", struct.pack("<I", bits))[0]


class _DeviceArray:
    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3}


def _view(ptr: int, n: int) -> torch.Tensor:
    return torch.as_tensor(_DeviceArray(ptr, n), device="cuda")


def _bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    return torch.equal(a.view(torch.int32), b.view(torch.int32))


def _step(fn, p, g, m, v, n, update, weight, clip_max=0.0):
    norm = C.c_uint32()
    err = k1.KernelError()
    rc = fn(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), n,
            *[etb.f32_bits(x) for x in OPTS], update, etb.f32_bits(weight),
            etb.f32_bits(clip_max) if clip_max else 0, None, C.byref(norm), C.byref(err))
    return rc, err, _f32(norm.value)


@pytest.mark.parametrize("clip_max", [0.0, 50.0])
def test_noalloc_step_matches_allocating_optimizer_two_updates(lib, cuda, clip_max):
    n = 300_001  # five 65,536-element partials, the last one partial
    fn = _entry(lib)
    p0 = etb.fill_normal(21, 0, n)
    pa = torch.from_numpy(p0.copy()).cuda()
    ga = torch.zeros(n, device="cuda")
    opt = etb.Optimizer([(pa.data_ptr(), ga.data_ptr(), n, *OPTS)],
                        clip_kind=1 if clip_max else 0, clip_max=clip_max)
    pb = torch.from_numpy(p0.copy()).cuda()
    gb = torch.zeros(n, device="cuda")
    mb = torch.zeros(n, device="cuda")
    vb = torch.zeros(n, device="cuda")
    weight = 2.0
    for update in (1, 2):
        g = etb.fill_normal(22 + update, 1, n, 0.0, 3.0)
        ga.copy_(torch.from_numpy(g))
        gb.copy_(torch.from_numpy(g))
        norm_a = opt.step(weight)
        rc, err, norm_b = _step(fn, pb, gb, mb, vb, n, update, weight, clip_max)
        assert rc == 0, str(err)
        torch.cuda.synchronize()
        assert abs(norm_b - norm_a) <= 1e-6 * norm_a, (update, norm_a, norm_b)
        if clip_max:
            assert norm_a > clip_max  # the clip branch is exercised
        ma_ptr, va_ptr = opt.moments(0)
        ma, va = _view(ma_ptr, n), _view(va_ptr, n)
        if norm_a == norm_b:
            assert _bits_equal(pa, pb), update
            assert _bits_equal(ma, mb), update
            assert _bits_equal(va, vb), update
        else:  # a one-ulp norm difference moves the clip factor by one ulp
            torch.testing.assert_close(pb, pa, rtol=1e-6, atol=0)
            torch.testing.assert_close(mb, ma, rtol=1e-6, atol=0)
            torch.testing.assert_close(vb, va, rtol=1e-6, atol=0)
    opt.close()


def test_noalloc_rejects_oversize_and_nonfinite(lib, cuda):
    fn = _entry(lib)
    n = 1000
    p = torch.ones(n, device="cuda")
    g = torch.ones(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    rc, err, _ = _step(fn, p, g, m, v, 8192 * 65536 + 1, 1, 1.0)
    assert rc == k1.ERROR_SHAPE_MISMATCH and b"536870912" in err.message
    g[17] = float("nan")
    before = p.clone()
    rc, err, _ = _step(fn, p, g, m, v, n, 1, 1.0)
    assert rc == k1.ERROR_INVALID_ARGUMENT
    assert torch.equal(p, before) and torch.all(m == 0) and torch.all(v == 0)
    g[17] = 0.5  # status words are cleared by the next call
    rc, err, norm = _step(fn, p, g, m, v, n, 1, 1.0)
    assert rc == 0, str(err)
    assert abs(norm - float(torch.linalg.vector_norm(g.double()))) <= 1e-6 * norm


def test_noalloc_leaves_tensors_untouched_on_any_nonfinite(lib, cuda):
    """All or nothing, as the reference's staged commit: an update that would
    overflow (finite gradient 1e20: its square is beyond f32), a nonfinite
    moment, and finite gradients whose norm is beyond f32 each return
    INVALID_ARGUMENT with the reference's message and leave parameter and
    moments bit-unchanged."""
    fn = _entry(lib)
    n = 70_000  # two norm partials
    p = torch.from_numpy(etb.fill_normal(31, 0, n)).cuda()
    m = torch.from_numpy(etb.fill_normal(31, 1, n, 0.0, 1e-3)).cuda()
    v = torch.from_numpy(np.abs(etb.fill_normal(31, 2, n, 0.0, 1e-3))).cuda()
    g = torch.from_numpy(etb.fill_normal(31, 3, n)).cuda()
    cases = []
    g1 = g.clone()
    g1[n - 5] = 1e20
    cases.append((g1, m.clone(), b"AdamW produced a nonfinite value"))
    m2 = m.clone()
    m2[3] = float("inf")
    cases.append((g.clone(), m2, b"parameter, gradient, or moment is nonfinite"))
    g3 = torch.full((n,), 1e38, device="cuda")
    cases.append((g3, m.clone(), b"gradient norm is unrepresentable"))
    for grad, mom, message in cases:
        pc, vc = p.clone(), v.clone()
        mc = mom.clone()
        rc, err, _ = _step(fn, pc, grad, mc, vc, n, 3, 1.0)
        assert rc == k1.ERROR_INVALID_ARGUMENT, message
        assert message in err.message, (message, err.message)
        assert _bits_equal(pc, p) and _bits_equal(mc, mom) and _bits_equal(vc, v), message
    rc, err, _ = _step(fn, p, g, m, v, n, 3, 1.0)  # and the next finite call applies
    assert rc == 0, str(err)

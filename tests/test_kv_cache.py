"""A2 KV cache, the parts that need no GPU: the ABI version handshake and the
argument checks that reject a call before any device work, compared call for
call with the reference's own CPU cache (native/a2_kv_cache.c:376-447,
compiled into oracle/_ref)."""
import ctypes as C

import pytest

from eshkol_transformer_b200.kv_cache import KvCacheApi
from oracle import oracle as orc

# K1 categories / codes (kernel_abi.h:50-68)
INVALID_ARGUMENT, SHAPE_MISMATCH, VERSION_MISMATCH = 1, 2, 7
NULL_ARGUMENT, ABI_MAJOR_MISMATCH, UNKNOWN_REQUIRED_FEATURE = 1, 7, 8
INVALID_SHAPE, INVALID_BUFFER = 12, 13


@pytest.fixture(scope="module")
def apis(lib):
    ref = orc.ref()
    if ref is None:
        pytest.skip("the reference library (oracle/_ref) is not built")
    return KvCacheApi(lib), KvCacheApi(ref)


def outcome(rc, err):
    return rc, err.category, err.code


def test_abi_version_and_require_match_reference(apis):
    ours, ref = apis
    assert ours.abi() == ref.abi() == (1, 0)
    for major, minor in ((1, 0), (2, 0), (0, 0), (1, 1)):
        a, b = ours.require(major, minor), ref.require(major, minor)
        assert outcome(*a) == outcome(*b), (major, minor)
    assert outcome(*ours.require(2, 0)) == (VERSION_MISMATCH, VERSION_MISMATCH, ABI_MAJOR_MISMATCH)
    assert outcome(*ours.require(1, 1))[2] == UNKNOWN_REQUIRED_FEATURE


@pytest.mark.parametrize("dims", [(0, 1, 1, 1, 1), (1, 0, 1, 1, 1), (1, 1, 0, 1, 1),
                                  (1, 1, 1, 0, 1), (1, 1, 1, 1, 0)])
def test_create_rejects_zero_dimensions_like_reference(apis, dims):
    ours, ref = apis
    a, b = ours.create(*dims), ref.create(*dims)
    assert outcome(a[0], a[1]) == outcome(b[0], b[1]) == (SHAPE_MISMATCH, SHAPE_MISMATCH,
                                                        INVALID_SHAPE)
    assert a[2].value is None


def test_create_rejects_null_and_occupied_slots_like_reference(apis, lib):
    ours, ref = apis
    for api in (ours, ref):
        err = type(ours.require(1, 0)[1])()
        rc = api.lib.et_a2_kv_cache_create_v1(1, 1, 1, 1, 1, None, C.byref(err))
        assert (rc, err.category, err.code) == (INVALID_ARGUMENT, INVALID_ARGUMENT, NULL_ARGUMENT)
        slot = C.c_void_p(0x1000)
        rc = api.lib.et_a2_kv_cache_create_v1(1, 1, 1, 1, 1, C.byref(slot), C.byref(err))
        assert (rc, err.category, err.code) == (INVALID_ARGUMENT, INVALID_ARGUMENT, INVALID_BUFFER)
        assert slot.value == 0x1000


def test_handles_from_nowhere_are_rejected_like_reference(apis):
    ours, ref = apis
    bogus = C.c_void_p(0x1234)
    for api in (ours, ref):
        rc, err = api.destroy(bogus)
        assert (rc, err.category, err.code) == (INVALID_ARGUMENT, INVALID_ARGUMENT, INVALID_BUFFER)
        rc, err, _ = api.begin(bogus, 1, [1])
        assert (rc, err.category, err.code) == (INVALID_ARGUMENT, INVALID_ARGUMENT, INVALID_BUFFER)

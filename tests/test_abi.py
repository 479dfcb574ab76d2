"""The C-ABI surface, checked without a GPU: the library loads, exports every
entry point include/ declares, keeps the K1 v1 struct layouts, and its host-
side pieces (seeded inputs, schedule rounding, provider descriptors) agree
with the oracle."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import eshkol_transformer_b200 as etb
from eshkol_transformer_b200 import k1
from helpers import bits_equal
from oracle import oracle as orc

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for header in (ROOT / "include").rglob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        for m in re.finditer(r"\b(et_[a-z0-9_]+)\s*\(", text):
            if not m.group(1).endswith("_t"):
                names.add(m.group(1))
    return sorted(names)


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_k1_layouts_match_reference_sizes():
    for name, size in k1.LAYOUT_SIZES.items():
        assert C.sizeof(getattr(k1, name)) == size, name
    assert k1.TensorView.shape.offset == 64
    assert k1.Call.outputs.offset == 80
    assert k1.Provider.invoke_call.offset == 88
    assert k1.Capability.shape_ranges.offset == 112


def test_header_compiles_standalone_c_and_cpp(tmp_path):
    import subprocess
    src = tmp_path / "t.c"
    src.write_text('#include "eshkol_b200/et_b200.h"\nint main(void){return 0;}\n')
    for compiler, name in (("gcc", "t.c"), ("g++", "t.cpp")):
        f = tmp_path / name
        f.write_text(src.read_text())
        subprocess.run([compiler, "-std=c11" if compiler == "gcc" else "-std=c++17", "-Wall",
                        "-Werror", f"-I{ROOT / 'include'}", "-fsyntax-only", str(f)], check=True)


@pytest.mark.parametrize("seed,stream,count", [(1, 0, 1000), (20261201, 7, 4096), (99, 12345, 33)])
def test_synthetic_inputs_identical_to_oracle(seed, stream, count):
    assert bits_equal(etb.fill_normal(seed, stream, count, 0.0, 0.02),
                      orc.fill_normal(seed, stream, count, 0.0, 0.02))
    assert np.array_equal(etb.fill_tokens(seed, stream, count, 32768),
                          orc.fill_tokens(seed, stream, count, 32768))
    assert np.array_equal(etb.fill_tokens(seed, stream, count, 1000),
                          orc.fill_tokens(seed, stream, count, 1000))


def test_schedule_factor_identical_to_oracle(lib):
    for warm, total, minimum in ((2, 6, 0.1), (0, 4, 0.25), (10, 1000, 0.0), (3, 7, 1e-40),
                                 (1, 3, 0.3333)):
        mb = orc.bits(minimum)
        for u in range(1, total + 3):
            assert lib.et_b200_o2_schedule_factor_v1(1, warm, total, mb, u) == \
                orc.schedule_factor(1, warm, total, mb, u), (warm, total, minimum, u)
    assert lib.et_b200_o2_schedule_factor_v1(0, 0, 0, 0, 5) == 0x3F800000


@pytest.mark.parametrize("accessor,caps", [
    ("et_a2_kernel_provider_v1", {"kernel.causal-attention", "kernel.rope"}),
    ("et_n2_kernel_provider_v1", {"kernel.matmul", "kernel.norm", "kernel.activation",
                                  "kernel.residual", "kernel.embedding-forward",
                                  "kernel.embedding-backward"}),
    ("et_n3k_kernel_provider_v1", {"n3k.linear"}),
    ("et_l2_indexed_cross_entropy_provider_v1", {"kernel.indexed-cross-entropy"}),
])
def test_provider_descriptors(lib, accessor, caps):
    p = k1.provider(lib, accessor)
    assert p.struct_size == 96 and p.abi_major == 1
    got = k1.capabilities(p)
    assert set(got) == caps
    for cap in got.values():
        assert cap["status"] == k1.CAPABILITY_VERIFIED and cap["deterministic"]
        assert set(cap["devices"]) == {"cpu", "cuda"} and cap["dtypes"] == ["f32"]
        assert cap["operations"] == sorted(cap["operations"])


def test_reference_k1_runtime_discovers_b200_providers(lib):
    """The reference's own K1 runtime (native/kernel_abi.c, compiled by
    oracle/Makefile.ref) accepts each provider descriptor unchanged."""
    ref = orc.ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    RESOLVER = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_char_p)
    for accessor in ("et_a2_kernel_provider_v1", "et_n2_kernel_provider_v1",
                     "et_n3k_kernel_provider_v1", "et_l2_indexed_cross_entropy_provider_v1"):
        fn = getattr(lib, accessor)
        fn.restype = C.c_void_p
        target = fn()
        resolver = RESOLVER(lambda ctx, sym, t=target: t)
        runtime = C.c_void_p()
        err = k1.KernelError()
        ref.et_kernel_runtime_discover.argtypes = [RESOLVER, C.c_void_p, C.POINTER(C.c_void_p),
                                                   C.POINTER(k1.KernelError)]
        rc = ref.et_kernel_runtime_discover(resolver, None, C.byref(runtime), C.byref(err))
        assert rc == 0, str(err)
        ref.et_kernel_runtime_destroy.argtypes = [C.c_void_p]
        ref.et_kernel_runtime_destroy(runtime)


def test_k1_precision_setter(lib):
    assert lib.et_b200_k1_precision_v1(etb.PRECISION_F32) == 0
    assert lib.et_b200_k1_precision_v1(etb.PRECISION_F16X3) == 0
    assert lib.et_b200_k1_precision_v1(4) != 0
    assert lib.et_b200_k1_precision_v1(9) != 0
    assert lib.et_b200_k1_precision_v1(etb.PRECISION_TF32X3) == 0


@pytest.mark.parametrize("precision,rejected", [(4, True), (99, True), (etb.PRECISION_F16X3, False)])
def test_lm_create_validates_contraction_mode_before_the_device(lib, precision, rejected):
    """The model's configuration is checked on the host before any device
    work: an unknown contraction mode is a shape/config error, while the
    split-f16 mode passes validation (and here, without a GPU, then fails on
    the device check instead)."""
    s = etb.TINY
    cfg = etb.LMConfig(C.sizeof(etb.LMConfig), s.layers, s.d_model, s.heads, s.ffn, s.vocabulary,
                       s.seq_len, s.batch, 0, etb.f32_bits(1e-5), precision, 10000.0,
                       etb.f32_bits(1e-3), etb.f32_bits(0.9), etb.f32_bits(0.999),
                       etb.f32_bits(1e-8), etb.f32_bits(0.01), 0)
    handle = C.c_void_p()
    err = k1.KernelError()
    rc = lib.et_b200_lm_create_v1(C.byref(cfg), C.byref(handle), C.byref(err))
    shape_error = rc == k1.ERROR_SHAPE_MISMATCH and err.code == 12  # INVALID_SHAPE (kernel_abi.h)
    if rejected:
        assert shape_error, (rc, err.category, err.code)
        assert handle.value is None
    else:
        assert not shape_error
        if rc == 0:  # a GPU is present after all
            lib.et_b200_lm_destroy_v1(C.byref(handle))


def test_f16_redone_steps_of_no_model_is_zero(lib):
    assert lib.et_b200_lm_f16_redone_steps_v1(None) == 0


def test_k2_resolver_and_audit_with_reference_runtime(lib):
    """The fixed resolver and the exact audit K2 needs for the B200 provider
    (native/k2_capabilities.c:493-561), through the reference's own K1
    runtime: discovery admits the composite provider and every B200
    capability is verified; the resolver answers only the K1 symbol with its
    private context; the audit tells the genuine descriptor from a copy whose
    callbacks or metadata differ."""
    ref = orc.ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    lib.et_b200_kernel_provider_v1.restype = C.c_void_p
    lib.et_b200_k2_resolver_context_v1.restype = C.c_void_p
    lib.et_b200_k2_resolver_v1.restype = C.c_void_p
    lib.et_b200_k2_resolver_v1.argtypes = [C.c_void_p, C.c_char_p]
    lib.et_b200_k2_audit_provider_v1.argtypes = [C.c_void_p]
    genuine = lib.et_b200_kernel_provider_v1()
    ctx = lib.et_b200_k2_resolver_context_v1()
    symbol = b"eshkol_transformer_kernel_provider_v1"
    assert lib.et_b200_k2_resolver_v1(ctx, symbol) == genuine
    assert lib.et_b200_k2_resolver_v1(None, symbol) is None
    assert lib.et_b200_k2_resolver_v1(ctx, b"another_symbol") is None
    # discovery through the reference's K1 runtime with the fixed resolver
    RESOLVER = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_char_p)
    resolver = RESOLVER(lambda c, s: lib.et_b200_k2_resolver_v1(c, s))
    runtime = C.c_void_p()
    err = k1.KernelError()
    ref.et_kernel_runtime_discover.argtypes = [RESOLVER, C.c_void_p, C.POINTER(C.c_void_p),
                                               C.POINTER(k1.KernelError)]
    assert ref.et_kernel_runtime_discover(resolver, ctx, C.byref(runtime), C.byref(err)) == 0, \
        str(err)
    ref.et_kernel_runtime_capability_find.restype = C.POINTER(k1.Capability)
    ref.et_kernel_runtime_capability_find.argtypes = [C.c_void_p, C.c_char_p]
    for name in ("kernel.causal-attention", "kernel.matmul", "kernel.indexed-cross-entropy",
                 "kernel.norm", "kernel.rope", "n3k.linear"):
        cap = ref.et_kernel_runtime_capability_find(runtime, name.encode())
        assert cap and cap.contents.status == k1.CAPABILITY_VERIFIED, name
        assert set(cap.contents.devices[i] for i in range(cap.contents.device_count)) == \
            {b"cpu", b"cuda"}
    ref.et_kernel_runtime_destroy.argtypes = [C.c_void_p]
    ref.et_kernel_runtime_destroy(runtime)
    # the audit: genuine, absent, a copy with a foreign callback, another version
    assert lib.et_b200_k2_audit_provider_v1(genuine) == 3
    assert lib.et_b200_k2_audit_provider_v1(None) == 0
    copy = k1.Provider.from_buffer_copy(k1.Provider.from_address(genuine))
    other = k1.provider(lib, "et_a2_kernel_provider_v1")
    copy.invoke_call = other.invoke_call
    assert lib.et_b200_k2_audit_provider_v1(C.addressof(copy)) == 2
    copy = k1.Provider.from_buffer_copy(k1.Provider.from_address(genuine))
    copy.capability_count = 9
    assert lib.et_b200_k2_audit_provider_v1(C.addressof(copy)) == 2
    copy = k1.Provider.from_buffer_copy(k1.Provider.from_address(genuine))
    copy.abi_minor = 7
    assert lib.et_b200_k2_audit_provider_v1(C.addressof(copy)) == 1

"""ctypes bindings of the O2 Eshkol bridge surface (include/eshkol_b200/o2_bridge.h)
with the extern signatures of native/o2_wave2_extension.esk:4-29 (i64 / ptr)."""
import ctypes as C

from eshkol_transformer_b200 import k1

I64, PTR = C.c_int64, C.c_void_p

SIGNATURES = {
    "et_o2_private_last_error_category_v1": (I64, []),
    "et_o2_private_builder_create_v1": (PTR, [I64] * 7),
    "et_o2_private_builder_set_v1": (I64, [PTR, I64, PTR, PTR] + [I64] * 5),
    "et_o2_private_builder_finish_v1": (PTR, [PTR]),
    "et_o2_private_builder_abort_v1": (I64, [PTR]),
    "et_o2_private_optimizer_step_v1": (I64, [PTR]),
    "et_o2_private_optimizer_zero_grad_v1": (I64, [PTR]),
    "et_o2_private_optimizer_require_absent_gradients_v1": (I64, [PTR]),
    "et_o2_private_optimizer_completed_updates_v1": (I64, [PTR]),
    "et_o2_private_optimizer_schedule_factor_bits_v1": (I64, [PTR]),
    "et_o2_private_optimizer_state_snapshot_v1": (PTR, [PTR]),
    "et_o2_private_optimizer_load_state_v1": (I64, [PTR, PTR]),
    "et_o2_private_optimizer_state_release_v1": (I64, [PTR]),
    "et_b200_o2_bridge_last_error_message_v1": (C.c_char_p, []),
    "et_b200_o2_bridge_destroy_v1": (None, [C.POINTER(PTR)]),
    "et_b200_o2_state_write_v1": (I64, [PTR, C.c_char_p]),
    "et_b200_o2_state_read_v1": (PTR, [C.c_char_p]),
    "et_b200_parameter_create_v1": (C.c_int32, [PTR, PTR, C.c_size_t, C.POINTER(PTR),
                                                C.POINTER(k1.KernelError)]),
    "et_b200_parameter_set_gradient_v1": (C.c_int32, [PTR, C.c_uint64, C.c_uint32,
                                                      C.POINTER(k1.KernelError)]),
    "et_b200_parameter_gradient_present_v1": (C.c_int32, [PTR]),
    "et_b200_parameter_destroy_v1": (None, [C.POINTER(PTR)]),
}


def bind(lib):
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib

"""ctypes mirror of the K1 kernel ABI v1 (include/eshkol_transformer/kernel_abi.h).

Struct layouts match the reference byte for byte (checked against the sizes
frozen at kernel_abi.h:176-234).  `KernelCall` builds a call descriptor from
numpy arrays (device "cpu") or CUDA torch tensors (device "cuda"), and
`dispatch` runs a provider's two phases the way K1's et_kernel_runtime_dispatch
does (native/kernel_abi.c:1287-1324): validate_call, then invoke_call only on
success.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

ABI_MAJOR = 1
ABI_MINOR = 0

# error categories (kernel_abi.h:37-48)
ERROR_NONE = 0
ERROR_INVALID_ARGUMENT = 1
ERROR_SHAPE_MISMATCH = 2
ERROR_DTYPE_MISMATCH = 3
ERROR_DEVICE_MISMATCH = 4
ERROR_NONCONTIGUOUS = 5
ERROR_UNSUPPORTED = 6
ERROR_VERSION_MISMATCH = 7
ERROR_INTERNAL = 8

# error codes (kernel_abi.h:50-68)
CODE_ALIASING_OUTPUT = 14
CODE_PROVIDER_REJECTED = 16

LAYOUT_DENSE_ROW_MAJOR = 1
CAPABILITY_VERIFIED = 1


class KernelError(C.Structure):
    _fields_ = [("category", C.c_uint32), ("code", C.c_uint32),
                ("operation", C.c_char * 64), ("message", C.c_char * 192)]

    def __str__(self) -> str:
        return (f"[{self.category}/{self.code}] {self.operation.decode(errors='replace')}: "
                f"{self.message.decode(errors='replace')}")


class DimensionRange(C.Structure):
    _fields_ = [("minimum", C.c_uint64), ("maximum", C.c_uint64),
                ("maximum_unbounded", C.c_uint8), ("reserved", C.c_uint8 * 7)]


class ShapeRange(C.Structure):
    _fields_ = [("rank", C.c_size_t), ("dimensions", C.POINTER(DimensionRange))]


class Capability(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("name", C.c_char_p), ("status", C.c_uint32),
                ("implementation", C.c_char_p), ("version", C.c_char_p),
                ("evidence", C.c_char_p), ("deterministic", C.c_uint8),
                ("reserved", C.c_uint8 * 7), ("operation_count", C.c_size_t),
                ("operations", C.POINTER(C.c_char_p)), ("dtype_count", C.c_size_t),
                ("dtypes", C.POINTER(C.c_char_p)), ("device_count", C.c_size_t),
                ("devices", C.POINTER(C.c_char_p)), ("shape_range_count", C.c_size_t),
                ("shape_ranges", C.POINTER(ShapeRange))]


class TensorView(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("data", C.c_void_p), ("byte_length", C.c_size_t),
                ("dtype", C.c_char_p), ("device", C.c_char_p), ("layout", C.c_uint32),
                ("offset_bytes", C.c_uint64), ("rank", C.c_size_t),
                ("shape", C.POINTER(C.c_uint64))]


class Request(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("operation", C.c_char_p), ("dtype", C.c_char_p),
                ("device", C.c_char_p), ("rank", C.c_size_t), ("shape", C.POINTER(C.c_uint64)),
                ("deterministic", C.c_uint8), ("reserved", C.c_uint8 * 7)]


class Call(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("capability", C.c_char_p),
                ("request", C.POINTER(Request)), ("input_count", C.c_size_t),
                ("input_stride", C.c_size_t), ("input_bytes", C.c_size_t),
                ("inputs", C.c_void_p), ("output_count", C.c_size_t),
                ("output_stride", C.c_size_t), ("output_bytes", C.c_size_t),
                ("outputs", C.c_void_p)]


VALIDATE = C.CFUNCTYPE(C.c_int32, C.POINTER(Call), C.POINTER(KernelError))
INVOKE = C.CFUNCTYPE(None, C.POINTER(Call))


class Provider(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("abi_major", C.c_uint32), ("abi_minor", C.c_uint32),
                ("required_features", C.c_uint64), ("name", C.c_char_p), ("version", C.c_char_p),
                ("evidence", C.c_char_p), ("capability_count", C.c_size_t),
                ("capability_stride", C.c_size_t), ("capability_bytes", C.c_size_t),
                ("capabilities", C.POINTER(Capability)), ("validate_call", VALIDATE),
                ("invoke_call", INVOKE)]


LAYOUT_SIZES = {"KernelError": 264, "TensorView": 72, "Request": 56, "Call": 88,
                "Provider": 96, "Capability": 120, "DimensionRange": 24, "ShapeRange": 16}

_DTYPE = {np.dtype(np.float32): "f32", np.dtype(np.int64): "i64", np.dtype(np.uint8): "bool",
          np.dtype(np.bool_): "bool"}
_TORCH_DTYPE = {"torch.float32": "f32", "torch.int64": "i64", "torch.uint8": "bool",
                "torch.bool": "bool"}


def _describe(t):
    """(pointer, byte_length, dtype, shape, device) of a numpy array or torch tensor."""
    if isinstance(t, np.ndarray):
        if not t.flags["C_CONTIGUOUS"]:
            raise ValueError("K1 views must be dense row-major")
        return t.ctypes.data, t.nbytes, _DTYPE[t.dtype], t.shape, "cpu"
    # torch tensor
    if not t.is_contiguous():
        raise ValueError("K1 views must be dense row-major")
    dev = "cuda" if t.is_cuda else "cpu"
    return t.data_ptr(), t.numel() * t.element_size(), _TORCH_DTYPE[str(t.dtype)], tuple(t.shape), dev


@dataclass
class KernelCall:
    """Owns every ctypes object a K1 call points to."""
    capability: str
    operation: str
    shape: tuple
    inputs: list
    outputs: list
    device: str | None = None
    dtype: str = "f32"

    def __post_init__(self):
        self._keep = []
        descs = [_describe(t) for t in self.inputs + self.outputs]
        device = self.device or (descs[0][4] if descs else "cpu")
        self._device = device.encode()
        self._req_shape = (C.c_uint64 * max(1, len(self.shape)))(*self.shape)
        self.request = Request(C.sizeof(Request), self.operation.encode(), self.dtype.encode(),
                               self._device, len(self.shape),
                               C.cast(self._req_shape, C.POINTER(C.c_uint64)), 1)
        n_in = len(self.inputs)
        self._in = (TensorView * max(1, n_in))()
        self._out = (TensorView * max(1, len(self.outputs)))()
        for i, (ptr, nbytes, dt, shape, dev) in enumerate(descs):
            arr = (C.c_uint64 * max(1, len(shape)))(*shape)
            self._keep.append(arr)
            # a scalar (rank 0) view carries no shape array
            view = TensorView(C.sizeof(TensorView), ptr, nbytes, dt.encode(), dev.encode(),
                              LAYOUT_DENSE_ROW_MAJOR, 0, len(shape),
                              C.cast(arr, C.POINTER(C.c_uint64)) if len(shape) else None)
            if i < n_in:
                self._in[i] = view
            else:
                self._out[i - n_in] = view
        vs = C.sizeof(TensorView)
        self.call = Call(C.sizeof(Call), self.capability.encode(), C.pointer(self.request),
                         n_in, vs, n_in * vs, C.cast(self._in, C.c_void_p) if n_in else None,
                         len(self.outputs), vs if self.outputs else 0, len(self.outputs) * vs,
                         C.cast(self._out, C.c_void_p) if self.outputs else None)


def provider(lib, accessor: str) -> Provider:
    fn = getattr(lib, accessor)
    fn.restype = C.POINTER(Provider)
    fn.argtypes = []
    return fn().contents


def capabilities(p: Provider) -> dict:
    out = {}
    for i in range(p.capability_count):
        cap = p.capabilities[i]
        out[cap.name.decode()] = {
            "operations": [cap.operations[j].decode() for j in range(cap.operation_count)],
            "devices": [cap.devices[j].decode() for j in range(cap.device_count)],
            "dtypes": [cap.dtypes[j].decode() for j in range(cap.dtype_count)],
            "deterministic": bool(cap.deterministic),
            "status": cap.status,
        }
    return out


def dispatch(p: Provider, kc: KernelCall) -> tuple[int, KernelError]:
    """validate_call then, on success, invoke_call (K1 dispatch order)."""
    err = KernelError()
    rc = p.validate_call(C.pointer(kc.call), C.pointer(err))
    if rc != 0:
        return rc, err
    p.invoke_call(C.pointer(kc.call))
    return 0, err

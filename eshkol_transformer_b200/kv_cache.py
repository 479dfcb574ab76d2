"""ctypes mirror of the A2 KV-cache C ABI (include/eshkol_transformer/
a2_kv_cache.h:42-147 in the reference; include/eshkol_b200/et_b200.h here).

The same functions with the same arguments exist in the reference's CPU
library and in libet_b200 (device storage), so one wrapper drives either.
Every method returns (rc, KernelError[, handle]) like the C calls; tensor
arguments are numpy arrays ("cpu" views) or CUDA torch tensors ("cuda"
views).  `read_view` copies a returned view (host or device) into numpy.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .k1 import LAYOUT_DENSE_ROW_MAJOR, KernelError, TensorView

_P = C.c_void_p
_PP = C.POINTER(C.c_void_p)
_ERR = C.POINTER(KernelError)
_TV = C.POINTER(TensorView)
_TVP = C.POINTER(_TV)

_SIGNATURES = {
    "et_a2_kv_cache_abi_major_v1": ([], C.c_int32),
    "et_a2_kv_cache_abi_minor_v1": ([], C.c_int32),
    "et_a2_kv_cache_abi_require_v1": ([C.c_uint32, C.c_uint32, _ERR], C.c_int32),
    "et_a2_kv_cache_create_v1": ([C.c_uint64] * 5 + [_PP, _ERR], C.c_int32),
    "et_a2_kv_cache_destroy_v1": ([_PP, _ERR], C.c_int32),
    "et_a2_kv_cache_transaction_begin_v1": ([_P, C.c_uint64, _TV, _PP, _ERR], C.c_int32),
    "et_a2_kv_cache_transaction_stage_layer_v1": ([_P, C.c_uint64, _TV, _TV, _ERR], C.c_int32),
    "et_a2_kv_cache_transaction_view_begin_v1": ([_P, C.c_uint64, _PP, _ERR], C.c_int32),
    "et_a2_kv_cache_transaction_view_tensors_v1": ([_P, _TVP, _TVP, _TVP, _TVP, _ERR], C.c_int32),
    "et_a2_kv_cache_transaction_view_end_v1": ([_PP, _ERR], C.c_int32),
    "et_a2_kv_cache_transaction_commit_v1": ([_PP, _ERR], C.c_int32),
    "et_a2_kv_cache_transaction_abort_v1": ([_PP, _ERR], C.c_int32),
    "et_a2_kv_cache_read_borrow_begin_v1": ([_P, _PP, _ERR], C.c_int32),
    "et_a2_kv_cache_read_borrow_layer_v1": ([_P, C.c_uint64, _TVP, _TVP, _TVP, _TVP, _ERR],
                                            C.c_int32),
    "et_a2_kv_cache_read_borrow_end_v1": ([_PP, _ERR], C.c_int32),
}

_NP_DTYPE = {"f32": np.float32, "i64": np.int64, "bool": np.uint8}


class _CudaArray:
    """__cuda_array_interface__ over a device pointer (zero copy into torch)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 2}


class View:
    """Owns the ctypes objects one tensor view points to."""

    def __init__(self, array, dtype: str | None = None):
        if hasattr(array, "is_cuda"):  # torch tensor
            if not array.is_contiguous():
                raise ValueError("views must be dense")
            ptr, nbytes = array.data_ptr(), array.numel() * array.element_size()
            dt = dtype or {"torch.float32": "f32", "torch.int64": "i64",
                           "torch.uint8": "bool"}[str(array.dtype)]
            dev = "cuda" if array.is_cuda else "cpu"
            shape = tuple(array.shape)
        else:
            array = np.ascontiguousarray(array)
            ptr, nbytes = array.ctypes.data, array.nbytes
            dt = dtype or {np.dtype(np.float32): "f32", np.dtype(np.int64): "i64",
                           np.dtype(np.uint8): "bool"}[array.dtype]
            dev = "cpu"
            shape = array.shape
        self._array = array
        self._shape = (C.c_uint64 * max(1, len(shape)))(*shape)
        self._dtype = dt.encode()
        self._device = dev.encode()
        self.view = TensorView(C.sizeof(TensorView), ptr, nbytes, self._dtype, self._device,
                               LAYOUT_DENSE_ROW_MAJOR, 0, len(shape),
                               C.cast(self._shape, C.POINTER(C.c_uint64)))

    def ref(self):
        return C.byref(self.view)


def read_view(view: TensorView) -> np.ndarray:
    """Copies the tensor a returned view describes (host or device) to numpy."""
    shape = tuple(view.shape[i] for i in range(view.rank))
    dt = _NP_DTYPE[view.dtype.decode()]
    if view.device.decode() == "cuda":
        import torch
        typestr = np.dtype(dt).str
        t = torch.as_tensor(_CudaArray(view.data, shape, typestr), device="cuda")
        return t.cpu().numpy().copy()
    count = int(np.prod(shape)) if shape else 1
    buf = (C.c_char * (count * np.dtype(dt).itemsize)).from_address(view.data)
    return np.frombuffer(bytes(buf), dtype=dt).reshape(shape)


class KvCacheApi:
    """The KV-cache entry points of one library (ours or the reference's)."""

    def __init__(self, lib):
        self.lib = lib
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res

    def _call(self, name, *args):
        err = KernelError()
        rc = getattr(self.lib, name)(*args, C.byref(err))
        return rc, err

    def abi(self):
        return (self.lib.et_a2_kv_cache_abi_major_v1(), self.lib.et_a2_kv_cache_abi_minor_v1())

    def require(self, major, minor):
        return self._call("et_a2_kv_cache_abi_require_v1", major, minor)

    def create(self, layers, batch, heads, capacity, dim):
        slot = C.c_void_p(None)
        rc, err = self._call("et_a2_kv_cache_create_v1", layers, batch, heads, capacity, dim,
                             C.byref(slot))
        return rc, err, slot

    def destroy(self, slot):
        return self._call("et_a2_kv_cache_destroy_v1", C.byref(slot))

    def begin(self, cache, width, counts):
        slot = C.c_void_p(None)
        cv = View(np.asarray(counts, np.int64))
        rc, err = self._call("et_a2_kv_cache_transaction_begin_v1", cache, width, cv.ref(),
                             C.byref(slot))
        return rc, err, slot

    def stage(self, txn, layer, keys, values):
        kv, vv = View(keys), View(values)
        return self._call("et_a2_kv_cache_transaction_stage_layer_v1", txn, layer, kv.ref(),
                          vv.ref())

    def view_begin(self, txn, layer):
        slot = C.c_void_p(None)
        rc, err = self._call("et_a2_kv_cache_transaction_view_begin_v1", txn, layer,
                             C.byref(slot))
        return rc, err, slot

    def view_tensors(self, view):
        outs = [_TV() for _ in range(4)]
        rc, err = self._call("et_a2_kv_cache_transaction_view_tensors_v1", view,
                             *[C.byref(o) for o in outs])
        return rc, err, [o.contents if o else None for o in outs]

    def view_end(self, view):
        return self._call("et_a2_kv_cache_transaction_view_end_v1", C.byref(view))

    def commit(self, txn):
        return self._call("et_a2_kv_cache_transaction_commit_v1", C.byref(txn))

    def abort(self, txn):
        return self._call("et_a2_kv_cache_transaction_abort_v1", C.byref(txn))

    def borrow_begin(self, cache):
        slot = C.c_void_p(None)
        rc, err = self._call("et_a2_kv_cache_read_borrow_begin_v1", cache, C.byref(slot))
        return rc, err, slot

    def borrow_layer(self, borrow, layer):
        outs = [_TV() for _ in range(4)]
        rc, err = self._call("et_a2_kv_cache_read_borrow_layer_v1", borrow, layer,
                             *[C.byref(o) for o in outs])
        return rc, err, [o.contents if o else None for o in outs]

    def borrow_end(self, borrow):
        return self._call("et_a2_kv_cache_read_borrow_end_v1", C.byref(borrow))

    def snapshot(self, cache, layers):
        """Committed (keys, values) per layer, lengths and mask via a read borrow."""
        rc, err, b = self.borrow_begin(cache)
        if rc != 0:
            raise RuntimeError(str(err))
        ks, vs, lengths, mask = [], [], None, None
        for layer in range(layers):
            rc, err, (k, v, ln, m) = self.borrow_layer(b, layer)
            if rc != 0:
                raise RuntimeError(str(err))
            ks.append(read_view(k))
            vs.append(read_view(v))
            lengths, mask = read_view(ln), read_view(m)
        rc, err = self.borrow_end(b)
        if rc != 0:
            raise RuntimeError(str(err))
        return np.stack(ks), np.stack(vs), lengths, mask

"""B200 (sm_100a) implementation of eshkol-transformer's f32 training-step hot path.

The product is the C-ABI library ``lib/libet_b200.so`` (declared in
``include/eshkol_b200/et_b200.h``).  This package loads it and offers thin
Python handles over its entry points:

* ``k1`` -- the K1 kernel ABI structs and provider dispatch;
* ``LanguageModel`` -- the native training step (et_b200_lm_*);
* ``Optimizer`` -- the O2-shaped device AdamW (et_b200_o2_*).

There is no fallback: loading fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import k1

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libet_b200.so"

PRECISION_TF32X3 = 0
PRECISION_TF32 = 1
PRECISION_F32 = 2
PRECISION_F16X3 = 3  # split-f16 operand pairs (f32-grade, 2x the TF32 tensor rate)

_lib = None


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def load() -> C.CDLL:
    """Loads libet_b200.so (built by __graft_entry__.build())."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() first")
    lib = C.CDLL(str(LIB_PATH), mode=C.RTLD_GLOBAL)
    E = C.POINTER(k1.KernelError)
    sig = {
        "et_b200_abi_major_v1": (C.c_int32, []),
        "et_b200_abi_minor_v1": (C.c_int32, []),
        "et_b200_launch_count_v1": (C.c_uint64, []),
        "et_b200_device_check_v1": (C.c_int32, [E]),
        "et_b200_k1_precision_v1": (C.c_int32, [C.c_uint32]),
        "et_b200_fill_normal_v1": (None, [C.c_uint64, C.c_uint64, C.c_size_t, C.c_double,
                                          C.c_double, C.c_void_p]),
        "et_b200_fill_tokens_v1": (None, [C.c_uint64, C.c_uint64, C.c_size_t, C.c_uint64,
                                          C.c_void_p]),
        "et_b200_lm_create_v1": (C.c_int32, [C.c_void_p, C.POINTER(C.c_void_p), E]),
        "et_b200_lm_destroy_v1": (None, [C.POINTER(C.c_void_p)]),
        "et_b200_lm_tensor_count_v1": (C.c_size_t, [C.c_void_p]),
        "et_b200_lm_parameter_count_v1": (C.c_size_t, [C.c_void_p]),
        "et_b200_lm_tensor_sizes_v1": (C.c_int32, [C.c_void_p, C.c_void_p]),
        "et_b200_lm_init_v1": (C.c_int32, [C.c_void_p, C.c_uint64, E]),
        "et_b200_lm_read_v1": (C.c_int32, [C.c_void_p, C.c_int32, C.c_void_p, C.c_size_t, E]),
        "et_b200_lm_write_v1": (C.c_int32, [C.c_void_p, C.c_int32, C.c_void_p, C.c_size_t, E]),
        "et_b200_lm_step_v1": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, E]),
        "et_b200_lm_step_device_v1": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p,
                                                  C.c_void_p, E]),
        "et_b200_lm_forward_backward_v1": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p,
                                                       C.c_void_p, E]),
        "et_b200_lm_stream_v1": (C.c_void_p, [C.c_void_p]),
        "et_b200_lm_set_loss_mask_v1": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_int32, E]),
        "et_b200_d2_row_count_v1": (C.c_int64, [C.c_uint64, C.c_int64]),
        "et_b200_d2_rows_v1": (C.c_int32, [C.c_void_p, C.c_uint64, C.c_int64, C.c_int64,
                                           C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p, E]),
        "et_b200_nccl_unique_id_v1": (C.c_int32, [C.c_void_p, E]),
        "et_b200_lm_enable_data_parallel_v1": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_int32,
                                                           C.c_int32, E]),
        "et_b200_lm_profile_v1": (C.c_int32, [C.c_void_p, C.c_int32]),
        "et_b200_lm_profile_collect_v1": (C.c_int32, [C.c_void_p]),
        "et_b200_lm_profile_read_v1": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_size_t]),
        "et_b200_lm_f16_redone_steps_v1": (C.c_int32, [C.c_void_p]),
        "et_b200_lm_update_counts_v1": (C.c_int32, [C.c_void_p, C.POINTER(C.c_uint64),
                                                    C.POINTER(C.c_uint64), E]),
        "et_b200_attention_workspace_bytes_v1": (C.c_size_t, [C.c_void_p]),
        "et_b200_rope_tables_v1": (None, [C.c_int64, C.c_int64, C.c_double, C.c_void_p,
                                          C.c_void_p]),
        "et_b200_attention_forward_v1": (C.c_int32, [C.c_void_p] + [C.c_void_p] * 6 +
                                         [C.c_void_p, C.c_size_t, C.c_void_p, E]),
        "et_b200_attention_backward_v1": (C.c_int32, [C.c_void_p] + [C.c_void_p] * 10 +
                                          [C.c_void_p, C.c_size_t, C.c_int32, C.c_void_p, E]),
        "et_b200_o2_optimizer_create_v1": (C.c_int32, [C.c_size_t, C.c_void_p, C.c_uint32,
                                                       C.c_uint32, C.c_uint32, C.c_uint64,
                                                       C.c_uint64, C.c_uint32,
                                                       C.POINTER(C.c_void_p), E]),
        "et_b200_o2_optimizer_step_v1": (C.c_int32, [C.c_void_p, C.c_uint32,
                                                     C.POINTER(C.c_uint32), E]),
        "et_b200_o2_optimizer_completed_updates_v1": (C.c_int32, [C.c_void_p,
                                                                  C.POINTER(C.c_uint64)]),
        "et_b200_o2_optimizer_moments_v1": (C.c_int32, [C.c_void_p, C.c_size_t,
                                                        C.POINTER(C.c_void_p),
                                                        C.POINTER(C.c_void_p)]),
        "et_b200_o2_optimizer_destroy_v1": (None, [C.POINTER(C.c_void_p)]),
        "et_b200_o2_schedule_factor_v1": (C.c_uint32, [C.c_uint32, C.c_uint64, C.c_uint64,
                                                       C.c_uint32, C.c_uint64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class B200Error(RuntimeError):
    def __init__(self, rc: int, err: k1.KernelError):
        super().__init__(f"libet_b200 error {rc}: {err}")
        self.category = rc
        self.error = err


def _check(rc: int, err: k1.KernelError) -> None:
    if rc != 0:
        raise B200Error(rc, err)


class LMConfig(C.Structure):
    """et_b200_lm_config_v1"""
    _fields_ = [("struct_size", C.c_size_t), ("layers", C.c_int64), ("d_model", C.c_int64),
                ("heads", C.c_int64), ("ffn", C.c_int64), ("vocabulary", C.c_int64),
                ("seq_len", C.c_int64), ("batch", C.c_int64), ("global_tokens", C.c_int64),
                ("ln_epsilon_bits", C.c_uint32), ("precision", C.c_uint32),
                ("rope_base", C.c_double), ("learning_rate_bits", C.c_uint32),
                ("beta1_bits", C.c_uint32), ("beta2_bits", C.c_uint32),
                ("epsilon_bits", C.c_uint32), ("weight_decay_bits", C.c_uint32),
                ("reserved", C.c_uint32)]


@dataclass(frozen=True)
class ModelShape:
    layers: int
    d_model: int
    heads: int
    ffn: int
    vocabulary: int
    seq_len: int
    batch: int


# The BASELINE decoder configurations (tiny / small / medium LM).
TINY = ModelShape(2, 128, 4, 512, 1024, 64, 8)
SMALL = ModelShape(6, 512, 8, 2048, 8192, 512, 16)
MEDIUM = ModelShape(12, 1024, 16, 4096, 32768, 1024, 64)


class LanguageModel:
    """Handle over et_b200_lm: the fused decoder-LM training step on one GPU."""

    def __init__(self, shape: ModelShape, precision: int = PRECISION_TF32X3,
                 global_tokens: int = 0, lr: float = 1e-3, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, weight_decay: float = 0.01,
                 ln_eps: float = 1e-5, rope_base: float = 10000.0):
        self.lib = load()
        self.shape = shape
        cfg = LMConfig(C.sizeof(LMConfig), shape.layers, shape.d_model, shape.heads, shape.ffn,
                       shape.vocabulary, shape.seq_len, shape.batch, global_tokens,
                       f32_bits(ln_eps), precision, rope_base, f32_bits(lr), f32_bits(beta1),
                       f32_bits(beta2), f32_bits(eps), f32_bits(weight_decay), 0)
        self._cfg = cfg
        self.handle = C.c_void_p()
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_create_v1(C.byref(cfg), C.byref(self.handle), C.byref(err)), err)
        self.tensor_count = self.lib.et_b200_lm_tensor_count_v1(self.handle)
        self.parameter_count = self.lib.et_b200_lm_parameter_count_v1(self.handle)
        sizes = (C.c_size_t * self.tensor_count)()
        self.lib.et_b200_lm_tensor_sizes_v1(self.handle, sizes)
        self.tensor_sizes = list(sizes)

    def close(self) -> None:
        if self.handle:
            self.lib.et_b200_lm_destroy_v1(C.byref(self.handle))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init(self, seed: int) -> None:
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_init_v1(self.handle, seed, C.byref(err)), err)

    def read(self, which: int = 0) -> np.ndarray:
        out = np.empty(self.parameter_count, np.float32)
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_read_v1(self.handle, which, out.ctypes.data, out.size,
                                           C.byref(err)), err)
        return out

    def write(self, values: np.ndarray, which: int = 0) -> None:
        values = np.ascontiguousarray(values, np.float32)
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_write_v1(self.handle, which, values.ctypes.data, values.size,
                                            C.byref(err)), err)

    def step(self, ids: np.ndarray, targets: np.ndarray) -> float:
        ids = np.ascontiguousarray(ids, np.int64)
        targets = np.ascontiguousarray(targets, np.int64)
        loss = C.c_float()
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_step_v1(self.handle, ids.ctypes.data, targets.ctypes.data,
                                           C.byref(loss), C.byref(err)), err)
        return loss.value

    def forward_backward(self, ids: np.ndarray, targets: np.ndarray) -> float:
        ids = np.ascontiguousarray(ids, np.int64)
        targets = np.ascontiguousarray(targets, np.int64)
        loss = C.c_float()
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_forward_backward_v1(self.handle, ids.ctypes.data,
                                                       targets.ctypes.data, C.byref(loss),
                                                       C.byref(err)), err)
        return loss.value

    def step_device(self, ids_ptr: int, targets_ptr: int, loss_ptr: int | None = None) -> None:
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_step_device_v1(self.handle, ids_ptr, targets_ptr, loss_ptr,
                                                  C.byref(err)), err)

    def set_loss_mask(self, mask=None, device_ptr: int | None = None) -> None:
        """Loss mask [batch, seq_len] (0 / 1 bytes) of the following steps: a
        host array, or a device pointer; None and no pointer restores the
        unmasked objective."""
        err = k1.KernelError()
        if device_ptr is not None:
            _check(self.lib.et_b200_lm_set_loss_mask_v1(self.handle, device_ptr, 1, C.byref(err)),
                   err)
            return
        if mask is None:
            _check(self.lib.et_b200_lm_set_loss_mask_v1(self.handle, None, 0, C.byref(err)), err)
            return
        m = np.ascontiguousarray(mask, np.uint8)
        _check(self.lib.et_b200_lm_set_loss_mask_v1(self.handle, m.ctypes.data, 0, C.byref(err)),
               err)

    def stream(self) -> int:
        return self.lib.et_b200_lm_stream_v1(self.handle)

    def enable_data_parallel(self, unique_id: bytes, rank: int, world: int) -> None:
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_enable_data_parallel_v1(self.handle, buf, rank, world,
                                                           C.byref(err)), err)

    def update_counts(self) -> tuple[int, int]:
        """(applied AdamW updates, device-enqueued steps whose update was skipped)."""
        done, skipped = C.c_uint64(), C.c_uint64()
        err = k1.KernelError()
        _check(self.lib.et_b200_lm_update_counts_v1(self.handle, C.byref(done), C.byref(skipped),
                                                    C.byref(err)), err)
        return done.value, skipped.value

    def f16_redone_steps(self) -> int:
        """Split-f16 steps redone in 3xTF32 after an operand overflow."""
        return self.lib.et_b200_lm_f16_redone_steps_v1(self.handle)

    def profile(self, enable: bool) -> None:
        self.lib.et_b200_lm_profile_v1(self.handle, 1 if enable else 0)

    PROFILE_CLASSES = ("gemm", "attention_forward", "attention_backward", "cross_entropy",
                       "adamw", "layer_norm", "elementwise", "embedding", "tf32_split",
                       "allreduce_wait", "adamw_check")

    def profile_read(self) -> dict:
        self.lib.et_b200_lm_profile_collect_v1(self.handle)
        n = 4 * len(self.PROFILE_CLASSES)
        out = (C.c_double * n)()
        self.lib.et_b200_lm_profile_read_v1(self.handle, out, n)
        return {name: {"launches": out[4 * i], "ms": out[4 * i + 1], "flop": out[4 * i + 2],
                       "bytes": out[4 * i + 3]} for i, name in enumerate(self.PROFILE_CLASSES)}


class AttentionShape(C.Structure):
    """et_b200_attention_v1"""
    _fields_ = [("struct_size", C.c_size_t), ("batch", C.c_int64), ("q_heads", C.c_int64),
                ("kv_heads", C.c_int64), ("q_len", C.c_int64), ("k_len", C.c_int64),
                ("head_dim", C.c_int64), ("q_positions", C.c_void_p),
                ("k_positions", C.c_void_p), ("keep", C.c_void_p), ("rope_cos", C.c_void_p),
                ("rope_sin", C.c_void_p), ("rope_batched", C.c_int32),
                ("contraction", C.c_int32)]


ATTENTION_DEFAULT = 0      # binary16 pairs at head_dim 128 and at head_dim 64 from
                           # q_len k_len = 768^2 up; 3xTF32 pairs otherwise
ATTENTION_BWD_PAIRS16 = 1  # binary16 pairs in the backward at head_dim 64 as well
ATTENTION_TF32 = 2         # one product of TF32-grade operands (11 significant bits)


def rope_tables(length: int, head_dim: int, base: float = 10000.0):
    """Host RoPE tables [length, head_dim / 2] (cos, sin) built as the reference does."""
    cos = np.empty((length, head_dim // 2), np.float32)
    sin = np.empty_like(cos)
    load().et_b200_rope_tables_v1(length, head_dim, base, cos.ctypes.data, sin.ctypes.data)
    return cos, sin


class Attention:
    """et_b200_attention_forward_v1 / _backward_v1 over torch CUDA tensors
    [batch, heads, len, head_dim] (f32), positions [batch, len] (i64) and
    optional RoPE tables; enqueued on `stream` (a cudaStream_t address, 0 =
    the legacy default stream)."""

    def __init__(self, batch, q_heads, kv_heads, q_len, k_len, head_dim, q_positions,
                 k_positions, keep=None, rope_cos=None, rope_sin=None, stream: int = 0,
                 contraction: int = 0):
        import torch
        self.lib = load()
        self.keepalive = [q_positions, k_positions, keep, rope_cos, rope_sin]
        ptr = lambda t: t.data_ptr() if t is not None else None
        self.shape = AttentionShape(C.sizeof(AttentionShape), batch, q_heads, kv_heads, q_len,
                                    k_len, head_dim, ptr(q_positions), ptr(k_positions),
                                    ptr(keep), ptr(rope_cos), ptr(rope_sin), 0, contraction)
        self.ws_bytes = self.lib.et_b200_attention_workspace_bytes_v1(C.byref(self.shape))
        if self.ws_bytes == 0:
            raise ValueError("attention shape rejected")
        self.ws = torch.empty(self.ws_bytes // 4 + 64, dtype=torch.float32, device="cuda")
        base = self.ws.data_ptr()
        self.ws_ptr = (base + 255) & ~255
        self.stream = stream

    def forward(self, q, k, v, o, row_max, row_sum) -> None:
        err = k1.KernelError()
        _check(self.lib.et_b200_attention_forward_v1(
            C.byref(self.shape), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
            row_max.data_ptr(), row_sum.data_ptr(), self.ws_ptr, self.ws_bytes, self.stream,
            C.byref(err)), err)

    def backward(self, q, k, v, o, dout, row_max, row_sum, dq, dk, dv,
                 workspace_from_forward: bool = True) -> None:
        err = k1.KernelError()
        _check(self.lib.et_b200_attention_backward_v1(
            C.byref(self.shape), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
            dout.data_ptr(), row_max.data_ptr(), row_sum.data_ptr(), dq.data_ptr(),
            dk.data_ptr(), dv.data_ptr(), self.ws_ptr, self.ws_bytes,
            1 if workspace_from_forward else 0, self.stream, C.byref(err)), err)


def d2_row_count(tokens: int, seq_len: int) -> int:
    """Rows of a packed D2 stream of `tokens` tokens (et_b200_d2_row_count_v1)."""
    return load().et_b200_d2_row_count_v1(tokens, seq_len)


def d2_rows(tokens: np.ndarray, seq_len: int, first_row: int, rows: int):
    """(ids, targets, mask) planes [rows, seq_len] of a packed D2 stream
    (et_b200_d2_rows_v1)."""
    toks = np.ascontiguousarray(tokens, np.int64)
    ids = np.empty((rows, seq_len), np.int64)
    targets = np.empty((rows, seq_len), np.int64)
    mask = np.empty((rows, seq_len), np.uint8)
    err = k1.KernelError()
    _check(load().et_b200_d2_rows_v1(toks.ctypes.data if toks.size else None, toks.size,
                                     seq_len, first_row, rows, ids.ctypes.data,
                                     targets.ctypes.data, mask.ctypes.data, C.byref(err)), err)
    return ids, targets, mask


def nccl_unique_id() -> bytes:
    lib = load()
    buf = (C.c_uint8 * 128)()
    err = k1.KernelError()
    _check(lib.et_b200_nccl_unique_id_v1(buf, C.byref(err)), err)
    return bytes(buf)


def launch_count() -> int:
    return load().et_b200_launch_count_v1()


def fill_normal(seed: int, stream: int, count: int, mean: float = 0.0,
                std: float = 1.0) -> np.ndarray:
    out = np.empty(count, np.float32)
    load().et_b200_fill_normal_v1(seed, stream, count, mean, std, out.ctypes.data)
    return out


def fill_tokens(seed: int, stream: int, count: int, vocabulary: int) -> np.ndarray:
    out = np.empty(count, np.int64)
    load().et_b200_fill_tokens_v1(seed, stream, count, vocabulary, out.ctypes.data)
    return out


def synthetic_batch(seed: int, batch: int, seq_len: int, vocabulary: int):
    """Token ids and next-token targets [batch, seq_len] from one uniform
    (seq_len + 1)-token stream per sequence (stream id 2^20)."""
    toks = fill_tokens(seed, 1 << 20, batch * (seq_len + 1), vocabulary).reshape(batch,
                                                                                  seq_len + 1)
    return np.ascontiguousarray(toks[:, :-1]), np.ascontiguousarray(toks[:, 1:])


class O2Parameter(C.Structure):
    """et_b200_o2_parameter_v1"""
    _fields_ = [("struct_size", C.c_size_t), ("value", C.c_void_p), ("gradient", C.c_void_p),
                ("count", C.c_size_t), ("learning_rate_bits", C.c_uint32),
                ("beta1_bits", C.c_uint32), ("beta2_bits", C.c_uint32),
                ("epsilon_bits", C.c_uint32), ("weight_decay_bits", C.c_uint32),
                ("reserved", C.c_uint32)]


class Optimizer:
    """Handle over et_b200_o2_optimizer (device AdamW, O2 semantics)."""

    def __init__(self, entries, clip_kind=0, clip_max=0.0, schedule_kind=0, warmup=0, total=0,
                 minimum_ratio=0.0):
        """entries: list of (value_ptr, grad_ptr, count, lr, beta1, beta2, eps, wd)."""
        self.lib = load()
        arr = (O2Parameter * len(entries))()
        for i, (v, g, n, lr, b1, b2, eps, wd) in enumerate(entries):
            arr[i] = O2Parameter(C.sizeof(O2Parameter), v, g, n, f32_bits(lr), f32_bits(b1),
                                 f32_bits(b2), f32_bits(eps), f32_bits(wd), 0)
        self.handle = C.c_void_p()
        err = k1.KernelError()
        _check(self.lib.et_b200_o2_optimizer_create_v1(
            len(entries), arr, clip_kind, f32_bits(clip_max) if clip_kind else 0, schedule_kind,
            warmup, total, f32_bits(minimum_ratio) if schedule_kind else 0,
            C.byref(self.handle), C.byref(err)), err)

    def step(self, weight: float = 1.0) -> float:
        norm = C.c_uint32()
        err = k1.KernelError()
        _check(self.lib.et_b200_o2_optimizer_step_v1(self.handle, f32_bits(weight),
                                                     C.byref(norm), C.byref(err)), err)
        return struct.unpack("<f", struct.pack("<I", norm.value))[0]

    def moments(self, index: int) -> tuple[int, int]:
        a, b = C.c_void_p(), C.c_void_p()
        self.lib.et_b200_o2_optimizer_moments_v1(self.handle, index, C.byref(a), C.byref(b))
        return a.value, b.value

    def close(self) -> None:
        if self.handle:
            self.lib.et_b200_o2_optimizer_destroy_v1(C.byref(self.handle))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

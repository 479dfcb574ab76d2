"""ctypes handles over the CPU oracle (liboracle.so) and, when built, the
reference's own C sources compiled unmodified (oracle/_ref/libref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, always as the checker or the CPU
baseline, never as the thing measured.
"""
from __future__ import annotations

import ctypes as C
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libref.so"

_lib = None
_ref = None


def build() -> None:
    subprocess.run(["make", "-s", "-f", str(HERE / "Makefile")], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build()
        _lib = C.CDLL(str(ORACLE_SO))
        _lib.orc_global_norm.restype = C.c_uint32
        _lib.orc_pow_bits.restype = C.c_uint32
        _lib.orc_schedule_factor.restype = C.c_uint32
        _lib.orc_schedule_factor.argtypes = [C.c_uint32, C.c_uint64, C.c_uint64, C.c_uint32,
                                             C.c_uint64]
        _lib.orc_mean_loss.restype = C.c_float
        _lib.orc_lm_forward_backward.restype = C.c_float
        _lib.orc_lm_forward_backward_masked.restype = C.c_float
        _lib.orc_lm_forward_backward_masked.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p,
                                                        C.c_void_p, C.c_void_p, C.c_float,
                                                        C.c_void_p]
        _lib.orc_masked_mean_loss.restype = C.c_float
        _lib.orc_masked_mean_loss.argtypes = [C.c_size_t, C.c_void_p, C.c_void_p]
        _lib.orc_lm_tensor_count.restype = C.c_size_t
        _lib.orc_lm_tensor_sizes.restype = C.c_size_t
        _lib.orc_fill_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_size_t, C.c_double,
                                         C.c_double, C.c_void_p]
        _lib.orc_fill_tokens.argtypes = [C.c_uint64, C.c_uint64, C.c_size_t, C.c_uint64,
                                         C.c_void_p]
        _lib.orc_lm_init.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p]
        _lib.orc_lm_forward_backward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                 C.c_double, C.c_void_p]
        _lib.orc_lm_adamw.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_uint64]
        _lib.orc_adamw_step.argtypes = [C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint32,
                                        C.c_uint32, C.c_uint32]
    return _lib


def ref() -> C.CDLL | None:
    """The reference compiled from its sources, or None when not built."""
    global _ref
    if _ref is None and REF_SO.exists():
        _ref = C.CDLL(str(REF_SO))
    return _ref


def _p(a: np.ndarray) -> C.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return C.c_void_p(a.ctypes.data)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32)


def i64(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.int64)


def bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def from_bits(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


# ---------------------------------------------------------------- inputs

def fill_normal(seed: int, stream: int, count: int, mean: float = 0.0,
                std: float = 1.0) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().orc_fill_normal(seed, stream, count, mean, std, _p(out))
    return out


def fill_tokens(seed: int, stream: int, count: int, vocabulary: int) -> np.ndarray:
    out = np.empty(count, np.int64)
    lib().orc_fill_tokens(seed, stream, count, vocabulary, _p(out))
    return out


# ---------------------------------------------------------------- A2

def attention_forward(shape, q, k, v, qpos, kpos, mask) -> np.ndarray:
    s = (C.c_int64 * 6)(*shape)
    q, k, v, qpos, kpos = f32(q), f32(k), f32(v), i64(qpos), i64(kpos)
    mask = np.ascontiguousarray(mask, np.uint8)
    out = np.empty_like(q)
    lib().orc_attention_forward(s, _p(q), _p(k), _p(v), _p(qpos), _p(kpos), _p(mask), _p(out))
    return out


def attention_backward(shape, q, k, v, qpos, kpos, mask, dout):
    s = (C.c_int64 * 6)(*shape)
    q, k, v, dout = f32(q), f32(k), f32(v), f32(dout)
    qpos, kpos = i64(qpos), i64(kpos)
    mask = np.ascontiguousarray(mask, np.uint8)
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    lib().orc_attention_backward(s, _p(q), _p(k), _p(v), _p(qpos), _p(kpos), _p(mask), _p(dout),
                                 _p(dq), _p(dk), _p(dv))
    return dq, dk, dv


def rope(shape, x, positions, inv_freq, backward=False) -> np.ndarray:
    s = (C.c_int64 * 4)(*shape)
    x, positions, inv_freq = f32(x), i64(positions), f32(inv_freq)
    y = np.empty_like(x)
    lib().orc_rope(s, _p(x), _p(positions), _p(inv_freq), 1 if backward else 0, _p(y))
    return y


# ---------------------------------------------------------------- N2

def linear_forward(x, w, bias=None) -> np.ndarray:
    x, w = f32(x), f32(w)
    rows, din = x.reshape(-1, x.shape[-1]).shape
    dout = w.shape[0]
    y = np.empty(x.shape[:-1] + (dout,), np.float32)
    b = f32(bias) if bias is not None else None
    lib().orc_linear_forward(C.c_size_t(rows), C.c_size_t(din), C.c_size_t(dout), _p(x), _p(w),
                             _p(b) if b is not None else None, _p(y))
    return y


def linear_backward(x, w, dy, with_bias=True):
    x, w, dy = f32(x), f32(w), f32(dy)
    rows, din = x.reshape(-1, x.shape[-1]).shape
    dout = w.shape[0]
    dx, dw = np.empty_like(x), np.empty_like(w)
    db = np.empty(dout, np.float32) if with_bias else None
    lib().orc_linear_backward(C.c_size_t(rows), C.c_size_t(din), C.c_size_t(dout), _p(x), _p(w),
                              _p(dy), _p(dx), _p(dw),
                              _p(db) if db is not None else None)
    return dx, dw, db


def layer_norm_forward(x, gamma, beta, eps) -> np.ndarray:
    x, gamma, beta = f32(x), f32(gamma), f32(beta)
    d = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_layer_norm_forward(C.c_size_t(x.size // d), C.c_size_t(d), _p(x), _p(gamma),
                                 _p(beta), C.c_float(eps), _p(y))
    return y


def layer_norm_backward(x, gamma, eps, dy):
    x, gamma, dy = f32(x), f32(gamma), f32(dy)
    d = x.shape[-1]
    dx, dg, db = np.empty_like(x), np.empty(d, np.float32), np.empty(d, np.float32)
    lib().orc_layer_norm_backward(C.c_size_t(x.size // d), C.c_size_t(d), _p(x), _p(gamma),
                                  C.c_float(eps), _p(dy), _p(dx), _p(dg), _p(db))
    return dx, dg, db


def gelu_forward(x) -> np.ndarray:
    x = f32(x)
    y = np.empty_like(x)
    lib().orc_gelu_forward(C.c_size_t(x.size), _p(x), _p(y))
    return y


def gelu_backward(x, dy) -> np.ndarray:
    x, dy = f32(x), f32(dy)
    dx = np.empty_like(x)
    lib().orc_gelu_backward(C.c_size_t(x.size), _p(x), _p(dy), _p(dx))
    return dx


def embedding_forward(ids, w) -> np.ndarray:
    ids, w = i64(ids), f32(w)
    y = np.empty(ids.shape + (w.shape[1],), np.float32)
    lib().orc_embedding_forward(C.c_size_t(ids.size), C.c_size_t(w.shape[0]),
                                C.c_size_t(w.shape[1]), _p(ids), _p(w), _p(y))
    return y


def embedding_backward(ids, dy, vocabulary) -> np.ndarray:
    ids, dy = i64(ids), f32(dy)
    d = dy.shape[-1]
    dw = np.empty((vocabulary, d), np.float32)
    lib().orc_embedding_backward(C.c_size_t(ids.size), C.c_size_t(vocabulary), C.c_size_t(d),
                                 _p(ids), _p(dy), _p(dw))
    return dw


# ---------------------------------------------------------------- L2 / O2

def ce_forward(logits, targets) -> np.ndarray:
    logits, targets = f32(logits), i64(targets)
    V = logits.shape[-1]
    loss = np.empty(logits.shape[:-1], np.float32)
    lib().orc_ce_forward(C.c_size_t(logits.size // V), C.c_size_t(V), _p(logits), _p(targets),
                         _p(loss))
    return loss


def ce_backward(logits, targets, upstream) -> np.ndarray:
    logits, targets, upstream = f32(logits), i64(targets), f32(upstream)
    V = logits.shape[-1]
    g = np.empty_like(logits)
    lib().orc_ce_backward(C.c_size_t(logits.size // V), C.c_size_t(V), _p(logits), _p(targets),
                          _p(upstream), _p(g))
    return g


class AdamwOptions(C.Structure):
    _fields_ = [("learning_rate_bits", C.c_uint32), ("beta1_bits", C.c_uint32),
                ("beta2_bits", C.c_uint32), ("epsilon_bits", C.c_uint32),
                ("weight_decay_bits", C.c_uint32)]


def adamw_options(lr, beta1, beta2, eps, wd) -> AdamwOptions:
    return AdamwOptions(bits(lr), bits(beta1), bits(beta2), bits(eps), bits(wd))


def adamw_step(p, g, m, v, options: AdamwOptions, update: int, weight: float = 1.0,
               schedule_factor_bits: int = 0x3F800000, clip: float = 1.0) -> int:
    """In place on p, m, v (float32 arrays); returns 0 or 1 (nonfinite)."""
    return lib().orc_adamw_step(p.size, _p(p), _p(f32(g)), _p(m), _p(v), C.byref(options),
                                update, bits(weight), schedule_factor_bits, bits(clip))


def global_norm(grads, weight: float = 1.0) -> float:
    arrs = [f32(g) for g in grads]
    ptrs = (C.c_void_p * len(arrs))(*[_p(a) for a in arrs])
    counts = (C.c_size_t * len(arrs))(*[a.size for a in arrs])
    return from_bits(lib().orc_global_norm(len(arrs), ptrs, counts, bits(weight)))


def schedule_factor(kind, warmup, total, minimum_ratio_bits, update) -> int:
    return lib().orc_schedule_factor(kind, warmup, total, minimum_ratio_bits, update)


def mean_loss(loss) -> float:
    loss = f32(loss)
    return lib().orc_mean_loss(C.c_size_t(loss.size), _p(loss))


def masked_mean_loss(loss, mask) -> float:
    loss = f32(loss)
    m = np.ascontiguousarray(mask, np.uint8)
    return lib().orc_masked_mean_loss(C.c_size_t(loss.size), _p(loss), _p(m))


def d2_rows(tokens, seq_len: int, first_row: int, rows: int):
    """The packed D2 row rule (docs/D2_SHARD_LOADER.md, "Rows, shift, mask,
    and ordering") in plain Python: (ids, targets, mask) planes [rows,
    seq_len] of rows first_row .. of the stream."""
    toks = list(int(t) for t in tokens)
    L = len(toks)
    count = 0 if L < 2 else 1 + (L - 2) // seq_len
    ids = np.zeros((rows, seq_len), np.int64)
    targets = np.zeros((rows, seq_len), np.int64)
    mask = np.zeros((rows, seq_len), np.uint8)
    for r in range(rows):
        if first_row + r >= count:
            break
        s = (first_row + r) * seq_len
        for t in range(seq_len):
            if s + t + 1 >= L:
                break
            ids[r, t], targets[r, t], mask[r, t] = toks[s + t], toks[s + t + 1], 1
    return ids, targets, mask


# ---------------------------------------------------------------- LM

class LMConfig(C.Structure):
    _fields_ = [("layers", C.c_int64), ("d_model", C.c_int64), ("heads", C.c_int64),
                ("ffn", C.c_int64), ("vocabulary", C.c_int64), ("seq_len", C.c_int64),
                ("batch", C.c_int64), ("ln_epsilon", C.c_float), ("rope_base", C.c_double)]


class LanguageModel:
    """The oracle's restatement of the decoder LM training step."""

    def __init__(self, layers, d_model, heads, ffn, vocabulary, seq_len, batch,
                 ln_eps=1e-5, rope_base=10000.0):
        self.cfg = LMConfig(layers, d_model, heads, ffn, vocabulary, seq_len, batch, ln_eps,
                            rope_base)
        n = lib().orc_lm_tensor_count(C.byref(self.cfg))
        sizes = (C.c_size_t * n)()
        self.total = lib().orc_lm_tensor_sizes(C.byref(self.cfg), sizes)
        self.tensor_sizes = list(sizes)

    def init(self, seed: int) -> np.ndarray:
        p = np.empty(self.total, np.float32)
        lib().orc_lm_init(C.byref(self.cfg), seed, _p(p))
        return p

    def forward_backward(self, params, ids, targets, token_scale: float = 0.0):
        grads = np.zeros(self.total, np.float32)
        params, ids, targets = f32(params), i64(ids), i64(targets)
        loss = lib().orc_lm_forward_backward(C.byref(self.cfg), _p(params), _p(ids),
                                             _p(targets), token_scale, _p(grads))
        return float(loss), grads

    def forward_backward_masked(self, params, ids, targets, loss_mask, upstream_scale: float):
        """The masked objective: loss = the L3S masked mean, gradients = the
        mask-weighted numerators times upstream_scale."""
        grads = np.zeros(self.total, np.float32)
        params, ids, targets = f32(params), i64(ids), i64(targets)
        m = np.ascontiguousarray(loss_mask, np.uint8)
        loss = lib().orc_lm_forward_backward_masked(C.byref(self.cfg), _p(params), _p(ids),
                                                    _p(targets), _p(m), upstream_scale,
                                                    _p(grads))
        return float(loss), grads

    def adamw(self, params, grads, m, v, options: AdamwOptions, update: int) -> int:
        return lib().orc_lm_adamw(C.byref(self.cfg), _p(params), _p(f32(grads)), _p(m), _p(v),
                                  C.byref(options), update)

    def split(self, flat: np.ndarray) -> list[np.ndarray]:
        out, off = [], 0
        for n in self.tensor_sizes:
            out.append(flat[off:off + n])
            off += n
        return out


def synthetic_batch(seed: int, batch: int, seq_len: int, vocabulary: int):
    """Token ids and next-token targets: one (seq_len + 1)-token stream per
    sequence drawn uniformly in [0, vocabulary)."""
    toks = fill_tokens(seed, 1 << 20, batch * (seq_len + 1), vocabulary).reshape(
        batch, seq_len + 1)
    return np.ascontiguousarray(toks[:, :-1]), np.ascontiguousarray(toks[:, 1:])

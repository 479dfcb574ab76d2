"""Shared helpers: golden-fixture decoding and tolerance checks."""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name: str) -> dict:
    return json.loads((GOLDEN / f"{name}.json").read_text())


def decode(t: dict) -> np.ndarray:
    """A tensor record of the reference's eshkol-oracle envelope."""
    shape = tuple(t["shape"])
    if t["dtype"] == "float32":
        vals = [struct.unpack(">f", bytes.fromhex(x))[0] for x in t["data"]]
        return np.array(vals, np.float32).reshape(shape)
    if t["dtype"] == "float64":
        vals = [struct.unpack(">d", bytes.fromhex(x))[0] for x in t["data"]]
        return np.array(vals, np.float64).reshape(shape)
    if t["dtype"] == "bool":
        return np.array([int(x) for x in t["data"]], np.uint8).reshape(shape)
    vals = [int.from_bytes(bytes.fromhex(x), "big", signed=True) for x in t["data"]]
    return np.array(vals, np.int64).reshape(shape)


def hex_f64(s: str) -> float:
    return struct.unpack(">d", bytes.fromhex(s))[0]


def decode_ref_vector(rec: dict) -> np.ndarray:
    """A tensor of reference_vectors.json (f32 as little-endian bit patterns)."""
    shape = tuple(rec["shape"])
    if "dtype" in rec and rec["dtype"] != "float32":
        return np.array(rec["hex"], np.dtype(rec["dtype"])).reshape(shape)
    return np.array([int(h, 16) for h in rec["hex"]], np.uint32).view(np.float32).reshape(shape)


def assert_close(actual, expected, atol, rtol, what=""):
    """|a - e| <= atol + rtol |e| elementwise (the fixtures' allclose rule)."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    err = np.abs(a - e)
    bound = atol + rtol * np.abs(e)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), a.shape)
        raise AssertionError(f"{what}: {bad.sum()} of {a.size} outside atol={atol} rtol={rtol};"
                             f" worst at {i}: {a[i]} vs {e[i]}")


def assert_close_norm(actual, expected, tol, what=""):
    """max |a - e| <= tol * max |e|: a tensor-wise relative bound for
    reductions whose summation order differs from the reference's."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    scale = max(np.abs(e).max(), 1e-30)
    err = np.abs(a - e).max()
    assert err <= tol * scale, f"{what}: max err {err:.3e} > {tol} * {scale:.3e}"


def bits_equal(a, b) -> bool:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))

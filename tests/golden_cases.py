"""The reference's golden fixture cases as uniform K1 calls.

Each case carries the K1 capability, operation, request shape, the input
arrays in the provider's tensor-table order, the expected outputs in output
order and the fixture's tolerance (|a - e| <= atol + rtol |e|).  The same cases
drive the oracle pin (CPU) and the B200 providers (GPU).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from helpers import decode, hex_f64, load_golden


@dataclass
class Case:
    name: str
    capability: str
    operation: str
    shape: tuple
    inputs: list
    outputs: list
    atol: float
    rtol: float


def _tensor(T, prefix, suffix):
    return decode(T[f"{prefix}.{suffix}"])


def a2_cases() -> list[Case]:
    g = load_golden("a2_attention")
    T = g["tensors"]
    out = []
    for c in g["cases"]:
        tol = c["tolerance"]
        atol, rtol = hex_f64(tol["absolute"]), hex_f64(tol["relative"])
        op = c["operation"]
        first = c["inputs"][0]
        prefix = first.split(".input.")[0]
        if op.startswith("causal-attention"):
            q, k, v = (_tensor(T, prefix, f"input.{n}") for n in ("q", "k", "v"))
            qpos, kpos = _tensor(T, prefix, "input.qpos"), _tensor(T, prefix, "input.kpos")
            mask = _tensor(T, prefix, "input.mask").astype(np.uint8)
            shape = (q.shape[0], q.shape[1], k.shape[1], q.shape[2], k.shape[2], q.shape[3])
            ins = [q, k, v, qpos, kpos, mask]
            if op.endswith("backward"):
                ins.append(_tensor(T, prefix, "input.upstream"))
                outs = [_tensor(T, prefix, f"gradient.{n}") for n in ("dq", "dk", "dv")]
            else:
                outs = [_tensor(T, prefix, "output.forward")]
            out.append(Case(c["name"], "kernel.causal-attention", op, shape, ins, outs, atol, rtol))
        elif op.startswith("rope"):
            x = _tensor(T, prefix, "input.upstream" if op.endswith("backward") else "input.x")
            pos = _tensor(T, prefix, "input.positions")
            inv = _tensor(T, prefix, "input.inv")
            y = _tensor(T, prefix, "gradient.dx" if op.endswith("backward") else "output.forward")
            out.append(Case(c["name"], "kernel.rope", op, x.shape, [x, pos, inv], [y], atol, rtol))
        # cached-incremental.forward exercises the KV cache (not a K1 op)
    return out


def n2_cases() -> list[Case]:
    g = load_golden("n2_primitives")
    T = g["tensors"]
    out = []
    for c in g["cases"]:
        tol = c["tolerance"]
        atol, rtol = hex_f64(tol["absolute"]), hex_f64(tol["relative"])
        op = c["operation"]
        names = c["inputs"]
        outs_n = c["expectation"]["outputs"]
        get = lambda n: decode(T[n])
        find = lambda key: next(n for n in names if n.endswith(key))
        if op.startswith("dropout"):
            continue  # Philox dropout is outside the training-step path
        if op == "embedding.forward":
            ids, w = get(find(".ids")), get(find(".weight"))
            shape = ids.shape + w.shape
            ins, cap = [ids, w], "kernel.embedding-forward"
        elif op == "embedding.backward":
            ids, up = get(find(".ids")), get(find(".upstream"))
            dw = get(outs_n[0])
            shape = ids.shape + dw.shape
            ins, cap = [ids, up], "kernel.embedding-backward"
        elif op.startswith("linear.forward"):
            x, w = get(find(".x")), get(find(".weight"))
            ins = [x, w] + ([get(find(".bias"))] if op == "linear.forward" else [])
            shape, cap = x.shape + (w.shape[0],), "kernel.matmul"
        elif op.startswith("linear.backward"):
            x, w, up = get(find(".x")), get(find(".weight")), get(find(".upstream"))
            ins, shape, cap = [x, w, up], x.shape + (w.shape[0],), "kernel.matmul"
        elif op == "layer-norm.forward":
            ins = [get(find(k)) for k in (".x", ".gamma", ".beta", ".epsilon")]
            shape, cap = ins[0].shape, "kernel.norm"
        elif op == "layer-norm.backward":
            ins = [get(find(k)) for k in (".x", ".gamma", ".epsilon", ".upstream")]
            shape, cap = ins[0].shape, "kernel.norm"
        elif op in ("gelu.forward", "relu.forward"):
            ins, cap = [get(find(".x"))], "kernel.activation"
            shape = ins[0].shape
        elif op in ("gelu.backward", "relu.backward"):
            ins, cap = [get(find(".x")), get(find(".upstream"))], "kernel.activation"
            shape = ins[0].shape
        elif op == "residual.forward":
            ins, cap = [get(find(".x")), get(find(".branch"))], "kernel.residual"
            shape = ins[0].shape
        elif op == "residual.backward":
            ins, cap = [get(find(".upstream"))], "kernel.residual"
            shape = ins[0].shape
        else:
            continue
        order = {"linear.backward": [".dx", ".dweight", ".dbias"],
                 "linear.backward-no-bias": [".dx", ".dweight"],
                 "layer-norm.backward": [".dx", ".dgamma", ".dbeta"],
                 "residual.backward": [".dx", ".dbranch"]}.get(op)
        if order:
            outs = [get(next(n for n in outs_n if n.endswith(k))) for k in order]
        else:
            outs = [get(outs_n[0])]
        out.append(Case(c["name"], cap, op, tuple(shape), ins, outs, atol, rtol))
    return out


def l2_cases() -> list[Case]:
    g = load_golden("indexed_cross_entropy")
    T = g["tensors"]
    out = []
    for c in g["cases"]:
        tol = c["tolerance"]
        atol, rtol = hex_f64(tol["absolute"]), hex_f64(tol["relative"])
        logits, targets = decode(T["input.logits"]), decode(T["input.targets"])
        if c["operation"].endswith("backward"):
            ins = [logits, targets, decode(T["input.upstream"])]
            outs = [decode(T["output.gradient"])]
        else:
            ins, outs = [logits, targets], [decode(T["output.loss"])]
        out.append(Case(c["name"], "kernel.indexed-cross-entropy", c["operation"], logits.shape,
                        ins, outs, atol, rtol))
    return out


def adamw_golden() -> dict:
    g = load_golden("adamw")
    T = g["tensors"]
    cases = {c["name"]: c for c in g["cases"]}
    return {"cases": cases, "get": lambda n: decode(T[n]),
            "tol": lambda c: (hex_f64(c["tolerance"]["absolute"]),
                              hex_f64(c["tolerance"]["relative"]))}

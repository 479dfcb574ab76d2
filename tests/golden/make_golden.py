"""Regenerates the golden fixtures under tests/golden from eshkol-transformer.

Two sources, both read only in this container (the GPU box has neither):

1. the reference's own PyTorch-generated fixtures (tests/a2/fixtures/
   a2_attention_v1.json, tests/q0/fixtures/indexed_cross_entropy_v1.json,
   tests/q0/fixtures/n2_primitives_v1.json, tests/o2/fixtures/adamw_v1.json),
   re-emitted case by case with their tensors and tolerances in the same
   hex encodings (the "eshkol-oracle" envelope of tests/q0/oracle_format.py);
2. outputs of the reference's C providers compiled unmodified into
   oracle/_ref/libref.so, on seeded inputs at small shapes
   (reference_vectors.json), so the GPU tests can check bit-level claims
   without the reference present.

Usage: python tests/golden/make_golden.py [/path/to/eshkol-transformer]
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

FIXTURES = {
    "a2_attention": "tests/a2/fixtures/a2_attention_v1.json",
    "indexed_cross_entropy": "tests/q0/fixtures/indexed_cross_entropy_v1.json",
    "n2_primitives": "tests/q0/fixtures/n2_primitives_v1.json",
    "adamw": "tests/o2/fixtures/adamw_v1.json",
}


def convert_fixture(reference: Path, name: str, rel: str) -> None:
    src = json.loads((reference / rel).read_text())
    payload = src["payload"]
    out = {
        "source": f"eshkol-transformer {rel}",
        "generator": payload.get("generator", {}),
        "cases": payload["cases"],
        "tensors": {t["name"]: {k: t[k] for k in ("dtype", "shape", "encoding", "data", "role")}
                    for t in payload["tensors"]},
    }
    (HERE / f"{name}.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")


def _hex_f32(a: np.ndarray) -> list[str]:
    return [format(int(x), "08x") for x in np.ascontiguousarray(a, np.float32).view(np.uint32).ravel()]


def reference_vectors() -> None:
    """Runs the reference's providers (oracle/_ref) on seeded inputs."""
    from eshkol_transformer_b200 import k1
    from oracle import oracle as orc

    ref = orc.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libref.so is not built (make -f oracle/Makefile.ref)")
    cases = []
    rng_seed = 20261201

    def record(kind, shape, inputs, outputs):
        cases.append({"kind": kind, "shape": list(shape),
                      "inputs": {k: {"dtype": str(v.dtype), "shape": list(v.shape),
                                     "hex": _hex_f32(v) if v.dtype == np.float32 else v.ravel().tolist()}
                                 for k, v in inputs.items()},
                      "outputs": {k: {"shape": list(v.shape), "hex": _hex_f32(v)}
                                  for k, v in outputs.items()}})

    a2 = k1.provider(ref, "et_a2_kernel_provider_v1")
    for si, shape in enumerate([(2, 4, 2, 16, 16, 8), (1, 2, 2, 33, 33, 16), (2, 4, 4, 24, 24, 32)]):
        N, Hq, Hkv, Tq, Tk, Dh = shape
        q = orc.fill_normal(rng_seed, 10 * si + 1, N * Hq * Tq * Dh).reshape(N, Hq, Tq, Dh)
        k = orc.fill_normal(rng_seed, 10 * si + 2, N * Hkv * Tk * Dh).reshape(N, Hkv, Tk, Dh)
        v = orc.fill_normal(rng_seed, 10 * si + 3, N * Hkv * Tk * Dh).reshape(N, Hkv, Tk, Dh)
        g = orc.fill_normal(rng_seed, 10 * si + 4, N * Hq * Tq * Dh).reshape(N, Hq, Tq, Dh)
        pos = np.tile(np.arange(Tq, dtype=np.int64), (N, 1))
        mask = np.ones((N, Tq, Tk), np.uint8)
        if si == 1:
            mask[:, 5, :] = 0  # a row with no admitted key
            mask[:, 9, 3] = 0
        o = np.zeros_like(q)
        call = k1.KernelCall("kernel.causal-attention", "causal-attention.forward", shape,
                             [q, k, v, pos, pos, mask], [o])
        rc, err = k1.dispatch(a2, call)
        assert rc == 0, str(err)
        dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
        call = k1.KernelCall("kernel.causal-attention", "causal-attention.backward", shape,
                             [q, k, v, pos, pos, mask, g], [dq, dk, dv])
        rc, err = k1.dispatch(a2, call)
        assert rc == 0, str(err)
        record("attention", shape, {"q": q, "k": k, "v": v, "pos": pos, "mask": mask, "dout": g},
               {"o": o, "dq": dq, "dk": dk, "dv": dv})
    for si, shape in enumerate([(2, 4, 16, 8), (1, 2, 40, 32)]):
        N, H, T, Dh = shape
        x = orc.fill_normal(rng_seed, 100 + si, N * H * T * Dh).reshape(N, H, T, Dh)
        pos = np.tile(np.arange(T, dtype=np.int64) * (3 if si else 1), (N, 1))
        inv = np.empty(Dh // 2, np.float32)
        orc.lib().orc_rope_inv_freq(C.c_int64(Dh), C.c_double(10000.0),
                                    inv.ctypes.data_as(C.c_void_p))
        outs = {}
        for op in ("forward", "backward"):
            y = np.zeros_like(x)
            call = k1.KernelCall("kernel.rope", f"rope.{op}", shape, [x, pos, inv], [y])
            rc, err = k1.dispatch(a2, call)
            assert rc == 0, str(err)
            outs[op] = y
        record("rope", shape, {"x": x, "pos": pos, "inv_freq": inv}, outs)
    l2 = k1.provider(ref, "et_l2_indexed_cross_entropy_provider_v1")
    for si, shape in enumerate([(2, 8, 64), (1, 5, 1000)]):
        N, T, V = shape
        logits = (orc.fill_normal(rng_seed, 200 + si, N * T * V) * 3).reshape(N, T, V).astype(np.float32)
        tgt = orc.fill_tokens(rng_seed, 210 + si, N * T, V).reshape(N, T)
        up = orc.fill_normal(rng_seed, 220 + si, N * T).reshape(N, T)
        loss = np.zeros((N, T), np.float32)
        rc, err = k1.dispatch(l2, k1.KernelCall("kernel.indexed-cross-entropy",
                                                "indexed-cross-entropy.forward", shape,
                                                [logits, tgt], [loss]))
        assert rc == 0, str(err)
        grad = np.zeros_like(logits)
        rc, err = k1.dispatch(l2, k1.KernelCall("kernel.indexed-cross-entropy",
                                                "indexed-cross-entropy.backward", shape,
                                                [logits, tgt, up], [grad]))
        assert rc == 0, str(err)
        record("cross_entropy", shape, {"logits": logits, "targets": tgt, "upstream": up},
               {"loss": loss, "grad": grad})
    body = {"source": "eshkol-transformer native providers compiled by oracle/Makefile.ref",
            "seed": rng_seed, "cases": cases}
    text = json.dumps(body, sort_keys=True)
    body["sha256"] = hashlib.sha256(text.encode()).hexdigest()
    (HERE / "reference_vectors.json").write_text(json.dumps(body, sort_keys=True) + "\n")


def main() -> None:
    reference = Path(sys.argv[1]) if len(sys.argv) > 1 else Path("/root/reference")
    for name, rel in FIXTURES.items():
        convert_fixture(reference, name, rel)
    reference_vectors()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()

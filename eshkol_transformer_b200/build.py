"""Builds libet_b200.so (sm_100a) in-tree.

Each CUDA translation unit is compiled by nvcc for sm_100a only, then linked
into eshkol_transformer_b200/lib/libet_b200.so.  Objects are rebuilt when
their source or any header is newer.  Run as a module to build:

    python -m eshkol_transformer_b200.build [--verbose-ptxas]
"""
from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = LIB_DIR / "obj"
LIB = LIB_DIR / "libet_b200.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3", f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path("/usr/local/cuda/bin/nvcc")
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found")


def _headers_mtime() -> float:
    paths = list(CSRC.glob("*.cuh")) + list(INCLUDE.rglob("*.h"))
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile(src: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    obj = OBJ_DIR / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj, ""
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stdout + proc.stderr


def build_library(ptxas_verbose: bool = False, jobs: int | None = None) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    logs = []
    with futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        results = list(pool.map(lambda s: _compile(s, ptxas_verbose), sources))
    objs = [r[0] for r in results]
    logs = [r[1] for r in results if r[1]]
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-ldl", "-lcuda"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    if ptxas_verbose:
        for log in logs:
            sys.stdout.write(log)
    return LIB


def build_oracle(reference: Path | None = None) -> None:
    """Builds the CPU oracle (test infrastructure) and, when the reference
    sources are present, the reference harness library oracle/_ref."""
    oracle = ROOT / "oracle"
    subprocess.run(["make", "-s", "-f", str(oracle / "Makefile")], check=True)
    if reference is not None and (reference / "native" / "kernel_abi.c").exists():
        subprocess.run(["make", "-s", "-f", str(oracle / "Makefile.ref"),
                        f"REF={reference}"], check=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build_library(ptxas_verbose=args.verbose_ptxas))


if __name__ == "__main__":
    main()

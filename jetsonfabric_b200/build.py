"""In-tree build of the native libraries.

    libjfm.so  host-only: JFM v2 loader (jf_* ABI), SHA-256, synthetic package
               writer (jfb_write_synthetic_package). No CUDA dependency.
    libjfb.so  the sm_100a kernel library and the native stage engine
               (jfb_* C ABI plus the jetsonfabric::native C++ API); links libjfm.

Both land in jetsonfabric_b200/lib/ so that they travel with the source tree.
Every CUDA file is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
REPO = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIB = PACKAGE / "lib"
BUILD = REPO / "_build"
INCLUDE = REPO / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = Path(NVCC).resolve().parent.parent
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

JFM_SOURCES = [
    CSRC / "jfm" / "jfm_loader.c",
    CSRC / "jfm" / "sha256.c",
    CSRC / "jfm" / "synth_package.cpp",
    CSRC / "jfm" / "gguf_import.cpp",
    CSRC / "tokenizer" / "bpe_tokenizer.cpp",
]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(map(str, cmd)) + "\n" + proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {Path(cmd[-1]).name if cmd else '?'}")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    deps = list(sources)
    for d in (CSRC, INCLUDE):
        deps += [p for p in d.rglob("*") if p.suffix in {".h", ".hpp", ".cuh"}]
    return any(p.stat().st_mtime > t for p in deps)


def build_jfm(force: bool = False) -> Path:
    target = LIB / "libjfm.so"
    if not force and not _stale(target, JFM_SOURCES):
        return target
    LIB.mkdir(parents=True, exist_ok=True)
    out = BUILD / "jfm"
    out.mkdir(parents=True, exist_ok=True)
    objects = []
    for src in JFM_SOURCES:
        obj = out / (src.name + ".o")
        if src.suffix == ".c":
            cmd = ["gcc", "-std=c11", "-O2", "-fPIC", "-Wall", "-Wextra", "-pthread"]
        else:
            cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-Wall", "-Wextra", "-pthread"]
        cmd += [f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
        _run(cmd)
        objects.append(str(obj))
    tmp = target.with_suffix(".so.tmp")
    _run(["g++", "-shared", "-pthread", "-o", str(tmp)] + objects)
    os.replace(tmp, target)
    return target


def build_all(force: bool = False) -> None:
    build_jfm(force)
    try:
        from . import build_cuda  # noqa: F401  (kernel library, added with the CUDA sources)
    except ImportError:
        return
    build_cuda.build(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)

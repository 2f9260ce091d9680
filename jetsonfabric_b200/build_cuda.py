"""Build of libjfb.so: the sm_100a kernel library plus the native engine.

Every .cu file is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a -lineinfo); the C++20 engine and the
C loader are compiled by g++/gcc; everything links into
jetsonfabric_b200/lib/libjfb.so against the CUDA runtime.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

from .build import BUILD, CSRC, CUDA_HOME, INCLUDE, LIB, NVCC, ARCH, JFM_SOURCES, _run, _stale

KERNELS = sorted((CSRC / "kernels").glob("*.cu"))
ENGINE = sorted((CSRC / "engine").glob("*.cpp")) + [CSRC / "transport" / "frame_channel.cpp"]

NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++20", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     f"-I{INCLUDE}", f"-I{CSRC}"]
CXX_FLAGS = ["-std=c++20", "-O2", "-fPIC", "-Wall", "-Wextra", "-pthread", f"-I{INCLUDE}", f"-I{CSRC}",
             f"-I{CUDA_HOME / 'include'}"]


def _compile(src: Path, out_dir: Path) -> str:
    obj = out_dir / (src.name + ".o")
    if obj.exists() and obj.stat().st_mtime > src.stat().st_mtime and not _stale(obj, [src]):
        return str(obj)
    if src.suffix == ".cu":
        cmd = [NVCC] + NVCC_FLAGS + ["-c", str(src), "-o", str(obj)]
    elif src.suffix == ".c":
        cmd = ["gcc", "-std=c11", "-O2", "-fPIC", "-Wall", "-pthread", f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++"] + CXX_FLAGS + ["-c", str(src), "-o", str(obj)]
    _run(cmd)
    return str(obj)


def build(force: bool = False) -> Path:
    target = LIB / "libjfb.so"
    sources = KERNELS + ENGINE + JFM_SOURCES
    if not force and not _stale(target, sources):
        return target
    LIB.mkdir(parents=True, exist_ok=True)
    out = BUILD / "jfb"
    out.mkdir(parents=True, exist_ok=True)
    if force:
        for o in out.glob("*.o"):
            o.unlink()
    with ThreadPoolExecutor(max_workers=max(2, min(8, os.cpu_count() or 2))) as pool:
        objects = list(pool.map(lambda s: _compile(s, out), sources))
    tmp = target.with_suffix(".so.tmp")
    _run(["g++", "-shared", "-pthread", "-o", str(tmp)] + objects +
         [f"-L{CUDA_HOME / 'lib64'}", "-lcudart", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}"])
    os.replace(tmp, target)
    return target

"""Builds oracle/_ref/transport_replay: the reference runtime's generation
runner, stage worker, activation codecs, Stagewire codec and stage executors,
compiled from where they lie under the reference tree, around this
repository's in-box StageTransport (jetsonfabric_b200/csrc/transport/) and
linked with libjfb.so (test infrastructure).

Nothing of the reference is modified or copied: its sources are compiled in
place with this repository's include/ ahead of them (so the native executor
binds the drop-in engine API). The reference's Stagewire codec needs the
single-header nlohmann JSON library, which the reference fetches at build
time; a copy that ships inside an installed Python package is used
(JFB_NLOHMANN_INCLUDE overrides the search).

Nothing is built when the reference tree is absent (on the GPU hosts the
prebuilt binary travels with the repository instead).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
OUT = REPO / "oracle" / "_ref"
BINARY = OUT / "transport_replay"
TRANSPORT = REPO / "jetsonfabric_b200" / "csrc" / "transport"

REFERENCE_SOURCES = [
    "protocol/stage.cpp", "protocol/stage_control.cpp", "protocol/utf8.cpp",
    "transport/stage_transport_factory.cpp",
    "pipeline_parallel/generation_runner.cpp", "pipeline_parallel/stage_worker.cpp",
    "pipeline_parallel/stage_assignment.cpp", "pipeline_parallel/synthetic_activation_executor.cpp",
    "inference/stage.cpp", "inference/token_payload.cpp",
    "activation/activation_codec_factory.cpp", "activation/builtin_activation_codecs.cpp",
    "adapters/native_stage_executor.cpp",
]


def reference_runtime() -> Path | None:
    root = Path(os.environ.get("JFB_REFERENCE", "/root/reference")) / "runtime"
    return root if (root / "transport" / "stage_transport.hpp").exists() else None


def nlohmann_include() -> Path | None:
    env = os.environ.get("JFB_NLOHMANN_INCLUDE")
    if env:
        return Path(env)
    for base in map(Path, sys.path):
        if not base.is_dir() or "site-packages" not in str(base):
            continue
        for hit in base.glob("**/nlohmann/json.hpp"):
            return hit.parent.parent
    return None


def build(force: bool = False) -> Path | None:
    ref = reference_runtime()
    if ref is None:
        return BINARY if BINARY.exists() else None
    lib = REPO / "jetsonfabric_b200" / "lib"
    inputs = [HERE / "transport_replay.cpp", HERE / "build.py", TRANSPORT / "inbox_stage_transport.cpp",
              TRANSPORT / "inbox_stage_transport.hpp", REPO / "include" / "jfb" / "jfb_stagewire.h",
              lib / "libjfb.so"]
    if not force and BINARY.exists() and all(BINARY.stat().st_mtime > p.stat().st_mtime for p in inputs):
        return BINARY
    nl = nlohmann_include()
    if nl is None:
        raise RuntimeError("the nlohmann JSON header is not available; set JFB_NLOHMANN_INCLUDE")
    OUT.mkdir(parents=True, exist_ok=True)
    objdir = OUT / "transport_obj"
    objdir.mkdir(exist_ok=True)
    flags = ["g++", "-std=c++20", "-O1", "-Wall", "-pthread", f"-I{REPO / 'include'}", f"-I{TRANSPORT}",
             f"-I{ref}", f"-I{nl}"]
    sources = [ref / s for s in REFERENCE_SOURCES] + [TRANSPORT / "inbox_stage_transport.cpp",
                                                     HERE / "transport_replay.cpp"]
    objects = []
    procs = []
    for src in sources:
        obj = objdir / (src.parent.name + "_" + src.stem + ".o")
        objects.append(str(obj))
        if not force and obj.exists() and obj.stat().st_mtime > max(p.stat().st_mtime for p in [src] + inputs[:5]):
            continue
        procs.append((src, subprocess.Popen(flags + ["-c", str(src), "-o", str(obj)])))
    for src, p in procs:
        if p.wait() != 0:
            raise RuntimeError(f"compiling {src} failed")
    tmp = BINARY.with_suffix(".tmp")
    subprocess.run(["g++", "-pthread", "-o", str(tmp)] + objects +
                   [f"-L{lib}", "-ljfb", "-Wl,-rpath,$ORIGIN/../../jetsonfabric_b200/lib"], check=True, cwd=REPO)
    os.replace(tmp, BINARY)
    return BINARY


if __name__ == "__main__":
    print(build(force=True))

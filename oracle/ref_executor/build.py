"""Builds oracle/_ref/native_executor_replay: the reference's own stage
executor linked against this repository's engine (test infrastructure).

The reference's runtime/adapters/native_stage_executor.{hpp,cpp},
runtime/inference/stage.cpp and runtime/inference/token_payload.cpp are
compiled from where they lie under the reference tree, with this
repository's include/ first on the include path, so that their
`#include "jetsonfabric/native_inference.hpp"` resolves to the drop-in header
and every engine call lands in libjfb.so. The executor gets one addition: the
`execute_batch` override of runtime/inference/executor.hpp:20-29, whose body
is this directory's execute_batch.inc. The reference files are read, the
declaration, the method and two includes are inserted at fixed anchors, and
the result is written under oracle/_ref/executor/ (git-ignored), never into
the repository. replay.cpp is the driver.

Nothing is built when the reference tree is absent (on the GPU hosts the
prebuilt binary travels with the repository instead).
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
OUT = REPO / "oracle" / "_ref"
BINARY = OUT / "native_executor_replay"


def reference_root() -> Path | None:
    root = Path(os.environ.get("JFB_REFERENCE", "/root/reference"))
    return root if (root / "runtime" / "adapters" / "native_stage_executor.cpp").exists() else None


def _insert(text: str, anchor: str, addition: str, before: bool = True) -> str:
    if text.count(anchor) != 1:
        raise RuntimeError(f"anchor not found exactly once in the reference executor: {anchor!r}")
    return text.replace(anchor, addition + anchor if before else anchor + addition)


def prepare_sources(ref: Path) -> Path:
    src = OUT / "executor"
    (src / "adapters").mkdir(parents=True, exist_ok=True)
    hpp = (ref / "runtime" / "adapters" / "native_stage_executor.hpp").read_text()
    hpp = _insert(hpp, "    void close_session(const std::string& session_id) const override;\n",
                  "    std::vector<inference::ExecutionResult> execute_batch(\n"
                  "        const std::vector<inference::StageInput>& inputs) const override;\n")
    hpp = _insert(hpp, "#include <memory>\n", "#include <vector>\n")
    cpp = (ref / "runtime" / "adapters" / "native_stage_executor.cpp").read_text()
    cpp = _insert(cpp, '#include "inference/token_payload.hpp"\n',
                  '#include "jetsonfabric/native_batch.hpp"\n\n#include <algorithm>\n', before=False)
    cpp = _insert(cpp, "    std::size_t session_count() const {\n", (HERE / "execute_batch.inc").read_text())
    cpp = _insert(cpp, "void NativeStageExecutor::close_session(",
                  "std::vector<inference::ExecutionResult> NativeStageExecutor::execute_batch(\n"
                  "    const std::vector<inference::StageInput>& inputs\n"
                  ") const {\n    return impl_->execute_batch(inputs);\n}\n\n")
    (src / "adapters" / "native_stage_executor.hpp").write_text(hpp)
    (src / "adapters" / "native_stage_executor.cpp").write_text(cpp)
    return src


CONFIG_BINARIES = {"reference": OUT / "worker_config_reference", "lifted": OUT / "worker_config_lifted"}
# the native engine's single-decode restriction in the reference worker
# (runtime/worker/config.cpp:159-162), removed in the "lifted" build
DECODE_BATCH_CHECK = (
    "        if (cfg.decode_batch_size != 1) {\n"
    "            throw std::invalid_argument(\n"
    "                \"native serving currently requires --decode-batch-size 1\"\n"
    "            );\n"
    "        }\n"
)


def build_config_checks(force: bool = False) -> dict | None:
    """The reference worker's config validation around config_check.cpp, as
    it is and with the decode-batch restriction lifted."""
    ref = reference_root()
    if ref is None:
        return CONFIG_BINARIES if all(p.exists() for p in CONFIG_BINARIES.values()) else None
    inputs = [HERE / "config_check.cpp", HERE / "build.py"]
    if not force and all(p.exists() and all(p.stat().st_mtime > i.stat().st_mtime for i in inputs)
                         for p in CONFIG_BINARIES.values()):
        return CONFIG_BINARIES
    rt = ref / "runtime"
    lifted_dir = OUT / "executor" / "worker"
    lifted_dir.mkdir(parents=True, exist_ok=True)
    text = (rt / "worker" / "config.cpp").read_text()
    if text.count(DECODE_BATCH_CHECK) != 1:
        raise RuntimeError("the reference worker's decode-batch check was not found exactly once")
    (lifted_dir / "config.cpp").write_text(text.replace(DECODE_BATCH_CHECK, ""))
    deps = [str(rt / "protocol" / "execution_mode.cpp"), str(rt / "pipeline_parallel" / "stage_assignment.cpp"),
            str(rt / "tensor_parallel" / "device_mesh.cpp")]
    for kind, config_src in (("reference", rt / "worker" / "config.cpp"), ("lifted", lifted_dir / "config.cpp")):
        target = CONFIG_BINARIES[kind]
        tmp = target.with_suffix(".tmp")
        subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", f"-I{rt}", str(HERE / "config_check.cpp"),
                        str(config_src)] + deps + ["-o", str(tmp)], check=True, cwd=REPO)
        os.replace(tmp, target)
    return CONFIG_BINARIES


def build(force: bool = False) -> Path | None:
    ref = reference_root()
    if ref is None:
        return BINARY if BINARY.exists() else None
    lib = REPO / "jetsonfabric_b200" / "lib"
    inputs = [HERE / "replay.cpp", HERE / "execute_batch.inc", HERE / "build.py", lib / "libjfb.so"]
    if not force and BINARY.exists() and all(BINARY.stat().st_mtime > p.stat().st_mtime for p in inputs):
        return BINARY
    src = prepare_sources(ref)
    tmp = BINARY.with_suffix(".tmp")
    cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-pthread",
           f"-I{src}", f"-I{REPO / 'include'}", f"-I{ref / 'runtime'}",
           str(src / "adapters" / "native_stage_executor.cpp"),
           str(ref / "runtime" / "inference" / "stage.cpp"),
           str(ref / "runtime" / "inference" / "token_payload.cpp"),
           str(ref / "runtime" / "pipeline_parallel" / "continuous_batching_executor.cpp"),
           str(HERE / "replay.cpp"),
           f"-L{lib}", "-ljfb", "-Wl,-rpath,$ORIGIN/../../jetsonfabric_b200/lib", "-o", str(tmp)]
    subprocess.run(cmd, check=True, cwd=REPO)
    os.replace(tmp, BINARY)
    return BINARY


if __name__ == "__main__":
    print(build(force=True))
    print(build_config_checks(force=True))

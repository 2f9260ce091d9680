"""The reference's own NativeStageExecutor over this repository's engine.

oracle/ref_executor/build.py compiles the reference's
runtime/adapters/native_stage_executor.cpp (plus the execute_batch override
this repository adds), runtime/inference/stage.cpp and token_payload.cpp
against include/jetsonfabric/native_inference.hpp and links libjfb.so. The
GPU test runs the resulting replay of the reference's executor test
(runtime/adapters/native_stage_executor_test.cpp:85-235) on the reference's
2-layer fixture package, on the CUDA backend, plus a batched decode through
execute_batch, and the reference's ContinuousBatchingExecutor coalescing
three concurrent decode steps into one execute_batch call.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "oracle" / "ref_executor"))
import build as executor_build  # noqa: E402


def replay_binary() -> Path | None:
    from jetsonfabric_b200 import build_cuda
    build_cuda.build()
    return executor_build.build()


def test_reference_executor_compiles_against_the_drop_in_headers():
    if executor_build.reference_root() is None and not executor_build.BINARY.exists():
        pytest.skip("the reference tree is not on this machine and no prebuilt replay exists")
    binary = replay_binary()
    assert binary is not None and binary.exists()
    # the executor's engine calls resolve in this repository's library
    out = subprocess.run(["ldd", str(binary)], capture_output=True, text=True).stdout
    assert "libjfb.so" in out


@pytest.mark.gpu
def test_reference_executor_replay_on_cuda(fixture_package):
    binary = replay_binary()
    if binary is None:
        pytest.fail("the replay binary was not built (oracle/ref_executor/build.py needs the reference tree once)")
    r = subprocess.run([str(binary), str(fixture_package)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "replay ok" in r.stdout


@pytest.mark.parametrize("args,reference,lifted", [
    (["4", "8", "cuda"], "rejected: native serving currently requires --decode-batch-size 1", "accepted"),
    (["1", "8", "cuda"], "accepted", "accepted"),
    (["9", "8", "cuda"], "rejected: --decode-batch-size must be between 1 and --parallel-sessions", None),
    (["4", "8", "rocm"], "rejected: native compute backend must be cpu or cuda", None),
])
def test_worker_config_lift(args, reference, lifted):
    """The reference worker's own config validation (runtime/worker/
    config.cpp), compiled as it is and with the native engine's
    decode_batch_size == 1 check removed: only that restriction changes, every
    other check stays."""
    binaries = executor_build.build_config_checks()
    if binaries is None:
        pytest.skip("the reference tree is not on this machine and no prebuilt config checks exist")
    out = {k: subprocess.run([str(p)] + args, capture_output=True, text=True, check=True).stdout.strip()
           for k, p in binaries.items()}
    assert out["reference"] == reference
    assert out["lifted"] == (lifted if lifted is not None else reference)

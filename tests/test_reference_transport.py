"""The in-box StageTransport inside the reference runtime.

oracle/ref_transport/build.py compiles the reference's GenerationRunner,
StageWorker, activation codecs, Stagewire codec and stage executors around
jetsonfabric_b200/csrc/transport/inbox_stage_transport.cpp, registered
through the reference's StageTransportFactory. The driver it builds runs
stage servers as separate processes and the reference's generation loop
against them:

- the refusal paths of HTTPStageTransport::invoke, restated for the channel
  (missing or wrong cluster token, a stage that is not in-box, no server,
  worker refusals as error frames, encoder refusals, oversized frames, a peer
  acknowledging another operation), then the channel still serving;
- three synthetic stages (the reference's SyntheticActivationExecutor, whose
  tokens hash the activation bytes it receives) served by three processes
  give exactly the tokens of the same workers called in-process;
- on a GPU, two native stages over this repository's engine, each in its own
  process, give exactly the CPU oracle's greedy tokens for the chained
  stages with the F16 codec at the boundary.
"""
from __future__ import annotations

import importlib.util
import json
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent


def _load_build():
    spec = importlib.util.spec_from_file_location("jfb_ref_transport_build",
                                                  REPO / "oracle" / "ref_transport" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


transport_build = _load_build()


def driver() -> Path:
    from jetsonfabric_b200 import build_cuda
    build_cuda.build()
    binary = transport_build.build()
    if binary is None:
        pytest.skip("the reference tree is not on this machine and no prebuilt transport driver exists")
    return binary


def _serve(binary, channel, token, args, env=None, idle_ms=3000):
    """A stage server process; it exits once no request has come for idle_ms."""
    return subprocess.Popen([str(binary), "serve", channel, token, str(idle_ms)] + args, stdout=subprocess.PIPE,
                            stderr=subprocess.PIPE, text=True, env=env)


def _finish(servers):
    outs = []
    for p in servers:
        try:
            out, err = p.communicate(timeout=60)
        except subprocess.TimeoutExpired:
            p.kill()
            out, err = p.communicate()
        outs.append((p.returncode, out, err))
    return outs


def test_transport_refusal_paths():
    binary = driver()
    r = subprocess.run([str(binary), "errors"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "errors ok" in r.stdout


def test_synthetic_stages_over_the_transport_match_in_process():
    binary = driver()
    tag = f"jfbt{os.getpid()}"
    servers = [_serve(binary, f"{tag}-{i}", "tok", ["synthetic", str(i), "3", str(i), str(i + 1)]) for i in range(3)]
    try:
        r = subprocess.run([str(binary), "generate", "tok", "6", "11 12 13 14", "sess"] +
                           [f"{tag}-{i}:{i}:{i + 1}" for i in range(3)], capture_output=True, text=True, timeout=120)
    finally:
        outs = _finish(servers)
    assert r.returncode == 0, r.stdout + r.stderr
    remote = json.loads(r.stdout.strip().splitlines()[-1])
    local = subprocess.run([str(binary), "local", "6", "11 12 13 14", "sess", "0:1", "1:2", "2:3"],
                           capture_output=True, text=True, timeout=60)
    assert local.returncode == 0, local.stderr
    expect = json.loads(local.stdout.strip().splitlines()[-1])
    assert remote["ok"] and len(remote["tokens"]) == 6
    assert remote["tokens"] == expect["tokens"]
    assert (remote["bytes_in"], remote["bytes_out"]) == (expect["bytes_in"], expect["bytes_out"])
    for rc, out, err in outs:
        assert rc == 0, err
        # prefill + 5 decode steps + close on every stage
        assert "served 7" in out


@pytest.mark.gpu
def test_native_stages_over_the_transport_match_oracle(small_q4k_package):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    from tests.test_gpu_pipeline import oracle_chain

    binary = driver()
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, 1024, 9).tolist()
    steps = 8
    ranges = [(0, 2), (2, 4)]
    tag = f"jfbn{os.getpid()}"
    gpus = torch.cuda.device_count()
    servers = []
    for i, (a, b) in enumerate(ranges):
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(i % gpus))
        servers.append(_serve(binary, f"{tag}-{i}", "tok",
                              ["native", str(small_q4k_package), str(i), "2", str(a), str(b), "64"], env=env,
                              idle_ms=15000))
    try:
        r = subprocess.run([str(binary), "generate", "tok", str(steps), " ".join(map(str, prompt)), "sess"] +
                           [f"{tag}-{i}:{a}:{b}" for i, (a, b) in enumerate(ranges)],
                           capture_output=True, text=True, timeout=300)
    finally:
        outs = _finish(servers)
    assert r.returncode == 0, r.stdout + r.stderr + "".join(e for _, _, e in outs)
    got = json.loads(r.stdout.strip().splitlines()[-1])
    assert got["ok"], got
    assert got["tokens"] == oracle_chain(small_q4k_package, ranges, [prompt], steps)[0]
    for rc, _, err in outs:
        assert rc == 0, err

"""Parity at the benchmark configurations' shapes, through the C ABI.

The engine tests elsewhere use small models. These run the shapes the
benchmark serves, against the CPU oracle (the GGML-CPU restatement):

- the full 28-layer configuration 1 (Qwen2 1.5B Q4_K_M: hidden 1536, 12/2
  heads, FFN 8960, 151,936 tokens): two concurrent 128-token prompts and 128
  greedy tokens each, batched exactly as the reference's bench serves it
  (runtime/benchmarks/native_inference_bench.cpp drives NativeEngine the same
  way), plus bit-exact prefill logits;
- two layers at the widths of configurations 3, 4 and 5: 7B (hidden 3584,
  28/4 heads so 7 query heads per kv head, FFN 18944 = 74 blocks), 14B
  (hidden 5120, 40/8 heads, FFN 13824) and 32B with Q2_K layers and a Q6_K
  head (FFN 27648), with the 152,064-token vocabulary. Nine sequences decode
  in one batch so the decode matmuls take the tensor-core path, as in the
  benchmark.

Greedy tokens must be identical and logits bit-identical (which implies the
2e-2 max-abs / 1e-3 relative tolerance, also asserted).
"""
from __future__ import annotations

import numpy as np
import pytest

from jetsonfabric_b200 import jfm
from oracle import binding as ob

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

LOGIT_MAX_ABS = 2e-2
LOGIT_REL = 1e-3


@pytest.fixture(scope="module")
def E():
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    from jetsonfabric_b200 import engine
    return engine


def check_logits(got: np.ndarray, ref: np.ndarray):
    max_abs = float(np.abs(got - ref).max())
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    assert max_abs <= LOGIT_MAX_ABS and rel <= LOGIT_REL, (max_abs, rel)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), ("not bit-identical", max_abs, rel)


def oracle_stream(oracle, prompt, steps):
    s = oracle.session(len(prompt) + steps)
    toks = [s.forward(True, tokens=prompt)["token"]]
    for _ in range(steps - 1):
        toks.append(s.forward(False, tokens=[toks[-1]])["token"])
    return toks


def engine_streams(eng, prompts, steps):
    sessions = [eng.create_session(len(p) + steps) for p in prompts]
    cur = [r.sampled_token for r in eng.prefill_stage_batch(sessions, prompts)]
    got = [[t] for t in cur]
    for _ in range(steps - 1):
        cur = [r.sampled_token for r in eng.decode_stage_batch(sessions, cur)]
        for g, t in zip(got, cur):
            g.append(t)
    for s in sessions:
        s.close()
    return got


@pytest.fixture(scope="module")
def cfg1_package(tmp_path_factory):
    d = tmp_path_factory.mktemp("cfg1") / "qwen2-1.5b.jfm"
    jfm.write_synthetic_package(d, **jfm.QWEN2_PRESETS["1.5b"], context_length=4096, seed=2026,
                                draw_norms=False, draw_biases=True)
    return d


def test_cfg1_full_depth_two_streams_128_tokens(E, cfg1_package):
    vocab = jfm.QWEN2_PRESETS["1.5b"]["vocabulary_size"]
    rng = np.random.default_rng(2026)
    prompts = [rng.integers(0, vocab, 128).tolist() for _ in range(2)]
    steps = 128
    oracle = ob.OracleStage(cfg1_package)
    ref = [oracle_stream(oracle, p, steps) for p in prompts]
    ref_logits = oracle.session(128).forward(True, tokens=prompts[0], want_logits=True)["logits"]
    oracle.close()
    with E.NativeEngine(cfg1_package, "cuda") as eng:
        assert eng.model_info().layer_count == 28
        got = engine_streams(eng, prompts, steps)
        check_logits(eng.logits(prompts[0]), ref_logits)
    for g, r in zip(got, ref):
        assert len(g) == steps
        first_diff = next((i for i, (a, b) in enumerate(zip(g, r)) if a != b), None)
        assert first_diff is None, f"greedy stream diverged at step {first_diff}"


WIDTHS = {
    "7b": jfm.QWEN2_PRESETS["7b"],
    "14b": jfm.QWEN2_PRESETS["14b"],
    "32b-q2k": jfm.QWEN2_PRESETS["32b"],
}


@pytest.mark.parametrize("name", list(WIDTHS))
def test_two_layers_at_config_width(E, tmp_path, name):
    shape = dict(WIDTHS[name])
    shape["layer_count"] = 2
    pkg = tmp_path / f"{name}.jfm"
    jfm.write_synthetic_package(pkg, **shape, context_length=4096, seed=31, draw_norms=True, draw_biases=True)
    vocab = shape["vocabulary_size"]
    rng = np.random.default_rng(77)
    # nine sequences: prefill of 9 ragged prompts (one batched call), then
    # 9-row decode steps, which run the tensor-core matmuls
    prompts = [rng.integers(0, vocab, n).tolist() for n in (24, 7, 31, 1, 16, 12, 40, 5, 19)]
    steps = 12
    oracle = ob.OracleStage(pkg)
    ref = [oracle_stream(oracle, p, steps) for p in prompts]
    ref_logits = [oracle.session(len(p)).forward(True, tokens=p, want_logits=True)["logits"] for p in prompts[:2]]
    oracle.close()
    with E.NativeEngine(pkg, "cuda") as eng:
        got = engine_streams(eng, prompts, steps)
        for p, r in zip(prompts[:2], ref_logits):
            check_logits(eng.logits(p), r)
    assert got == ref

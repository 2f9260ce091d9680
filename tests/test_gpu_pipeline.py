"""Pipeline stages on one GPU: two NativeEngine stages over layer ranges,
chained through the device-resident stage entry point
(jfb_engine_stage_batch_device) and the device F16 codec, must give exactly
the greedy tokens of the CPU oracle's chained stages with the same codec at
the boundary. The multi-GPU benchmark runs the same stages with NCCL between
processes (jetsonfabric_b200/pipeline.py, checked on CPU by
test_pipeline_gloo.py).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import binding as ob

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def E():
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    from jetsonfabric_b200 import engine
    return engine


def oracle_chain(package, ranges, prompts, steps):
    stages = [ob.OracleStage(package, a, b) for a, b in ranges]
    capacity = max(len(p) for p in prompts) + steps
    out = []
    for prompt in prompts:
        sessions = [st.session(capacity) for st in stages]
        tokens, feed = [], list(prompt)
        for step in range(steps):
            x = None
            for k, sess in enumerate(sessions):
                r = sess.forward(step == 0, tokens=feed) if k == 0 else sess.forward(step == 0, activations=x)
                if k + 1 < len(sessions):
                    x = r["activations"].astype(np.float16).astype(np.float32)
                else:
                    tokens.append(r["token"])
            feed = [tokens[-1]]
        out.append(tokens)
    return out


def test_two_device_stages_match_oracle_chain(E, small_q4k_package):
    from jetsonfabric_b200 import kernels as K
    from jetsonfabric_b200 import pipeline as PL

    ranges = PL.stage_ranges(4, 2)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 1024, n).tolist() for n in (9, 4, 13)]
    steps = 8
    capacity = max(len(p) for p in prompts) + steps
    engines = [E.NativeEngine(small_q4k_package, "cuda", layer_start=a, layer_end=b) for a, b in ranges]
    try:
        sessions = [[eng.create_session(capacity) for _ in prompts] for eng in engines]
        hidden = engines[0].model_info().embedding_length
        counts = [len(p) for p in prompts]
        prompt_dev = torch.tensor([t for p in prompts for t in p], dtype=torch.int32, device="cuda")
        got = [[] for _ in prompts]
        tokens = None
        for step in range(steps):
            prefill = step == 0
            rows = sum(counts) if prefill else len(prompts)
            acts = torch.empty((rows, hidden), dtype=torch.float32, device="cuda")
            engines[0].stage_batch_device(sessions[0], prefill, counts if prefill else None,
                                          tokens_ptr=(prompt_dev if prefill else tokens).data_ptr(),
                                          activations_out_ptr=acts.data_ptr())
            engines[0].synchronize()
            payload = torch.empty((rows, hidden), dtype=torch.float16, device="cuda")
            K.codec_f32_to_f16(acts, payload)
            back = torch.empty_like(acts)
            K.codec_f16_to_f32(payload, back)
            torch.cuda.synchronize()
            tokens = torch.empty(len(prompts), dtype=torch.int32, device="cuda")
            engines[1].stage_batch_device(sessions[1], prefill, counts if prefill else None,
                                          activations_ptr=back.data_ptr(), tokens_out_ptr=tokens.data_ptr())
            engines[1].synchronize()
            for i, t in enumerate(tokens.cpu().tolist()):
                got[i].append(t)
        assert got == oracle_chain(small_q4k_package, ranges, prompts, steps)
        # wrong input kind for a stage is rejected before any launch
        with pytest.raises(E.InvalidArgument):
            engines[1].stage_batch_device(sessions[1], False, tokens_ptr=tokens.data_ptr(),
                                          tokens_out_ptr=tokens.data_ptr())
        for group in sessions:
            for s in group:
                s.close()
    finally:
        for eng in engines:
            eng.close()

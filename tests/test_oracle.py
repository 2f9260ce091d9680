"""Pins the CPU oracle before it is trusted as the parity checker.

- K-quant dequantization is bit-exact against gguf-py 0.19's NumPy
  dequantizers (an independent implementation of GGML's formats).
- The reference's known-answer tests on its 2-layer F32 fixture:
  prompt [2] -> greedy [7, 7] (runtime/compiler/compiler_integration_test.cmake:55-81),
  alternate prompt [2, 2] -> [7] (114-139), token 8 rejected (163-180), and the
  two-stage 0-1 / 1-2 split also yields 7 (adapters/native_stage_executor_test.cpp:139-235).
- Q8_K quantization properties, RoPE and F16 codec edge cases.
"""
from __future__ import annotations

import numpy as np
import pytest

from jetsonfabric_b200 import jfm
from oracle import binding as ob

gguf = pytest.importorskip("gguf")
from gguf.quants import dequantize as gguf_dequantize  # noqa: E402

GGUF_TYPES = {jfm.JF_TENSOR_Q4_K: gguf.GGMLQuantizationType.Q4_K,
              jfm.JF_TENSOR_Q6_K: gguf.GGMLQuantizationType.Q6_K,
              jfm.JF_TENSOR_Q2_K: gguf.GGMLQuantizationType.Q2_K}


@pytest.mark.parametrize("jf_type", list(GGUF_TYPES))
def test_dequant_bit_exact_vs_gguf_py(jf_type):
    rng = np.random.default_rng(jf_type)
    values = np.concatenate([rng.normal(0, 0.02, 256 * 32), rng.normal(0, 3.0, 256 * 8),
                             np.zeros(256), -np.abs(rng.normal(0, 1, 256))]).astype(np.float32)
    raw = jfm.quantize_blocks(jf_type, values)
    mine = ob.dequantize(jf_type, raw, values.size)
    ref = gguf_dequantize(np.frombuffer(raw, dtype=np.uint8), GGUF_TYPES[jf_type]).ravel()
    assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32))


def test_dequant_bit_exact_on_package_tensors(small_q4k_package):
    with jfm.Model(small_q4k_package) as m:
        for t in m.tensors():
            if t.type not in GGUF_TYPES:
                continue
            n = t.shape[0] * t.shape[1]
            mine = ob.dequantize(t.type, t.bytes(), n)
            ref = gguf_dequantize(np.frombuffer(t.bytes(), dtype=np.uint8), GGUF_TYPES[t.type]).ravel()
            assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32)), t.name


BLOCK_BYTES = {jfm.JF_TENSOR_Q4_K: 144, jfm.JF_TENSOR_Q6_K: 210, jfm.JF_TENSOR_Q2_K: 84}
# byte offsets of the f16 block scales (d, dmin) inside each block
SCALE_OFFSETS = {jfm.JF_TENSOR_Q4_K: (0, 2), jfm.JF_TENSOR_Q6_K: (208,), jfm.JF_TENSOR_Q2_K: (80, 82)}


@pytest.mark.parametrize("jf_type", list(GGUF_TYPES))
def test_vectorised_dot_matches_scalar_dot(jf_type):
    """orc_matmul's AVX2 path forms the same integer sums as the scalar
    restatement of ggml_vec_dot_*_q8_K: random raw blocks over the full code,
    scale and min ranges, random Q8_K blocks with codes in [-127, 127]."""
    import ctypes as C
    L = ob.lib()
    assert L.orc_q8k_block_bytes() == 292
    rng = np.random.default_rng(100 + jf_type)
    for nb in (1, 3, 14, 74):
        for trial in range(8):
            w = rng.integers(0, 256, nb * BLOCK_BYTES[jf_type], dtype=np.uint8).reshape(nb, -1)
            for off in SCALE_OFFSETS[jf_type]:
                w[:, off:off + 2] = np.frombuffer(rng.normal(0, 0.05, nb).astype(np.float16).tobytes(),
                                                  dtype=np.uint8).reshape(nb, 2)
            if trial == 0:  # extreme codes and scales
                w[:, :] = 0xFF
                for off in SCALE_OFFSETS[jf_type]:
                    w[:, off:off + 2] = np.frombuffer(np.float16(0.5).tobytes(), dtype=np.uint8)
            qs = rng.integers(-127, 128, (nb, 256)).astype(np.int8)
            if trial == 1:
                qs[:] = -127
            a = np.zeros((nb, 292), dtype=np.uint8)
            a[:, 0:4] = np.frombuffer(rng.uniform(1e-4, 1e-1, nb).astype(np.float32).tobytes(), dtype=np.uint8).reshape(nb, 4)
            a[:, 4:260] = qs.view(np.uint8)
            a[:, 260:292] = qs.astype(np.int16).reshape(nb, 16, 16).sum(axis=2).astype(np.int16).view(np.uint8).reshape(nb, 32)
            wp, ap = np.ascontiguousarray(w), np.ascontiguousarray(a)
            s = L.orc_dot_kquant_scalar(jf_type, wp.ctypes.data, ap.ctypes.data, nb)
            v = L.orc_dot_kquant_vector(jf_type, wp.ctypes.data, ap.ctypes.data, nb)
            assert np.float32(s).view(np.uint32) == np.float32(v).view(np.uint32), (nb, trial, s, v)


def test_q8_k_quantization_properties():
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 256 * 8).astype(np.float32)
    x[256:512] = 0.0                      # all-zero block
    x[512 + 7] = -5.0                     # negative extreme: iscale = -127/-5 > 0
    x[768:1024] *= 0.1
    x[768 + 3], x[768 + 9] = 2.0, -2.0    # tie in magnitude: the first (+2) sets the sign
    d, qs, bs = ob.split_q8_k(ob.quantize_q8_k(x), x.size)
    assert d[1] == 0 and not qs[256:512].any()
    assert qs[512 + 7] == -127 and d[2] > 0
    assert qs[768 + 3] == -127 and qs[768 + 9] == 127 and d[3] < 0
    assert np.all(qs >= -127) and np.all(qs <= 127)
    assert np.array_equal(bs, qs.reshape(-1, 16).astype(np.int32).sum(1).astype(np.int16))
    recon = (qs.reshape(8, 256).astype(np.float32) * d[:, None]).ravel()
    assert np.abs(recon - x).max() <= np.abs(x).reshape(8, 256).max(1).max() / 127 * 0.5001 + 1e-7


def test_reference_fixture_greedy_tokens(fixture_package):
    stage = ob.OracleStage(fixture_package)
    s = stage.session(2)  # prompt 1 + max_tokens 2 - 1
    first = s.forward(True, tokens=[2])["token"]
    second = s.forward(False, tokens=[first])["token"]
    assert [first, second] == [7, 7]
    alt = stage.session(2).forward(True, tokens=[2, 2])["token"]
    assert alt == 7
    with pytest.raises(ob.OracleError, match="outside model vocabulary"):
        stage.session(2).forward(True, tokens=[8])


def test_reference_fixture_two_stage_split(fixture_package):
    a, b = ob.OracleStage(fixture_package, 0, 1), ob.OracleStage(fixture_package, 1, 2)
    sa, sb = a.session(2), b.session(2)
    x = sa.forward(True, tokens=[2])["activations"]
    assert x.shape == (1, 4)
    t1 = sb.forward(True, activations=x)["token"]
    t2 = sb.forward(False, activations=sa.forward(False, tokens=[t1])["activations"])["token"]
    assert [t1, t2] == [7, 7]


def test_session_position_rules(fixture_package):
    stage = ob.OracleStage(fixture_package)
    s = stage.session(4)
    with pytest.raises(ob.OracleError, match="decode is outside"):
        s.forward(False, tokens=[1])
    s.forward(True, tokens=[1, 2])
    with pytest.raises(ob.OracleError, match="prefill is outside"):
        s.forward(True, tokens=[1])
    s.forward(False, tokens=[3])
    s.forward(False, tokens=[3])
    with pytest.raises(ob.OracleError, match="decode is outside"):
        s.forward(False, tokens=[3])
    with pytest.raises(ob.OracleError, match="rollback"):
        s.rollback(3)
    s.rollback(2)
    assert s.position == 2


def test_rollback_replays_identically(small_q4k_package):
    stage = ob.OracleStage(small_q4k_package)
    s = stage.session(16)
    prompt = [5, 17, 300, 2]
    t = s.forward(True, tokens=prompt)["token"]
    a = s.forward(False, tokens=[t], want_logits=True)
    b = s.forward(False, tokens=[a["token"]], want_logits=True)
    s.rollback(2)
    a2 = s.forward(False, tokens=[t], want_logits=True)
    b2 = s.forward(False, tokens=[a2["token"]], want_logits=True)
    assert np.array_equal(a["logits"], a2["logits"]) and np.array_equal(b["logits"], b2["logits"])


def test_incremental_decode_matches_full_prefill(small_q4k_package):
    """Decode with the KV cache equals a fresh prefill of the whole prefix for
    the same last row (the oracle's cache semantics are self-consistent)."""
    stage = ob.OracleStage(small_q4k_package)
    prompt = [11, 22, 33, 44, 55]
    s = stage.session(8)
    s.forward(True, tokens=prompt[:3])
    s.forward(False, tokens=[prompt[3]])
    inc = s.forward(False, tokens=[prompt[4]], want_logits=True)["logits"]
    full = stage.session(8).forward(True, tokens=prompt, want_logits=True)["logits"]
    np.testing.assert_allclose(inc, full, rtol=0, atol=1e-5)


def test_rope_neox_rotation():
    x = np.arange(2 * 8, dtype=np.float32).reshape(2, 8).copy()
    orig = x.copy()
    ob.lib().orc_rope_neox(x.ctypes.data, 2, 8, 8, 0, 10000.0)
    assert np.array_equal(x, orig)  # position 0 is the identity
    ob.lib().orc_rope_neox(x.ctypes.data, 2, 8, 8, 3, 10000.0)
    theta_scale = np.float32(10000.0) ** np.float32(-2.0 / 8)
    theta = np.float32(3.0)
    for i in range(4):
        c, s = np.cos(theta), np.sin(theta)
        np.testing.assert_allclose(x[0, i], orig[0, i] * c - orig[0, i + 4] * s, rtol=1e-6)
        np.testing.assert_allclose(x[0, i + 4], orig[0, i] * s + orig[0, i + 4] * c, rtol=1e-6)
        theta = np.float32(theta * theta_scale)


def test_f16_codec_matches_reference_rules():
    L = ob.lib()
    cases = {1.0: 0x3C00, -2.0: 0xC000, 65504.0: 0x7BFF, 65520.0: 0x7C00, 1e-8: 0x0000,
             5.960464477539063e-08: 0x0001, float("inf"): 0x7C00, -0.0: 0x8000}
    for v, h in cases.items():
        assert L.orc_codec_float_to_half(v) == h, v
    # NaN keeps payload bits and is made quiet
    import struct
    nan = struct.unpack("<f", struct.pack("<I", 0x7F800001 | (0x155 << 13)))[0]
    assert L.orc_codec_float_to_half(nan) == (0x7C00 | 0x155 | 0x200)
    for h in [0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0xFC00, 0x8001]:
        v = L.orc_codec_half_to_float(h)
        assert L.orc_codec_float_to_half(v) == h

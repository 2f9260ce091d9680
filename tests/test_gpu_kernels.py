"""Kernel-level parity of the sm_100a library against the CPU oracle.

Every op is bit-exact against the oracle: K-quant dequantization (also
against gguf-py), Q8_K activation quantization, RMSNorm, the K-quant and
float matmuls (exact integer sub-block sums, per-block float terms summed in
double), SwiGLU and its exp, RoPE with the KV append, attention, the F16
activation codec and argmax.
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np
import pytest

from jetsonfabric_b200 import jfm
from oracle import binding as ob

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KQ = [jfm.JF_TENSOR_Q4_K, jfm.JF_TENSOR_Q6_K, jfm.JF_TENSOR_Q2_K]


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    from jetsonfabric_b200 import kernels
    return kernels


def make_weight(K, jf_type, rows, cols, seed, std=0.02):
    rng = np.random.default_rng(seed)
    values = rng.normal(0, std, rows * cols).astype(np.float32)
    if jf_type == jfm.JF_TENSOR_F32:
        raw = values.tobytes()
    elif jf_type == jfm.JF_TENSOR_F16:
        raw = values.astype(np.float16).tobytes()
    else:
        raw = jfm.quantize_blocks(jf_type, values)
    return K.DeviceWeight(jf_type, rows, cols, raw), raw


@pytest.mark.parametrize("jf_type", KQ + [jfm.JF_TENSOR_F32, jfm.JF_TENSOR_F16])
def test_dequantize_bit_exact(K, jf_type):
    rows, cols = 48, 1024
    w, raw = make_weight(K, jf_type, rows, cols, 1)
    gpu = w.dequantize().cpu().numpy().ravel()
    ref = ob.dequantize(jf_type, raw, rows * cols)
    assert np.array_equal(gpu.view(np.uint32), ref.view(np.uint32))
    if jf_type in KQ:
        from gguf.quants import dequantize as gd
        import gguf
        gt = {jfm.JF_TENSOR_Q4_K: gguf.GGMLQuantizationType.Q4_K, jfm.JF_TENSOR_Q6_K: gguf.GGMLQuantizationType.Q6_K,
              jfm.JF_TENSOR_Q2_K: gguf.GGMLQuantizationType.Q2_K}[jf_type]
        assert np.array_equal(gpu.view(np.uint32), gd(np.frombuffer(raw, np.uint8), gt).ravel().view(np.uint32))


def q8_reference(x: np.ndarray):
    raw = ob.quantize_q8_k(x)
    return ob.split_q8_k(raw, x.size)


def test_quantize_q8k_bit_exact(K):
    rng = np.random.default_rng(2)
    rows, cols = 37, 2048
    x = rng.normal(0, 1, (rows, cols)).astype(np.float32)
    x[3, :256] = 0.0                                   # zero block
    x[5, 10], x[5, 20] = 4.0, -4.0                      # magnitude tie
    x[7] *= 1e-30                                      # tiny values
    x[9, 300] = 1e6                                    # extreme
    xt = torch.from_numpy(x).cuda()
    out = K.Q8Buffer(rows, cols)
    K.quantize_q8k(xt, out)
    torch.cuda.synchronize()
    for r in range(rows):
        d, qs, bs = q8_reference(x[r])
        assert np.array_equal(out.qs[r].cpu().numpy(), qs), r
        assert np.array_equal(out.d[r].cpu().numpy().view(np.uint32), d.view(np.uint32)), r
        assert np.array_equal(out.bsums[r].cpu().numpy(), bs), r


@pytest.mark.parametrize("cols", [4, 1536, 2048, 5120, 1540, 1538, 3])
def test_rmsnorm_quant_bit_exact(K, cols):
    rng = np.random.default_rng(cols)
    rows = 9
    x = rng.normal(0, 2, (rows, cols)).astype(np.float32)
    w = (1 + rng.normal(0, 0.1, cols)).astype(np.float32)
    xt, wt = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out = torch.empty_like(xt)
    q8 = K.Q8Buffer(rows, cols) if cols % 256 == 0 else None
    K.rmsnorm_quant(xt, wt, 1e-6, out_f32=out, out_q8=q8)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for r in range(rows):
        ref = np.empty(cols, np.float32)
        ob.lib().orc_rms_norm(x[r].ctypes.data, w.ctypes.data, cols, C.c_float(1e-6), ref.ctypes.data)
        assert np.array_equal(got[r].view(np.uint32), ref.view(np.uint32)), r
        if q8 is not None:
            d, qs, bs = q8_reference(ref)
            assert np.array_equal(q8.qs[r].cpu().numpy(), qs)
            assert np.array_equal(q8.d[r].cpu().numpy().view(np.uint32), d.view(np.uint32))


def test_rmsnorm_row_gather(K):
    rng = np.random.default_rng(4)
    x = rng.normal(0, 1, (6, 512)).astype(np.float32)
    w = np.ones(512, np.float32)
    idx = torch.tensor([5, 0, 3], dtype=torch.int32, device="cuda")
    out = torch.empty((3, 512), dtype=torch.float32, device="cuda")
    K.rmsnorm_quant(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), 1e-6, out_f32=out, row_index=idx, rows=3)
    torch.cuda.synchronize()
    for i, r in enumerate([5, 0, 3]):
        ref = np.empty(512, np.float32)
        ob.lib().orc_rms_norm(x[r].ctypes.data, w.ctypes.data, 512, C.c_float(1e-6), ref.ctypes.data)
        assert np.array_equal(out[i].cpu().numpy(), ref)


@pytest.mark.parametrize("jf_type", KQ)
@pytest.mark.parametrize("rows_in", [1, 3, 8, 13, 32])
def test_matmul_matches_oracle(K, jf_type, rows_in):
    N, Kdim = 96, 2048
    w, raw = make_weight(K, jf_type, N, Kdim, 10 + jf_type)
    rng = np.random.default_rng(rows_in)
    x = rng.normal(0, 1, (rows_in, Kdim)).astype(np.float32)
    q8 = K.Q8Buffer(rows_in, Kdim)
    K.quantize_q8k(torch.from_numpy(x).cuda(), q8)
    bias = torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda()
    out = torch.empty((rows_in, N), dtype=torch.float32, device="cuda")
    K.matmul(w, rows_in, out, x_q8=q8, epilogue=K.EPILOGUE_BIAS, bias=bias)
    torch.cuda.synchronize()
    raw_np = np.frombuffer(raw, np.uint8)
    t = ob.OrcTensor(jf_type, 0, Kdim, N, raw_np.ctypes.data)
    ref = np.empty((rows_in, N), np.float32)
    ob.lib().orc_matmul(C.byref(t), x.ctypes.data, rows_in, ref.ctypes.data)
    ref += bias.cpu().numpy()
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("jf_type", [jfm.JF_TENSOR_F32, jfm.JF_TENSOR_F16])
def test_float_matmul_residual(K, jf_type):
    N, Kdim, rows_in = 40, 96, 5
    w, raw = make_weight(K, jf_type, N, Kdim, 3)
    rng = np.random.default_rng(6)
    x = rng.normal(0, 1, (rows_in, Kdim)).astype(np.float32)
    res = rng.normal(0, 1, (rows_in, N)).astype(np.float32)
    out = torch.from_numpy(res.copy()).cuda()
    K.matmul(w, rows_in, out, x_f32=torch.from_numpy(x).cuda(), epilogue=K.EPILOGUE_RESIDUAL, residual=out)
    torch.cuda.synchronize()
    t = ob.OrcTensor(jf_type, 0, Kdim, N, np.frombuffer(raw, np.uint8).ctypes.data)
    ref = np.empty((rows_in, N), np.float32)
    ob.lib().orc_matmul(C.byref(t), x.ctypes.data, rows_in, ref.ctypes.data)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), (ref + res).view(np.uint32))


def test_swiglu_quant(K):
    rng = np.random.default_rng(8)
    g = rng.normal(0, 4, (4, 1024)).astype(np.float32)
    g[0, :8] = [0.0, -0.0, 88.0, -88.0, 103.0, -103.0, 120.0, -120.0]   # exp range edges
    u = rng.normal(0, 2, (4, 1024)).astype(np.float32)
    out = torch.empty((4, 1024), dtype=torch.float32, device="cuda")
    q8 = K.Q8Buffer(4, 1024)
    K.swiglu_quant(torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda(), out_f32=out, out_q8=q8)
    torch.cuda.synchronize()
    L = ob.lib()
    ref = np.array([[L.orc_silu_mul(float(a), float(b)) for a, b in zip(gr, ur)] for gr, ur in zip(g, u)],
                   dtype=np.float32)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    d, qs, bs = q8_reference(ref[1])
    assert np.array_equal(q8.qs[1].cpu().numpy(), qs)


def test_argmax_first_max(K):
    x = np.random.default_rng(1).normal(0, 1, (4, 151936)).astype(np.float32)
    x[0, 17] = x[0, 99999] = 50.0          # tie: first index wins
    x[1, :] = -np.inf
    x[2, 5] = np.nan
    x[2, 6] = 30.0
    out = torch.empty(4, dtype=torch.int32, device="cuda")
    K.argmax(torch.from_numpy(x).cuda(), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().tolist()
    assert got[0] == 17 and got[1] == 0 and got[2] == 6
    assert got[3] == ob.lib().orc_argmax(x[3].ctypes.data, x.shape[1])


def test_codec_bit_exact(K):
    rng = np.random.default_rng(5)
    specials = [0.0, -0.0, 1.0, 65504.0, 65519.99, 65520.0, 1e-8, 5.96e-8, 6.1e-5, 6.0e-5, np.inf, -np.inf]
    vals = np.concatenate([rng.normal(0, 100, 20000), rng.normal(0, 1e-5, 5000), specials]).astype(np.float32)
    nan_bits = np.array([0x7F800001, 0x7FC00000, 0xFFBFFFFF, 0x7F801000 | (0x2AA << 13)], dtype=np.uint32)
    vals = np.concatenate([vals, nan_bits.view(np.float32)])
    x = torch.from_numpy(vals).cuda()
    h = torch.empty(vals.size, dtype=torch.int16, device="cuda")
    K.codec_f32_to_f16(x, h)
    back = torch.empty(vals.size, dtype=torch.float32, device="cuda")
    K.codec_f16_to_f32(h, back)
    torch.cuda.synchronize()
    got = h.cpu().numpy().view(np.uint16)
    ref = np.array([ob.lib().orc_codec_float_to_half(float(v)) for v in vals], dtype=np.uint16)
    # ctypes passes floats through a double: NaN payloads must be checked bitwise separately
    finite = np.isfinite(vals) | np.isinf(vals)
    assert np.array_equal(got[finite], ref[finite])
    for bits, g in zip(nan_bits, got[-4:]):
        mant = int(bits) & 0x7FFFFF
        assert g == (((int(bits) >> 16) & 0x8000) | 0x7C00 | (mant >> 13) | 0x200)
    widened = back.cpu().numpy().view(np.uint32)
    for g, w in zip(got[:50], widened[:50]):
        assert struct.unpack("<I", struct.pack("<f", ob.lib().orc_codec_half_to_float(int(g))))[0] == w


@pytest.mark.parametrize("heads,kv_heads,hd", [(16, 2, 128), (12, 2, 128), (1, 1, 4), (40, 8, 128)])
def test_rope_kv_and_attention(K, heads, kv_heads, hd):
    rng = np.random.default_rng(heads)
    cap, layers, layer = 300, 2, 1
    kvd = kv_heads * hd
    n_seq = 3
    positions = [0, 77, 299]  # one row per sequence (decode-like), covering 1..5 key chunks
    kbuf = [torch.zeros((layers, cap, kvd), dtype=torch.float16, device="cuda") for _ in range(n_seq)]
    vbuf = [torch.zeros((layers, cap, kvd), dtype=torch.float16, device="cuda") for _ in range(n_seq)]
    hist_k = [rng.normal(0, 1, (cap, kvd)).astype(np.float16) for _ in range(n_seq)]
    hist_v = [rng.normal(0, 1, (cap, kvd)).astype(np.float16) for _ in range(n_seq)]
    for i in range(n_seq):
        kbuf[i][layer] = torch.from_numpy(hist_k[i]).cuda()
        vbuf[i][layer] = torch.from_numpy(hist_v[i]).cuda()
    slots = (K.KvSlot * n_seq)()
    for i in range(n_seq):
        slots[i] = K.KvSlot(kbuf[i].data_ptr(), vbuf[i].data_ptr(), cap, 0)
    slots_dev = torch.frombuffer(bytearray(bytes(slots)), dtype=torch.uint8).cuda()
    q = rng.normal(0, 1, (n_seq, heads * hd)).astype(np.float32)
    k = rng.normal(0, 1, (n_seq, kvd)).astype(np.float32)
    v = rng.normal(0, 1, (n_seq, kvd)).astype(np.float32)
    seq = torch.arange(n_seq, dtype=torch.int32, device="cuda")
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    qt = torch.from_numpy(q.copy()).cuda()
    table = K.rope_table(cap, hd, 1e6)
    K.rope_kv_append(qt, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), seq, pos, heads, kv_heads, hd, hd,
                     table, slots_dev, layer)
    scratch = torch.empty(K.attention_scratch_bytes(n_seq, heads, hd, cap), dtype=torch.uint8, device="cuda")
    out = torch.empty((n_seq, heads * hd), dtype=torch.float32, device="cuda")
    K.attention(qt, seq, pos, heads, kv_heads, hd, cap, slots_dev, layer, scratch, out)
    torch.cuda.synchronize()
    L = ob.lib()
    for i, p in enumerate(positions):
        qr, kr = q[i].copy(), k[i].copy()
        L.orc_rope_neox(qr.ctypes.data, heads, hd, hd, p, C.c_float(1e6))
        L.orc_rope_neox(kr.ctypes.data, kv_heads, hd, hd, p, C.c_float(1e6))
        assert np.array_equal(qt[i].cpu().numpy().view(np.uint32), qr.view(np.uint32))
        kc = kbuf[i][layer].cpu().numpy()
        vc = vbuf[i][layer].cpu().numpy()
        assert np.array_equal(kc[p], kr.astype(np.float16))
        assert np.array_equal(vc[p], v[i].astype(np.float16))
        assert np.array_equal(kc[p + 1:], hist_k[i][p + 1:])  # nothing else touched
        ref = np.empty(heads * hd, np.float32)
        qrot = qt[i].cpu().numpy().copy()
        kcu = np.ascontiguousarray(kc.view(np.uint16))
        vcu = np.ascontiguousarray(vc.view(np.uint16))
        L.orc_attention_row(qrot.ctypes.data, kcu.ctypes.data, vcu.ctypes.data, p, heads, kv_heads, hd, ref.ctypes.data)
        got = out[i].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), np.abs(got - ref).max()


def _attention_case(K, rng, heads, kv_heads, hd, lengths, rows):
    """KV caches of random f16 rows; `rows` = [(sequence, position)]: the
    query rows of one jfb_attention call, with max_keys the longest row."""
    kvd = kv_heads * hd
    cap = max(lengths)
    kbuf = [torch.from_numpy(rng.normal(0, 1, (1, cap, kvd)).astype(np.float16)).cuda() for _ in lengths]
    vbuf = [torch.from_numpy(rng.normal(0, 1, (1, cap, kvd)).astype(np.float16)).cuda() for _ in lengths]
    slots = (K.KvSlot * len(lengths))()
    for i in range(len(lengths)):
        slots[i] = K.KvSlot(kbuf[i].data_ptr(), vbuf[i].data_ptr(), cap, 0)
    slots_dev = torch.frombuffer(bytearray(bytes(slots)), dtype=torch.uint8).cuda()
    n = len(rows)
    q = rng.normal(0, 1, (n, heads * hd)).astype(np.float32)
    seq = torch.tensor([s for s, _ in rows], dtype=torch.int32, device="cuda")
    pos = torch.tensor([p for _, p in rows], dtype=torch.int32, device="cuda")
    max_keys = max(p for _, p in rows) + 1
    scratch = torch.empty(K.attention_scratch_bytes(n, heads, hd, max_keys), dtype=torch.uint8, device="cuda")
    out = torch.empty((n, heads * hd), dtype=torch.float32, device="cuda")
    q8 = K.Q8Buffer(n, heads * hd) if (heads * hd) % 256 == 0 else None
    K.attention(torch.from_numpy(q).cuda(), seq, pos, heads, kv_heads, hd, max_keys, slots_dev, 0, scratch, out,
                out_q8=q8)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    L = ob.lib()
    kc = [np.ascontiguousarray(b[0].cpu().numpy().view(np.uint16)) for b in kbuf]
    vc = [np.ascontiguousarray(b[0].cpu().numpy().view(np.uint16)) for b in vbuf]
    for i, (s, p) in enumerate(rows):
        ref = np.empty(heads * hd, np.float32)
        L.orc_attention_row(q[i].ctypes.data, kc[s].ctypes.data, vc[s].ctypes.data, p, heads, kv_heads, hd,
                            ref.ctypes.data)
        assert np.array_equal(got[i].view(np.uint32), ref.view(np.uint32)), (i, s, p, np.abs(got[i] - ref).max())
    if q8 is not None:  # the fused Q8_K output equals quantizing the rows
        again = K.Q8Buffer(n, heads * hd)
        K.quantize_q8k(out, again)
        torch.cuda.synchronize()
        for a, b in [(q8.qs, again.qs), (q8.d, again.d), (q8.bsums, again.bsums), (q8.qs_f16, again.qs_f16),
                     (q8.d_t, again.d_t)]:
            assert torch.equal(a, b)


@pytest.mark.parametrize("heads,kv_heads,lengths", [
    (16, 2, [300, 340]),   # 640 causal rows: 8 rows per CTA, one CTA per key range
    (16, 2, [600, 100]),   # 700 rows, rows up to 600 keys: 4 rows per CTA (two warps per row)
    (40, 8, [200]),        # 5 query heads per kv head: padded MMA rows, separate quantization
    (28, 4, [900, 77]),    # the 7B heads (7 per kv head), rows up to 900 keys: 4 rows per CTA
    (28, 4, [1100, 200]),  # rows up to 1100 keys: 2 rows per CTA (four warps per row)
    (16, 2, [2100]),       # beyond 2048 keys: 8 rows per CTA over clusters of 5 CTAs
])
def test_prefill_attention_matches_oracle(K, heads, kv_heads, lengths):
    """Every causal row of whole prompts in one call (the prefill shape)."""
    rng = np.random.default_rng(sum(lengths) + heads)
    rows = [(s, p) for s, length in enumerate(lengths) for p in range(length)]
    _attention_case(K, rng, heads, kv_heads, 128, lengths, rows)


@pytest.mark.parametrize("positions", [[0, 4500, 9000], [8191, 17, 5000, 1, 0, 3000]])
def test_long_decode_attention_matches_oracle(K, positions):
    """Decode rows with long contexts: keys split over clusters of up to 8 CTAs."""
    rng = np.random.default_rng(len(positions))
    lengths = [p + 1 for p in positions]
    _attention_case(K, rng, 16, 2, 128, lengths, list(enumerate(positions)))


@pytest.mark.parametrize("n_rows", [64, 40, 30])
def test_wide_decode_attention_matches_oracle(K, n_rows):
    """Decode rows at the 7B heads (7 per kv head): 64 and 40 rows give more
    one-row CTAs than SMs (the two-per-SM kernel), 30 rows fewer."""
    rng = np.random.default_rng(n_rows)
    positions = rng.integers(0, 1200, n_rows).tolist()
    lengths = [p + 1 for p in positions]
    _attention_case(K, rng, 28, 4, 128, lengths, list(enumerate(positions)))


@pytest.mark.parametrize("cols", [1028, 1030, 5])
def test_swiglu_f32_ragged_rows(K, cols):
    """Rows whose length leaves a partial 8-value group (the element-wise tail)
    or is not a multiple of 4 (no 16-byte vectors at all)."""
    rng = np.random.default_rng(cols)
    g = rng.normal(0, 4, (3, cols)).astype(np.float32)
    u = rng.normal(0, 2, (3, cols)).astype(np.float32)
    out = torch.empty((3, cols), dtype=torch.float32, device="cuda")
    K.swiglu_quant(torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda(), out_f32=out)
    torch.cuda.synchronize()
    L = ob.lib()
    ref = np.array([[L.orc_silu_mul(float(a), float(b)) for a, b in zip(gr, ur)] for gr, ur in zip(g, u)],
                   dtype=np.float32)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))

"""Bit-exact parity of the tcgen05 K-quant matmul (jfb_matmul_tc).

The tensor-core path must give the same bits as the CPU oracle
(ggml_vec_dot_{q4_K,q6_K,q2_K}_q8_K restated, block terms summed in double)
and as the CUDA-core jfb_matmul, for any block contents. Weights are random
raw GGML blocks, so every scale, min and code value occurs, Q6_K scales
included over their whole signed int8 range. "Extreme" rows put every scale
and code at its maximum under constant activations, which drives each
accumulator chain to its largest possible sum (just below 2^24) and the
integer block sum above 2^24, where the CPU's (float)isum rounds.

Shapes cover:
- partial row tiles and partial token tiles;
- few tiles, scheduled on clusters: a tile's K blocks split across 2, 4 or 8
  CTAs (the slices added over distributed shared memory), uneven slices,
  32-token tiles (sums in shared memory) and 64-token tiles (sums staged);
- many tiles, scheduled stream-K: CTA ranges that straddle tiles, which
  exercises the global-memory fixup and the partial slots;
- repeated calls on one workspace, which must leave its counters at zero
  (stream-K) or untouched (clusters).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from jetsonfabric_b200 import jfm
from oracle import binding as ob

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KQ = [jfm.JF_TENSOR_Q4_K, jfm.JF_TENSOR_Q6_K, jfm.JF_TENSOR_Q2_K]
BLOCK_BYTES = {jfm.JF_TENSOR_Q4_K: 144, jfm.JF_TENSOR_Q6_K: 210, jfm.JF_TENSOR_Q2_K: 84}


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    from jetsonfabric_b200 import kernels
    return kernels


def _f16_bits(values) -> np.ndarray:
    return np.asarray(values, dtype=np.float16).view(np.uint16)


def random_blocks(jf_type: int, rows: int, cols: int, seed: int, extreme_rows=()) -> bytes:
    """Raw GGML blocks with uniformly random scales, mins and codes."""
    rng = np.random.default_rng(seed)
    nb = rows * cols // 256
    size = BLOCK_BYTES[jf_type]
    raw = rng.integers(0, 256, (nb, size), dtype=np.uint8)
    if jf_type == jfm.JF_TENSOR_Q4_K:  # d, dmin, scales[12], qs[128]
        raw[:, 0:2] = _f16_bits(rng.uniform(1e-4, 2e-3, nb)).view(np.uint8).reshape(nb, 2)
        raw[:, 2:4] = _f16_bits(rng.uniform(1e-4, 2e-3, nb)).view(np.uint8).reshape(nb, 2)
    elif jf_type == jfm.JF_TENSOR_Q6_K:  # ql[128], qh[64], scales[16], d
        raw[:, 208:210] = _f16_bits(rng.uniform(-2e-4, 2e-4, nb)).view(np.uint8).reshape(nb, 2)
    else:  # scales[16], qs[64], d, dmin
        raw[:, 80:82] = _f16_bits(rng.uniform(1e-4, 2e-3, nb)).view(np.uint8).reshape(nb, 2)
        raw[:, 82:84] = _f16_bits(rng.uniform(1e-4, 2e-3, nb)).view(np.uint8).reshape(nb, 2)
    per_row = cols // 256
    for r in extreme_rows:
        blk = raw[r * per_row:(r + 1) * per_row]
        if jf_type == jfm.JF_TENSOR_Q4_K:
            blk[:, 4:16] = 0xFF          # every 6-bit scale and min = 63
            blk[:, 16:144] = 0xFF        # every code = 15
        elif jf_type == jfm.JF_TENSOR_Q6_K:
            blk[:, 0:192] = 0x00         # every code = 0 -> code - 32 = -32
            blk[:, 192:208] = 0x80       # every scale = -128
        else:
            blk[:, 0:16] = 0xFF          # scale 15, min 15
            blk[:, 16:80] = 0xFF         # every code = 3
    return raw.tobytes()


def oracle_matmul(jf_type, raw: bytes, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    raw_np = np.frombuffer(raw, np.uint8)
    t = ob.OrcTensor(jf_type, 0, cols, rows, raw_np.ctypes.data)
    ref = np.empty((x.shape[0], rows), np.float32)
    ob.lib().orc_matmul(C.byref(t), np.ascontiguousarray(x).ctypes.data, x.shape[0], ref.ctypes.data)
    return ref


def activations(n: int, cols: int, seed: int, constant_rows=()) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (n, cols)).astype(np.float32)
    for r in constant_rows:
        if r < n:
            x[r] = 1.0 if r % 2 == 0 else -1.0
    return x


def run_tc(K, w, x, workspace=None, epilogue=None, bias=None, residual=None):
    n, cols = x.shape
    q8 = K.Q8Buffer(n, cols)
    K.quantize_q8k(torch.from_numpy(x).cuda(), q8)
    if workspace is None:
        workspace = torch.zeros(K.matmul_tc_workspace_bytes(w.rows, cols, n), dtype=torch.uint8, device="cuda")
    out = torch.empty((n, w.rows), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.matmul_tc(w, n, out, q8, workspace, epilogue=K.EPILOGUE_STORE if epilogue is None else epilogue, bias=bias,
                residual=residual, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out, q8, workspace


def bits(a) -> np.ndarray:
    a = a.cpu().numpy() if hasattr(a, "cpu") else a
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("jf_type", KQ)
@pytest.mark.parametrize("rows,cols,n", [
    (96, 256, 1),       # one block of K, one partial tile
    (96, 2048, 5),      # one tile split into 8 one-block slices
    (300, 2560, 32),    # 3 row tiles x 10 blocks, a full token tile: uneven slices
    (1000, 11008, 32),  # clusters: 8 tiles x 43 blocks in slices of 5 and 6 blocks
    (1000, 11008, 33),  # stream-K over 8 tiles of 64 tokens x 43 blocks: ranges straddle tiles
    (200, 1024, 100),   # 2 x 2 tiles of 64 tokens, partial token tile
    (520, 2048, 130),   # 5 x 3 tiles of 64 tokens
    (19000, 256, 20),   # stream-K over 149 tiles of one block
    (9600, 2560, 24),   # stream-K over 75 tiles x 10 blocks: ranges straddle tiles
])
def test_tc_matches_oracle_and_cuda_core(K, jf_type, rows, cols, n):
    raw = random_blocks(jf_type, rows, cols, 7 + rows + jf_type, extreme_rows=(0, rows - 1))
    w = K.DeviceWeight(jf_type, rows, cols, raw)
    x = activations(n, cols, n + cols, constant_rows=(0, n - 1))
    got, q8, _ = run_tc(K, w, x)
    ref = oracle_matmul(jf_type, raw, rows, cols, x)
    assert np.array_equal(bits(got), bits(ref))
    core = torch.empty((n, rows), dtype=torch.float32, device="cuda")
    K.matmul(w, n, core, x_q8=q8)
    torch.cuda.synchronize()
    assert np.array_equal(bits(got), bits(core))


@pytest.mark.parametrize("jf_type", KQ)
def test_tc_encoder_weights_with_epilogues(K, jf_type):
    rows, cols, n = 384, 2048, 32
    rng = np.random.default_rng(jf_type)
    raw = jfm.quantize_blocks(jf_type, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    w = K.DeviceWeight(jf_type, rows, cols, raw)
    x = activations(n, cols, 3)
    ref = oracle_matmul(jf_type, raw, rows, cols, x)
    bias_np = rng.normal(0, 0.1, rows).astype(np.float32)
    res_np = rng.normal(0, 1, (n, rows)).astype(np.float32)
    got, _, ws = run_tc(K, w, x, epilogue=K.EPILOGUE_BIAS, bias=torch.from_numpy(bias_np).cuda())
    assert np.array_equal(bits(got), bits(ref + bias_np))
    res = torch.from_numpy(res_np).cuda()
    got, _, ws = run_tc(K, w, x, workspace=ws, epilogue=K.EPILOGUE_RESIDUAL, residual=res)
    assert np.array_equal(bits(got), bits(ref + res_np))


@pytest.mark.parametrize("jf_type,rows,cols,n,clustered", [
    (jfm.JF_TENSOR_Q4_K, 1000, 11008, 32, True),
    (jfm.JF_TENSOR_Q4_K, 1000, 11008, 33, False),
    (jfm.JF_TENSOR_Q6_K, 2048, 2048, 32, True),
    (jfm.JF_TENSOR_Q4_K, 20000, 2048, 33, False),
])
def test_tc_repeated_calls_are_identical(K, jf_type, rows, cols, n, clustered):
    """Split tiles are added in a fixed order, so repeated calls give the same
    bits. Stream-K launches leave their arrival counters at zero; clustered
    launches add the slices on chip and never write the workspace."""
    raw = random_blocks(jf_type, rows, cols, 99)
    w = K.DeviceWeight(jf_type, rows, cols, raw)
    x = activations(n, cols, 5)
    first, _, ws = run_tc(K, w, x)
    for _ in range(3):
        again, _, ws = run_tc(K, w, x, workspace=ws)
        assert np.array_equal(bits(again), bits(first))
    if clustered:
        assert int(ws.sum().item()) == 0
    else:
        # partial slots: two per SM, sized for the widest token tile (64)
        partial_bytes = 2 * torch.cuda.get_device_properties(0).multi_processor_count * 128 * 64 * 8
        counters = ws[partial_bytes:].view(torch.int32)
        assert int(counters.abs().sum().item()) == 0


def test_tc_shapes_share_one_workspace(K):
    """Calls of different grids and tile counts interleaved on one workspace,
    as a stage runs its weights: each stays bit-exact."""
    shapes = [(jfm.JF_TENSOR_Q4_K, 1000, 11008, 33), (jfm.JF_TENSOR_Q4_K, 256, 1536, 24),
              (jfm.JF_TENSOR_Q6_K, 1536, 8960, 24), (jfm.JF_TENSOR_Q2_K, 96, 2048, 5), (jfm.JF_TENSOR_Q6_K, 4000, 1536, 1)]
    size = max(K.matmul_tc_workspace_bytes(r, c, n) for _, r, c, n in shapes)
    ws = torch.zeros(size, dtype=torch.uint8, device="cuda")
    cases = []
    for i, (t, r, c, n) in enumerate(shapes):
        raw = random_blocks(t, r, c, 50 + i)
        x = activations(n, c, 60 + i)
        cases.append((K.DeviceWeight(t, r, c, raw), x, oracle_matmul(t, raw, r, c, x)))
    for _ in range(2):
        for w, x, ref in cases:
            got, _, ws = run_tc(K, w, x, workspace=ws)
            assert np.array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("n,cols", [(1, 256), (37, 2048), (130, 11008)])
def test_quantizer_writes_tensor_core_operands(K, n, cols):
    """Every quantizer also writes the codes and partial sums as f16 and d
    transposed; the tensor-core matmul loads those instead of the int8 codes."""
    x = torch.from_numpy(activations(n, cols, 11, constant_rows=(0,))).cuda()
    q8 = K.Q8Buffer(n, cols)
    K.quantize_q8k(x, q8)
    torch.cuda.synchronize()
    assert torch.equal(q8.qs_f16.float(), q8.qs.float())
    assert torch.equal(q8.bsums_f16.float(), q8.bsums.float())
    assert torch.equal(q8.d_t[:, :n], q8.d.t())
    gate = torch.from_numpy(activations(n, cols, 12)).cuda()
    K.swiglu_quant(gate, x, out_q8=q8)
    torch.cuda.synchronize()
    assert torch.equal(q8.qs_f16.float(), q8.qs.float())
    assert torch.equal(q8.d_t[:, :n], q8.d.t())
    if cols <= 8192:
        norm_w = torch.from_numpy(np.random.default_rng(1).normal(1, 0.1, cols).astype(np.float32)).cuda()
        K.rmsnorm_quant(x, norm_w, 1e-6, out_q8=q8)
        torch.cuda.synchronize()
        assert torch.equal(q8.bsums_f16.float(), q8.bsums.float())
        assert torch.equal(q8.d_t[:, :n], q8.d.t())


def test_tc_rejects_bad_arguments(K):
    from jetsonfabric_b200.engine import InvalidArgument, NativeExecutionError
    rows, cols, n = 128, 512, 4
    raw = random_blocks(jfm.JF_TENSOR_Q4_K, rows, cols, 1)
    w = K.DeviceWeight(jfm.JF_TENSOR_Q4_K, rows, cols, raw)
    q8 = K.Q8Buffer(n, cols)
    out = torch.empty((n, rows), dtype=torch.float32, device="cuda")
    need = K.matmul_tc_workspace_bytes(rows, cols, n)
    small = torch.zeros(need - 8, dtype=torch.uint8, device="cuda")
    with pytest.raises(InvalidArgument):
        K.matmul_tc(w, n, out, q8, small)
    plain = K.Q8Buffer(n, cols, tensor_core=False)  # no f16 operands for the tensor cores
    with pytest.raises(InvalidArgument):
        K.matmul_tc(w, n, out, plain, torch.zeros(need, dtype=torch.uint8, device="cuda"))
    f32 = K.DeviceWeight(jfm.JF_TENSOR_F32, 8, 256, np.zeros(8 * 256, np.float32).tobytes())
    with pytest.raises(NativeExecutionError):
        K.matmul_tc(f32, n, out, q8, torch.zeros(need, dtype=torch.uint8, device="cuda"))


@pytest.mark.parametrize("jf_type", KQ)
def test_tc_segments_over_stacked_rows(K, jf_type):
    """One launch over a weight stacking three matrices (as the engine stacks
    Q/K/V) writes each member's rows to its own output with its own bias;
    row views of the stacked weight through both matmul paths agree."""
    cols, n = 2048, 24
    parts = [(300, 31), (128, 32), (200, 33)]
    raws = [random_blocks(jf_type, r, cols, seed) for r, seed in parts]
    total = sum(r for r, _ in parts)
    w = K.DeviceWeight(jf_type, total, cols, b"".join(raws))
    x = activations(n, cols, 17)
    q8 = K.Q8Buffer(n, cols)
    K.quantize_q8k(torch.from_numpy(x).cuda(), q8)
    ws = torch.zeros(K.matmul_tc_workspace_bytes(total, cols, n), dtype=torch.uint8, device="cuda")
    rng = np.random.default_rng(5)
    outs, biases, segs, end = [], [], [], 0
    for r, _ in parts:
        end += r
        bias = torch.from_numpy(rng.normal(0, 0.1, r).astype(np.float32)).cuda()
        out = torch.empty((n, r), dtype=torch.float32, device="cuda")
        outs.append(out)
        biases.append(bias)
        segs.append((end, K.EPILOGUE_BIAS, bias, None, out))
    K.matmul_tc_segments(w, n, q8, segs, ws)
    torch.cuda.synchronize()
    row = 0
    for (r, _), raw, out, bias in zip(parts, raws, outs, biases):
        ref = oracle_matmul(jf_type, raw, r, cols, x) + bias.cpu().numpy()
        assert np.array_equal(bits(out), bits(ref))
        view = K.WeightView(w, row, r)
        core = torch.empty((n, r), dtype=torch.float32, device="cuda")
        K.matmul(view, n, core, x_q8=q8, epilogue=K.EPILOGUE_BIAS, bias=bias)
        torch.cuda.synchronize()
        assert np.array_equal(bits(core), bits(ref))
        row += r

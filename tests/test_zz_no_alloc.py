"""jfb_attention_static_scratch: attention for callers that cannot call
cudaMalloc (their device memory belongs to another allocator, or a
cudaMalloc's implicit synchronisation is not allowed on their path). It must
give exactly what jfb_attention gives with caller-provided scratch, call after
call, although every call reuses the same file-scope device array.

Kept in a file of its own that pytest collects last, and self-contained, so it
passes alone in a fresh process as well as after the other GPU tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def bind():
    from jetsonfabric_b200 import engine, kernels
    kernels._bind()
    L = engine.lib()
    fn = L.jfb_attention_static_scratch
    fn.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                   C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p]
    fn.restype = engine.Status
    return L, engine, kernels


def make_case(K, rng, heads, kv_heads, hd, cap, positions, layers=2, layer=1):
    kvd = kv_heads * hd
    bufs = []
    slots = (K.KvSlot * len(positions))()
    for i in range(len(positions)):
        kb = torch.from_numpy(rng.normal(0, 1, (layers, cap, kvd)).astype(np.float16)).cuda()
        vb = torch.from_numpy(rng.normal(0, 1, (layers, cap, kvd)).astype(np.float16)).cuda()
        bufs += [kb, vb]
        slots[i] = K.KvSlot(kb.data_ptr(), vb.data_ptr(), cap, 0)
    slots_dev = torch.frombuffer(bytearray(bytes(slots)), dtype=torch.uint8).cuda()
    q = torch.from_numpy(rng.normal(0, 1, (len(positions), heads * hd)).astype(np.float32)).cuda()
    seq = torch.arange(len(positions), dtype=torch.int32, device="cuda")
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    return dict(q=q, seq=seq, pos=pos, slots=slots_dev, bufs=bufs, heads=heads, kv_heads=kv_heads, hd=hd, cap=cap,
                layer=layer)


def run_static(L, engine, K, case, out, q8=None):
    stream = torch.cuda.current_stream().cuda_stream
    st = L.jfb_attention_static_scratch(case["q"].data_ptr(), case["q"].shape[0], case["seq"].data_ptr(),
                                        case["pos"].data_ptr(), case["heads"], case["kv_heads"], case["hd"],
                                        case["cap"], case["slots"].data_ptr(), case["layer"], out.data_ptr(),
                                        None if q8 is None else C.byref(q8.desc), stream)
    engine.check(st)


def run_reference_entry(K, case, out, q8=None):
    n = case["q"].shape[0]
    scratch = torch.empty(K.attention_scratch_bytes(n, case["heads"], case["hd"], case["cap"]), dtype=torch.uint8,
                          device="cuda")
    K.attention(case["q"], case["seq"], case["pos"], case["heads"], case["kv_heads"], case["hd"], case["cap"],
                case["slots"], case["layer"], scratch, out, out_q8=q8)


def uses_scratch(case) -> bool:
    """Whether jfb_attention takes its four-launch form, the one that keeps
    scores, statistics and partial sums in the scratch buffer: head dims other
    than 64 and 128, or more than 8 query heads per kv head. (The single
    launch on the FP64 tensor cores keeps everything on chip and would leave
    the static array untouched.)"""
    return case["hd"] not in (64, 128) or case["heads"] // case["kv_heads"] > 8


def test_static_scratch_attention_matches_scratch_attention_twice():
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    L, engine, K = bind()
    rng = np.random.default_rng(77)
    # calls of different shapes in a row, through the scratch-using form: each
    # must not see the previous call's leftovers in the shared array
    wide = make_case(K, rng, 16, 1, 128, 700, [699, 5, 300, 64, 128, 0, 511, 333])  # 16 query heads per kv head
    odd = make_case(K, rng, 4, 2, 96, 200, [199, 63, 1])                              # head_dim 96
    for case in (wide, odd, wide):
        assert uses_scratch(case)
        n, width = case["q"].shape[0], case["heads"] * case["hd"]
        quantize = width % 256 == 0
        want = torch.empty((n, width), dtype=torch.float32, device="cuda")
        want_q8 = K.Q8Buffer(n, width) if quantize else None
        run_reference_entry(K, case, want, want_q8)
        got = torch.full((n, width), float("nan"), dtype=torch.float32, device="cuda")
        got_q8 = K.Q8Buffer(n, width) if quantize else None
        run_static(L, engine, K, case, got, got_q8)
        torch.cuda.synchronize()
        # the attention tests' tolerance is bit equality
        assert torch.equal(got.view(torch.int32), want.view(torch.int32))
        if quantize:
            assert torch.equal(got_q8.qs, want_q8.qs)
            assert torch.equal(got_q8.d.view(torch.int32), want_q8.d.view(torch.int32))


def test_static_scratch_rejects_oversized_calls():
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    L, engine, K = bind()
    limit = 16 * 1024 * 1024
    n, heads, hd, keys = 64, 40, 128, 8192
    assert K.attention_scratch_bytes(n, heads, hd, keys) > limit
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(engine.InvalidArgument, match="static scratch"):
        engine.check(L.jfb_attention_static_scratch(dummy.data_ptr(), n, dummy.data_ptr(), dummy.data_ptr(), heads, 8,
                                                    hd, keys, dummy.data_ptr(), 0, dummy.data_ptr(), None, None))

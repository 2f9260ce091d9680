"""ctypes binding of the jfb kernel C ABI (include/jfb/jfb_kernels.h).

Arguments are torch CUDA tensors (or raw device pointers); PyTorch only
provides device memory and streams here. Used by the kernel-level GPU tests
and by bench.py to time the dominant kernel in isolation.
"""
from __future__ import annotations

import ctypes as C

from .engine import Status, check, lib

_VP = C.c_void_p


class Weight(C.Structure):
    _fields_ = [("type", C.c_uint32), ("rows", C.c_uint32), ("cols", C.c_uint32), ("reserved", C.c_uint32),
                ("plane", C.c_void_p * 3)]


class Q8K(C.Structure):
    _fields_ = [("qs", C.c_void_p), ("d", C.c_void_p), ("bsums", C.c_void_p), ("qs_f16", C.c_void_p),
                ("bsums_f16", C.c_void_p), ("d_t", C.c_void_p), ("d_stride", C.c_uint32), ("reserved", C.c_uint32)]


class Segment(C.Structure):
    _fields_ = [("row_end", C.c_uint32), ("epilogue", C.c_uint32), ("bias", C.c_void_p), ("residual", C.c_void_p),
                ("out", C.c_void_p)]


class KvSlot(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("capacity", C.c_uint32), ("reserved", C.c_uint32)]


_bound = False

EPILOGUE_STORE, EPILOGUE_BIAS, EPILOGUE_RESIDUAL = 0, 1, 2


def _bind():
    global _bound
    if _bound:
        return lib()
    L = lib()
    sig = {
        "jfb_weight_device_bytes": ([C.c_uint32, C.c_uint32, C.c_uint32], C.c_uint64),
        "jfb_weight_repack": ([C.c_uint32, C.c_uint32, C.c_uint32, _VP, _VP, C.POINTER(Weight), _VP], Status),
        "jfb_dequantize": ([C.POINTER(Weight), _VP, _VP], Status),
        "jfb_embed_rows": ([C.POINTER(Weight), _VP, C.c_uint32, _VP, _VP, _VP], Status),
        "jfb_rmsnorm_quant": ([_VP, _VP, _VP, C.c_uint32, C.c_uint32, C.c_float, _VP, C.POINTER(Q8K), _VP], Status),
        "jfb_quantize_q8k": ([_VP, C.c_uint32, C.c_uint32, C.POINTER(Q8K), _VP], Status),
        "jfb_swiglu_quant": ([_VP, _VP, C.c_uint32, C.c_uint32, _VP, C.POINTER(Q8K), _VP], Status),
        "jfb_matmul": ([C.POINTER(Weight), C.POINTER(Q8K), _VP, C.c_uint32, C.c_uint32, _VP, _VP, _VP, _VP], Status),
        "jfb_matmul_tc_supported": ([C.POINTER(Weight)], C.c_int),
        "jfb_matmul_tc_segments": ([C.POINTER(Weight), C.POINTER(Q8K), C.c_uint32, C.POINTER(Segment), C.c_uint32, _VP,
                                    C.c_uint64, _VP, _VP], Status),
        "jfb_weight_row_view": ([C.POINTER(Weight), C.c_uint32, C.c_uint32, C.POINTER(Weight)], Status),
        "jfb_matmul_tc_workspace_bytes": ([C.c_uint32, C.c_uint32, C.c_uint32], C.c_uint64),
        "jfb_matmul_tc": ([C.POINTER(Weight), C.POINTER(Q8K), C.c_uint32, C.c_uint32, _VP, _VP, _VP, _VP, C.c_uint64,
                           _VP, _VP], Status),
        "jfb_rope_kv_append": ([_VP, _VP, _VP, C.c_uint32, _VP, _VP, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                _VP, C.c_uint32, _VP, C.c_uint32, _VP], Status),
        "jfb_rope_table_host": ([_VP, C.c_uint32, C.c_uint32, C.c_float], None),
        "jfb_attention_scratch_bytes": ([C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32], C.c_uint64),
        "jfb_attention": ([_VP, C.c_uint32, _VP, _VP, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, _VP, C.c_uint32,
                           _VP, C.c_uint64, _VP, C.POINTER(Q8K), _VP], Status),
        "jfb_argmax": ([_VP, C.c_uint32, C.c_uint32, _VP, _VP], Status),
        "jfb_codec_f32_to_f16": ([_VP, _VP, C.c_uint64, _VP], Status),
        "jfb_codec_f16_to_f32": ([_VP, _VP, C.c_uint64, _VP], Status),
        "jfb_crc32_scratch_bytes": ([C.c_uint64], C.c_uint64),
        "jfb_crc32": ([_VP, C.c_uint64, _VP, _VP, C.c_uint64, _VP], Status),
        "jfb_stagewire_stamp_crc": ([_VP, _VP, C.c_uint32, _VP], Status),
        "jfb_stagewire_check_crc": ([_VP, _VP, C.c_uint32, _VP, _VP], Status),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _bound = True
    return L


def ptr(t) -> int | None:
    if t is None:
        return None
    return t if isinstance(t, int) else t.data_ptr()


def stream_ptr(stream=None) -> int | None:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class DeviceWeight:
    """A weight uploaded and repacked into the planar device layout."""

    def __init__(self, jf_type: int, rows: int, cols: int, raw: bytes | bytearray | memoryview):
        import numpy as np
        import torch
        L = _bind()
        nbytes = L.jfb_weight_device_bytes(jf_type, rows, cols)
        self.buffer = torch.empty(int(nbytes), dtype=torch.uint8, device="cuda")
        src = torch.from_numpy(np.frombuffer(bytes(raw), dtype=np.uint8).copy()).cuda()
        self.desc = Weight()
        check(L.jfb_weight_repack(jf_type, rows, cols, src.data_ptr(), self.buffer.data_ptr(), C.byref(self.desc),
                                  stream_ptr()))
        torch.cuda.synchronize()
        self.rows, self.cols, self.type = rows, cols, jf_type

    def dequantize(self):
        import torch
        out = torch.empty((self.rows, self.cols), dtype=torch.float32, device="cuda")
        check(_bind().jfb_dequantize(C.byref(self.desc), out.data_ptr(), stream_ptr()))
        return out


class Q8Buffer:
    """Q8_K activations [rows][cols] on the device. With `tensor_core` (the
    default) the buffer also keeps the operands of the tensor-core matmul that
    every quantizer writes: the codes and partial sums as f16 and d
    transposed with a row stride of rows rounded up to 4."""

    def __init__(self, rows: int, cols: int, tensor_core: bool = True):
        import torch
        self.qs = torch.zeros((rows, cols), dtype=torch.int8, device="cuda")
        self.d = torch.zeros((rows, cols // 256), dtype=torch.float32, device="cuda")
        self.bsums = torch.zeros((rows, cols // 16), dtype=torch.int16, device="cuda")
        self.qs_f16 = self.bsums_f16 = self.d_t = None
        self.d_stride = 0
        if tensor_core:
            self.d_stride = (rows + 3) // 4 * 4
            self.qs_f16 = torch.zeros((rows, cols), dtype=torch.float16, device="cuda")
            self.bsums_f16 = torch.zeros((rows, cols // 16), dtype=torch.float16, device="cuda")
            self.d_t = torch.zeros((cols // 256, self.d_stride), dtype=torch.float32, device="cuda")
        self.desc = Q8K(self.qs.data_ptr(), self.d.data_ptr(), self.bsums.data_ptr(),
                        None if self.qs_f16 is None else self.qs_f16.data_ptr(),
                        None if self.bsums_f16 is None else self.bsums_f16.data_ptr(),
                        None if self.d_t is None else self.d_t.data_ptr(), self.d_stride, 0)


def rmsnorm_quant(x, weight, eps, out_f32=None, out_q8: Q8Buffer | None = None, row_index=None, rows=None):
    n = rows if rows is not None else x.shape[0]
    check(_bind().jfb_rmsnorm_quant(ptr(x), ptr(row_index), ptr(weight), n, x.shape[1], eps, ptr(out_f32),
                                    None if out_q8 is None else C.byref(out_q8.desc), stream_ptr()))


def quantize_q8k(x, out: Q8Buffer):
    check(_bind().jfb_quantize_q8k(ptr(x), x.shape[0], x.shape[1], C.byref(out.desc), stream_ptr()))


def swiglu_quant(gate, up, out_f32=None, out_q8: Q8Buffer | None = None):
    check(_bind().jfb_swiglu_quant(ptr(gate), ptr(up), gate.shape[0], gate.shape[1], ptr(out_f32),
                                   None if out_q8 is None else C.byref(out_q8.desc), stream_ptr()))


def matmul(w: DeviceWeight, n: int, out, x_q8: Q8Buffer | None = None, x_f32=None, epilogue=EPILOGUE_STORE,
           bias=None, residual=None, stream=None):
    check(_bind().jfb_matmul(C.byref(w.desc), None if x_q8 is None else C.byref(x_q8.desc), ptr(x_f32), n,
                             epilogue, ptr(bias), ptr(residual), ptr(out), stream_ptr(stream)))


def matmul_tc_workspace_bytes(rows: int, cols: int, n: int) -> int:
    return int(_bind().jfb_matmul_tc_workspace_bytes(rows, cols, n))


def matmul_tc(w: DeviceWeight, n: int, out, x_q8: Q8Buffer, workspace, epilogue=EPILOGUE_STORE, bias=None,
              residual=None, error_flag=None, stream=None, workspace_bytes=None):
    """The tcgen05 path (jfb_matmul_tc); `workspace` is a zero-filled uint8 CUDA tensor."""
    size = workspace.numel() if workspace_bytes is None else workspace_bytes
    check(_bind().jfb_matmul_tc(C.byref(w.desc), C.byref(x_q8.desc), n, epilogue, ptr(bias), ptr(residual), ptr(out),
                                ptr(workspace), size, ptr(error_flag), stream_ptr(stream)))


def matmul_tc_segments(w: DeviceWeight, n: int, x_q8: Q8Buffer, segments, workspace, error_flag=None, stream=None):
    """jfb_matmul_tc_segments; `segments` is a list of (row_end, epilogue, bias, residual, out)."""
    arr = (Segment * len(segments))(*[Segment(r, e, ptr(b), ptr(res), ptr(o)) for r, e, b, res, o in segments])
    check(_bind().jfb_matmul_tc_segments(C.byref(w.desc), C.byref(x_q8.desc), n, arr, len(segments), ptr(workspace),
                                         workspace.numel(), ptr(error_flag), stream_ptr(stream)))


class WeightView:
    """Rows [row_begin, row_begin + rows) of a DeviceWeight (jfb_weight_row_view); keeps the parent alive."""

    def __init__(self, parent: DeviceWeight, row_begin: int, rows: int):
        self.parent = parent
        self.desc = Weight()
        check(_bind().jfb_weight_row_view(C.byref(parent.desc), row_begin, rows, C.byref(self.desc)))
        self.rows, self.cols, self.type = rows, parent.cols, parent.type


def argmax(logits, out):
    check(_bind().jfb_argmax(ptr(logits), logits.shape[0], logits.shape[1], ptr(out), stream_ptr()))


def codec_f32_to_f16(x, out, stream=None):
    check(_bind().jfb_codec_f32_to_f16(ptr(x), ptr(out), x.numel(), stream_ptr(stream)))


def codec_f16_to_f32(x, out, stream=None):
    check(_bind().jfb_codec_f16_to_f32(ptr(x), ptr(out), x.numel(), stream_ptr(stream)))


def crc32_scratch_bytes(n: int) -> int:
    return int(_bind().jfb_crc32_scratch_bytes(n))


def crc32(data, crc_out, scratch, stream=None):
    """crc_out[0] (a 4-byte device word) = CRC-32/IEEE of the bytes of `data`."""
    n = data.numel() * data.element_size()
    check(_bind().jfb_crc32(ptr(data), n, ptr(crc_out), ptr(scratch), scratch.numel() * scratch.element_size(),
                            stream_ptr(stream)))


def stagewire_stamp_crc(crc, frame, offset: int, stream=None):
    check(_bind().jfb_stagewire_stamp_crc(ptr(crc), ptr(frame), offset, stream_ptr(stream)))


def stagewire_check_crc(crc, frame, offset: int, mismatch, stream=None):
    check(_bind().jfb_stagewire_check_crc(ptr(crc), ptr(frame), offset, ptr(mismatch), stream_ptr(stream)))


def attention_scratch_bytes(n, heads, head_dim, max_keys) -> int:
    return int(_bind().jfb_attention_scratch_bytes(n, heads, head_dim, max_keys))


def rope_table(positions: int, rope_dims: int, freq_base: float):
    """Host-built GGML rope cache (cos, sin) [positions][rope_dims/2][2] as a CUDA tensor."""
    import numpy as np
    import torch
    t = np.empty((positions, rope_dims // 2, 2), dtype=np.float32)
    _bind().jfb_rope_table_host(t.ctypes.data, positions, rope_dims, freq_base)
    return torch.from_numpy(t).cuda()


def rope_kv_append(q, k, v, seq, pos, heads, kv_heads, head_dim, rope_dims, table, slots, layer):
    check(_bind().jfb_rope_kv_append(ptr(q), ptr(k), ptr(v), q.shape[0], ptr(seq), ptr(pos), heads, kv_heads,
                                     head_dim, rope_dims, ptr(table), table.shape[0], ptr(slots), layer, stream_ptr()))


def attention(q, seq, pos, heads, kv_heads, head_dim, max_keys, slots, layer, scratch, out, out_q8=None):
    check(_bind().jfb_attention(ptr(q), q.shape[0], ptr(seq), ptr(pos), heads, kv_heads, head_dim, max_keys,
                                ptr(slots), layer, ptr(scratch), scratch.numel(), ptr(out),
                                None if out_q8 is None else C.byref(out_q8.desc), stream_ptr()))

"""ctypes binding of the JFM v2 loader (jf_* C ABI) and the synthetic package
writer, both in lib/libjfm.so.

The Python names follow the C ABI of include/jetsonfabric/engine.h, which is
the reference loader ABI (runtime/engines/native/include/jetsonfabric/engine.h).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"

JF_TENSOR_F32 = 1
JF_TENSOR_F16 = 2
JF_TENSOR_I8 = 23
JF_TENSOR_Q2_K = 9
JF_TENSOR_Q4_K = 11
JF_TENSOR_Q6_K = 13
JF_ALL_LAYERS = 0xFFFFFFFF

JF_STATUS_OK = 0
JF_STATUS_INVALID_ARGUMENT = 1
JF_STATUS_IO_ERROR = 2
JF_STATUS_FORMAT_ERROR = 3
JF_STATUS_NOT_FOUND = 4
JF_STATUS_OUT_OF_MEMORY = 5


class Status(C.Structure):
    _fields_ = [("code", C.c_int), ("message", C.c_char * 256)]


class StagePlan(C.Structure):
    _fields_ = [("layer_start", C.c_uint32), ("layer_end", C.c_uint32),
                ("verify_hashes", C.c_uint32), ("evict_before_open", C.c_uint32)]


class ModelStats(C.Structure):
    _fields_ = [("layer_start", C.c_uint32), ("layer_end", C.c_uint32), ("layer_count", C.c_uint32),
                ("selected_weight_bytes", C.c_uint64), ("total_weight_bytes", C.c_uint64),
                ("mapped_bytes", C.c_uint64), ("selected_tensor_count", C.c_uint64),
                ("total_tensor_count", C.c_uint64)]


class TensorView(C.Structure):
    _fields_ = [("name", C.c_void_p), ("name_length", C.c_size_t), ("type", C.c_uint32),
                ("rank", C.c_uint32), ("storage_block_elements", C.c_uint32),
                ("storage_block_bytes", C.c_uint32), ("shape", C.c_uint64 * 4),
                ("layer", C.c_int32), ("data", C.c_void_p), ("size", C.c_uint64)]


class SynthSpec(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("layer_count", C.c_uint32), ("embedding_length", C.c_uint32),
                ("head_count", C.c_uint32), ("kv_head_count", C.c_uint32),
                ("feed_forward_length", C.c_uint32), ("vocabulary_size", C.c_uint32),
                ("context_length", C.c_uint32), ("rope_freq_base", C.c_float),
                ("rms_epsilon", C.c_float), ("layer_type", C.c_uint32),
                ("embedding_type", C.c_uint32), ("output_type", C.c_uint32),
                ("more_bits_q6k", C.c_uint32), ("seed", C.c_uint64), ("weight_std", C.c_float),
                ("draw_norms", C.c_uint32), ("draw_biases", C.c_uint32), ("threads", C.c_uint32)]


class SynthReport(C.Structure):
    _fields_ = [("weight_bytes", C.c_uint64), ("tensor_count", C.c_uint64), ("file_bytes", C.c_uint64)]


class ImportReport(C.Structure):
    _fields_ = [("layer_count", C.c_uint32), ("reserved", C.c_uint32), ("tensor_count", C.c_uint64),
                ("tensor_bytes", C.c_uint64), ("package_bytes", C.c_uint64), ("source_sha256", C.c_uint8 * 32),
                ("architecture", C.c_char * 64)]


class JfmError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = LIB_DIR / "libjfm.so"
        if not path.exists():
            raise RuntimeError(f"{path} is missing; run python -m jetsonfabric_b200.build")
        L = C.CDLL(str(path))
        L.jf_model_open.argtypes = [C.c_char_p, C.POINTER(StagePlan), C.POINTER(C.c_void_p)]
        L.jf_model_open.restype = Status
        L.jf_model_close.argtypes = [C.c_void_p]
        L.jf_model_close.restype = None
        L.jf_model_get_stats.argtypes = [C.c_void_p]
        L.jf_model_get_stats.restype = ModelStats
        L.jf_model_tensor_count.argtypes = [C.c_void_p]
        L.jf_model_tensor_count.restype = C.c_size_t
        L.jf_model_tensor_at.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(TensorView)]
        L.jf_model_tensor_at.restype = Status
        L.jf_model_find_tensor.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(TensorView)]
        L.jf_model_find_tensor.restype = Status
        L.jf_model_prefetch.argtypes = [C.c_void_p, C.POINTER(C.c_uint64)]
        L.jf_model_prefetch.restype = Status
        L.jf_model_prefetch_parallel.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(C.c_uint64)]
        L.jf_model_prefetch_parallel.restype = Status
        L.jf_model_get_source_sha256.argtypes = [C.c_void_p, C.POINTER(C.c_uint8 * 32)]
        L.jf_model_get_source_sha256.restype = Status
        L.jf_model_get_gguf_metadata.argtypes = [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
        L.jf_model_get_gguf_metadata.restype = Status
        L.jf_tensor_type_layout.argtypes = [C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]
        L.jf_tensor_type_layout.restype = Status
        L.jf_status_code_name.argtypes = [C.c_int]
        L.jf_status_code_name.restype = C.c_char_p
        L.jf_sha256_buffer.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(C.c_uint8 * 32)]
        L.jf_sha256_buffer.restype = None
        L.jfb_write_synthetic_package.argtypes = [C.POINTER(SynthSpec), C.c_char_p, C.POINTER(SynthReport)]
        L.jfb_write_synthetic_package.restype = Status
        L.jfb_quantize_blocks.argtypes = [C.c_uint32, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
        L.jfb_quantize_blocks.restype = Status
        L.jfb_import_gguf.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(ImportReport)]
        L.jfb_import_gguf.restype = Status
        L.jfb_tokenizer_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
        L.jfb_tokenizer_open.restype = Status
        L.jfb_tokenizer_close.argtypes = [C.c_void_p]
        L.jfb_tokenizer_close.restype = None
        L.jfb_tokenizer_tokenize.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_int32), C.c_size_t,
                                             C.POINTER(C.c_size_t)]
        L.jfb_tokenizer_tokenize.restype = Status
        L.jfb_tokenizer_token_piece.argtypes = [C.c_void_p, C.c_int32, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]
        L.jfb_tokenizer_token_piece.restype = Status
        L.jfb_tokenizer_is_end_token.argtypes = [C.c_void_p, C.c_int32]
        L.jfb_tokenizer_is_end_token.restype = C.c_int
        _lib = L
    return _lib


def _check(status: Status) -> None:
    if status.code != 0:
        raise JfmError(status.code, status.message.decode(errors="replace"))


def sha256(data: bytes) -> bytes:
    out = (C.c_uint8 * 32)()
    buf = C.create_string_buffer(data, len(data))
    lib().jf_sha256_buffer(buf, len(data), C.byref(out))
    return bytes(out)


def import_gguf(gguf_path: str | Path, package_dir: str | Path) -> dict:
    """Converts a GGUF file into a new JFM v2 package directory (jfb_import_gguf);
    the equivalent of the reference's `jf-model-compile --input --output`."""
    rep = ImportReport()
    _check(lib().jfb_import_gguf(str(gguf_path).encode(), str(package_dir).encode(), C.byref(rep)))
    return {"format": "jfm-v2", "architecture": rep.architecture.decode(), "source_sha256": bytes(rep.source_sha256).hex(),
            "layer_count": rep.layer_count, "tensor_count": rep.tensor_count, "tensor_bytes": rep.tensor_bytes,
            "package_bytes": rep.package_bytes}


class Tokenizer:
    """The package's text tokenizer (jfb_tokenizer_*): the reference tokenizer
    interface's tokenize / token_piece / is_end_token (tokenizer.hpp:9-16)."""

    def __init__(self, package_dir: str | Path):
        h = C.c_void_p()
        _check(lib().jfb_tokenizer_open(str(package_dir).encode(), C.byref(h)))
        self._h = h

    def close(self) -> None:
        if self._h:
            lib().jfb_tokenizer_close(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tokenize(self, text: str | bytes) -> list[int]:
        data = text.encode() if isinstance(text, str) else bytes(text)
        cap = len(data) + 8
        while True:
            buf = (C.c_int32 * cap)()
            n = C.c_size_t()
            _check(lib().jfb_tokenizer_tokenize(self._h, data, len(data), buf, cap, C.byref(n)))
            if n.value <= cap:
                return list(buf[:n.value])
            cap = n.value

    def token_piece(self, token: int) -> bytes:
        n = C.c_size_t()
        _check(lib().jfb_tokenizer_token_piece(self._h, token, None, 0, C.byref(n)))
        buf = C.create_string_buffer(max(n.value, 1))
        _check(lib().jfb_tokenizer_token_piece(self._h, token, buf, n.value, C.byref(n)))
        return buf.raw[:n.value]

    def is_end_token(self, token: int) -> bool:
        return bool(lib().jfb_tokenizer_is_end_token(self._h, token))


def type_layout(jf_type: int) -> tuple[int, int]:
    e, b = C.c_uint32(), C.c_uint32()
    _check(lib().jf_tensor_type_layout(jf_type, C.byref(e), C.byref(b)))
    return e.value, b.value


@dataclass
class Tensor:
    name: str
    type: int
    rank: int
    shape: tuple[int, int, int, int]
    layer: int
    block_elements: int
    block_bytes: int
    data: int
    size: int

    def bytes(self) -> bytes:
        return C.string_at(self.data, self.size)


class Model:
    """One opened stage view of a JFM package (jf_model_open)."""

    def __init__(self, path: str | Path, layer_start: int = 0, layer_end: int = JF_ALL_LAYERS,
                 verify_hashes: bool = True, evict_before_open: bool = False):
        plan = StagePlan(layer_start, layer_end, int(verify_hashes), int(evict_before_open))
        handle = C.c_void_p()
        _check(lib().jf_model_open(str(path).encode(), C.byref(plan), C.byref(handle)))
        self._h = handle

    def close(self) -> None:
        if self._h:
            lib().jf_model_close(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stats(self) -> ModelStats:
        return lib().jf_model_get_stats(self._h)

    def tensors(self) -> list[Tensor]:
        return [self.tensor_at(i) for i in range(lib().jf_model_tensor_count(self._h))]

    @staticmethod
    def _view(v: TensorView) -> Tensor:
        return Tensor(C.string_at(v.name, v.name_length).decode(), v.type, v.rank, tuple(v.shape),
                      v.layer, v.storage_block_elements, v.storage_block_bytes, v.data, v.size)

    def tensor_at(self, index: int) -> Tensor:
        v = TensorView()
        _check(lib().jf_model_tensor_at(self._h, index, C.byref(v)))
        return self._view(v)

    def find(self, name: str) -> Tensor:
        v = TensorView()
        _check(lib().jf_model_find_tensor(self._h, name.encode(), C.byref(v)))
        return self._view(v)

    def prefetch(self, threads: int = 1) -> int:
        checksum = C.c_uint64()
        _check(lib().jf_model_prefetch_parallel(self._h, threads, C.byref(checksum)))
        return checksum.value

    def source_sha256(self) -> bytes:
        out = (C.c_uint8 * 32)()
        _check(lib().jf_model_get_source_sha256(self._h, C.byref(out)))
        return bytes(out)

    def gguf_metadata(self) -> bytes:
        p, n = C.c_void_p(), C.c_size_t()
        _check(lib().jf_model_get_gguf_metadata(self._h, C.byref(p), C.byref(n)))
        return C.string_at(p, n.value) if p.value else b""


def write_synthetic_package(directory: str | Path, *, kind: int = 0, layer_count: int = 2,
                            embedding_length: int = 256, head_count: int = 2, kv_head_count: int = 1,
                            feed_forward_length: int = 512, vocabulary_size: int = 512,
                            context_length: int = 256, rope_freq_base: float = 1.0e6,
                            rms_epsilon: float = 1.0e-6, layer_type: int = JF_TENSOR_Q4_K,
                            embedding_type: int = JF_TENSOR_Q4_K, output_type: int = JF_TENSOR_Q6_K,
                            more_bits_q6k: bool = True, seed: int = 1234, weight_std: float = 0.02,
                            draw_norms: bool = False, draw_biases: bool = True,
                            threads: int = 0) -> SynthReport:
    spec = SynthSpec(kind, layer_count, embedding_length, head_count, kv_head_count, feed_forward_length,
                     vocabulary_size, context_length, rope_freq_base, rms_epsilon, layer_type,
                     embedding_type, output_type, int(more_bits_q6k), seed, weight_std, int(draw_norms),
                     int(draw_biases), threads)
    report = SynthReport()
    _check(lib().jfb_write_synthetic_package(C.byref(spec), str(directory).encode(), C.byref(report)))
    return report


def write_reference_fixture(directory: str | Path) -> SynthReport:
    """The reference's 2-layer constant F32 Qwen2 fixture (model_fixture.cpp:76-133)."""
    return write_synthetic_package(directory, kind=1)


def quantize_blocks(jf_type: int, values) -> bytes:
    import numpy as np

    x = np.ascontiguousarray(values, dtype=np.float32).ravel()
    _, block_bytes = type_layout(jf_type)
    out = np.zeros(x.size // 256 * block_bytes, dtype=np.uint8)
    _check(lib().jfb_quantize_blocks(jf_type, x.ctypes.data, x.size, out.ctypes.data, out.size))
    return out.tobytes()


# Preset model shapes of the configurations (hidden, heads, kv heads, ffn, vocab).
QWEN2_PRESETS = {
    "1.5b": dict(layer_count=28, embedding_length=1536, head_count=12, kv_head_count=2,
                 feed_forward_length=8960, vocabulary_size=151936),
    "3b": dict(layer_count=36, embedding_length=2048, head_count=16, kv_head_count=2,
               feed_forward_length=11008, vocabulary_size=151936),
    "7b": dict(layer_count=28, embedding_length=3584, head_count=28, kv_head_count=4,
               feed_forward_length=18944, vocabulary_size=152064),
    "14b": dict(layer_count=48, embedding_length=5120, head_count=40, kv_head_count=8,
                feed_forward_length=13824, vocabulary_size=152064),
    "32b": dict(layer_count=64, embedding_length=5120, head_count=40, kv_head_count=8,
                feed_forward_length=27648, vocabulary_size=152064, layer_type=JF_TENSOR_Q2_K,
                embedding_type=JF_TENSOR_Q2_K, more_bits_q6k=False),
}


def main(argv: list[str] | None = None) -> int:
    """`python -m jetsonfabric_b200.jfm --input model.gguf --output model.jfm`: the
    command line of the reference's jf-model-compile (jf_model_compile.cpp:374-396),
    printing the same JSON summary on success."""
    import argparse
    import json
    import sys

    ap = argparse.ArgumentParser(prog="jetsonfabric_b200.jfm", description="Convert a GGUF file to a JFM v2 package")
    ap.add_argument("--input", required=True)
    ap.add_argument("--output", required=True)
    args = ap.parse_args(argv)
    try:
        report = import_gguf(args.input, args.output)
    except JfmError as e:
        print(f"jf-model-compile: {e}", file=sys.stderr)
        return 1
    print(json.dumps(report, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

"""Python mirror of the native engine API over the jfb C ABI (lib/libjfb.so).

Names and argument meaning follow the reference C++ API
(runtime/engines/native/include/jetsonfabric/native_inference.hpp):
NativeEngine(package_path, backend=..., ...), create_session(capacity),
NativeSession.prefill_stage_tokens / prefill_stage_activations /
decode_stage_token / decode_stage_activation / prefill_greedy /
decode_greedy / rollback, NativeEngine.logits / forced_decode_logits /
generate. Invalid input raises InvalidArgument (a ValueError), the
counterpart of std::invalid_argument; any other failure raises
NativeExecutionError.

There is no CPU path: the library is CUDA-only, and importing this module
without a built libjfb.so, or opening an engine without a CUDA device, fails
loudly.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from pathlib import Path
from typing import Sequence

import numpy as np

LIB_DIR = Path(__file__).resolve().parent / "lib"

BACKENDS = {"cpu": 0, "cuda": 1}
ATTENTION_KERNELS = {"automatic": 0, "unfused": 1, "flash": 2}
ATTENTION_NAMES = {v: k for k, v in ATTENTION_KERNELS.items()}

JFB_STATUS_INVALID_ARGUMENT = 1


class InvalidArgument(ValueError):
    """std::invalid_argument of the reference engine (HTTP 400 in the executor)."""


class NativeExecutionError(RuntimeError):
    """Any other engine failure (HTTP 502 in the reference executor)."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class Status(C.Structure):
    _fields_ = [("code", C.c_int), ("message", C.c_char * 256)]


class EngineOptions(C.Structure):
    _fields_ = [("backend", C.c_uint32), ("prefill_attention_kernel", C.c_uint32),
                ("decode_attention_kernel", C.c_uint32), ("threads", C.c_int32), ("layer_start", C.c_uint32),
                ("layer_end", C.c_uint32), ("device", C.c_int32)]


class ModelInfoC(C.Structure):
    _fields_ = [("architecture", C.c_char * 32), ("source_sha256", C.c_char * 72), ("compute_backend", C.c_char * 32),
                ("compute_device", C.c_char * 128), ("layer_count", C.c_uint32), ("embedding_length", C.c_uint32),
                ("context_length", C.c_uint32), ("vocabulary_size", C.c_uint32), ("weight_bytes", C.c_uint64),
                ("total_weight_bytes", C.c_uint64), ("tensor_count", C.c_uint64),
                ("resident_layer_start", C.c_uint32), ("resident_layer_end", C.c_uint32),
                ("prefill_attention_kernel", C.c_uint32), ("decode_attention_kernel", C.c_uint32),
                ("load_time_ms", C.c_double)]


class GenerationStats(C.Structure):
    _fields_ = [("time_to_first_token_ms", C.c_double), ("inter_token_latency_ms", C.c_double),
                ("decode_tokens_per_second", C.c_double), ("end_to_end_tokens_per_second", C.c_double),
                ("kv_cache_bytes", C.c_uint64), ("scratch_bytes", C.c_uint64)]


class KernelTimingC(C.Structure):
    _fields_ = [("matmul_launches", C.c_uint64), ("matmul_ms", C.c_double), ("matmul_bytes", C.c_double),
                ("attention_launches", C.c_uint64), ("attention_ms", C.c_double), ("attention_bytes", C.c_double)]


class StageOutputC(C.Structure):
    _fields_ = [("sampled_token", C.c_int32), ("activation_rows", C.c_uint32)]


_lib = None
_VP, _SZ, _I32P, _U32P, _F32P = C.c_void_p, C.c_size_t, C.POINTER(C.c_int32), C.POINTER(C.c_uint32), C.c_void_p


def library_path() -> Path:
    return LIB_DIR / "libjfb.so"


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = library_path()
        if not path.exists():
            raise RuntimeError(f"{path} is missing: the CUDA engine is not built "
                               "(run python -c 'import __graft_entry__; __graft_entry__.build()')")
        L = C.CDLL(str(path))
        sig = {
            "jfb_engine_open": ([C.c_char_p, C.POINTER(EngineOptions), C.POINTER(_VP)], Status),
            "jfb_engine_close": ([_VP], None),
            "jfb_engine_info": ([_VP, C.POINTER(ModelInfoC)], Status),
            "jfb_session_open": ([_VP, _SZ, C.POINTER(_VP)], Status),
            "jfb_session_close": ([_VP], None),
            "jfb_session_capacity": ([_VP], _SZ),
            "jfb_session_position": ([_VP], _SZ),
            "jfb_session_prefill_tokens": ([_VP, _VP, _SZ, C.POINTER(StageOutputC), _VP, _SZ], Status),
            "jfb_session_prefill_activations": ([_VP, _VP, _SZ, C.POINTER(StageOutputC), _VP, _SZ], Status),
            "jfb_session_decode_token": ([_VP, C.c_int32, C.POINTER(StageOutputC), _VP, _SZ], Status),
            "jfb_session_decode_activation": ([_VP, _VP, C.POINTER(StageOutputC), _VP, _SZ], Status),
            "jfb_session_prefill_greedy": ([_VP, _VP, _SZ, _I32P], Status),
            "jfb_session_decode_greedy": ([_VP, C.c_int32, _I32P], Status),
            "jfb_session_rollback": ([_VP, _SZ], Status),
            "jfb_session_reset": ([_VP], Status),
            "jfb_engine_logits": ([_VP, _VP, _SZ, _VP, _SZ], Status),
            "jfb_engine_forced_decode_logits": ([_VP, _VP, _SZ, _VP, _SZ, _VP, _SZ], Status),
            "jfb_engine_generate": ([_VP, _VP, _SZ, C.c_uint32, _VP, C.POINTER(GenerationStats)], Status),
            "jfb_engine_release_session": ([_VP], None),
            "jfb_engine_prefill_batch": ([_VP, _VP, _SZ, _VP, _VP, _VP, _VP, _SZ], Status),
            "jfb_engine_prefill_batch_activations": ([_VP, _VP, _SZ, _VP, _VP, _VP, _VP, _SZ], Status),
            "jfb_engine_decode_batch": ([_VP, _VP, _SZ, _VP, _VP, _VP, _SZ], Status),
            "jfb_engine_decode_batch_activations": ([_VP, _VP, _SZ, _VP, _VP, _VP, _SZ], Status),
            "jfb_engine_decode_batch_device": ([_VP, _VP, _SZ, _VP, _VP], Status),
            "jfb_engine_prefill_batch_device": ([_VP, _VP, _SZ, _VP, _VP, _VP], Status),
            "jfb_engine_stage_batch_device": ([_VP, _VP, _SZ, C.c_int, _VP, _VP, _VP, _VP, _VP], Status),
            "jfb_engine_synchronize": ([_VP], Status),
            "jfb_engine_stream": ([_VP], _VP),
            "jfb_engine_last_launch_count": ([_VP], C.c_uint64),
            "jfb_engine_set_kernel_timing": ([_VP, C.c_int], Status),
            "jfb_engine_kernel_timing": ([_VP, C.POINTER(KernelTimingC)], Status),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: Status) -> None:
    if status.code == 0:
        return
    message = status.message.decode(errors="replace")
    if status.code == JFB_STATUS_INVALID_ARGUMENT:
        raise InvalidArgument(message)
    raise NativeExecutionError(status.code, message)


def _i32(values) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(values, dtype=np.int32).ravel())


@dataclass
class ModelInfo:
    architecture: str
    source_sha256: str
    compute_backend: str
    compute_device: str
    layer_count: int
    embedding_length: int
    context_length: int
    vocabulary_size: int
    weight_bytes: int
    total_weight_bytes: int
    tensor_count: int
    resident_layer_start: int
    resident_layer_end: int


@dataclass
class StageResult:
    activation: np.ndarray | None = None   # f32 [rows, hidden] on intermediate stages
    sampled_token: int = -1

    def has_activations(self) -> bool:
        return self.activation is not None

    def has_sampled_token(self) -> bool:
        return self.sampled_token >= 0


@dataclass
class GenerationResult:
    sampled_tokens: list[int] = field(default_factory=list)
    time_to_first_token_ms: float = 0.0
    inter_token_latency_ms: float = 0.0
    decode_tokens_per_second: float = 0.0
    end_to_end_tokens_per_second: float = 0.0
    kv_cache_bytes: int = 0
    scratch_bytes: int = 0


class NativeSession:
    """A session; it must not outlive its engine, so NativeEngine.close()
    closes every session still open on it first."""

    def __init__(self, engine: "NativeEngine", handle: C.c_void_p):
        self.engine = engine
        self._h = handle

    def close(self) -> None:
        if self._h:
            if self.engine._h:
                lib().jfb_session_close(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def capacity(self) -> int:
        return lib().jfb_session_capacity(self._h)

    def position(self) -> int:
        return lib().jfb_session_position(self._h)

    def _result(self, out: StageOutputC, acts: np.ndarray | None) -> StageResult:
        if out.sampled_token >= 0 or acts is None:
            return StageResult(sampled_token=out.sampled_token)
        return StageResult(activation=acts[: out.activation_rows].copy())

    def _acts(self, rows: int) -> np.ndarray | None:
        if self.engine.last_stage:
            return None
        return np.empty((rows, self.engine.hidden), dtype=np.float32)

    def prefill_stage_tokens(self, tokens: Sequence[int]) -> StageResult:
        t = _i32(tokens)
        acts = self._acts(t.size)
        out = StageOutputC()
        check(lib().jfb_session_prefill_tokens(self._h, t.ctypes.data, t.size, C.byref(out),
                                                None if acts is None else acts.ctypes.data,
                                                0 if acts is None else acts.size))
        return self._result(out, acts)

    def _check_activation(self, a: np.ndarray) -> None:
        # f32[sequence_length, hidden_size] (runtime/adapters/native_stage_executor.cpp:16-45)
        if a.ndim != 2 or a.shape[0] == 0 or a.shape[1] != self.engine.hidden:
            raise InvalidArgument("native stage activation shape is invalid")

    def prefill_stage_activations(self, activation: np.ndarray) -> StageResult:
        a = np.ascontiguousarray(activation, dtype=np.float32)
        self._check_activation(a)
        rows = a.shape[0]
        acts = self._acts(max(rows, 1))
        out = StageOutputC()
        check(lib().jfb_session_prefill_activations(self._h, a.ctypes.data, rows, C.byref(out),
                                                     None if acts is None else acts.ctypes.data,
                                                     0 if acts is None else acts.size))
        return self._result(out, acts)

    def decode_stage_token(self, token: int) -> StageResult:
        acts = self._acts(1)
        out = StageOutputC()
        check(lib().jfb_session_decode_token(self._h, int(token), C.byref(out),
                                              None if acts is None else acts.ctypes.data,
                                              0 if acts is None else acts.size))
        return self._result(out, acts)

    def decode_stage_activation(self, activation: np.ndarray) -> StageResult:
        a = np.ascontiguousarray(activation, dtype=np.float32)
        self._check_activation(a)
        if a.shape[0] != 1:
            raise InvalidArgument("native decode activation must contain one token row")
        acts = self._acts(1)
        out = StageOutputC()
        check(lib().jfb_session_decode_activation(self._h, a.ctypes.data, C.byref(out),
                                                   None if acts is None else acts.ctypes.data,
                                                   0 if acts is None else acts.size))
        return self._result(out, acts)

    def prefill_greedy(self, tokens: Sequence[int]) -> int:
        t = _i32(tokens)
        tok = C.c_int32(-1)
        check(lib().jfb_session_prefill_greedy(self._h, t.ctypes.data, t.size, C.byref(tok)))
        return tok.value

    def decode_greedy(self, token: int) -> int:
        tok = C.c_int32(-1)
        check(lib().jfb_session_decode_greedy(self._h, int(token), C.byref(tok)))
        return tok.value

    def rollback(self, token_count: int) -> None:
        check(lib().jfb_session_rollback(self._h, int(token_count)))

    def reset(self) -> None:
        check(lib().jfb_session_reset(self._h))


class NativeEngine:
    def __init__(self, package_path: str | Path, backend: str = "cuda", threads: int = 1, *,
                 prefill_attention_kernel: str = "automatic", decode_attention_kernel: str = "automatic",
                 layer_start: int = 0, layer_end: int | None = None, device: int = -1):
        opts = EngineOptions(BACKENDS[backend], ATTENTION_KERNELS[prefill_attention_kernel],
                             ATTENTION_KERNELS[decode_attention_kernel], threads, layer_start,
                             0xFFFFFFFF if layer_end is None else layer_end, device)
        handle = C.c_void_p()
        import weakref
        self._sessions = weakref.WeakSet()
        check(lib().jfb_engine_open(str(package_path).encode(), C.byref(opts), C.byref(handle)))
        self._h = handle
        info = ModelInfoC()
        check(lib().jfb_engine_info(self._h, C.byref(info)))
        self._info = info
        self.hidden = info.embedding_length
        self.vocabulary = info.vocabulary_size
        self.first_stage = info.resident_layer_start == 0
        self.last_stage = info.resident_layer_end == info.layer_count

    def close(self) -> None:
        if getattr(self, "_h", None):
            for s in list(self._sessions):
                s.close()
            lib().jfb_engine_close(self._h)
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
    def handle(self) -> C.c_void_p:
        return self._h

    def model_info(self) -> ModelInfo:
        i = self._info
        return ModelInfo(i.architecture.decode(), i.source_sha256.decode(), i.compute_backend.decode(),
                         i.compute_device.decode(), i.layer_count, i.embedding_length, i.context_length,
                         i.vocabulary_size, i.weight_bytes, i.total_weight_bytes, i.tensor_count,
                         i.resident_layer_start, i.resident_layer_end)

    def prefill_attention_kernel(self) -> str:
        return ATTENTION_NAMES[self._info.prefill_attention_kernel]

    def decode_attention_kernel(self) -> str:
        return ATTENTION_NAMES[self._info.decode_attention_kernel]

    def load_time_ms(self) -> float:
        return self._info.load_time_ms

    def create_session(self, capacity: int) -> NativeSession:
        h = C.c_void_p()
        check(lib().jfb_session_open(self._h, int(capacity), C.byref(h)))
        session = NativeSession(self, h)
        self._sessions.add(session)
        return session

    def logits(self, tokens: Sequence[int]) -> np.ndarray:
        t = _i32(tokens)
        out = np.empty(self.vocabulary, dtype=np.float32)
        check(lib().jfb_engine_logits(self._h, t.ctypes.data, t.size, out.ctypes.data, out.size))
        return out

    def forced_decode_logits(self, prompt_tokens: Sequence[int], forced_tokens: Sequence[int]) -> np.ndarray:
        p, f = _i32(prompt_tokens), _i32(forced_tokens)
        out = np.empty((f.size + 1, self.vocabulary), dtype=np.float32)
        check(lib().jfb_engine_forced_decode_logits(self._h, p.ctypes.data, p.size, f.ctypes.data, f.size,
                                                     out.ctypes.data, out.size))
        return out

    def generate(self, prompt_tokens: Sequence[int], max_tokens: int) -> GenerationResult:
        p = _i32(prompt_tokens)
        out = np.empty(max(int(max_tokens), 1), dtype=np.int32)
        st = GenerationStats()
        check(lib().jfb_engine_generate(self._h, p.ctypes.data, p.size, int(max_tokens), out.ctypes.data, C.byref(st)))
        return GenerationResult(out[:max_tokens].tolist(), st.time_to_first_token_ms, st.inter_token_latency_ms,
                                st.decode_tokens_per_second, st.end_to_end_tokens_per_second, st.kv_cache_bytes,
                                st.scratch_bytes)

    def release_session(self) -> None:
        lib().jfb_engine_release_session(self._h)

    # ---- batched stage passes (continuous batching) ----

    @staticmethod
    def _handles(sessions: Sequence[NativeSession]):
        arr = (C.c_void_p * max(len(sessions), 1))()
        for i, s in enumerate(sessions):
            arr[i] = s.handle.value
        return arr

    def _batch_outputs(self, rows: int, n: int):
        tokens = np.full(n, -1, dtype=np.int32)
        acts = None if self.last_stage else np.empty((rows, self.hidden), dtype=np.float32)
        return tokens, acts

    def _split(self, tokens, acts, counts) -> list[StageResult]:
        if acts is None:
            return [StageResult(sampled_token=int(t)) for t in tokens]
        out, off = [], 0
        for c in counts:
            out.append(StageResult(activation=acts[off:off + c].copy()))
            off += c
        return out

    def prefill_stage_batch(self, sessions: Sequence[NativeSession], prompts: Sequence[Sequence[int]]) -> list[StageResult]:
        counts = np.asarray([len(p) for p in prompts], dtype=np.uint32)
        flat = _i32(np.concatenate([np.asarray(p, dtype=np.int32) for p in prompts]) if prompts else [])
        tokens, acts = self._batch_outputs(int(counts.sum()), len(sessions))
        check(lib().jfb_engine_prefill_batch(self._h, self._handles(sessions), len(sessions), flat.ctypes.data,
                                              counts.ctypes.data, tokens.ctypes.data,
                                              None if acts is None else acts.ctypes.data,
                                              0 if acts is None else acts.size))
        return self._split(tokens, acts, counts.tolist())

    def prefill_stage_batch_activations(self, sessions: Sequence[NativeSession],
                                        activations: Sequence[np.ndarray]) -> list[StageResult]:
        counts = np.asarray([a.shape[0] for a in activations], dtype=np.uint32)
        flat = np.ascontiguousarray(np.concatenate(activations, axis=0), dtype=np.float32)
        tokens, acts = self._batch_outputs(int(counts.sum()), len(sessions))
        check(lib().jfb_engine_prefill_batch_activations(self._h, self._handles(sessions), len(sessions),
                                                          flat.ctypes.data, counts.ctypes.data, tokens.ctypes.data,
                                                          None if acts is None else acts.ctypes.data,
                                                          0 if acts is None else acts.size))
        return self._split(tokens, acts, counts.tolist())

    def decode_stage_batch(self, sessions: Sequence[NativeSession], tokens_in: Sequence[int]) -> list[StageResult]:
        t = _i32(tokens_in)
        tokens, acts = self._batch_outputs(len(sessions), len(sessions))
        check(lib().jfb_engine_decode_batch(self._h, self._handles(sessions), len(sessions), t.ctypes.data,
                                             tokens.ctypes.data, None if acts is None else acts.ctypes.data,
                                             0 if acts is None else acts.size))
        return self._split(tokens, acts, [1] * len(sessions))

    def decode_stage_batch_activations(self, sessions: Sequence[NativeSession],
                                       activations: np.ndarray) -> list[StageResult]:
        a = np.ascontiguousarray(activations, dtype=np.float32)
        tokens, acts = self._batch_outputs(len(sessions), len(sessions))
        check(lib().jfb_engine_decode_batch_activations(self._h, self._handles(sessions), len(sessions),
                                                         a.ctypes.data, tokens.ctypes.data,
                                                         None if acts is None else acts.ctypes.data,
                                                         0 if acts is None else acts.size))
        return self._split(tokens, acts, [1] * len(sessions))

    # ---- device-resident passes (benchmark loop) ----

    def prefill_batch_device(self, sessions: Sequence[NativeSession], tokens_device_ptr: int,
                             counts: Sequence[int], tokens_out_device_ptr: int) -> None:
        c = np.asarray(counts, dtype=np.uint32)
        check(lib().jfb_engine_prefill_batch_device(self._h, self._handles(sessions), len(sessions),
                                                     C.c_void_p(tokens_device_ptr), c.ctypes.data,
                                                     C.c_void_p(tokens_out_device_ptr)))

    def decode_batch_device(self, sessions: Sequence[NativeSession], tokens_device_ptr: int,
                            tokens_out_device_ptr: int, handles=None) -> None:
        check(lib().jfb_engine_decode_batch_device(self._h, handles if handles is not None else self._handles(sessions),
                                                    len(sessions), C.c_void_p(tokens_device_ptr),
                                                    C.c_void_p(tokens_out_device_ptr)))

    def stage_batch_device(self, sessions: Sequence[NativeSession], prefill: bool, counts: Sequence[int] | None = None,
                           tokens_ptr: int = 0, activations_ptr: int = 0, tokens_out_ptr: int = 0,
                           activations_out_ptr: int = 0, handles=None) -> None:
        """One device-resident pass of this engine's stage (jfb_engine_stage_batch_device): the first
        stage reads token ids, later stages f32 activations; the last stage writes greedy tokens, the
        others f32 activations. Pointers are device addresses; nothing is synchronised."""
        c = None if counts is None else np.asarray(counts, dtype=np.uint32)
        check(lib().jfb_engine_stage_batch_device(
            self._h, handles if handles is not None else self._handles(sessions), len(sessions), int(prefill),
            None if c is None else c.ctypes.data, C.c_void_p(tokens_ptr or None), C.c_void_p(activations_ptr or None),
            C.c_void_p(tokens_out_ptr or None), C.c_void_p(activations_out_ptr or None)))

    def synchronize(self) -> None:
        check(lib().jfb_engine_synchronize(self._h))

    def stream(self) -> int:
        return lib().jfb_engine_stream(self._h) or 0

    def last_launch_count(self) -> int:
        return lib().jfb_engine_last_launch_count(self._h)

    def set_kernel_timing(self, enabled: bool) -> None:
        check(lib().jfb_engine_set_kernel_timing(self._h, int(enabled)))

    def kernel_timing(self) -> dict:
        t = KernelTimingC()
        check(lib().jfb_engine_kernel_timing(self._h, C.byref(t)))
        return {f: getattr(t, f) for f, _ in KernelTimingC._fields_}

"""ctypes binding of the CPU oracle (oracle/liboracle.so) — TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker; the product never imports it.

`OracleStage` opens one stage of a JFM package with the product's loader
(jetsonfabric_b200.jfm, itself checked against the reference's golden package)
and hands the raw GGML-encoded tensor bytes to the C restatement.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


class OrcTensor(C.Structure):
    _fields_ = [("type", C.c_uint32), ("pad_", C.c_uint32), ("ne0", C.c_uint64), ("ne1", C.c_uint64),
                ("data", C.c_void_p)]


_LAYER_FIELDS = ["attn_norm", "attn_q", "attn_q_bias", "attn_k", "attn_k_bias", "attn_v", "attn_v_bias",
                 "attn_output", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"]
_LAYER_NAMES = {"attn_norm": "attn_norm.weight", "attn_q": "attn_q.weight", "attn_q_bias": "attn_q.bias",
                "attn_k": "attn_k.weight", "attn_k_bias": "attn_k.bias", "attn_v": "attn_v.weight",
                "attn_v_bias": "attn_v.bias", "attn_output": "attn_output.weight",
                "ffn_norm": "ffn_norm.weight", "ffn_gate": "ffn_gate.weight", "ffn_up": "ffn_up.weight",
                "ffn_down": "ffn_down.weight"}


class OrcLayer(C.Structure):
    _fields_ = [(f, OrcTensor) for f in _LAYER_FIELDS]


class OrcModel(C.Structure):
    _fields_ = [("layer_count", C.c_uint32), ("embedding_length", C.c_uint32), ("head_count", C.c_uint32),
                ("kv_head_count", C.c_uint32), ("feed_forward_length", C.c_uint32),
                ("context_length", C.c_uint32), ("vocabulary_size", C.c_uint32),
                ("rope_dimension_count", C.c_uint32), ("rope_freq_base", C.c_float),
                ("rms_epsilon", C.c_float), ("layer_start", C.c_uint32), ("layer_end", C.c_uint32),
                ("token_embd", OrcTensor), ("output_norm", OrcTensor), ("output", OrcTensor),
                ("output_bias", OrcTensor), ("layers", C.POINTER(OrcLayer))]


_lib = None


def build() -> Path:
    """Compiles liboracle.so (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return HERE / "liboracle.so"


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        L = C.CDLL(str(path))
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_dequantize_row.argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_int64]
        L.orc_quantize_row_q8_k.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.orc_matmul.argtypes = [C.POINTER(OrcTensor), C.c_void_p, C.c_int64, C.c_void_p]
        for name in ("orc_dot_kquant_scalar", "orc_dot_kquant_vector"):
            getattr(L, name).argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_int64]
            getattr(L, name).restype = C.c_float
        L.orc_q8k_block_bytes.restype = C.c_size_t
        L.orc_rms_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_float, C.c_void_p]
        L.orc_rope_neox.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_float]
        L.orc_argmax.argtypes = [C.c_void_p, C.c_int64]
        L.orc_argmax.restype = C.c_int32
        L.orc_expf.argtypes = [C.c_float]
        L.orc_expf.restype = C.c_float
        L.orc_silu_mul.argtypes = [C.c_float, C.c_float]
        L.orc_silu_mul.restype = C.c_float
        L.orc_attention_row.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                        C.c_int64, C.c_void_p]
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_codec_float_to_half.argtypes = [C.c_float]
        L.orc_codec_float_to_half.restype = C.c_uint16
        L.orc_codec_half_to_float.argtypes = [C.c_uint16]
        L.orc_codec_half_to_float.restype = C.c_float
        L.orc_session_create.argtypes = [C.POINTER(OrcModel), C.c_size_t]
        L.orc_session_create.restype = C.c_void_p
        L.orc_session_destroy.argtypes = [C.c_void_p]
        L.orc_session_position.argtypes = [C.c_void_p]
        L.orc_session_position.restype = C.c_size_t
        L.orc_session_rollback.argtypes = [C.c_void_p, C.c_size_t]
        L.orc_session_rollback.restype = C.c_int
        L.orc_session_forward.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                          C.c_void_p, C.POINTER(C.c_int32), C.c_char_p, C.c_size_t]
        L.orc_session_forward.restype = C.c_int
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def dequantize(jf_type: int, raw: bytes | np.ndarray, count: int) -> np.ndarray:
    src = np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray)) else raw
    src = np.ascontiguousarray(src)
    out = np.empty(count, dtype=np.float32)
    lib().orc_dequantize_row(jf_type, src.ctypes.data, out.ctypes.data, count)
    return out


def quantize_q8_k(x: np.ndarray) -> np.ndarray:
    """Returns the raw 292-byte GGML block_q8_K records."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(x.size // 256 * 292, dtype=np.uint8)
    lib().orc_quantize_row_q8_k(x.ctypes.data, out.ctypes.data, x.size)
    return out


def split_q8_k(raw: np.ndarray, k: int):
    """Splits block_q8_K records into (d [nb], qs [nb*256] int8, bsums [nb*16] int16)."""
    nb = raw.size // 292
    rec = raw.reshape(nb, 292)
    d = rec[:, 0:4].copy().view(np.float32).ravel()
    qs = rec[:, 4:260].copy().view(np.int8).ravel()
    bs = rec[:, 260:292].copy().view(np.int16).ravel()
    return d, qs, bs


class GgufMeta:
    """Minimal GGUF v3 key/value reader for the oracle's hyper-parameters."""

    def __init__(self, blob: bytes):
        import struct
        self.kv = {}
        if blob[:4] != b"GGUF":
            raise ValueError("not GGUF")
        _, n_tensors, n_kv = struct.unpack_from("<IQQ", blob, 4)
        off = 24

        def string(o):
            (n,) = struct.unpack_from("<Q", blob, o)
            return blob[o + 8:o + 8 + n].decode(), o + 8 + n

        scalar = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
                  12: "<d"}

        def value(t, o):
            if t in scalar:
                v = struct.unpack_from(scalar[t], blob, o)[0]
                return v, o + struct.calcsize(scalar[t])
            if t == 8:
                return string(o)
            if t == 9:
                et, n = struct.unpack_from("<IQ", blob, o)
                o += 12
                vals = []
                for _ in range(n):
                    v, o = value(et, o)
                    vals.append(v)
                return vals, o
            raise ValueError(f"GGUF type {t}")

        for _ in range(n_kv):
            key, off = string(off)
            (t,) = struct.unpack_from("<I", blob, off)
            v, off = value(t, off + 4)
            self.kv[key] = v


class OracleStage:
    """A stage of a JFM package, executed by the C oracle."""

    def __init__(self, package, layer_start: int = 0, layer_end: int | None = None):
        from jetsonfabric_b200 import jfm

        self.jfm_model = jfm.Model(package, layer_start, jfm.JF_ALL_LAYERS if layer_end is None else layer_end)
        st = self.jfm_model.stats
        meta = GgufMeta(self.jfm_model.gguf_metadata()).kv
        m = OrcModel()
        m.layer_count = meta["qwen2.block_count"]
        m.embedding_length = meta["qwen2.embedding_length"]
        m.head_count = meta["qwen2.attention.head_count"]
        m.kv_head_count = meta["qwen2.attention.head_count_kv"]
        m.feed_forward_length = meta["qwen2.feed_forward_length"]
        m.context_length = meta["qwen2.context_length"]
        m.rope_dimension_count = meta.get("qwen2.rope.dimension_count", m.embedding_length // m.head_count)
        m.rope_freq_base = meta["qwen2.rope.freq_base"]
        m.rms_epsilon = meta["qwen2.attention.layer_norm_rms_epsilon"]
        m.layer_start, m.layer_end = st.layer_start, st.layer_end
        tensors = {t.name: t for t in self.jfm_model.tensors()}

        def ot(name):
            t = tensors.get(name)
            if t is None:
                return OrcTensor(0, 0, 0, 0, None)
            return OrcTensor(t.type, 0, t.shape[0], t.shape[1], t.data)

        vocab_src = tensors.get("token_embd.weight") or tensors.get("output.weight")
        m.vocabulary_size = vocab_src.shape[1] if vocab_src is not None else 0  # a middle stage has neither
        m.token_embd = ot("token_embd.weight")
        m.output_norm = ot("output_norm.weight")
        m.output = ot("output.weight")
        m.output_bias = ot("output.bias")
        n_layers = st.layer_end - st.layer_start
        self._layers = (OrcLayer * n_layers)()
        for i in range(n_layers):
            prefix = f"blk.{st.layer_start + i}."
            for f in _LAYER_FIELDS:
                setattr(self._layers[i], f, ot(prefix + _LAYER_NAMES[f]))
        m.layers = self._layers
        self.model = m
        self.hidden = m.embedding_length
        self.vocab = m.vocabulary_size
        self.first = st.layer_start == 0
        self.last = st.layer_end == m.layer_count

    def session(self, capacity: int) -> "OracleSession":
        return OracleSession(self, capacity)

    def close(self):
        self.jfm_model.close()


class OracleError(ValueError):
    pass


class OracleSession:
    def __init__(self, stage: OracleStage, capacity: int):
        self.stage = stage
        self.h = lib().orc_session_create(C.byref(stage.model), capacity)
        if not self.h:
            raise OracleError("native Qwen2 cache capacity is outside model context")

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_session_destroy(self.h)
            self.h = None

    @property
    def position(self) -> int:
        return lib().orc_session_position(self.h)

    def rollback(self, n: int) -> None:
        if lib().orc_session_rollback(self.h, n) != 0:
            raise OracleError("native Qwen2 rollback exceeds the decoded suffix")

    def forward(self, prefill: bool, tokens=None, activations=None, want_logits: bool = False):
        st = self.stage
        n = len(tokens) if tokens is not None else activations.shape[0]
        tok = np.ascontiguousarray(tokens, dtype=np.int32) if tokens is not None else None
        act = np.ascontiguousarray(activations, dtype=np.float32) if activations is not None else None
        out_act = None if st.last else np.empty((n, st.hidden), dtype=np.float32)
        logits = np.empty(st.vocab, dtype=np.float32) if (st.last and want_logits) else None
        token = C.c_int32(-1)
        err = C.create_string_buffer(256)
        rc = lib().orc_session_forward(self.h, int(prefill), None if tok is None else tok.ctypes.data,
                                       None if act is None else act.ctypes.data, n,
                                       None if out_act is None else out_act.ctypes.data,
                                       None if logits is None else logits.ctypes.data, C.byref(token), err, 256)
        if rc != 0:
            raise OracleError(err.value.decode())
        return {"activations": out_act, "logits": logits, "token": token.value if st.last else None}

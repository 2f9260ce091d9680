"""Stagewire v2 frames for stage-to-stage traffic.

The reference moves every stage operation as one Stagewire v2 frame
(internal/stagewire/frame.go:36-136, types.go): a 20-byte big-endian header
(magic "JFST", version 2, flags 0, metadata length u32, payload length u64),
JSON metadata, then the raw payload, whose CRC-32 the metadata carries. This
module restates that contract:

  - `marshal` / `unmarshal` / `validate`: the frame codec with the reference's
    defaults (normalizeFrame, frame.go:245-276) and every rejection of
    Encode/Decode/Validate (frame.go:48-355), on host bytes;
  - `FramePlan` / `StagewireLink`: the same frames between pipeline stages on
    GPUs. Header and metadata of every (step, micro-batch) frame are built on
    the host once, with the metadata padded by JSON whitespace so that header
    plus metadata fill a fixed 256-byte-aligned prefix; the payload is written
    straight behind the prefix, its CRC-32 is computed and stamped into the
    metadata on the device (include/jfb/jfb_stagewire.h), and the whole frame
    goes out as one message. The receiver checksums the payload on the
    device, compares it with the received field into an error word, and
    keeps the received prefixes; `verify()` (called by `flush`) reads them
    back once and applies the full host validation. A frame is therefore
    executed before its metadata has been looked at on the host, and a bad
    frame fails the run at the next `verify()`, not before its step.

Frames built here decode with the reference's own decoder: the transport
field keeps the reference's value, since the frame layout, not the carrier,
is what it names.
"""
from __future__ import annotations

import json
import struct
import zlib
from dataclasses import dataclass, field, fields
from typing import Sequence

VERSION = 2
HEADER_SIZE = 20
MAX_METADATA_BYTES = 1 << 20
MAX_PAYLOAD_BYTES = 512 << 20
MAGIC = b"JFST"
TRANSPORT = "http_binary_v1"
CONTENT_TYPE = "application/vnd.jetsonfabric.stage.v2+octet-stream"
CRC_FIELD = 10  # JFB_STAGEWIRE_CRC_FIELD

OPERATIONS = ("execute", "close_session", "rollback_session")
PHASES = ("prefill", "decode")
PAYLOAD_KINDS = ("text", "tokens", "activation", "sampled_token", "sampled_tokens")
TENSOR_KINDS = ("tokens", "activation", "sampled_token", "sampled_tokens")
DTYPE_WIDTHS = {"u8": 1, "i8": 1, "f16": 2, "bf16": 2, "i32": 4, "u32": 4, "f32": 4, "i64": 8, "u64": 8, "f64": 8}


class StagewireError(ValueError):
    """A frame that the reference's codec rejects."""


class InvalidMagic(StagewireError):
    pass


class UnsupportedVersion(StagewireError):
    pass


class FrameTooLarge(StagewireError):
    pass


class TruncatedFrame(StagewireError):
    pass


class TrailingData(StagewireError):
    pass


class ChecksumMismatch(StagewireError):
    pass


# JSON field kinds: (lo, hi) integer ranges, "str", or ("list", lo, hi)
_U16, _U32, _U64 = (0, 0xFFFF), (0, 0xFFFFFFFF), (0, 2**64 - 1)
_I64 = (-(2**63), 2**63 - 1)


@dataclass
class Metadata:
    """types.go:46-102 Metadata, field for field and in its order (the
    embedded DeploymentIdentity's three fields sit after model_id). Each
    field's "k" is its Go type's range and "omit" its omitempty tag."""

    protocol_version: int = field(default=0, metadata={"k": _U16, "omit": False})
    operation: str = field(default="", metadata={"k": "str", "omit": False})
    session_id: str = field(default="", metadata={"k": "str", "omit": False})
    request_id: str = field(default="", metadata={"k": "str", "omit": False})
    model_id: str = field(default="", metadata={"k": "str", "omit": False})
    deployment_id: str = field(default="", metadata={"k": "str", "omit": True})
    deployment_epoch: int = field(default=0, metadata={"k": _U64, "omit": True})
    model_sha256: str = field(default="", metadata={"k": "str", "omit": True})
    phase: str = field(default="", metadata={"k": "str", "omit": False})
    decode_step: int = field(default=0, metadata={"k": _I64, "omit": False})
    stage_index: int = field(default=0, metadata={"k": _I64, "omit": False})
    stage_count: int = field(default=0, metadata={"k": _I64, "omit": False})
    node_name: str = field(default="", metadata={"k": "str", "omit": False})
    layer_start: int = field(default=0, metadata={"k": _I64, "omit": False})
    layer_end: int = field(default=0, metadata={"k": _I64, "omit": False})
    payload_kind: str = field(default="", metadata={"k": "str", "omit": False})
    encoding: str = field(default="", metadata={"k": "str", "omit": True})
    dtype: str = field(default="", metadata={"k": "str", "omit": True})
    shape: list = field(default_factory=list, metadata={"k": ("list",) + _I64, "omit": True})
    byte_order: str = field(default="", metadata={"k": "str", "omit": True})
    layout: str = field(default="", metadata={"k": "str", "omit": True})
    payload_bytes: int = field(default=0, metadata={"k": _I64, "omit": False})
    payload_crc32: int = field(default=0, metadata={"k": _U32, "omit": False})
    transport: str = field(default="", metadata={"k": "str", "omit": False})
    max_tokens: int = field(default=0, metadata={"k": _I64, "omit": True})
    rollback_tokens: int = field(default=0, metadata={"k": _I64, "omit": True})
    bytes_in: int = field(default=0, metadata={"k": _I64, "omit": True})
    bytes_out: int = field(default=0, metadata={"k": _I64, "omit": True})
    prompt_tokens: int = field(default=0, metadata={"k": _I64, "omit": True})
    prompt_token_ids: list = field(default_factory=list, metadata={"k": ("list",) + _U32, "omit": True})
    completion_tokens: int = field(default=0, metadata={"k": _I64, "omit": True})
    execution_batch_size: int = field(default=0, metadata={"k": _I64, "omit": True})
    verification_width: int = field(default=0, metadata={"k": _I64, "omit": True})
    latency_ms: int = field(default=0, metadata={"k": _I64, "omit": True})
    execution_us: int = field(default=0, metadata={"k": _I64, "omit": True})
    activation_decode_us: int = field(default=0, metadata={"k": _I64, "omit": True})
    activation_encode_us: int = field(default=0, metadata={"k": _I64, "omit": True})
    stage_total_us: int = field(default=0, metadata={"k": _I64, "omit": True})
    token_text_offsets: list = field(default_factory=list, metadata={"k": ("list",) + _U32, "omit": True})
    token_eog: list = field(default_factory=list, metadata={"k": ("list",) + _U32, "omit": True})
    error: str = field(default="", metadata={"k": "str", "omit": True})
    message: str = field(default="", metadata={"k": "str", "omit": True})
    message_bytes: list = field(default_factory=list, metadata={"k": ("list",) + _I64, "omit": True})


_FIELDS = [(f.name, f.metadata["k"], f.metadata["omit"]) for f in fields(Metadata)]
_BY_FOLD = {name.lower(): (name, kind) for name, kind, _ in _FIELDS}


@dataclass
class Frame:
    metadata: Metadata
    payload: bytes = b""


# ---- JSON -------------------------------------------------------------------


def _json_string(s: str) -> str:
    # encoding/json's default escaping: quotes, backslash, control
    # characters, and the HTML-sensitive <, >, & plus U+2028/U+2029
    out = ['"']
    for ch in s:
        o = ord(ch)
        if ch == '"':
            out.append('\\"')
        elif ch == "\\":
            out.append("\\\\")
        elif ch == "\n":
            out.append("\\n")
        elif ch == "\r":
            out.append("\\r")
        elif ch == "\t":
            out.append("\\t")
        elif o < 0x20 or ch in "<>&" or o in (0x2028, 0x2029):
            out.append(f"\\u{o:04x}")
        else:
            out.append(ch)
    out.append('"')
    return "".join(out)


def _encode_metadata(m: Metadata, crc_placeholder: bool = False) -> tuple[bytes, int]:
    """Compact JSON of `m` in field order with omitempty; with
    `crc_placeholder`, payload_crc32 is written as CRC_FIELD spaces and its
    byte offset in the result is returned (else -1)."""
    parts: list[str] = []
    offset = -1
    for name, kind, omit in _FIELDS:
        v = getattr(m, name)
        if omit and (v == 0 or v == "" or v == [] or v is None):
            continue
        prefix = ("," if parts else "{") + f'"{name}":'
        if name == "payload_crc32" and crc_placeholder:
            parts.append(prefix)
            offset = len("".join(parts).encode())
            parts.append(" " * CRC_FIELD)
            continue
        if kind == "str":
            parts.append(prefix + _json_string(v))
        elif isinstance(kind, tuple) and kind[0] == "list":
            parts.append(prefix + "[" + ",".join(str(int(x)) for x in v) + "]")
        else:
            parts.append(prefix + str(int(v)))
    parts.append("}")
    return "".join(parts).encode("utf-8"), offset


class _Pairs(list):
    """A decoded JSON object as its (key, value) pairs in document order."""


def _decode_metadata(raw: bytes) -> Metadata:
    """json.Decoder with DisallowUnknownFields into Metadata: keys match
    case-insensitively, the last duplicate wins, null leaves a field zero,
    numbers must be integers within the field's Go type."""
    try:
        text = raw.decode("utf-8")
    except UnicodeDecodeError as e:
        raise StagewireError(f"decode stagewire metadata: {e}") from None

    def no_constants(name):
        raise ValueError(f"invalid character in {name}")

    try:
        obj = json.loads(text, object_pairs_hook=_Pairs, parse_constant=no_constants)
    except ValueError as e:
        raise StagewireError(f"decode stagewire metadata: {e}") from None
    if obj is None:
        return Metadata()
    if not isinstance(obj, _Pairs):
        raise StagewireError("decode stagewire metadata: not a JSON object")
    m = Metadata()
    for key, value in obj:
        hit = _BY_FOLD.get(key.lower()) if isinstance(key, str) else None
        if hit is None:
            raise StagewireError(f'decode stagewire metadata: json: unknown field "{key}"')
        name, kind = hit
        if value is None:
            continue
        setattr(m, name, _typed(name, kind, value))
    return m


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _typed(name: str, kind, value):
    if kind == "str":
        if not isinstance(value, str):
            raise StagewireError(f"decode stagewire metadata: {name} must be a string")
        return value
    if isinstance(kind, tuple) and kind[0] == "list":
        if not isinstance(value, list) or isinstance(value, _Pairs):
            raise StagewireError(f"decode stagewire metadata: {name} must be an array")
        lo, hi = kind[1], kind[2]
        out = []
        for x in value:
            if x is None:
                out.append(0)
                continue
            if not _is_int(x) or not lo <= x <= hi:
                raise StagewireError(f"decode stagewire metadata: {name} element {x!r} out of range")
            out.append(x)
        return out
    lo, hi = kind
    if not _is_int(value) or not lo <= value <= hi:
        raise StagewireError(f"decode stagewire metadata: {name} value {value!r} out of range")
    return value


def _check_encoded_max_tokens(raw: bytes) -> None:
    """frame.go:138-155: an explicit max_tokens of zero (or null) is refused."""
    try:
        obj = json.loads(raw.decode("utf-8"), object_pairs_hook=_Pairs)
    except ValueError as e:
        raise StagewireError(f"decode stagewire metadata fields: {e}") from None
    if obj is None:
        return
    if not isinstance(obj, _Pairs):
        raise StagewireError("decode stagewire metadata fields: not a JSON object")
    present, value = False, None
    for k, v in obj:
        if k == "max_tokens":
            present, value = True, v
    if not present:
        return
    if value is not None and not _is_int(value):
        raise StagewireError("decode max_tokens: not an integer")
    if value is None or value == 0:
        raise StagewireError("max_tokens must be omitted or between 1 and 1024")


# ---- rules ------------------------------------------------------------------


def tensor_byte_length(dtype: str, shape: Sequence[int]) -> int:
    """frame.go:324-354."""
    width = DTYPE_WIDTHS.get(dtype)
    if width is None:
        raise StagewireError(f'unsupported dtype "{dtype}"')
    count = 1
    for dim in shape:
        if dim <= 0:
            raise StagewireError(f"shape dimensions must be positive, got {dim}")
        if count > MAX_PAYLOAD_BYTES // dim:
            raise FrameTooLarge("stagewire frame is too large")
        count *= dim
    if count > MAX_PAYLOAD_BYTES // width:
        raise FrameTooLarge("stagewire frame is too large")
    return count * width


def _validate_payload_metadata(m: Metadata, payload_len: int) -> None:
    """frame.go:288-322."""
    if m.error != "":
        return
    if m.payload_kind == "text":
        if m.encoding != "utf-8":
            raise StagewireError("text payload encoding must be utf-8")
        if m.shape or m.dtype or m.byte_order or m.layout:
            raise StagewireError("text payload must not declare tensor metadata")
    elif m.payload_kind in TENSOR_KINDS:
        if m.dtype.strip() == "":
            raise StagewireError("tensor payload dtype is required")
        if not m.shape:
            raise StagewireError("tensor payload shape is required")
        if m.byte_order != "little":
            raise StagewireError("tensor payload byte_order must be little")
        if m.layout != "row_major":
            raise StagewireError("tensor payload layout must be row_major")
        expected = tensor_byte_length(m.dtype, m.shape)
        if expected != payload_len:
            raise StagewireError(f"tensor metadata requires {expected} bytes, got {payload_len}")


def _validate_identity(m: Metadata) -> None:
    """frame.go:229-243."""
    if not (m.deployment_id or m.deployment_epoch or m.model_sha256):
        return
    if m.deployment_id.strip() == "" or m.deployment_epoch == 0:
        raise StagewireError("managed stagewire identity requires deployment_id and positive deployment_epoch")
    if len(m.model_sha256) != 64:
        raise StagewireError("managed stagewire identity requires a 64-character model_sha256")
    try:
        bytes.fromhex(m.model_sha256)
    except ValueError:
        raise StagewireError("managed stagewire identity requires a hexadecimal model_sha256") from None


def validate_metadata(m: Metadata, payload_len: int, payload_crc: int) -> None:
    """frame.go:157-227 Validate, given the payload's length and CRC-32."""
    if m.protocol_version != VERSION:
        raise StagewireError(f"protocol_version must be {VERSION}")
    if m.operation not in OPERATIONS:
        raise StagewireError(f'invalid operation "{m.operation}"')
    if m.operation == "rollback_session" and m.rollback_tokens <= 0:
        raise StagewireError("rollback_session requires positive rollback_tokens")
    if m.operation != "rollback_session" and m.rollback_tokens != 0:
        raise StagewireError("rollback_tokens is only valid for rollback_session")
    if m.max_tokens != 0 and not 1 <= m.max_tokens <= 1024:
        raise StagewireError("max_tokens must be between 1 and 1024")
    if m.execution_batch_size < 1:
        raise StagewireError("execution_batch_size must be positive")
    if m.verification_width < 1:
        raise StagewireError("verification_width must be positive")
    if any(v > 1 for v in m.token_eog):
        raise StagewireError("token_eog values must be 0 or 1")
    if any(v < 0 or v > 255 for v in m.message_bytes):
        raise StagewireError("message_bytes values must be between 0 and 255")
    for name in ("session_id", "request_id", "model_id"):
        if getattr(m, name).strip() == "":
            raise StagewireError(f"{name} is required")
    _validate_identity(m)
    if m.phase not in PHASES:
        raise StagewireError(f'invalid phase "{m.phase}"')
    if m.stage_count <= 0:
        raise StagewireError("stage count must be greater than zero")
    if m.stage_index < 0 or m.stage_index >= m.stage_count:
        raise StagewireError(f"stage index {m.stage_index} must be in [0,{m.stage_count})")
    if m.layer_start < 0 or m.layer_end <= m.layer_start:
        raise StagewireError(f"invalid layer range [{m.layer_start}:{m.layer_end})")
    if m.payload_kind not in PAYLOAD_KINDS:
        raise StagewireError(f'invalid payload_kind "{m.payload_kind}"')
    if m.payload_bytes != payload_len:
        raise StagewireError(f"payload_bytes={m.payload_bytes} does not match payload length {payload_len}")
    if m.payload_bytes > MAX_PAYLOAD_BYTES:
        raise FrameTooLarge("stagewire frame is too large")
    if payload_crc != m.payload_crc32:
        raise ChecksumMismatch(f"stagewire payload checksum mismatch: metadata={m.payload_crc32:08x} "
                               f"actual={payload_crc:08x}")
    if m.transport != TRANSPORT:
        raise StagewireError(f'transport must be "{TRANSPORT}"')
    _validate_payload_metadata(m, payload_len)


def validate(frame: Frame) -> None:
    validate_metadata(frame.metadata, len(frame.payload), zlib.crc32(frame.payload))


def _telemetry_defaults(m: Metadata) -> None:
    if m.execution_batch_size == 0:
        m.execution_batch_size = 1
    if m.verification_width == 0:
        m.verification_width = 1


def normalize(m: Metadata, payload_len: int, payload_crc: int) -> Metadata:
    """frame.go:245-276 normalizeFrame on a copy of `m`."""
    m = Metadata(**{f.name: (list(getattr(m, f.name)) if isinstance(getattr(m, f.name), list)
                             else getattr(m, f.name)) for f in fields(Metadata)})
    _telemetry_defaults(m)
    m.protocol_version = VERSION
    if m.operation == "":
        m.operation = "execute"
    if m.operation == "execute" and m.max_tokens == 0:
        m.max_tokens = 128
    if m.phase == "":
        m.phase = "prefill" if m.decode_step == 0 else "decode"
    if m.payload_kind == "text" and m.encoding == "":
        m.encoding = "utf-8"
    if m.payload_kind in TENSOR_KINDS:
        if m.byte_order == "":
            m.byte_order = "little"
        if m.layout == "":
            m.layout = "row_major"
    m.payload_bytes = payload_len
    m.payload_crc32 = payload_crc
    m.transport = TRANSPORT
    return m


def _header(metadata_len: int, payload_len: int) -> bytes:
    return MAGIC + struct.pack(">HHIQ", VERSION, 0, metadata_len, payload_len)


def marshal(frame: Frame) -> bytes:
    """frame.go:36-79 Marshal/Encode."""
    payload = bytes(frame.payload)
    m = normalize(frame.metadata, len(payload), zlib.crc32(payload))
    validate(Frame(m, payload))
    meta, _ = _encode_metadata(m)
    if len(meta) > MAX_METADATA_BYTES or len(payload) > MAX_PAYLOAD_BYTES:
        raise FrameTooLarge("stagewire frame is too large")
    return _header(len(meta), len(payload)) + meta + payload


def parse_prefix(data: bytes) -> tuple[int, int]:
    """Header checks of frame.go:81-104; returns (metadata_len, payload_len)."""
    if len(data) < HEADER_SIZE:
        raise TruncatedFrame("truncated stagewire frame: header")
    if data[:4] != MAGIC:
        raise InvalidMagic("invalid stagewire magic")
    version, flags, meta_len, payload_len = struct.unpack(">HHIQ", data[4:HEADER_SIZE])
    if version != VERSION:
        raise UnsupportedVersion(f"unsupported stagewire version: {version}")
    if flags != 0:
        raise StagewireError(f"stagewire flags must be zero, got {flags}")
    if meta_len == 0 or meta_len > MAX_METADATA_BYTES or payload_len > MAX_PAYLOAD_BYTES:
        raise FrameTooLarge("stagewire frame is too large")
    return meta_len, payload_len


def decode_metadata(raw: bytes, payload_len: int, payload_crc: int) -> Metadata:
    """frame.go:117-135 after the bytes are read: metadata decoding, the
    explicit-zero max_tokens check, the version match, the telemetry
    defaults and Validate."""
    m = _decode_metadata(raw)
    _check_encoded_max_tokens(raw)
    if m.protocol_version != VERSION:
        raise StagewireError(f"metadata protocol_version {m.protocol_version} does not match frame version {VERSION}")
    _telemetry_defaults(m)
    validate_metadata(m, payload_len, payload_crc)
    return m


def unmarshal(data: bytes) -> Frame:
    """frame.go:44-136 Unmarshal/Decode."""
    data = bytes(data)
    meta_len, payload_len = parse_prefix(data)
    if len(data) < HEADER_SIZE + meta_len:
        raise TruncatedFrame("truncated stagewire frame: metadata")
    raw = data[HEADER_SIZE:HEADER_SIZE + meta_len]
    end = HEADER_SIZE + meta_len + payload_len
    if len(data) < end:
        raise TruncatedFrame("truncated stagewire frame: payload")
    if len(data) > end:
        raise TrailingData("stagewire frame has trailing data")
    payload = data[HEADER_SIZE + meta_len:end]
    return Frame(decode_metadata(raw, payload_len, zlib.crc32(payload)), payload)


# ---- frames between pipeline stages ---------------------------------------------


def frame_prefix(m: Metadata, payload_len: int, prefix_bytes: int) -> tuple[bytes, int]:
    """Header plus metadata of a frame whose payload is not known yet, padded
    with trailing JSON whitespace to exactly `prefix_bytes`. Returns the
    prefix and the offset of the CRC_FIELD-wide payload_crc32 value within
    it. Every rule except the checksum is checked here."""
    m = normalize(m, payload_len, 0)
    validate_metadata(m, payload_len, 0)
    meta, off = _encode_metadata(m, crc_placeholder=True)
    room = prefix_bytes - HEADER_SIZE
    if len(meta) > room:
        raise FrameTooLarge(f"stagewire metadata of {len(meta)} bytes exceeds the {room}-byte prefix")
    meta = meta + b" " * (room - len(meta))
    return _header(len(meta), payload_len) + meta, HEADER_SIZE + off


@dataclass
class FramePlan:
    """Who sends what: the frame metadata of every message of a
    `pipeline.run_schedule` run, from the same (step, micro-batch) order
    that every rank follows. `stage_layers` are the ranks' layer ranges;
    activations travel as F16 codec bits [rows, hidden] to stage r + 1,
    sampled tokens as u32 [count] from the last stage to stage 0."""

    model_id: str
    stage_layers: Sequence[tuple[int, int]]
    batches: Sequence[Sequence[int]]
    prompt_lengths: Sequence[int]
    steps: int
    hidden: int
    request_id: str = "pipeline"
    max_tokens: int = 0
    prefix_bytes: int = 1024

    def rows(self, step: int, m: int) -> int:
        mb = self.batches[m]
        return sum(self.prompt_lengths[s] for s in mb) if step == 0 else len(mb)

    def _common(self, step: int, m: int, to_stage: int) -> Metadata:
        a, b = self.stage_layers[to_stage]
        mb = self.batches[m]
        return Metadata(
            operation="execute", session_id=f"{self.request_id}-mb{m}-s{mb[0]}-{mb[-1]}",
            request_id=f"{self.request_id}-step{step}-mb{m}-stage{to_stage}", model_id=self.model_id,
            phase="prefill" if step == 0 else "decode", decode_step=step, stage_index=to_stage,
            stage_count=len(self.stage_layers), node_name=f"stage-{to_stage}", layer_start=a, layer_end=b,
            max_tokens=self.max_tokens or min(1024, max(1, self.steps)), execution_batch_size=len(mb))

    def activation(self, step: int, m: int, to_stage: int) -> tuple[Metadata, int]:
        rows = self.rows(step, m)
        md = self._common(step, m, to_stage)
        md.payload_kind, md.dtype, md.shape = "activation", "f16", [rows, self.hidden]
        return md, rows * self.hidden * 2

    def tokens(self, step: int, m: int) -> tuple[Metadata, int]:
        n = len(self.batches[m])
        md = self._common(step + 1, m, 0)
        md.payload_kind, md.dtype, md.shape = "sampled_tokens", "u32", [n]
        return md, n * 4


class StagewireLink:
    """`pipeline.TorchLink` traffic as Stagewire v2 frames (one message per
    frame). Works on CUDA tensors over NCCL, where checksums are formed and
    compared on the device, and on CPU tensors over gloo, where they are
    formed on the host as the reference's Go codec does."""

    def __init__(self, base, rank: int, plan: FramePlan, device=None, stream=None):
        import torch

        self.torch, self.base, self.rank, self.plan = torch, base, rank, plan
        self.world = len(plan.stage_layers)
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.cuda = self.device.type == "cuda"
        self.stream = stream
        self.P = plan.prefix_bytes
        if self.P % 256 != 0 or self.P <= HEADER_SIZE:
            raise ValueError("the frame prefix must be a positive multiple of 256 bytes")
        M = len(plan.batches)
        self.M = M
        first, last = rank == 0, rank == self.world - 1
        # outgoing prefixes, one row per message this rank sends, uploaded once
        self.out_offsets: list[int] = []
        rows = []
        if not last:
            for step in range(plan.steps):
                for m in range(M):
                    md, n = plan.activation(step, m, rank + 1)
                    pre, off = frame_prefix(md, n, self.P)
                    rows.append(pre)
                    self.out_offsets.append(off)
        elif self.world > 1:
            for step in range(plan.steps - 1):
                for m in range(M):
                    md, n = plan.tokens(step, m)
                    pre, off = frame_prefix(md, n, self.P)
                    rows.append(pre)
                    self.out_offsets.append(off)
        self.out_prefix = self._table(rows)
        # what this rank expects to receive, in receive order
        self.expect: list[tuple[bytes, int, int]] = []  # (prefix, crc offset, payload bytes)
        if not first:
            for step in range(plan.steps):
                for m in range(M):
                    md, n = plan.activation(step, m, rank)
                    pre, off = frame_prefix(md, n, self.P)
                    self.expect.append((pre, off, n))
        elif self.world > 1:
            for step in range(plan.steps - 1):
                for m in range(M):
                    md, n = plan.tokens(step, m)
                    pre, off = frame_prefix(md, n, self.P)
                    self.expect.append((pre, off, n))
        R = max(1, len(self.expect))
        self.recv_log = torch.zeros((R, self.P), dtype=torch.uint8, device=self.device)
        self.recv_crc = torch.zeros(R, dtype=torch.int64 if not self.cuda else torch.int32, device=self.device)
        self.send_crc = torch.zeros(max(1, len(self.out_offsets)), dtype=torch.int32, device=self.device)
        self.mismatch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.sent = self.received = self.verified = 0
        self.scratch = None
        if self.cuda:
            from . import kernels

            self.kernels = kernels
            biggest = max([n for _, _, n in self.expect] + [self._out_payload(k) for k in range(len(self.out_offsets))]
                          + [0])
            self.scratch = torch.empty(max(256, kernels.crc32_scratch_bytes(biggest)), dtype=torch.uint8,
                                       device=self.device)

    def _table(self, rows: list[bytes]):
        torch = self.torch
        if not rows:
            return torch.zeros((1, self.P), dtype=torch.uint8, device=self.device)
        host = torch.frombuffer(bytearray(b"".join(rows)), dtype=torch.uint8).view(len(rows), self.P)
        return host.to(self.device)

    def _out_payload(self, k: int) -> int:
        step, m = divmod(k, self.M)
        if self.rank == self.world - 1:
            return self.plan.tokens(step, m)[1]
        return self.plan.activation(step, m, self.rank + 1)[1]

    # -- sending --------------------------------------------------------------

    def _frame_out(self, nbytes: int):
        k = self.sent
        if k >= len(self.out_offsets):
            raise StagewireError("more frames sent than the schedule holds")
        if nbytes != self._out_payload(k):
            raise StagewireError(f"frame {k}: payload of {nbytes} bytes, the schedule says {self._out_payload(k)}")
        frame = self.torch.empty(self.P + nbytes, dtype=self.torch.uint8, device=self.device)
        frame[:self.P].copy_(self.out_prefix[k])
        return k, frame

    def _seal(self, k: int, frame) -> None:
        off = self.out_offsets[k]
        payload = frame[self.P:]
        if self.cuda:
            crc = self.send_crc[k:k + 1]
            self.kernels.crc32(payload, crc, self.scratch, stream=self.stream)
            self.kernels.stagewire_stamp_crc(crc, frame, off, stream=self.stream)
        else:
            value = zlib.crc32(payload.numpy().tobytes())
            frame[off:off + CRC_FIELD] = self.torch.frombuffer(bytearray(f"{value:>{CRC_FIELD}d}".encode()),
                                                               dtype=self.torch.uint8)
        self.sent = k + 1

    def send_activation(self, stage, activations) -> None:
        rows = activations.shape[0]
        k, frame = self._frame_out(rows * stage.hidden * 2)
        payload = frame[self.P:].view(self.torch.float16).view(rows, stage.hidden)
        stage.encode(activations, out=payload)
        self._seal(k, frame)
        self.base.send_next(frame)

    def send_tokens(self, tokens) -> None:
        k, frame = self._frame_out(tokens.numel() * 4)
        frame[self.P:].view(self.torch.int32).copy_(tokens.reshape(-1))
        self._seal(k, frame)
        self.base.send_tokens(frame)

    # -- receiving ------------------------------------------------------------

    def _frame_in(self, nbytes: int):
        k = self.received
        if k >= len(self.expect):
            raise StagewireError("more frames received than the schedule holds")
        if nbytes != self.expect[k][2]:
            raise StagewireError(f"frame {k}: expected a payload of {self.expect[k][2]} bytes, asked for {nbytes}")
        return k, self.torch.empty(self.P + nbytes, dtype=self.torch.uint8, device=self.device)

    def _check(self, k: int, frame) -> None:
        off = self.expect[k][1]
        payload = frame[self.P:]
        if self.cuda:
            crc = self.recv_crc[k:k + 1]
            self.kernels.crc32(payload, crc, self.scratch, stream=self.stream)
            self.kernels.stagewire_check_crc(crc, frame, off, self.mismatch, stream=self.stream)
        else:
            self.recv_crc[k] = zlib.crc32(payload.numpy().tobytes())
        self.recv_log[k].copy_(frame[:self.P])
        self.received = k + 1

    def recv_activation(self, stage, rows: int):
        k, frame = self._frame_in(rows * stage.hidden * 2)
        self.base.recv_prev(frame)
        self._check(k, frame)
        return frame[self.P:].view(self.torch.float16).view(rows, stage.hidden)

    def recv_tokens(self, tokens) -> None:
        k, frame = self._frame_in(tokens.numel() * 4)
        self.base.recv_tokens(frame)
        self._check(k, frame)
        tokens.reshape(-1).copy_(frame[self.P:].view(self.torch.int32))

    def flush(self) -> None:
        """End of a schedule: waits for the sends, verifies every received
        frame, and rewinds the frame counters for the next run."""
        self.base.flush()
        self.verify()
        if self.sent not in (0, len(self.out_offsets)) or self.received not in (0, len(self.expect)):
            raise StagewireError(f"schedule ended after {self.sent} of {len(self.out_offsets)} sends and "
                                 f"{self.received} of {len(self.expect)} receives")
        self.sent = self.received = self.verified = 0

    def verify(self) -> int:
        """Host validation of every frame received since the last call: the
        received prefix must pass the reference decoder's checks with the
        device-computed payload CRC, and must be the frame the schedule
        says this stage gets. Returns the number of frames checked."""
        if self.cuda:
            if self.stream is None:
                self.torch.cuda.current_stream(self.device).synchronize()
            else:
                self.stream.synchronize()
        lo, hi = self.verified, self.received
        if hi == lo:
            return 0
        log = self.recv_log[lo:hi].cpu().numpy()
        crcs = self.recv_crc[lo:hi].cpu().numpy()
        if self.cuda and int(self.mismatch.item()) != 0:
            raise ChecksumMismatch("stagewire payload checksum mismatch (device check)")
        for i in range(hi - lo):
            k = lo + i
            pre = log[i].tobytes()
            expected, off, n = self.expect[k]
            crc = int(crcs[i]) & 0xFFFFFFFF
            stamped = expected[:off] + f"{crc:>{CRC_FIELD}d}".encode() + expected[off + CRC_FIELD:]
            if pre == stamped:
                # the expected prefix passed every rule when it was built, and
                # its checksum field matches the received payload
                continue
            # anything else: the decoder's own error first, then the mismatch
            meta_len, payload_len = parse_prefix(pre)
            if HEADER_SIZE + meta_len != self.P:
                raise StagewireError(f"frame {k}: metadata does not fill the {self.P}-byte prefix")
            if payload_len != n:
                raise StagewireError(f"frame {k}: payload length {payload_len}, expected {n}")
            md = decode_metadata(pre[HEADER_SIZE:], payload_len, crc)
            raise StagewireError(f"frame {k}: metadata differs from the schedule's "
                                 f"(request {md.request_id!r}, stage {md.stage_index})")
        self.verified = hi
        return hi - lo


# ---- the in-box frame channel (include/jfb/jfb_stagewire.h) -----------------------

JFB_STATUS_TIMEOUT = 9


class ChannelTimeout(TimeoutError):
    """A bounded wait of the frame channel gave up."""


class FrameChannel:
    """ctypes binding of `jfb_frame_channel_*`: Stagewire frames between
    processes on one host through shared memory. `FrameChannel.create(name)`
    is the server side (`receive` / `reply`), `FrameChannel.open(name)` the
    caller side (`call`). Needs no GPU."""

    _bound = None

    def __init__(self, handle, server: bool):
        self._h, self.server = handle, server

    @classmethod
    def _lib(cls):
        if cls._bound is None:
            import ctypes as C

            from .engine import Status, lib

            L = lib()
            vp, u64, u32, i32 = C.c_void_p, C.c_uint64, C.c_uint32, C.c_int32
            sig = {
                "jfb_frame_channel_create": ([C.c_char_p, u64, C.POINTER(vp)], Status),
                "jfb_frame_channel_open": ([C.c_char_p, u32, C.POINTER(vp)], Status),
                "jfb_frame_channel_capacity": ([vp], u64),
                "jfb_frame_channel_call": ([vp, C.c_char_p, u64, C.c_char_p, u64, u32, C.POINTER(i32), C.POINTER(i32),
                                            C.POINTER(C.POINTER(C.c_uint8)), C.POINTER(u64)], Status),
                "jfb_frame_channel_receive": ([vp, u32, C.POINTER(C.POINTER(C.c_uint8)), C.POINTER(u64)], Status),
                "jfb_frame_channel_reply": ([vp, i32, i32, C.c_char_p, u64, C.c_char_p, u64], Status),
                "jfb_frame_channel_close": ([vp], None),
            }
            for name, (args, res) in sig.items():
                fn = getattr(L, name)
                fn.argtypes, fn.restype = args, res
            cls._bound = L
        return cls._bound

    @staticmethod
    def _check(st) -> None:
        from .engine import check

        if st.code == JFB_STATUS_TIMEOUT:
            raise ChannelTimeout(st.message.decode(errors="replace"))
        check(st)

    @classmethod
    def create(cls, name: str, capacity: int = 0) -> "FrameChannel":
        import ctypes as C

        h = C.c_void_p()
        cls._check(cls._lib().jfb_frame_channel_create(name.encode(), capacity, C.byref(h)))
        return cls(h, True)

    @classmethod
    def open(cls, name: str, timeout_ms: int = 5000) -> "FrameChannel":
        import ctypes as C

        h = C.c_void_p()
        cls._check(cls._lib().jfb_frame_channel_open(name.encode(), timeout_ms, C.byref(h)))
        return cls(h, False)

    @property
    def capacity(self) -> int:
        return int(self._lib().jfb_frame_channel_capacity(self._h))

    def call(self, head: bytes, body: bytes = b"", timeout_ms: int = 5000) -> tuple[int, bool, bytes]:
        """Sends head || body; returns (status, is_frame, reply bytes)."""
        import ctypes as C

        status, is_frame = C.c_int32(), C.c_int32()
        reply, n = C.POINTER(C.c_uint8)(), C.c_uint64()
        self._check(self._lib().jfb_frame_channel_call(self._h, head, len(head), body, len(body), timeout_ms,
                                                       C.byref(status), C.byref(is_frame), C.byref(reply),
                                                       C.byref(n)))
        return status.value, bool(is_frame.value), C.string_at(reply, n.value) if n.value else b""

    def receive(self, timeout_ms: int = 5000) -> bytes:
        import ctypes as C

        frame, n = C.POINTER(C.c_uint8)(), C.c_uint64()
        self._check(self._lib().jfb_frame_channel_receive(self._h, timeout_ms, C.byref(frame), C.byref(n)))
        return C.string_at(frame, n.value) if n.value else b""

    def reply(self, status: int, is_frame: bool, head: bytes, body: bytes = b"") -> None:
        self._check(self._lib().jfb_frame_channel_reply(self._h, status, 1 if is_frame else 0, head, len(head),
                                                        body, len(body)))

    def close(self) -> None:
        if self._h:
            self._lib().jfb_frame_channel_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

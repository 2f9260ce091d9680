"""Stagewire v2 frame codec (jetsonfabric_b200/stagewire.py) against the
reference's contract.

The cases restate the reference's own codec tests
(internal/stagewire/frame_test.go:14-265, operation_test.go:9-70): binary
activation round trip with the CRC of Go's crc32.ChecksumIEEE (zlib's
crc32), text and full v2 metadata round trips, the rollback and telemetry
rules, every Marshal rejection, and the Decode rejections of a corrupted,
truncated or extended frame. Go is not installed here, so no frame bytes of
the reference's encoder are pinned; the rules are.

The CRC-32 combine method that the device kernel uses is checked here on the
host against zlib; the device kernel itself is checked in the GPU test.
"""
from __future__ import annotations

import json
import struct
import zlib
from pathlib import Path

import numpy as np
import pytest

from jetsonfabric_b200 import stagewire as sw
from jetsonfabric_b200.stagewire import Frame, Metadata


def _activation_frame() -> bytes:
    return sw.marshal(Frame(Metadata(session_id="s", request_id="r", model_id="m", stage_index=0, stage_count=2,
                                     node_name="node", layer_start=0, layer_end=1, payload_kind="activation",
                                     dtype="f32", shape=[1]), b"\0\0\0\0"))


def _with_metadata(encoded: bytes, edit) -> bytes:
    meta_len = struct.unpack(">I", encoded[8:12])[0]
    md = json.loads(encoded[sw.HEADER_SIZE:sw.HEADER_SIZE + meta_len])
    edit(md)
    raw = json.dumps(md, separators=(",", ":")).encode()
    header = bytearray(encoded[:sw.HEADER_SIZE])
    header[8:12] = struct.pack(">I", len(raw))
    return bytes(header) + raw + encoded[sw.HEADER_SIZE + meta_len:]


def test_activation_round_trip_keeps_binary_payload():
    payload = bytearray((i * 37) % 251 for i in range(4 * 16 * 4))
    payload[3] = 0
    payload[127] = 0
    payload = bytes(payload)
    encoded = sw.marshal(Frame(Metadata(session_id="session-1", request_id="request-1", model_id="model",
                                        phase="prefill", stage_index=1, stage_count=2, node_name="stage-1",
                                        layer_start=14, layer_end=28, payload_kind="activation", dtype="f32",
                                        shape=[4, 16], execution_us=1200, activation_decode_us=10,
                                        activation_encode_us=20, stage_total_us=1300), payload))
    assert b"AA==" not in encoded[sw.HEADER_SIZE:]
    assert encoded[:4] == b"JFST" and struct.unpack(">HH", encoded[4:8]) == (2, 0)
    assert struct.unpack(">Q", encoded[12:20])[0] == len(payload)
    f = sw.unmarshal(encoded)
    assert f.payload == payload
    assert f.metadata.payload_crc32 == zlib.crc32(payload)
    assert f.metadata.payload_bytes == len(payload) and f.metadata.dtype == "f32" and f.metadata.shape == [4, 16]
    m = f.metadata
    assert (m.execution_us, m.activation_decode_us, m.activation_encode_us, m.stage_total_us) == (1200, 10, 20, 1300)
    # Go's encoder: compact, struct field order, omitempty fields dropped
    meta = encoded[sw.HEADER_SIZE:sw.HEADER_SIZE + struct.unpack(">I", encoded[8:12])[0]].decode()
    assert meta.startswith('{"protocol_version":2,"operation":"execute","session_id":"session-1",')
    assert '"deployment_id"' not in meta and '"rollback_tokens"' not in meta
    keys = list(json.loads(meta).keys())
    order = [f.name for f in sw.fields(Metadata)]
    assert keys == sorted(keys, key=order.index)


def test_text_round_trip_with_identity():
    ident = dict(deployment_id="deployment-a", deployment_epoch=3, model_sha256="a" * 64)
    encoded = sw.marshal(Frame(Metadata(session_id="s", request_id="r", model_id="m", stage_index=0, stage_count=1,
                                        node_name="node", layer_start=0, layer_end=1, payload_kind="text", **ident),
                               b"hello"))
    f = sw.unmarshal(encoded)
    assert f.payload == b"hello" and f.metadata.encoding == "utf-8" and f.metadata.phase == "prefill"
    assert (f.metadata.deployment_id, f.metadata.deployment_epoch, f.metadata.model_sha256) == tuple(ident.values())


def test_version_two_metadata_round_trip():
    md = Metadata(operation="execute", session_id="session-v2", request_id="request-v2", model_id="model-v2",
                  phase="decode", decode_step=7, stage_index=1, stage_count=2, node_name="stage-1", layer_start=14,
                  layer_end=28, payload_kind="sampled_tokens", dtype="u32", shape=[2], max_tokens=128,
                  bytes_in=24576, bytes_out=8, prompt_tokens=4, prompt_token_ids=[1, 2, 3, 4], completion_tokens=2,
                  execution_batch_size=1, verification_width=2, latency_ms=12, execution_us=9000,
                  activation_decode_us=100, activation_encode_us=200, stage_total_us=9500,
                  token_text_offsets=[0, 3, 8], token_eog=[0, 1], message_bytes=[111, 107])
    payload = bytes([11, 0, 0, 0, 12, 0, 0, 0])
    f = sw.unmarshal(sw.marshal(Frame(md, payload)))
    m = f.metadata
    assert m.protocol_version == 2 and m.operation == "execute" and m.verification_width == 2
    assert m.execution_batch_size == 1 and m.prompt_token_ids == [1, 2, 3, 4]
    assert m.token_text_offsets == [0, 3, 8] and m.token_eog == [0, 1] and f.payload == payload


def test_rollback_needs_positive_tokens():
    md = Metadata(operation="rollback_session", session_id="s", request_id="r", model_id="m", stage_index=0,
                  stage_count=1, node_name="node", layer_start=0, layer_end=1, payload_kind="text")
    with pytest.raises(sw.StagewireError):
        sw.marshal(Frame(md))
    md.rollback_tokens = 2
    sw.marshal(Frame(md))
    md.operation, md.rollback_tokens = "execute", 1
    with pytest.raises(sw.StagewireError, match="only valid for rollback_session"):
        sw.marshal(Frame(md, b"x"))


def test_decode_defaults_omitted_telemetry_widths():
    def strip(md):
        md.pop("execution_batch_size", None)
        md.pop("verification_width", None)

    f = sw.unmarshal(_with_metadata(_activation_frame(), strip))
    assert f.metadata.execution_batch_size == 1 and f.metadata.verification_width == 1


@pytest.mark.parametrize("edit", [
    dict(execution_batch_size=-1), dict(verification_width=-1), dict(token_eog=[2]), dict(message_bytes=[256]),
    dict(max_tokens=1025), dict(message_bytes=[-1]), dict(phase="warmup"), dict(operation="restart"),
    dict(stage_index=1, stage_count=1), dict(stage_count=0), dict(layer_start=1, layer_end=1),
    dict(layer_start=-1), dict(payload_kind="logits"), dict(session_id="  "), dict(request_id=""),
    dict(model_id=""),
])
def test_marshal_rejects_invalid_metadata(edit):
    md = Metadata(session_id="s", request_id="r", model_id="m", stage_index=0, stage_count=1, node_name="node",
                  layer_start=0, layer_end=1, payload_kind="text")
    for k, v in edit.items():
        setattr(md, k, v)
    with pytest.raises(sw.StagewireError):
        sw.marshal(Frame(md, b"hello"))


@pytest.mark.parametrize("ident", [
    dict(deployment_id="deployment-a"), dict(deployment_id="deployment-a", deployment_epoch=1),
    dict(deployment_id="deployment-a", deployment_epoch=1, model_sha256="not-a-digest"),
    dict(deployment_id="deployment-a", deployment_epoch=1, model_sha256="g" * 64),
])
def test_marshal_rejects_partial_deployment_identity(ident):
    md = Metadata(session_id="s", request_id="r", model_id="m", stage_index=0, stage_count=1, node_name="node",
                  layer_start=0, layer_end=1, payload_kind="text", **ident)
    with pytest.raises(sw.StagewireError):
        sw.marshal(Frame(md, b"hello"))


def test_decode_rejects_corruption_and_truncation():
    encoded = _activation_frame()
    bad = bytearray(encoded)
    bad[0] = ord("X")
    with pytest.raises(sw.InvalidMagic):
        sw.unmarshal(bytes(bad))
    bad = bytearray(encoded)
    bad[4:6] = struct.pack(">H", 99)
    with pytest.raises(sw.UnsupportedVersion):
        sw.unmarshal(bytes(bad))
    with pytest.raises(sw.TruncatedFrame):
        sw.unmarshal(encoded[:-1])
    with pytest.raises(sw.TruncatedFrame):
        sw.unmarshal(encoded[:10])
    bad = bytearray(encoded)
    bad[-1] ^= 0xFF
    with pytest.raises(sw.ChecksumMismatch):
        sw.unmarshal(bytes(bad))
    with pytest.raises(sw.TrailingData):
        sw.unmarshal(encoded + b"\x01")
    bad = bytearray(encoded)
    bad[6:8] = struct.pack(">H", 1)
    with pytest.raises(sw.StagewireError, match="flags"):
        sw.unmarshal(bytes(bad))
    bad = bytearray(encoded)
    bad[8:12] = struct.pack(">I", 0)
    with pytest.raises(sw.FrameTooLarge):
        sw.unmarshal(bytes(bad))
    bad = bytearray(encoded)
    bad[12:20] = struct.pack(">Q", sw.MAX_PAYLOAD_BYTES + 1)
    with pytest.raises(sw.FrameTooLarge):
        sw.unmarshal(bytes(bad))


def test_decode_metadata_rules():
    encoded = _activation_frame()
    for edit in (lambda md: md.update(unexpected=1),                       # DisallowUnknownFields
                 lambda md: md.pop("operation"),                            # operation required on decode
                 lambda md: md.update(max_tokens=0),                        # explicit zero max_tokens
                 lambda md: md.update(max_tokens=None),
                 lambda md: md.update(protocol_version=1),                  # version mismatch
                 lambda md: md.update(transport="grpc"),
                 lambda md: md.update(payload_bytes=5),
                 lambda md: md.update(stage_index=1.5),                     # not an integer
                 lambda md: md.update(payload_crc32=-1),                    # out of the uint32 range
                 lambda md: md.update(shape=[0]),                           # dimensions must be positive
                 lambda md: md.update(byte_order="big"),
                 lambda md: md.update(layout="column_major"),
                 lambda md: md.update(dtype="f8")):
        with pytest.raises(sw.StagewireError):
            sw.unmarshal(_with_metadata(encoded, edit))
    # keys match case-insensitively and null leaves a field at its zero value
    f = sw.unmarshal(_with_metadata(encoded, lambda md: md.update(Session_ID=md.pop("session_id"), error=None)))
    assert f.metadata.session_id == "s"
    # a JSON array is not an object
    meta_len = struct.unpack(">I", encoded[8:12])[0]
    raw = b'[["session_id","s"]]'
    arr = encoded[:8] + struct.pack(">I", len(raw)) + encoded[12:20] + raw + encoded[sw.HEADER_SIZE + meta_len:]
    with pytest.raises(sw.StagewireError):
        sw.unmarshal(arr)


def test_tensor_length_mismatch_and_sizes():
    md = Metadata(session_id="s", request_id="r", model_id="m", stage_index=0, stage_count=2, node_name="node",
                  layer_start=0, layer_end=1, payload_kind="activation", dtype="f32", shape=[2, 2])
    with pytest.raises(sw.StagewireError, match="requires 16 bytes"):
        sw.marshal(Frame(md, bytes(12)))
    assert sw.tensor_byte_length("bf16", [3, 5]) == 30
    with pytest.raises(sw.FrameTooLarge):
        sw.tensor_byte_length("f64", [1 << 20, 1 << 20])
    with pytest.raises(sw.StagewireError, match="unsupported dtype"):
        sw.tensor_byte_length("f8", [1])


def test_execute_is_the_default_operation_and_close_allows_empty_payload():
    md = Metadata(session_id="session", request_id="request", model_id="model", phase="prefill", stage_index=0,
                  stage_count=1, node_name="node", layer_start=0, layer_end=1, payload_kind="text", encoding="utf-8")
    f = sw.unmarshal(sw.marshal(Frame(md, b"prompt")))
    assert f.metadata.operation == "execute" and f.metadata.max_tokens == 128
    md.operation, md.stage_count, md.request_id = "close_session", 2, "request-close"
    sw.marshal(Frame(md))
    # the phase defaults from decode_step
    md2 = Metadata(session_id="s", request_id="r", model_id="m", stage_index=0, stage_count=1, node_name="n",
                   layer_start=0, layer_end=1, payload_kind="text", decode_step=3)
    assert sw.unmarshal(sw.marshal(Frame(md2, b"t"))).metadata.phase == "decode"


def test_json_string_escaping_decodes_back():
    s = 'a"b\\c\n\t<tag>& \x01é'
    md = Metadata(session_id=s, request_id="r", model_id="m", stage_index=0, stage_count=1, node_name="n",
                  layer_start=0, layer_end=1, payload_kind="text")
    encoded = sw.marshal(Frame(md, b"x"))
    assert b"<" not in encoded and b"\\u003c" in encoded
    assert sw.unmarshal(encoded).metadata.session_id == s


def test_frame_prefix_is_a_valid_frame_once_stamped():
    """The device frame layout: header + metadata padded with JSON whitespace
    to a fixed prefix, payload behind it, CRC stamped right-aligned into a
    10-character field. Stamped the way jfb_stagewire_stamp_crc does it, the
    bytes must decode with the codec's full rules."""
    plan = sw.FramePlan(model_id="qwen2", stage_layers=[(0, 14), (14, 28)], batches=[[0, 1], [2]],
                        prompt_lengths=[5, 3, 4], steps=4, hidden=8)
    rng = np.random.default_rng(0)
    for step in range(plan.steps):
        for m in range(2):
            md, n = plan.activation(step, m, 1)
            pre, off = sw.frame_prefix(md, n, 1024)
            assert len(pre) == 1024 and pre[off:off + sw.CRC_FIELD] == b" " * sw.CRC_FIELD
            payload = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
            crc = zlib.crc32(payload)
            frame = pre[:off] + f"{crc:>10d}".encode() + pre[off + 10:] + payload
            f = sw.unmarshal(frame)
            assert f.metadata.payload_crc32 == crc and f.metadata.shape == [plan.rows(step, m), 8]
            assert f.metadata.phase == ("prefill" if step == 0 else "decode") and f.metadata.stage_index == 1
            bad = bytearray(frame)
            bad[-1] ^= 1
            with pytest.raises(sw.ChecksumMismatch):
                sw.unmarshal(bytes(bad))
    md, n = plan.tokens(0, 1)
    pre, off = sw.frame_prefix(md, n, 1024)
    assert sw.unmarshal(pre[:off] + f"{zlib.crc32(bytes(4)):>10d}".encode() + pre[off + 10:] + bytes(4)).metadata \
        .payload_kind == "sampled_tokens"
    with pytest.raises(sw.FrameTooLarge):
        sw.frame_prefix(md, n, 256)


# ---- the combine arithmetic of the device CRC ---------------------------------------

_POLY = 0xEDB88320


def _mulmod(a: int, b: int) -> int:
    p = 0
    for i in range(32):
        if a & (0x80000000 >> i):
            p ^= b
        b = (b >> 1) ^ _POLY if b & 1 else b >> 1
    return p


def _xpow_bytes(n: int) -> int:
    r, x = 0x80000000, 0x00800000
    while n:
        if n & 1:
            r = _mulmod(r, x)
        x = _mulmod(x, x)
        n >>= 1
    return r


def _raw(data: bytes) -> int:
    # register after feeding `data` from 0: crc32 with pre/post conditioning undone
    return zlib.crc32(data) ^ 0xFFFFFFFF ^ _mulmod(0xFFFFFFFF, _xpow_bytes(len(data)))


@pytest.mark.parametrize("n", [1, 5, 64, 1023, 1024, 1025, 70000])
def test_crc_combine_matches_zlib(n):
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    for cut in sorted({0, 1, n // 3, n // 2, n - 1, n}):
        a, b = data[:cut], data[cut:]
        joined = _mulmod(_raw(a), _xpow_bytes(len(b))) ^ _raw(b)
        assert ~(joined ^ _mulmod(0xFFFFFFFF, _xpow_bytes(n))) & 0xFFFFFFFF == zlib.crc32(data)


# ---- against the reference runtime's own C++ codec ----------------------------------

GOLDEN = Path(__file__).resolve().parent / "golden" / "stagewire_frames.jsonl"


def _golden_frames():
    return [json.loads(line) for line in GOLDEN.read_text().splitlines() if line.strip()]


def test_reference_encoder_frames_decode():
    """Frames written by the reference's C++ encoder (tests/golden/
    make_stagewire_frames.py) decode here to what the reference's own decoder
    read from them."""
    frames = _golden_frames()
    assert len(frames) == 8
    for f in frames:
        got = sw.unmarshal(bytes.fromhex(f["frame"]))
        m = got.metadata
        assert m.operation == f["operation"], f["name"]
        ref = f.get("reference_decode")
        if ref is not None:
            assert ref["ok"]
            for key in ("session_id", "request_id", "phase", "decode_step", "stage_index", "layer_start",
                        "layer_end", "payload_kind", "dtype", "shape", "payload_bytes", "payload_crc32",
                        "max_tokens"):
                assert getattr(m, key) == ref[key], (f["name"], key)
            assert zlib.crc32(got.payload) == ref["payload_crc32"]
    by_name = {f["name"]: sw.unmarshal(bytes.fromhex(f["frame"])) for f in frames}
    managed = by_name["activation_decode_managed"].metadata
    assert (managed.deployment_id, managed.deployment_epoch, managed.model_sha256) == ("deployment-a", 3, "a" * 64)
    resp = by_name["response_sampled_token"]
    assert resp.payload == bytes([42, 0, 0, 0]) and resp.metadata.message == "<42>"
    assert resp.metadata.token_text_offsets == [0, 4] and resp.metadata.execution_us == 812
    assert by_name["rollback"].metadata.rollback_tokens == 2
    # one flipped payload bit in a reference frame is refused here as well
    bad = bytearray(bytes.fromhex(frames[1]["frame"]))
    bad[-1] ^= 4
    with pytest.raises(sw.ChecksumMismatch):
        sw.unmarshal(bytes(bad))


def _reference_decode(frames: list[bytes]) -> list[dict]:
    import importlib.util
    import subprocess

    repo = Path(__file__).resolve().parent.parent
    spec = importlib.util.spec_from_file_location("jfb_ref_transport_build",
                                                  repo / "oracle" / "ref_transport" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    from jetsonfabric_b200 import build_cuda
    build_cuda.build()
    binary = mod.build()
    if binary is None:
        pytest.skip("the reference tree is not on this machine and no prebuilt transport driver exists")
    out = subprocess.run([str(binary), "decode"], input="\n".join(f.hex() for f in frames) + "\n",
                         capture_output=True, text=True, timeout=60, check=True).stdout
    return [json.loads(line) for line in out.splitlines() if line.strip()]


def test_frames_made_here_decode_with_the_reference_decoder():
    """marshal's frames and the device link's padded, stamped frames pass the
    reference's C++ request decoder with the same fields; corrupted ones do
    not."""
    rng = np.random.default_rng(3)
    frames, expect, offsets = [], [], [None]
    md = Metadata(session_id="s-1", request_id="r-1", model_id="qwen2", stage_index=1, stage_count=2,
                  node_name="stage-1", layer_start=14, layer_end=28, payload_kind="activation", dtype="f16",
                  shape=[5, 16], max_tokens=64)
    payload = rng.integers(0, 256, 160, dtype=np.uint8).tobytes()
    frames.append(sw.marshal(Frame(md, payload)))
    expect.append(dict(operation="execute", phase="prefill", shape=[5, 16], payload_crc32=zlib.crc32(payload)))
    plan = sw.FramePlan(model_id="qwen2", stage_layers=[(0, 14), (14, 28)], batches=[[0, 1], [2]],
                        prompt_lengths=[5, 3, 4], steps=3, hidden=16)
    for step in range(plan.steps):
        for m in range(2):
            a, n = plan.activation(step, m, 1)
            pre, off = sw.frame_prefix(a, n, 1024)
            p = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
            frames.append(pre[:off] + f"{zlib.crc32(p):>10d}".encode() + pre[off + 10:] + p)
            offsets.append(off)
            expect.append(dict(operation="execute", phase="prefill" if step == 0 else "decode", decode_step=step,
                               shape=[plan.rows(step, m), 16], payload_crc32=zlib.crc32(p)))
    t, n = plan.tokens(0, 1)
    pre, off = sw.frame_prefix(t, n, 1024)
    frames.append(pre[:off] + f"{zlib.crc32(bytes(4)):>10d}".encode() + pre[off + 10:] + bytes(4))
    expect.append(dict(operation="execute", payload_kind="sampled_tokens", stage_index=0, shape=[1]))
    good = len(frames)
    bad = bytearray(frames[1])
    bad[-1] ^= 1
    frames.append(bytes(bad))
    bad = bytearray(frames[2])  # the stamped checksum's last digit changed
    last = offsets[2] + 9
    bad[last] = ord("0") + (bad[last] - ord("0") + 1) % 10
    frames.append(bytes(bad))
    res = _reference_decode(frames)
    assert len(res) == len(frames)
    for r, e in zip(res[:good], expect):
        assert r["ok"], r
        for k, v in e.items():
            assert r[k] == v, (k, r)
    assert not res[good]["ok"] and "checksum" in res[good]["error"]
    assert not res[good + 1]["ok"] and "checksum" in res[good + 1]["error"]


class _HostLoopback:
    """A base link whose sends are the next receives (CPU tensors), with an
    optional edit applied to a sent frame's bytes."""

    def __init__(self, edit=None):
        self.q, self.edit = [], edit

    def send_next(self, frame):
        frame = frame.clone()
        if self.edit is not None:
            self.edit(frame)
        self.q.append(frame)

    send_tokens = send_next

    def recv_prev(self, frame):
        frame.copy_(self.q.pop(0))

    recv_tokens = recv_prev

    def flush(self):
        pass


class _HostCodec:
    hidden = 16

    def encode(self, activations, out=None):
        import torch

        out.copy_(torch.from_numpy(np.asarray(activations, dtype=np.float32).astype(np.float16)))
        return out


def _plan():
    return sw.FramePlan(model_id="m", stage_layers=[(0, 1), (1, 2)], batches=[[0]], prompt_lengths=[3], steps=2,
                        hidden=16)


def test_host_link_round_trip_and_schedule_limits():
    base = _HostLoopback()
    tx, rx = sw.StagewireLink(base, 0, _plan()), sw.StagewireLink(base, 1, _plan())
    stage = _HostCodec()
    for step, rows in ((0, 3), (1, 1)):
        act = np.random.default_rng(step).normal(0, 1, (rows, 16)).astype(np.float32)
        tx.send_activation(stage, act)
        got = rx.recv_activation(stage, rows)
        assert np.array_equal(got.numpy(), act.astype(np.float16))
    with pytest.raises(sw.StagewireError, match="more frames sent"):
        tx.send_activation(stage, np.zeros((1, 16), np.float32))
    tx.flush()
    rx.flush()
    # a run that stops early is reported at flush
    tx.send_activation(stage, np.zeros((3, 16), np.float32))
    with pytest.raises(sw.StagewireError, match="schedule ended after 1 of 2 sends"):
        tx.flush()


def test_host_link_rejects_metadata_that_is_not_the_schedules():
    """A frame whose checksum holds but whose metadata names another step
    (a digit of decode_step changed in flight) fails verification."""
    def edit(frame):
        raw = bytes(frame[:1024].numpy())
        at = raw.index(b'"decode_step":0') + len(b'"decode_step":')
        frame[at] = ord("7")

    base = _HostLoopback(edit)
    tx, rx = sw.StagewireLink(base, 0, _plan()), sw.StagewireLink(base, 1, _plan())
    tx.send_activation(_HostCodec(), np.ones((3, 16), np.float32))
    rx.recv_activation(_HostCodec(), 3)
    with pytest.raises(sw.StagewireError, match="differs from the schedule"):
        rx.verify()

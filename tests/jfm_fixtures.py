"""Hand-built JFM v2 packages for loader tests, written byte by byte from the
format description (docs/jfm-v2-format.md in the reference). Mirrors the
package the reference's loader test builds (engine_test.cpp:135-245): one
I8 tensor per segment, a shared segment, two layers."""
from __future__ import annotations

import struct
from pathlib import Path

from jetsonfabric_b200 import jfm

JF_SEGMENT_SHARED, JF_SEGMENT_INPUT, JF_SEGMENT_LAYER, JF_SEGMENT_OUTPUT, JF_SEGMENT_METADATA = 0, 1, 2, 3, 4


def segment_bytes(layer: int, tensor_name: str, data: bytes) -> bytes:
    index_bytes = (80 + len(tensor_name) + 7) // 8 * 8
    data_offset = (64 + index_bytes + 63) // 64 * 64
    out = bytearray(b"JFSEGM02" + struct.pack("<IIQQ", 2, 1, index_bytes, len(data)))
    out += bytes(64 - len(out))
    out += struct.pack("<IIiI", jfm.JF_TENSOR_I8, 1, layer, 0)
    out += struct.pack("<QQQQ", len(data), 1, 1, 1)
    out += struct.pack("<QQIIII", data_offset, len(data), len(tensor_name), 1, 1, 0)
    out += tensor_name.encode()
    out += bytes((-len(out)) % 8)
    out += bytes(data_offset - len(out))
    out += data
    return bytes(out)


def default_segments():
    return [
        dict(kind=JF_SEGMENT_METADATA, layer=-1, path="metadata.gguf", name="", data=b"GGUF\x03\x00\x00\x00"),
        dict(kind=JF_SEGMENT_SHARED, layer=-1, path="shared.jfs", name="shared.scale", data=bytes([1, 2])),
        dict(kind=JF_SEGMENT_INPUT, layer=-1, path="input.jfs", name="token_embd.weight", data=bytes([3, 4, 5])),
        dict(kind=JF_SEGMENT_LAYER, layer=0, path="layer-00000.jfs", name="blk.0.weight", data=bytes([6, 7, 8, 9])),
        dict(kind=JF_SEGMENT_LAYER, layer=1, path="layer-00001.jfs", name="blk.1.weight",
             data=bytes([10, 11, 12, 13, 14])),
        dict(kind=JF_SEGMENT_OUTPUT, layer=-1, path="output.jfs", name="output.weight",
             data=bytes([15, 16, 17, 18, 19, 20])),
    ]


def write_segment(directory: Path, seg: dict) -> None:
    body = seg["data"] if seg["kind"] == JF_SEGMENT_METADATA else segment_bytes(seg["layer"], seg["name"], seg["data"])
    (directory / seg["path"]).write_bytes(body)
    seg["file_size"] = len(body)
    seg["sha256"] = jfm.sha256(body)


def write_manifest(directory: Path, segments: list[dict], path_override: str | None = None) -> None:
    out = bytearray(b"JFMODEL2" + struct.pack("<IIQ", 2, 2, 1) + bytes(range(32)) + struct.pack("<II", len(segments), 0))
    for i, seg in enumerate(segments):
        path = path_override if (i == 0 and path_override) else seg["path"]
        meta = seg["kind"] == JF_SEGMENT_METADATA
        out += struct.pack("<IiQQQ", seg["kind"], seg["layer"], 0 if meta else 1, 0 if meta else len(seg["data"]),
                           seg["file_size"])
        out += seg["sha256"] + struct.pack("<II", len(path), 0) + path.encode()
    (directory / "manifest.jfm").write_bytes(bytes(out))


def make_package(directory: Path) -> list[dict]:
    directory.mkdir(parents=True, exist_ok=True)
    segments = default_segments()
    for seg in segments:
        write_segment(directory, seg)
    write_manifest(directory, segments)
    return segments


def overwrite(path: Path, offset: int, fmt: str, value: int) -> None:
    data = bytearray(path.read_bytes())
    struct.pack_into(fmt, data, offset, value)
    path.write_bytes(bytes(data))

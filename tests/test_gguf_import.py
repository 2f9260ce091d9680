"""GGUF -> JFM v2 importer (jfb_import_gguf), the GGML-free replacement of
the reference's jf-model-compile (runtime/compiler/jf_model_compile.cpp).

Parity is pinned on the reference's frozen golden package
(runtime/engines/native/tests/fixtures/jfm-v2-golden, copied to
tests/golden/jfm-v2-golden by make_jfm_golden.py): the source GGUF is rebuilt
from the package (metadata.gguf is the exact source prefix; each payload goes
back to its directory offset in the data section), the rebuild is checked
against the source size and SHA-256 the golden manifest records, and importing
it must reproduce every golden file byte for byte.

The error cases follow jf_model_compile.cpp: an existing output, split GGUFs,
tied embeddings, empty layers, malformed block names, unknown tensor types and
malformed GGUF headers all fail and leave nothing behind.
"""
from __future__ import annotations

import hashlib
import shutil
import struct
from pathlib import Path

import numpy as np
import pytest

from jetsonfabric_b200 import jfm

GOLDEN = Path(__file__).resolve().parent / "golden" / "jfm-v2-golden"
FILES = ["manifest.jfm", "metadata.gguf", "input.jfs", "layer-00000.jfs", "layer-00001.jfs", "output.jfs"]

# GGUF value types (public GGUF specification)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)


def golden_bytes() -> dict[str, bytes]:
    return {name: bytes.fromhex("".join((GOLDEN / f"{name}.hex").read_text().split())) for name in FILES}


# ---- a small GGUF reader and writer (test infrastructure) ---------------------------

def read_gguf_directory(meta: bytes):
    """(alignment, data offset, [(name, dims, ggml type, offset)]) of a GGUF prefix."""
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from("<" + fmt, meta, pos)
        pos += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string():
        n = take("Q")
        nonlocal pos
        s = meta[pos:pos + n].decode()
        pos += n
        return s

    sizes = {U8: 1, I8: 1, U16: 2, I16: 2, U32: 4, I32: 4, F32: 4, BOOL: 1, U64: 8, I64: 8, F64: 8}
    assert meta[:4] == b"GGUF"
    pos = 4
    take("I")
    n_tensors, n_kv = take("Q"), take("Q")
    alignment = 32
    for _ in range(n_kv):
        key = string()
        t = take("I")
        if t == STRING:
            string()
        elif t == ARRAY:
            et, count = take("I"), take("Q")
            for _ in range(count):
                if et == STRING:
                    string()
                else:
                    pos += sizes[et]
        else:
            value = struct.unpack_from("<" + {4: "I", 5: "i", 10: "Q", 11: "q"}.get(t, "B"), meta, pos)[0]
            if key == "general.alignment":
                alignment = value
            pos += sizes[t]
    tensors = []
    for _ in range(n_tensors):
        name = string()
        nd = take("I")
        dims = [take("Q") for _ in range(nd)]
        gtype, offset = take("I"), take("Q")
        tensors.append((name, dims, gtype, offset))
    data_offset = (pos + alignment - 1) // alignment * alignment
    return alignment, data_offset, tensors


def gguf_bytes(kv: list, tensors: list, alignment: int = 32, version: int = 3) -> bytes:
    """A GGUF file: kv = [(key, type, value)], tensors = [(name, dims, ggml type, payload bytes)]."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv)))

    def string(s: str):
        b = s.encode()
        out.extend(struct.pack("<Q", len(b)) + b)

    for key, t, value in kv:
        string(key)
        out.extend(struct.pack("<I", t))
        if t == STRING:
            string(value)
        else:
            out.extend(struct.pack("<" + {U8: "B", U32: "I", I32: "i", U64: "Q", F32: "f"}[t], value))
    offset = 0
    placed = []
    for name, dims, gtype, payload in tensors:
        string(name)
        out.extend(struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims))
        out.extend(struct.pack("<IQ", gtype, offset))
        placed.append((offset, payload))
        offset = (offset + len(payload) + alignment - 1) // alignment * alignment
    data = (len(out) + alignment - 1) // alignment * alignment
    out.extend(b"\0" * (data - len(out)))
    for off, payload in placed:
        out.extend(b"\0" * (data + off - len(out)))
        out.extend(payload)
    return bytes(out)


def rebuild_source(package: dict[str, bytes], source_size: int) -> bytes:
    """The source GGUF of a package: metadata.gguf, then every payload at its
    directory offset (found by name in the segments, through the loader's
    segment format), zero elsewhere."""
    meta = package["metadata.gguf"]
    _, data_offset, tensors = read_gguf_directory(meta)
    payloads = {}
    for name, blob in package.items():
        if not name.endswith(".jfs"):
            continue
        count, = struct.unpack_from("<I", blob, 12)
        pos = 64
        for _ in range(count):
            rec = blob[pos:pos + 80]
            off, size, name_len = struct.unpack_from("<QQI", rec, 48)
            tname = blob[pos + 80:pos + 80 + name_len].decode()
            payloads[tname] = blob[off:off + size]
            pos += (80 + name_len + 7) // 8 * 8
    src = bytearray(source_size)
    src[:len(meta)] = meta
    for name, _, _, offset in tensors:
        p = payloads[name]
        src[data_offset + offset:data_offset + offset + len(p)] = p
    return bytes(src)


def qwen2_kv(layers: int) -> list:
    return [("general.architecture", STRING, "qwen2"), ("qwen2.block_count", U32, layers)]


def f32(values) -> bytes:
    return np.asarray(values, np.float32).tobytes()


def small_model(layers: int = 2, tied: bool = False, extra=()) -> list:
    t = [("token_embd.weight", [4, 8], 0, f32(np.arange(32) * 0.1))]
    for layer in range(layers):
        t.append((f"blk.{layer}.attn_norm.weight", [4], 0, f32([1, 1, 1, 1])))
        t.append((f"blk.{layer}.attn_q.weight", [4, 4], 0, f32(np.arange(16) * 0.01 + layer)))
    t.append(("output_norm.weight", [4], 0, f32([1, 1, 1, 1])))
    if not tied:
        t.append(("output.weight", [4, 8], 0, f32(np.arange(32) * 0.01)))
    return t + list(extra)


# ---- golden parity -----------------------------------------------------------------

def test_importer_reproduces_the_golden_package(tmp_path):
    golden = golden_bytes()
    manifest = golden["manifest.jfm"]
    source_size, = struct.unpack_from("<Q", manifest, 16)
    source_sha = manifest[24:56]
    source = rebuild_source(golden, source_size)
    # the rebuild is the reference's source file: its size and digest are the manifest's
    assert hashlib.sha256(source).digest() == source_sha
    src = tmp_path / "model.gguf"
    src.write_bytes(source)
    out = tmp_path / "model.jfm"
    report = jfm.import_gguf(src, out)
    assert report["layer_count"] == 2 and report["architecture"] == "qwen2"
    assert report["source_sha256"] == source_sha.hex()
    assert sorted(p.name for p in out.iterdir()) == sorted(FILES)
    for name in FILES:
        assert (out / name).read_bytes() == golden[name], name
    assert report["package_bytes"] == sum(len(golden[n]) for n in FILES)
    assert report["tensor_count"] == 7
    assert not list(tmp_path.glob("model.jfm.tmp.*"))


def test_imported_package_opens_and_keeps_payloads(tmp_path):
    tensors = small_model(layers=3, extra=[("rope_freqs.weight", [4], 0, f32([1, 2, 3, 4]))])
    src = tmp_path / "m.gguf"
    src.write_bytes(gguf_bytes(qwen2_kv(3) + [("general.alignment", U32, 64)], tensors, alignment=64))
    out = tmp_path / "m.jfm"
    report = jfm.import_gguf(src, out)
    # a tensor that belongs to no layer, input or output goes to the shared segment
    assert (out / "shared.jfs").exists()
    assert report["tensor_count"] == len(tensors)
    with jfm.Model(out) as m:
        got = {t.name: t for t in m.tensors()}
        for name, dims, _, payload in tensors:
            t = got[name]
            assert t.bytes() == payload
            assert list(t.shape[:len(dims)]) == dims
            assert t.layer == (int(name.split(".")[1]) if name.startswith("blk.") else -1)


def test_imported_synthetic_qwen2_matches_its_writer(tmp_path):
    """The synthetic writer emits a GGUF directory plus segments; a GGUF rebuilt
    from them imports to the same segment files (K-quant payloads included)."""
    spec = dict(layer_count=2, embedding_length=256, head_count=2, kv_head_count=1, feed_forward_length=512,
                vocabulary_size=512, context_length=64, layer_type=jfm.JF_TENSOR_Q4_K,
                embedding_type=jfm.JF_TENSOR_Q6_K, output_type=jfm.JF_TENSOR_Q6_K, seed=3)
    synth = tmp_path / "synth"
    jfm.write_synthetic_package(synth, **spec)
    package = {p.name: p.read_bytes() for p in synth.iterdir()}
    meta = package["metadata.gguf"]
    _, data_offset, tensors = read_gguf_directory(meta)
    # size: after the last payload, whatever its length (found in the segments)
    sizes = {}
    for name, blob in package.items():
        if name.endswith(".jfs"):
            count, = struct.unpack_from("<I", blob, 12)
            pos = 64
            for _ in range(count):
                off, size, name_len = struct.unpack_from("<QQI", blob, pos + 48)
                sizes[blob[pos + 80:pos + 80 + name_len].decode()] = size
                pos += (80 + name_len + 7) // 8 * 8
    source_size = max(data_offset + off + sizes[n] for n, _, _, off in tensors)
    src = tmp_path / "synth.gguf"
    src.write_bytes(rebuild_source(package, source_size))
    out = tmp_path / "imported"
    jfm.import_gguf(src, out)
    for name, blob in package.items():
        if name != "manifest.jfm":
            assert (out / name).read_bytes() == blob, name


# ---- rejections --------------------------------------------------------------------

def expect_failure(tmp_path, data: bytes, fragment: str, code=None):
    src = tmp_path / "bad.gguf"
    src.write_bytes(data)
    out = tmp_path / "bad.jfm"
    with pytest.raises(jfm.JfmError) as err:
        jfm.import_gguf(src, out)
    assert fragment in str(err.value)
    if code is not None:
        assert err.value.code == code
    assert not out.exists()
    assert not list(tmp_path.glob("bad.jfm.tmp.*"))


def test_rejects_existing_output(tmp_path):
    src = tmp_path / "m.gguf"
    src.write_bytes(gguf_bytes(qwen2_kv(2), small_model()))
    out = tmp_path / "m.jfm"
    out.mkdir()
    with pytest.raises(jfm.JfmError, match="already exists"):
        jfm.import_gguf(src, out)


def test_rejects_tied_embeddings(tmp_path):
    expect_failure(tmp_path, gguf_bytes(qwen2_kv(2), small_model(tied=True)), "output.weight is required")


def test_rejects_split_gguf(tmp_path):
    expect_failure(tmp_path, gguf_bytes(qwen2_kv(2) + [("split.count", U32, 2)], small_model()), "split GGUF")


def test_rejects_missing_layer(tmp_path):
    expect_failure(tmp_path, gguf_bytes(qwen2_kv(3), small_model(layers=2)), "no tensors for layer-00002.jfs")


def test_rejects_layer_beyond_block_count(tmp_path):
    expect_failure(tmp_path, gguf_bytes(qwen2_kv(1), small_model(layers=2)), "exceeds model block count")


def test_rejects_malformed_block_name(tmp_path):
    bad = small_model(extra=[("blk.x.weight", [4], 0, f32([0, 0, 0, 0]))])
    expect_failure(tmp_path, gguf_bytes(qwen2_kv(2), bad), "invalid block tensor name")


def test_rejects_unknown_tensor_type(tmp_path):
    bad = small_model(extra=[("rope.weight", [32], 31, b"\0" * 32)])
    expect_failure(tmp_path, gguf_bytes(qwen2_kv(2), bad), "GGML type id 31")


def test_rejects_missing_input_and_metadata(tmp_path):
    no_input = [t for t in small_model() if not t[0].startswith("token_embd")]
    expect_failure(tmp_path, gguf_bytes(qwen2_kv(2), no_input), "no input embedding")
    expect_failure(tmp_path, gguf_bytes([("qwen2.block_count", U32, 2)], small_model()), "general.architecture")
    expect_failure(tmp_path, gguf_bytes([("general.architecture", STRING, "qwen2")], small_model()), "block_count")


def test_rejects_malformed_headers(tmp_path):
    good = gguf_bytes(qwen2_kv(2), small_model())
    expect_failure(tmp_path, b"GGML" + good[4:], "bad magic", jfm.JF_STATUS_FORMAT_ERROR)
    expect_failure(tmp_path, good[:4] + struct.pack("<I", 1) + good[8:], "version 1")
    expect_failure(tmp_path, good[:200], "past the end")
    # a payload that runs past the end of the file
    expect_failure(tmp_path, good[:-16], "exceeds the source GGUF")


def test_truncated_and_corrupted_sources_fail_cleanly(tmp_path):
    """Every prefix of a valid GGUF and seeded single-byte corruptions of it:
    the importer either publishes a package or raises JfmError, never reads
    out of bounds, and never leaves a staging directory or a partial
    package behind."""
    import random

    good = gguf_bytes(qwen2_kv(2), small_model())
    src = tmp_path / "x.gguf"
    out = tmp_path / "x.jfm"

    def attempt(data: bytes) -> bool:
        src.write_bytes(data)
        try:
            jfm.import_gguf(src, out)
        except jfm.JfmError:
            assert not out.exists()
            assert not list(tmp_path.glob("x.jfm.tmp.*"))
            return False
        assert not list(tmp_path.glob("x.jfm.tmp.*"))
        with jfm.Model(out):
            pass
        shutil.rmtree(out)
        return True

    for n in range(len(good)):
        assert not attempt(good[:n]), n
    rng = random.Random(5)
    published = 0
    for _ in range(300):
        data = bytearray(good)
        at = rng.randrange(len(data))
        data[at] ^= 1 << rng.randrange(8)
        published += attempt(bytes(data))
    assert 0 < published < 300  # payload flips still import; header flips are rejected
    assert attempt(good)


def test_command_line(tmp_path, capsys):
    import json

    src = tmp_path / "m.gguf"
    src.write_bytes(gguf_bytes(qwen2_kv(2), small_model()))
    assert jfm.main(["--input", str(src), "--output", str(tmp_path / "m.jfm")]) == 0
    report = json.loads(capsys.readouterr().out)
    assert report["format"] == "jfm-v2" and report["layer_count"] == 2
    assert report["source_sha256"] == hashlib.sha256(src.read_bytes()).hexdigest()
    assert jfm.main(["--input", str(src), "--output", str(tmp_path / "m.jfm")]) == 1
    assert "already exists" in capsys.readouterr().err

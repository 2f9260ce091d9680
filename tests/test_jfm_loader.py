"""JFM v2 loader tests (CPU). Mirrors the reference's loader test
runtime/engines/native/tests/engine_test.cpp: golden package (95), stage
residency (247), rejection of invalid packages (319), SHA-256 (444) and the
tensor-layout contract (457)."""
from __future__ import annotations

import shutil
from pathlib import Path

import pytest

from jetsonfabric_b200 import jfm
from tests import jfm_fixtures as fx

GOLDEN = Path(__file__).resolve().parent / "golden" / "jfm-v2-golden"


def decode_golden(target: Path) -> Path:
    target.mkdir(parents=True, exist_ok=True)
    for hexfile in GOLDEN.glob("*.hex"):
        (target / hexfile.stem).write_bytes(bytes.fromhex("".join(hexfile.read_text().split())))
    return target


def test_golden_package_opens_both_stage_ranges(tmp_path):
    package = decode_golden(tmp_path / "golden")
    with jfm.Model(package, 0, 1) as first:
        assert first.stats.selected_tensor_count == 3
        assert {t.name for t in first.tensors()} == {"blk.0.attn_norm.weight", "blk.0.attn_q.weight",
                                                      "token_embd.weight"}
    with jfm.Model(package, 1, 2) as last:
        assert last.stats.selected_tensor_count == 4
        assert "output.weight" in {t.name for t in last.tensors()}


def test_sha256_known_answer():
    assert jfm.sha256(b"abc").hex() == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    assert jfm.sha256(b"").hex() == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"
    # 56 and 64 byte inputs cross the padding boundary
    assert jfm.sha256(b"a" * 64) != jfm.sha256(b"a" * 63)


def test_tensor_layout_contract():
    for t in range(jfm.JF_TENSOR_F32, 36):
        e, b = jfm.type_layout(t)
        assert e > 0 and b > 0
    assert jfm.type_layout(jfm.JF_TENSOR_Q4_K) == (256, 144)
    assert jfm.type_layout(jfm.JF_TENSOR_Q6_K) == (256, 210)
    assert jfm.type_layout(jfm.JF_TENSOR_Q2_K) == (256, 84)
    with pytest.raises(jfm.JfmError) as err:
        jfm.type_layout(0)
    assert err.value.code == jfm.JF_STATUS_FORMAT_ERROR


def test_stage_residency(tmp_path):
    package = tmp_path / "pkg"
    fx.make_package(package)
    with jfm.Model(package, 0, 1) as first:
        s = first.stats
        assert (s.layer_start, s.layer_end, s.layer_count) == (0, 1, 2)
        assert s.selected_weight_bytes == 9 and s.total_weight_bytes == 20
        assert s.selected_tensor_count == 3 and s.total_tensor_count == 5
        t = first.find("blk.0.weight")
        assert t.layer == 0 and t.size == 4 and t.type == jfm.JF_TENSOR_I8
        assert (t.block_elements, t.block_bytes) == (1, 1)
        with pytest.raises(jfm.JfmError) as err:
            first.find("output.weight")
        assert err.value.code == jfm.JF_STATUS_NOT_FOUND
        assert first.prefetch() != 0
        assert first.prefetch(threads=4) == first.prefetch(threads=1)
        meta = first.gguf_metadata()
        assert len(meta) == 8 and meta[:4] == b"GGUF"
        digest = first.source_sha256()
        assert digest[0] == 0 and digest[31] == 31
    with jfm.Model(package, 1, 2) as last:
        assert last.stats.selected_weight_bytes == 13 and last.stats.selected_tensor_count == 3
        with pytest.raises(jfm.JfmError):
            last.find("token_embd.weight")
        assert last.find("output.weight").size == 6
    with jfm.Model(package, 0, 2) as full:
        assert full.stats.selected_weight_bytes == 20 and full.stats.selected_tensor_count == 5
    with jfm.Model(package, 0, jfm.JF_ALL_LAYERS) as all_layers:
        assert all_layers.stats.layer_end == 2 and all_layers.stats.selected_weight_bytes == 20


def _rejects(path, code, start=0, end=1, verify=False):
    with pytest.raises(jfm.JfmError) as err:
        jfm.Model(path, start, end, verify_hashes=verify)
    assert err.value.code == code, str(err.value)


def test_rejects_invalid_inputs(tmp_path):
    package = tmp_path / "pkg"
    segments = fx.make_package(package)
    _rejects(package, jfm.JF_STATUS_INVALID_ARGUMENT, 1, 1)
    _rejects(package, jfm.JF_STATUS_INVALID_ARGUMENT, 0, 3)
    _rejects(tmp_path / "missing", jfm.JF_STATUS_IO_ERROR)

    unsafe = tmp_path / "unsafe"
    unsafe.mkdir()
    fx.write_manifest(unsafe, segments, "../escape.jfs")
    _rejects(unsafe, jfm.JF_STATUS_FORMAT_ERROR)

    corrupt = tmp_path / "corrupt"
    fx.make_package(corrupt)
    data = bytearray((corrupt / "layer-00000.jfs").read_bytes())
    data[-1] = 0xFF
    (corrupt / "layer-00000.jfs").write_bytes(bytes(data))
    _rejects(corrupt, jfm.JF_STATUS_FORMAT_ERROR, verify=True)
    # the same corruption is not detected without verification, and a stage
    # that does not map the corrupted segment is unaffected
    jfm.Model(corrupt, 0, 1, verify_hashes=False).close()
    jfm.Model(corrupt, 1, 2, verify_hashes=True).close()

    missing_layer = tmp_path / "missing_layer"
    segs = fx.make_package(missing_layer)
    del segs[4]
    fx.write_manifest(missing_layer, segs)
    _rejects(missing_layer, jfm.JF_STATUS_FORMAT_ERROR)

    dup_path = tmp_path / "dup_path"
    segs = fx.make_package(dup_path)
    segs[2]["path"] = segs[1]["path"]
    fx.write_manifest(dup_path, segs)
    _rejects(dup_path, jfm.JF_STATUS_FORMAT_ERROR)

    wrong_layer = tmp_path / "wrong_layer"
    fx.make_package(wrong_layer)
    fx.overwrite(wrong_layer / "layer-00000.jfs", 64 + 8, "<I", 1)
    _rejects(wrong_layer, jfm.JF_STATUS_FORMAT_ERROR)

    reserved = tmp_path / "reserved"
    fx.make_package(reserved)
    fx.overwrite(reserved / "manifest.jfm", 60, "<I", 1)
    _rejects(reserved, jfm.JF_STATUS_FORMAT_ERROR)

    bad_layout = tmp_path / "bad_layout"
    fx.make_package(bad_layout)
    fx.overwrite(bad_layout / "layer-00000.jfs", 64, "<I", jfm.JF_TENSOR_Q4_K)
    _rejects(bad_layout, jfm.JF_STATUS_FORMAT_ERROR)

    bad_offset = tmp_path / "bad_offset"
    fx.make_package(bad_offset)
    fx.overwrite(bad_offset / "layer-00000.jfs", 64 + 48, "<Q", 0)
    _rejects(bad_offset, jfm.JF_STATUS_FORMAT_ERROR)

    dup_name = tmp_path / "dup_name"
    segs = fx.make_package(dup_name)
    segs[2]["name"] = segs[1]["name"]
    fx.write_segment(dup_name, segs[2])
    fx.write_manifest(dup_name, segs)
    _rejects(dup_name, jfm.JF_STATUS_FORMAT_ERROR)


@pytest.mark.parametrize("name", ["manifest.jfm", "input.jfs", "layer-00000.jfs", "layer-00001.jfs", "output.jfs",
                                  "metadata.gguf"])
def test_truncated_golden_files_are_rejected(tmp_path, name):
    """Every proper prefix of each golden package file, opened for the whole
    model without hash verification: the structural checks alone reject it
    (no mapping past the end of a file)."""
    package = decode_golden(tmp_path / "pkg")
    full = (package / name).read_bytes()
    with jfm.Model(package, 0, 2, verify_hashes=False):
        pass
    for n in range(len(full)):
        (package / name).write_bytes(full[:n])
        with pytest.raises(jfm.JfmError):
            jfm.Model(package, 0, 2, verify_hashes=False)
    (package / name).write_bytes(full)


def test_reference_fixture_residency(fixture_package):
    """compiler_integration_test.cmake:29-52: 27 tensors total, 13 on stage 0-1."""
    with jfm.Model(fixture_package, 0, 1) as first:
        assert first.stats.selected_tensor_count == 13
        assert first.stats.total_tensor_count == 27
    with jfm.Model(fixture_package) as full:
        assert full.stats.layer_count == 2
        assert full.stats.selected_tensor_count == 27


@pytest.mark.parametrize("preset,expected_bytes,expected_tensors", [
    ("1.5b", 1_111_370_240, 339),
])
def test_q4_k_m_map_reproduces_published_weight_bytes(tmp_path, preset, expected_bytes, expected_tensors):
    """The synthetic Q4_K_M type map reproduces the reference's published
    resident weight bytes (docs/benchmarks/2026-08-03-native-distributed-stages.md:47-51)."""
    report = jfm.write_synthetic_package(tmp_path / preset, **jfm.QWEN2_PRESETS[preset], context_length=4096)
    assert report.weight_bytes == expected_bytes
    assert report.tensor_count == expected_tensors
    with jfm.Model(tmp_path / preset) as m:
        assert m.stats.selected_weight_bytes == expected_bytes
    shutil.rmtree(tmp_path / preset)


def test_synthetic_package_is_deterministic(tmp_path):
    kw = dict(layer_count=2, embedding_length=256, head_count=2, kv_head_count=1, feed_forward_length=512,
              vocabulary_size=256, seed=99)
    jfm.write_synthetic_package(tmp_path / "a", threads=1, **kw)
    jfm.write_synthetic_package(tmp_path / "b", threads=8, **kw)
    for f in (tmp_path / "a").iterdir():
        assert f.read_bytes() == (tmp_path / "b" / f.name).read_bytes(), f.name

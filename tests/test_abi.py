"""The C-ABI libraries load without a GPU and export every symbol their
headers declare (every C header under include/)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
HEADERS = sorted((REPO / "include").glob("*/*.h"))
# the host-only library (loader, importer, tokenizer) and the headers it serves
JFM_HEADERS = [REPO / "include" / "jetsonfabric" / "engine.h", REPO / "include" / "jfb" / "jfb_model.h",
               REPO / "include" / "jfb" / "jfb_tokenizer.h"]


def declared_functions(header: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    names = re.findall(r"\b((?:jf|jfb)_[a-z0-9_]+)\s*\(", text)
    return sorted(set(n for n in names if not n.endswith("_t")))


def test_headers_are_all_listed():
    names = {h.name for h in HEADERS}
    assert {"engine.h", "jfb_kernels.h", "jfb_engine.h", "jfb_model.h", "jfb_status.h", "jfb_tokenizer.h"} <= names
    assert all(declared_functions(h) for h in HEADERS if h.name != "jfb_status.h")


def test_jfb_library_exports_every_declared_symbol():
    from jetsonfabric_b200 import build_cuda
    path = build_cuda.build()
    lib = C.CDLL(str(path))
    missing = [n for h in HEADERS for n in declared_functions(h) if not hasattr(lib, n)]
    assert not missing, missing


def test_jfm_library_exports_loader_abi():
    from jetsonfabric_b200 import jfm
    lib = jfm.lib()
    for h in JFM_HEADERS:
        missing = [n for n in declared_functions(h) if not hasattr(lib, n)]
        assert not missing, missing


def test_engine_module_fails_loudly_without_a_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from jetsonfabric_b200 import engine
    with pytest.raises((engine.NativeExecutionError, engine.InvalidArgument)):
        engine.NativeEngine(REPO / "does-not-exist", "cuda")

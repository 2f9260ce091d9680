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
    assert {"engine.h", "jfb_kernels.h", "jfb_engine.h", "jfb_model.h", "jfb_status.h", "jfb_tokenizer.h",
            "jfb_stagewire.h"} <= names
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


ENGINE_CONSUMER = r"""
#include "jetsonfabric/native_inference.hpp"

#include <cstdio>
#include <cstring>
#include <stdexcept>

using namespace jetsonfabric::native;

static const char * open_engine(const char * path, Backend backend) {
    try {
        NativeEngine engine(path, backend, 1);
        return engine.model_info().architecture.empty() ? "opened-empty" : "opened";
    } catch (const std::invalid_argument &) {
        return "invalid_argument";
    } catch (const std::exception &) {
        return "exception";
    }
}

int main(int argc, char ** argv) {
    if (argc != 2) return 2;
    std::printf("%s %s\n", backend_name(Backend::Cpu), backend_name(Backend::Cuda));
    std::printf("%s %s %s\n", attention_kernel_name(AttentionKernel::Automatic),
                attention_kernel_name(AttentionKernel::Unfused), attention_kernel_name(AttentionKernel::Flash));
    EngineOptions options;
    std::printf("%s %u\n", options.backend == Backend::Cpu ? "cpu-default" : "other", options.layer_start);
    std::printf("%s\n", open_engine(argv[1], Backend::Cpu));
    std::printf("%s\n", open_engine((std::string(argv[1]) + "/missing").c_str(), Backend::Cuda));
    return 0;
}
"""


def test_engine_cpp_api_compiles_links_and_rejects_without_a_device(tmp_path):
    """A caller written against the reference's engine header
    (include/jetsonfabric/native_inference.hpp) compiles, links against
    libjfb.so and runs without a GPU: the name helpers return the reference's
    strings, Backend::Cpu is rejected with std::invalid_argument (no CPU
    fallback), and a missing package raises a std::exception."""
    import shutil
    import subprocess

    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    if shutil.which("g++") is None:
        pytest.skip("no C++ compiler")
    from jetsonfabric_b200 import build_cuda
    lib = build_cuda.build()
    src = tmp_path / "engine_consumer.cpp"
    src.write_text(ENGINE_CONSUMER)
    exe = tmp_path / "engine_consumer"
    subprocess.run(["g++", "-std=c++20", "-O1", f"-I{REPO / 'include'}", str(src), "-o", str(exe),
                    f"-L{lib.parent}", "-ljfb", f"-Wl,-rpath,{lib.parent}"], check=True)
    golden = REPO / "tests" / "golden" / "jfm-v2-golden"
    package = tmp_path / "pkg"
    package.mkdir()
    for hexfile in golden.glob("*.hex"):
        (package / hexfile.stem).write_bytes(bytes.fromhex("".join(hexfile.read_text().split())))
    out = subprocess.run([str(exe), str(package)], check=True, capture_output=True, text=True).stdout.split("\n")
    assert out[:4] == ["cpu cuda", "automatic unfused flash", "cpu-default 0", "invalid_argument"]
    assert out[4] in ("invalid_argument", "exception")


@pytest.mark.parametrize("header", HEADERS, ids=lambda h: h.name)
@pytest.mark.parametrize("compiler", [("gcc", "-std=c11", "c"), ("g++", "-std=c++20", "c++")], ids=["c11", "c++20"])
def test_header_compiles_alone(header, compiler):
    """Each C header is self-contained and warning-free as C (what cgo and
    other FFI generators parse) and as C++."""
    import shutil
    import subprocess

    cc, std, lang = compiler
    if shutil.which(cc) is None:
        pytest.skip(f"no {cc}")
    rel = header.relative_to(REPO / "include")
    subprocess.run([cc, std, "-x", lang, "-Wall", "-Wextra", "-Werror", f"-I{REPO / 'include'}", "-fsyntax-only", "-"],
                   input=f'#include "{rel}"\n', text=True, check=True)


CGO_SIDE = r"""
#include <stdint.h>
#include <stdlib.h>

#include "jfb/jfb_engine.h"
#include "jfb/jfb_model.h"
#include "jfb/jfb_stagewire.h"

/* what the cgo stubs of the integration guide touch, written in C */
int open_stage(const char * pkg, uint32_t start, uint32_t end, int device, jfb_engine ** eng) {
    jfb_engine_options opts = {0};
    opts.backend = 1;
    opts.layer_start = start;
    opts.layer_end = end;
    opts.device = (int32_t) device;
    jfb_status st = jfb_engine_open(pkg, &opts, eng);
    return st.code != 0 ? (int) st.message[0] : 0;
}

int import_gguf(const char * src, const char * dst) {
    jfb_import_report rep;
    jfb_status st = jfb_import_gguf(src, dst, &rep);
    return st.code != JFB_STATUS_OK ? (int) st.message[0] : 0;
}

int call_inbox(jfb_frame_channel * ch, const void * head, uint64_t head_len, const void * frame, uint64_t len,
               uint32_t timeout_ms) {
    int32_t status = 0, is_frame = 0;
    const uint8_t * reply = NULL;
    uint64_t n = 0;
    jfb_status st = jfb_frame_channel_call(ch, head, head_len, frame, len, timeout_ms, &status, &is_frame, &reply, &n);
    return st.code != JFB_STATUS_OK ? (int) st.message[0] : (int) status + is_frame + (int) n + (reply != NULL);
}
"""


def test_cgo_stub_calls_compile_as_c():
    """The fields, calls and constants the integration guide's cgo stubs use
    exist with those types in the C headers."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("no gcc")
    subprocess.run(["gcc", "-std=c11", "-x", "c", "-Wall", "-Wextra", "-Werror", f"-I{REPO / 'include'}",
                    "-fsyntax-only", "-"], input=CGO_SIDE, text=True, check=True)

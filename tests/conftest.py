import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _native_libraries():
    """Builds the host-only libraries (libjfm, oracle) once per session."""
    from jetsonfabric_b200 import build
    build.build_jfm()
    from oracle import binding
    binding.build()
    yield


@pytest.fixture(scope="session")
def fixture_package(tmp_path_factory):
    """The reference's 2-layer constant F32 Qwen2 fixture as a JFM package."""
    from jetsonfabric_b200 import jfm
    d = tmp_path_factory.mktemp("fixture") / "fixture.jfm"
    jfm.write_reference_fixture(d)
    return d


@pytest.fixture(scope="session")
def small_q4k_package(tmp_path_factory):
    """A small seeded Q4_K_M-style Qwen2 package (4 layers, hidden 512)."""
    from jetsonfabric_b200 import jfm
    d = tmp_path_factory.mktemp("small") / "small.jfm"
    jfm.write_synthetic_package(d, layer_count=4, embedding_length=512, head_count=4, kv_head_count=2,
                                feed_forward_length=1024, vocabulary_size=1024, context_length=512,
                                seed=7, draw_norms=True, draw_biases=True)
    return d

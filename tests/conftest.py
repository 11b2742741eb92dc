"""Shared pytest setup: the `gpu` marker, the package loader and model fixtures."""
from __future__ import annotations

import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libz2b.so")


def load_pkg():
    """Import zonos2.cpp_b200/ under the module name z2b."""
    if "z2b" in sys.modules:
        return sys.modules["z2b"]
    spec = importlib.util.spec_from_file_location(
        "z2b", os.path.join(ROOT, "zonos2.cpp_b200", "__init__.py"),
        submodule_search_locations=[os.path.join(ROOT, "zonos2.cpp_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["z2b"] = mod
    spec.loader.exec_module(mod)
    return mod


load_pkg()


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("Z2B_MODEL_DIR") or str(tmp_path_factory.mktemp("models"))
    os.makedirs(d, exist_ok=True)
    return d


@pytest.fixture(scope="session")
def tiny_path(model_dir):
    import z2b.synth as S
    return S.cached("tiny", directory=model_dir)


@pytest.fixture(scope="session")
def dummy_path(model_dir):
    """The reference's CI fixture model, regenerated from its recipe."""
    from tests.golden.make_dummy import write
    p = os.path.join(model_dir, "dummy-zonos2.gguf")
    if not os.path.exists(p):
        write(p + ".tmp")
        os.replace(p + ".tmp", p)
    return p

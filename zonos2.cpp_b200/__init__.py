"""zonos2.cpp_b200 — B200-native batched MoE backbone decode step for zonos2.cpp.

The directory name is not an identifier, so load it under the name ``z2b``::

    import importlib.util, sys
    spec = importlib.util.spec_from_file_location(
        "z2b", "<repo>/zonos2.cpp_b200/__init__.py",
        submodule_search_locations=["<repo>/zonos2.cpp_b200"])
    z2b = importlib.util.module_from_spec(spec); sys.modules["z2b"] = z2b
    spec.loader.exec_module(z2b)

Submodules: ``z2b.runtime`` (ctypes binding of include/z2b.h), ``z2b.synth``
(synthetic GGUF files), ``z2b.build`` (nvcc build recipe).
"""
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)

"""The C ABI libraries load and export every function the public headers declare;
calls fail with an error code (no crash) when their preconditions are not met."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

import z2b.build as B
from tests.conftest import ROOT

HEADERS = ["z2b.h", "z2b_tools.h"]


def _declared(header):
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(z2b_[a-z0-9_]+)\s*\(", src)))


def test_headers_declare_entry_points():
    names = _declared("z2b.h")
    for n in ["z2b_model_load", "z2b_ctx_create", "z2b_slot_prefill", "z2b_step", "z2b_step_logits",
              "z2b_last_error"]:
        assert n in names


@pytest.mark.parametrize("header", HEADERS)
def test_every_declared_symbol_exported(header):
    libs = [ctypes.CDLL(B.LIB), ctypes.CDLL(B.SYNTH_LIB)]
    missing = [n for n in _declared(header) if not any(hasattr(L, n) for L in libs)]
    assert not missing, missing


def test_load_errors_are_reported(tmp_path):
    import z2b.runtime as R
    with pytest.raises(R.Z2BError) as e:
        R.Model(str(tmp_path / "missing.gguf"))
    assert e.value.rc in (2, 4)        # IO error, or no CUDA device on a CPU-only host
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"not a gguf file at all")
    with pytest.raises(R.Z2BError):
        R.Model(str(bad))

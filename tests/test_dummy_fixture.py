"""The reference's CI fixture model (tests/fixtures/dummy-zonos2.gguf) is reproduced
byte for byte by tests/golden/make_dummy.py, so GPU tests can use it on any machine."""
from __future__ import annotations

import hashlib
import os

import pytest

# sha256 of the reference's own tests/fixtures/dummy-zonos2.gguf
SHA256 = "4ffebf4f4b702d772b4920b09ccf94db4f097bb8edc9e8b738dd22a43591cce7"
# optional: a checkout of the reference, to compare with its fixture file directly
REF = os.path.join(os.environ.get("Z2B_REFERENCE_DIR", ""), "tests", "fixtures", "dummy-zonos2.gguf")


def _sha(p):
    return hashlib.sha256(open(p, "rb").read()).hexdigest()


def test_regenerated_fixture_hash(dummy_path):
    assert _sha(dummy_path) == SHA256


@pytest.mark.skipif(not os.environ.get("Z2B_REFERENCE_DIR") or not os.path.exists(REF),
                    reason="Z2B_REFERENCE_DIR not set to a reference checkout")
def test_matches_reference_fixture(dummy_path):
    assert open(dummy_path, "rb").read() == open(REF, "rb").read()

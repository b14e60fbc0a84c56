"""The C-ABI library loads on the CPU and exports every function include/*.h declares."""

import re
from pathlib import Path

import pytest

from shellsmith_b200 import _capi

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(?:int|size_t)\s+(sc_\w+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def library():
    from shellsmith_b200 import _build

    _build.build()
    return _capi.lib()


def test_every_declared_symbol_is_exported(library):
    declared = _declared()
    assert declared, "no declarations found"
    missing = [name for name in sorted(declared) if not hasattr(library, name)]
    assert not missing, missing


def test_every_declared_symbol_has_a_binding():
    assert _declared() == set(_capi.SIGNATURES)


def test_workspace_size_query_without_gpu(library):
    """sc_gdn_decode_glue_workspace is pure arithmetic: 256-byte aligned buffers for
    q, k, v, the pre-norm output, g and beta."""
    n = library.sc_gdn_decode_glue_workspace(256, 16, 32)
    qk, vy, gb = 256 * 16 * 128 * 2, 256 * 32 * 128 * 2, 256 * 32 * 4
    assert n == 2 * qk + 2 * vy + 2 * gb
    assert library.sc_gdn_decode_glue_workspace(0, 16, 32) == 0


def test_version_and_error_text_without_gpu(library):
    assert library.sc_version() >= 100
    # Argument validation runs on the host before any CUDA call.
    code = library.sc_gdn_decode(None, None, None, None, None, None, None, None, 1, 1, 1, 128,
                                 128, 1, None)
    assert code == 1
    assert "null pointer" in _capi.last_error()
    code = library.sc_paged_decode_attention(1, 1, 10, 1, 1, None, 1, 16, 2, 256, 8, 4, 64, 1,
                                             0.1, None, None, 1, None, None)
    assert code == 2 and "page size" in _capi.last_error()

"""The C-ABI library builds, loads without a GPU and exports every entry point
declared in include/affmae_b200.h (no compute calls: those need a GPU)."""
import re

import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def lib():
    from affmae_b200 import build, _native
    build.build()
    return _native.lib()


def declared():
    text = (ROOT / "include" / "affmae_b200.h").read_text()
    return sorted(set(re.findall(r"\b(affb_\w+)\s*\(", text)))


def test_header_declares_all_bound_symbols():
    from affmae_b200 import _native
    assert set(declared()) == set(_native.SIGNATURES) | set(_native.OTHER_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared():
        assert hasattr(lib, name), name


def test_abi_version_and_error_channel(lib):
    assert lib.affb_abi_version() == 1
    assert isinstance(lib.affb_last_error(), bytes)


def test_argument_errors_are_reported_before_any_launch(lib):
    from affmae_b200 import _native
    # K larger than N is rejected by the host-side checks (no GPU work enqueued)
    rc = lib.affb_knn(None, None, 0, 1, 1, 4, 2, 8, None, None)
    assert rc == 1
    assert b"exceeds" in lib.affb_last_error()
    with pytest.raises(RuntimeError, match="head_dim"):
        _native.call("affb_nbhd_attn_fwd", None, None, None, None, None, None, 1, None, None, 0,
                     1, 1, 8, 12, 8, 1.0, None, None, None)


def test_workspace_size_is_monotone(lib):
    a = lib.affb_deform_workspace_bytes(1, 1000)
    b = lib.affb_deform_workspace_bytes(2, 1000)
    c = lib.affb_deform_workspace_bytes(1, 100000)
    assert 0 < a < b and a < c and a % 256 == 0

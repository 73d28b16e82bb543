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


def test_dropout_masks_of_two_seeds_are_independent(lib):
    """The fused LayerNorm's dropout mask (evaluated on the host by the same
    Philox code the kernels run): the keep rate is 1 - p, masks of different
    seeds are uncorrelated, and neither is an index-shuffled copy of the other
    (an XOR or a shift of the element index)."""
    import ctypes
    import numpy as np
    n, p = 1 << 20, 0.1
    masks = {}
    for seed in (1, 2, 1234567):
        buf = (ctypes.c_uint8 * n)()
        assert lib.affb_dropout_keep_mask(seed, p, 0, n, buf) == 0
        masks[seed] = np.frombuffer(buf, dtype=np.uint8).astype(np.float64)
    for m in masks.values():
        assert abs(m.mean() - (1 - p)) < 3e-3
    a, b = masks[1], masks[2]
    corr = np.corrcoef(a, b)[0, 1]
    assert abs(corr) < 0.01, corr
    e = np.arange(n)
    for shuffled in (a[e ^ (1 ^ 2)], np.roll(a, 1), np.roll(a, 3)):
        assert abs(np.corrcoef(shuffled, b)[0, 1]) < 0.01
    # a sub-range starting mid-stream equals the same slice of the whole stream
    buf = (ctypes.c_uint8 * 1000)()
    lib.affb_dropout_keep_mask(1, p, 12345, 1000, buf)
    assert np.array_equal(np.frombuffer(buf, dtype=np.uint8), masks[1][12345:13345].astype(np.uint8))

"""The C-ABI library loads and exports every symbol include/intcrush_b200.h declares (no GPU needed)."""

import ctypes
import os
import re

from int_crush_converter_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "intcrush_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ic_[a-z0-9_]+)\s*\(", src)))


def test_header_symbols_exported():
    lib = ctypes.CDLL(_native.LIB_PATH)
    names = declared()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), n


def test_binding_covers_header():
    assert set(declared()) == set(_native.SIGNATURES)


def test_version_and_no_device():
    lib = _native.load()
    assert b"sm_100a" in lib.ic_version()


def test_binding_rejects_wrong_argument_count():
    import pytest
    lib = _native.load()
    with pytest.raises(TypeError):
        lib.ic_rotate_hessian(None, 1, 4, 4, 4, None, None, 4, 4, None)  # one too many
    with pytest.raises(TypeError):
        lib.ic_version(1)


def test_greedy_gemm_passes_validated_before_any_device_use(monkeypatch):
    """The cross-term precision is 1 or 3 passes, from the keyword or the
    IC_GREEDY_GEMM_PASSES environment variable; anything else is a ValueError
    raised before a GPU is looked for."""
    import pytest
    import torch

    from int_crush_converter_b200 import greedy
    W = torch.zeros(2, 4)
    Q = torch.zeros(2, 4)
    with pytest.raises(ValueError, match="gemm_passes"):
        greedy.greedy_local_search(W, Q, torch.ones(2, 4), torch.eye(4), 1, -8, 7, gemm_passes=2)
    monkeypatch.setenv("IC_GREEDY_GEMM_PASSES", "5")
    with pytest.raises(ValueError, match="gemm_passes"):
        greedy.greedy_local_search(W, Q, torch.ones(2, 4), torch.eye(4), 1, -8, 7)

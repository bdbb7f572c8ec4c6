"""The C-ABI library loads on the CPU and exports exactly what include/gns_b200.h declares."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from gram_newton_schulz_ampere_b200 import _native, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "gns_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^GNS_API\s+[\w\s\*]+?\b(gns_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def library() -> ctypes.CDLL:
    if build.is_stale():
        build.build()
    return _native.load()


def test_header_declares_the_abi():
    names = declared_functions()
    assert "gns_gemm" in names and "gns_gram_newton_schulz" in names and "gns_dion3_select_rows" in names
    assert len(names) >= 15


def test_every_declared_symbol_is_exported(library):
    for name in declared_functions():
        assert hasattr(library, name), f"{name} missing from {_native.library_path()}"


def test_python_binding_covers_the_header():
    assert sorted(_native.SIGNATURES) == declared_functions()


def test_calls_that_need_no_gpu(library):
    assert library.gns_version() == 100
    assert library.gns_newton_schulz_workspace_size(64, 1024, 4096) > 64 * 1024 * 4096 * 2 * 2
    assert library.gns_dion3_select_workspace_size(16, 4096) >= 16 * 4096 * 4
    # Argument validation happens before any CUDA call.
    rc = library.gns_gemm(5, 1, 8, 8, 8, None, 0, 0, 0, None, 0, 0, 0, None, 0, 0, 0, None, 0, 0, 0,
                          1.0, 0.0, 0, None)
    assert rc == -1
    assert b"dtype" in library.gns_last_error()
    rc = library.gns_gram_newton_schulz(1, 1, 4, 8, None, 0, 0, None, 1, 0, 0, None, 0, 0, 1e-7, None, 0, None)
    assert rc == -1  # no coefficients
    assert library.gns_muon_momentum(0, None, None, None, None, 1, 1, 1, 0.9, 1, None) == 0


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setenv("GNS_B200_LIB", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="native library not found"):
        _native.load()

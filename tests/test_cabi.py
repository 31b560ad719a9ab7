"""The C-ABI library loads on a CPU-only host and exports every entry point
that include/harsh4b_b200.h declares (no GPU work is done here)."""
import ctypes
import re
from pathlib import Path

import pytest

from harsh4b_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "harsh4b_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|long long)\s+(h4b_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_bound_entry_points():
    assert declared_functions() == sorted(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    if not _lib.LIBRARY.exists():
        pytest.skip("library not built (run __graft_entry__.build())")
    library = ctypes.CDLL(str(_lib.LIBRARY))
    for name in declared_functions():
        assert hasattr(library, name), name


def test_no_cpu_fallback_without_a_device(monkeypatch):
    import torch

    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    _lib.lib.cache_clear()
    try:
        with pytest.raises(RuntimeError, match="no CPU fallback"):
            _lib.lib()
    finally:
        _lib.lib.cache_clear()

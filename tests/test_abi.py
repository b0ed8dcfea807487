"""CPU checks of the C ABI boundary: libq4k.so loads, exports exactly what
include/q4k.h declares, and rejects bad calls without touching a GPU."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "q4k.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^Q4K_API\s+[\w\s\*]+?\b(q4k_\w+)\s*\(", text, flags=re.M))


@pytest.fixture(scope="module")
def L():
    import q4k._lib as ql

    return ql.lib()


def test_header_declares_entry_points():
    names = declared()
    assert {"q4k_create", "q4k_destroy", "q4k_matmul_quant", "q4k_gemv", "q4k_lmhead_select"} <= names


def test_library_exports_every_declared_symbol(L):
    import q4k._lib as ql

    out = subprocess.run(["nm", "-D", "--defined-only", str(ql.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (q4k_\w+)", out))
    missing = declared() - exported
    assert not missing, f"declared but not exported: {missing}"
    for name in declared():
        assert hasattr(L, name)


def test_binding_table_matches_header():
    import q4k._lib as ql

    assert set(ql.SIGNATURES) == declared()


def test_version_and_null_context(L):
    assert L.q4k_version() >= 100
    assert L.q4k_last_error(None) == b"null context"
    # Every compute entry point rejects a null context before any CUDA call.
    assert L.q4k_gemv(None, None, None, None, 1, 256, 1, None) == -1
    assert L.q4k_matmul_quant(None, None, None, None, 1, 256, None) == -1
    assert L.q4k_lmhead_select(None, None, None, 1, 256, 30.0, 0, None, None, None, None, None) == -1
    assert L.q4k_merge_candidates(None, None, None, 1, None, None, None, None) == -1


def test_create_without_gpu_fails_cleanly(L):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    rc = L.q4k_create(0, ctypes.byref(h))
    assert rc != 0 and h.value is None

"""The C-ABI library loads on a machine without a GPU and exports every entry point include/kd_b200.h declares;
the ctypes declarations cover the same set. No kernel is called."""

import ctypes
import re
from pathlib import Path

import pytest

from karpo_decision_b200 import _lib
from karpo_decision_b200.build import LIBRARY, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "kd_b200.h"


def declared() -> set[str]:
    return set(re.findall(r"^int (kd_\w+)\(", HEADER.read_text(), re.M))


@pytest.fixture(scope="module")
def library():
    build()
    return ctypes.CDLL(str(LIBRARY))


def test_header_declares_entry_points():
    names = declared()
    assert {"kd_gemm_bf16", "kd_gemm_fp8", "kd_attention_varlen", "kd_readout"} <= names


def test_library_exports_every_declared_symbol(library):
    missing = [n for n in sorted(declared()) if not hasattr(library, n)]
    assert not missing, missing


def test_ctypes_signatures_match_header():
    assert set(_lib.SIGNATURES) == declared()


def test_version_and_error_channel_without_gpu(library):
    assert _lib.load().kd_version() >= 100
    assert isinstance(_lib.last_error(), str)


def test_argument_errors_launch_nothing():
    """A rejected call returns a negative status and a message before touching the device."""
    lib = _lib.load()
    rc = lib.kd_gemm_bf16(None, 0, None, 0, None, 0, None, 0, 16, 30, 64, 0, None, None)  # N % 32 != 0
    assert rc == -1
    assert "gemm" in _lib.last_error()
    rc = lib.kd_attention_varlen(None, 0, None, 0, None, 0, None, 0, None, 0, None, None, 2, 8, 16, 16, 3, 2, 128,
                                 1.0, -1, 0, None, None, None)  # 3 query heads over 2 kv heads
    assert rc == -1

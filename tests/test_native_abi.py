"""The C-ABI library loads and exports every symbol include/ima_b200.h declares
(no compute calls: this runs without a GPU)."""

from __future__ import annotations

import ctypes
import os
import re

from int_model_approximation_b200 import _native as nat

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ima_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ima_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("ima_int_gemm", "ima_hawkeye_replay", "ima_freivalds_fp8", "ima_quantize_per_token"):
        assert required in names


def test_library_exports_every_declared_symbol():
    handle = ctypes.CDLL(nat.library_path())
    missing = [n for n in declared_functions() if not hasattr(handle, n)]
    assert not missing, f"libima_b200.so lacks {missing}"


def test_python_binding_covers_header():
    assert set(declared_functions()) <= set(nat.SIGNATURES), set(declared_functions()) - set(nat.SIGNATURES)
    lib = nat.lib()
    assert lib.ima_abi_version() >= 1
    assert lib.ima_status_string(nat.IMA_ERR_TIMEOUT).decode() == "device wait timed out"


def test_descriptor_struct_layouts_match_the_header():
    sizes = (ctypes.c_int64 * 3)()
    assert nat.lib().ima_struct_sizes(sizes, 3) == 0
    assert list(sizes) == [
        ctypes.sizeof(nat.QuantizeProblem),
        ctypes.sizeof(nat.GemmProblem),
        ctypes.sizeof(nat.FreivaldsRowsProblem),
    ]


def test_host_only_queries():
    lib = nat.lib()
    assert lib.ima_scheme_planes(nat.IMA_SCHEME_DIGITS3) == 3
    assert lib.ima_scheme_planes(nat.IMA_SCHEME_DIGITS5) == 5
    assert lib.ima_hawkeye_operand_pitch(1) == 128
    assert lib.ima_hawkeye_operand_bytes(100, 33) == 128 * 2 * (32 * 8 + 16 * 4 + 4)
    assert lib.ima_freivalds_workspace_bytes(10) == 80


def test_argument_errors_are_reported_before_any_launch():
    lib = nat.lib()
    assert lib.ima_int_gemm(None, 16, None, 16, 1, 1, 1, 3, None, 1, None, None, None, None, 0, 1, None) == \
        nat.IMA_ERR_INVALID_ARGUMENT
    assert lib.ima_hawkeye_replay(1, 1, 1, 1, 1, 1, 32, 64, 14, -139, 1, 1, None, 1, None) == nat.IMA_ERR_UNSUPPORTED
    assert lib.ima_hawkeye_replay(1, 1, 1, 1, 1, 1, 32, 32, 12, -139, 1, 1, None, 1, None) == nat.IMA_ERR_UNSUPPORTED
    assert lib.ima_quantize_per_token(1, 7, 1, 1, 1, 1, 1, 1, None, 1, None, None, 16, None) == \
        nat.IMA_ERR_INVALID_ARGUMENT

"""ctypes binding of libima_b200.so (the C ABI declared in include/ima_b200.h).

This is the only place Python touches the native library.  There is no CPU or
PyTorch fallback: if the library is missing, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_native", "libima_b200.so")
_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

IMA_OK = 0
IMA_ERR_INVALID_ARGUMENT = 1
IMA_ERR_UNSUPPORTED = 2
IMA_ERR_CUDA = 3
IMA_ERR_TIMEOUT = 4
IMA_ERR_DEVICE_BOUNDS = 5
IMA_ERR_OVERFLOW = 6

IMA_DTYPE_F32 = 0
IMA_DTYPE_BF16 = 1
IMA_DTYPE_F16 = 2

IMA_SCHEME_DIGITS3 = 3
IMA_SCHEME_DIGITS5 = 5

_VP = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int

IMA_FREIVALDS_A_FP8 = 0
IMA_FREIVALDS_A_INT32 = 1


class QuantizeProblem(ctypes.Structure):
    """ima_quantize_problem"""

    _fields_ = [
        ("x", _VP), ("x_dtype", ctypes.c_int32), ("M", _I64), ("K", _I64), ("ldx", _I64), ("q_fp8", _VP),
        ("ldq", _I64), ("scale", _VP), ("codebook", _VP), ("ldc", _I64), ("code_scale", _VP), ("planes", _VP),
        ("ldp", _I64),
    ]


class GemmProblem(ctypes.Structure):
    """ima_gemm_problem"""

    _fields_ = [
        ("a_planes", _VP), ("lda", _I64), ("b_planes", _VP), ("ldb", _I64), ("M", _I64), ("N", _I64), ("K", _I64),
        ("c", _VP), ("ldc", _I64), ("x_scale", _VP), ("w_scale", _VP), ("bias", _VP), ("y", _VP),
        ("y_dtype", ctypes.c_int32), ("ldy", _I64),
    ]


class GemmYCopies(ctypes.Structure):
    """ima_gemm_y_copies"""

    _fields_ = [("y", _VP * 8)]


class CopyDesc(ctypes.Structure):
    """ima_copy_desc"""

    _fields_ = [("dst", _VP), ("src", _VP), ("bytes", _I64)]


class FreivaldsRowsProblem(ctypes.Structure):
    """ima_freivalds_rows_problem"""

    _fields_ = [
        ("a", _VP), ("lda", _I64), ("t", _VP), ("c", _VP), ("ldc", _I64), ("r", _VP), ("M", _I64), ("N", _I64),
        ("K", _I64), ("a_kind", ctypes.c_int32), ("mismatch_rows", _VP),
    ]


# name -> (restype, argtypes); mirrors include/ima_b200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ima_abi_version": (_I32, []),
    "ima_struct_sizes": (_I32, [_VP, _I32]),
    "ima_int32_issue_probe": (_I32, [_I64, _I32, _VP, _VP]),
    "ima_quant_fast_selftest": (_I32, [_I32, _VP, _VP]),
    "ima_quantize_grouped": (_I32, [_VP, _I32, _VP]),
    "ima_int_gemm_grouped": (_I32, [_VP, _I32, _I32, _VP]),
    "ima_int_gemm_grouped_copies": (_I32, [_VP, _VP, _I32, _I32, _VP]),
    "ima_set_gemm_sm_limit": (_I32, [_I32]),
    "ima_set_gemm_wait_test": (_I32, [_I64]),
    "ima_ipc_handle_bytes": (_I32, []),
    "ima_ipc_alloc": (_I32, [_I64, _VP, _VP]),
    "ima_ipc_free": (_I32, [_VP]),
    "ima_ipc_open": (_I32, [_VP, _VP]),
    "ima_ipc_close": (_I32, [_VP]),
    "ima_copy_async": (_I32, [_VP, _VP, _I64, _VP]),
    "ima_copy_many": (_I32, [_VP, _I32, _I32, _VP]),
    "ima_freivalds_weight_vector": (_I32, [_VP, _I64, _VP, _I64, _I64, _VP, _VP]),
    "ima_freivalds_rows_grouped": (_I32, [_VP, _I32, _VP]),
    "ima_status_string": (ctypes.c_char_p, [_I32]),
    "ima_last_cuda_error": (_I32, []),
    "ima_device_status": (_I32, [_I32, _VP, _VP, _VP, _I32]),
    "ima_quantize_per_token": (
        _I32,
        [_VP, _I32, _I64, _I64, _I64, _VP, _I64, _VP, _VP, _I64, _VP, _VP, _I64, _VP],
    ),
    "ima_codebook_from_fp8": (_I32, [_VP, _I64, _I64, _I64, _VP, _I64, _VP]),
    "ima_class_presence": (_I32, [_VP, _I64, _I64, _I64, _I64, _VP, _VP]),
    "ima_class_count_operand_bytes": (_I64, [_I64, _I64]),
    "ima_class_count_prepare": (_I32, [_VP, _I64, _I64, _I64, _VP, _VP]),
    "ima_class_count_weight_tiles_bytes": (_I64, [_I64, _I64]),
    "ima_class_count_weight_tiles": (_I32, [_VP, _I64, _I64, ctypes.c_uint64, _VP, _VP]),
    "ima_class_count_tile_entries": (_I64, [_I64, _I64, _I64]),
    "ima_class_count_replay": (
        _I32,
        [_VP, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP],
    ),
    "ima_planes_from_fp8": (_I32, [_VP, _I64, _I64, _I64, _VP, _I64, _VP, _VP]),
    "ima_planes_from_int32": (_I32, [_VP, _I64, _I64, _I64, _I64, _I32, _VP, _I64, _VP]),
    "ima_scheme_planes": (_I32, [_I32]),
    "ima_int32_maxabs": (_I32, [_VP, _I64, _I64, _I64, _I64, _VP, _VP]),
    "ima_int_gemm": (
        _I32,
        [_VP, _I64, _VP, _I64, _I64, _I64, _I64, _I32, _VP, _I64, _VP, _VP, _VP, _VP, _I32, _I64, _VP],
    ),
    "ima_hawkeye_operand_pitch": (_I64, [_I64]),
    "ima_hawkeye_operand_bytes": (_I64, [_I64, _I64]),
    "ima_hawkeye_prepare": (_I32, [_VP, _I64, _I64, _I64, _VP, _VP]),
    "ima_hawkeye_quantize_prepare": (_I32, [_VP, _I32, _I64, _I64, _I64, _VP, _VP, _I64, _VP, _VP]),
    "ima_hawkeye_replay": (
        _I32,
        [_VP, _VP, _VP, _VP, _I64, _I64, _I64, _I32, _I32, _I32, _VP, _I64, _VP, _I64, _VP],
    ),
    "ima_freivalds_workspace_bytes": (_I64, [_I64]),
    "ima_freivalds_fp8": (
        _I32,
        [_VP, _I64, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _VP],
    ),
    "ima_freivalds_fp8_noalloc": (
        _I32,
        [_VP, _I64, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP],
    ),
    "ima_freivalds_i32": (
        _I32,
        [_VP, _I64, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _VP],
    ),
}


def library_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is not built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    f"the B200 kernel library {_LIB_PATH} is not built; "
                    "run `python -c 'import __graft_entry__ as g; g.build()'` (there is no CPU execution path)"
                )
            handle = ctypes.CDLL(_LIB_PATH)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _check_struct_layouts(handle)
            _LIB = handle
    return _LIB


def _check_struct_layouts(handle: ctypes.CDLL) -> None:
    """Refuse a library whose descriptor structs differ from the ctypes mirrors above: a
    stale build would otherwise read the grouped launches' descriptors at wrong offsets."""
    mirrors = (QuantizeProblem, GemmProblem, FreivaldsRowsProblem)
    sizes = (ctypes.c_int64 * len(mirrors))()
    if handle.ima_struct_sizes(sizes, len(mirrors)) != IMA_OK:
        raise RuntimeError(f"{_LIB_PATH}: ima_struct_sizes failed")
    expected = [ctypes.sizeof(m) for m in mirrors]
    if list(sizes) != expected:
        raise RuntimeError(
            f"{_LIB_PATH} was built from a different include/ima_b200.h: descriptor sizes {list(sizes)}, "
            f"binding expects {expected}; rebuild with `python -m int_model_approximation_b200.build`"
        )


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        text = lib().ima_status_string(status).decode()
        detail = ""
        if status == IMA_ERR_CUDA:
            detail = f" (cudaError {lib().ima_last_cuda_error()})"
        super().__init__(f"{fn} failed: {text}{detail}")


def check(fn: str, status: int) -> None:
    if status != IMA_OK:
        raise NativeError(fn, status)


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def tensor_version(t: torch.Tensor) -> int | None:
    """The tensor's in-place version counter (None for inference tensors, which have none)."""
    try:
        return t._version
    except RuntimeError:
        return None


def require_device(device: torch.device, *named: tuple[str, torch.Tensor | None]) -> None:
    """Refuse (before any launch) tensors that are not on `device`: a host or
    other-device pointer must never reach a kernel."""
    for label, t in named:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError(f"{label} must be on CUDA; this repo has no CPU execution path")
        if t.device != device:
            raise RuntimeError(f"{label} is on {t.device}, expected {device}")


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(device: int = 0, clear: bool = True) -> tuple[int, int, int]:
    """(code, where, detail) of the device status word; synchronises the device."""
    code, where, detail = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(
        "ima_device_status",
        lib().ima_device_status(
            device, ctypes.byref(code), ctypes.byref(where), ctypes.byref(detail), 1 if clear else 0
        ),
    )
    return code.value, where.value, detail.value


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return IMA_DTYPE_F32
    if dtype == torch.bfloat16:
        return IMA_DTYPE_BF16
    if dtype == torch.float16:
        return IMA_DTYPE_F16
    raise RuntimeError(f"unsupported dtype {dtype}; expected float32, bfloat16 or float16")

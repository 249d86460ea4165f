"""Exact FP8-codebook integer GEMM: quantiser, digit planes and the tcgen05 GEMM.

Kernel-level host API over the C ABI (include/ima_b200.h).  The reference
equivalents live in the reference package's __main__.py:
  per_token_fp8 / per_token_fp8_codebook   <- _per_token_fp8 :148-154, _per_token_fp8_int32 :161-163
  codebook_planes_from_fp8                 <- CodebookLinear.__init__ :429-432 (weight prepack)
  int_gemm                                 <- _int32_raw_matmul :228-253, _int32_matmul :301-333
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat

FP8_E4M3_MAX = 448.0
FP8_E4M3_CODE_SCALE = 512.0
DIGITS3_MAX_ABS = 1_064_960  # largest |v| the three balanced base-128 digits represent


def _round16(k: int) -> int:
    return max(16, (k + 15) // 16 * 16)


@dataclass
class DigitPlanes:
    """int8 digit planes [P, rows, ld] of an integer matrix [rows, K] (K-major)."""

    planes: torch.Tensor
    rows: int
    k: int
    scheme: int

    @property
    def ld(self) -> int:
        return int(self.planes.shape[2])

    @staticmethod
    def empty(rows: int, k: int, scheme: int, device: torch.device) -> "DigitPlanes":
        count = 3 if scheme == nat.IMA_SCHEME_DIGITS3 else 5
        planes = torch.empty((count, rows, _round16(k)), dtype=torch.int8, device=device)
        return DigitPlanes(planes, rows, k, scheme)


def _require_cuda(t: torch.Tensor, label: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(f"{label} must be on CUDA; this repo has no CPU execution path")


def per_token_fp8(x: torch.Tensor, *, codebook: bool = False, planes: bool = False):
    """Per-token e4m3 quantisation of x [..., K] in one kernel.

    Returns (q_fp8 [M,K], scale [M,1] fp32, codebook int32 [M,K] or None,
    code_scale [M,1] or None, DigitPlanes or None).  Bit-identical to the
    reference's torch expression as it runs on CUDA (amax / 448 as a multiplication by the
    fp32 reciprocal, clamp 1e-12, fp32 division of the elements, e4m3 RNE).
    """
    _require_cuda(x, "FP8 activation")
    rows = x.reshape(-1, x.shape[-1])
    if rows.stride(-1) != 1:
        rows = rows.contiguous()
    m, k = rows.shape
    dev = rows.device
    q = torch.empty((m, k), dtype=torch.uint8, device=dev)
    scale = torch.empty((m, 1), dtype=torch.float32, device=dev)
    with torch.inference_mode(False):
        # a normal tensor even inside inference mode: its version counter lets a cache of
        # its digit planes notice in-place edits (inference tensors have no counter)
        cb = torch.empty((m, k), dtype=torch.int32, device=dev) if codebook else None
    cs = torch.empty((m, 1), dtype=torch.float32, device=dev) if codebook else None
    dp = DigitPlanes.empty(m, k, nat.IMA_SCHEME_DIGITS3, dev) if planes else None
    with torch.cuda.device(dev):
        nat.call(
            "ima_quantize_per_token",
            rows.data_ptr(),
            nat.dtype_code(rows.dtype),
            m,
            k,
            rows.stride(0) if m > 1 else k,
            q.data_ptr(),
            k,
            scale.data_ptr(),
            nat.ptr(cb),
            k,
            nat.ptr(cs),
            nat.ptr(dp.planes) if dp is not None else None,
            dp.ld if dp is not None else 16,
            nat.stream_of(dev),
        )
    return q.view(torch.float8_e4m3fn), scale, cb, cs, dp


def codebook_planes_from_fp8(w_fp8: torch.Tensor, *, with_codebook_t: bool = False):
    """Digit planes (DIGITS3) of the codebook values of an e4m3 matrix [rows, K] (a weight, prepared once).

    Optionally also returns the reference's `weight_t` = int32 codebook transposed [K, rows].
    """
    _require_cuda(w_fp8, "FP8 codebook weight")
    w = w_fp8.contiguous().view(torch.uint8)
    rows, k = w.shape
    dp = DigitPlanes.empty(rows, k, nat.IMA_SCHEME_DIGITS3, w.device)
    with torch.inference_mode(False):   # versioned even inside inference mode (see per_token_fp8)
        cbt = torch.empty((k, rows), dtype=torch.int32, device=w.device) if with_codebook_t else None
    with torch.cuda.device(w.device):
        nat.call(
            "ima_planes_from_fp8", w.data_ptr(), rows, k, k, dp.planes.data_ptr(), dp.ld, nat.ptr(cbt),
            nat.stream_of(w.device),
        )
    return dp, cbt


def int32_maxabs(t: torch.Tensor) -> int:
    """max |t| of a 2-D int32 CUDA tensor (one device reduction, one host sync)."""
    out = torch.zeros((1,), dtype=torch.int64, device=t.device)
    with torch.cuda.device(t.device):
        nat.call(
            "ima_int32_maxabs", t.data_ptr(), t.shape[0], t.shape[1], t.stride(0), t.stride(1), out.data_ptr(),
            nat.stream_of(t.device),
        )
    return int(out.item())


def planes_from_int32(t: torch.Tensor, *, transpose: bool = False, scheme: int | None = None) -> DigitPlanes:
    """Digit planes of an int32 matrix.  t is [rows, K], or [K, rows] with transpose=True
    (the reference's weight_t layout).  The scheme defaults to the cheapest exact one."""
    rows, k = (t.shape[1], t.shape[0]) if transpose else (t.shape[0], t.shape[1])
    sr, sk = (t.stride(1), t.stride(0)) if transpose else (t.stride(0), t.stride(1))
    if scheme is None:
        scheme = nat.IMA_SCHEME_DIGITS3 if int32_maxabs(t) <= DIGITS3_MAX_ABS else nat.IMA_SCHEME_DIGITS5
    dp = DigitPlanes.empty(rows, k, scheme, t.device)
    with torch.cuda.device(t.device):
        nat.call(
            "ima_planes_from_int32", t.data_ptr(), rows, k, sr, sk, scheme, dp.planes.data_ptr(), dp.ld,
            nat.stream_of(t.device),
        )
    return dp


def int_gemm(
    a: DigitPlanes,
    b: DigitPlanes,
    *,
    want_c: bool = True,
    x_scale: torch.Tensor | None = None,
    w_scale: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    y_dtype: torch.dtype | None = None,
    c_out: torch.Tensor | None = None,
    y_out: torch.Tensor | None = None,
):
    """C = A B^T exactly (int64) and/or y = (fp32(C) * x_scale[m]) * w_scale[n] (+ bias).

    a: planes of the left operand [M, K]; b: planes of the right operand given as [N, K].
    Returns (c int64 [M,N] or None, y [M,N] or None).
    """
    if a.scheme != b.scheme:
        raise RuntimeError("int_gemm operands use different digit schemes")
    if a.k != b.k:
        raise RuntimeError(f"int32 matmul shape mismatch: K={a.k} vs K={b.k}")
    dev = a.planes.device
    m, n, k = a.rows, b.rows, a.k
    c = c_out if c_out is not None else (torch.empty((m, n), dtype=torch.int64, device=dev) if want_c else None)
    y = None
    if y_dtype is not None or y_out is not None:
        if x_scale is None or w_scale is None:
            raise RuntimeError("int_gemm needs x_scale and w_scale for the rescaled output")
        y = y_out if y_out is not None else torch.empty((m, n), dtype=y_dtype, device=dev)
        x_scale = x_scale.reshape(-1).to(torch.float32).contiguous()
        w_scale = w_scale.reshape(-1).to(torch.float32).contiguous()
        if bias is not None:
            bias = bias.reshape(-1).to(torch.float32).contiguous()
        if x_scale.numel() != m or w_scale.numel() != n or (bias is not None and bias.numel() != n):
            raise RuntimeError(
                f"int_gemm scale/bias sizes {x_scale.numel()}, {w_scale.numel()} do not match M={m}, N={n}"
            )
    nat.require_device(
        dev, ("B planes", b.planes), ("int64 output", c), ("output", y), ("x_scale", x_scale),
        ("w_scale", w_scale), ("bias", bias),
    )
    with torch.cuda.device(dev):
        nat.call(
            "ima_int_gemm",
            a.planes.data_ptr(),
            a.ld,
            b.planes.data_ptr(),
            b.ld,
            m,
            n,
            k,
            a.scheme,
            nat.ptr(c),
            c.stride(0) if c is not None else n,
            nat.ptr(x_scale) if y is not None else None,
            nat.ptr(w_scale) if y is not None else None,
            nat.ptr(bias) if y is not None else None,
            nat.ptr(y),
            nat.dtype_code(y.dtype) if y is not None else 0,
            y.stride(0) if y is not None else n,
            nat.stream_of(dev),
        )
    return c, y

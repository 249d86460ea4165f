"""Freivalds check of claimed int64 products on B200.

The reference checks its int64 products only in tests
(tests/test_real_integer_gemms.py:67-93: _exact_matvec and
_assert_freivalds_verifies_int_product, with Python big integers).  Here the
check is a production operation: A (B r) == C r evaluated modulo 2^64 by two
bandwidth-bound GEMV kernels (csrc/freivalds.cu).  A correct product always
passes; a product with one entry off by d is rejected whenever d * r[n] != 0 mod 2^64.
"""

from __future__ import annotations

import torch

from . import _native as nat

FREIVALDS_VECTOR_BITS = 20  # r is uniform in [0, 2^20)


def freivalds_vector(n: int, seed: int, device: torch.device | str = "cpu") -> torch.Tensor:
    """Seeded int64 vector uniform in [0, 2^20) (CPU generator, then moved)."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    r = torch.randint(0, 1 << FREIVALDS_VECTOR_BITS, (n,), generator=g, dtype=torch.int64)
    return r.to(device)


def weight_vector(w_fp8: torch.Tensor, r: torch.Tensor) -> torch.Tensor:
    """t = codebook(w)^T r (int64 [K], wrapping): the weight half of the check, fixed for
    a given weight and vector, so it is computed once per linear."""
    w = w_fp8.contiguous().view(torch.uint8)
    n, k = w.shape
    if r.dtype != torch.int64 or r.numel() != n:
        raise RuntimeError("Freivalds vector must be int64 with one entry per weight row")
    r = r.reshape(-1).contiguous()
    nat.require_device(w.device, ("vector", r))
    t = torch.empty((max(k, 1),), dtype=torch.int64, device=w.device)
    with torch.cuda.device(w.device):
        nat.call("ima_freivalds_weight_vector", w.data_ptr(), k, r.data_ptr(), n, k, t.data_ptr(),
                 nat.stream_of(w.device))
    return t[:k]


def _workspace(k: int, device: torch.device) -> torch.Tensor:
    nbytes = int(nat.lib().ima_freivalds_workspace_bytes(k))
    return torch.empty((nbytes // 8,), dtype=torch.int64, device=device)


def mismatch_rows_codebook(
    x_fp8: torch.Tensor,
    w_fp8: torch.Tensor,
    c: torch.Tensor,
    r: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Rows m where codebook(x) (codebook(w)^T r) != C r (mod 2^64), counted into a
    device int32 scalar (accumulated into `out` when given).  No host sync."""
    if c.dtype != torch.int64 or r.dtype != torch.int64:
        raise RuntimeError("Freivalds check needs an int64 product and an int64 vector")
    x = x_fp8.contiguous().view(torch.uint8)
    w = w_fp8.contiguous().view(torch.uint8)
    m, k = x.shape
    n, k2 = w.shape
    if k != k2 or tuple(c.shape) != (m, n) or r.numel() != n:
        raise RuntimeError(f"Freivalds shape mismatch: x {tuple(x.shape)}, w {tuple(w.shape)}, c {tuple(c.shape)}")
    if c.stride(1) != 1:
        c = c.contiguous()
    r = r.reshape(-1).contiguous()
    dev = c.device
    if out is None:
        out = torch.zeros((1,), dtype=torch.int32, device=dev)
    nat.require_device(dev, ("product", c), ("activations", x), ("weights", w), ("vector", r), ("counter", out))
    ws = _workspace(k, dev)
    with torch.cuda.device(dev):
        nat.call(
            "ima_freivalds_fp8", x.data_ptr(), k, w.data_ptr(), k, c.data_ptr(), c.stride(0), r.data_ptr(), m, n, k,
            ws.data_ptr(), out.data_ptr(), nat.stream_of(dev),
        )
    return out


def mismatch_rows_int32(
    a: torch.Tensor,
    b: torch.Tensor,
    c: torch.Tensor,
    r: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Same check for int32 operands a [M,K] and b [K,N] (the reference's weight_t)."""
    if a.dtype != torch.int32 or b.dtype != torch.int32:
        raise RuntimeError("Freivalds check received non-int32 operands")
    if c.dtype != torch.int64 or r.dtype != torch.int64:
        raise RuntimeError("Freivalds check needs an int64 product and an int64 vector")
    a = a.contiguous()
    b = b.contiguous()
    m, k = a.shape
    k2, n = b.shape
    if k != k2 or tuple(c.shape) != (m, n) or r.numel() != n:
        raise RuntimeError(f"Freivalds shape mismatch: a {tuple(a.shape)}, b {tuple(b.shape)}, c {tuple(c.shape)}")
    if c.stride(1) != 1:
        c = c.contiguous()
    r = r.reshape(-1).contiguous()
    dev = c.device
    if out is None:
        out = torch.zeros((1,), dtype=torch.int32, device=dev)
    nat.require_device(dev, ("product", c), ("a", a), ("b", b), ("vector", r), ("counter", out))
    ws = _workspace(k, dev)
    with torch.cuda.device(dev):
        nat.call(
            "ima_freivalds_i32", a.data_ptr(), k, b.data_ptr(), n, c.data_ptr(), c.stride(0), r.data_ptr(), m, n, k,
            ws.data_ptr(), out.data_ptr(), nat.stream_of(dev),
        )
    return out


def verify_int32_product(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, r: torch.Tensor) -> bool:
    """True iff the claimed product c of a [M,K] and b [K,N] passes the check (host sync)."""
    return int(mismatch_rows_int32(a, b, c, r).item()) == 0


def verify_codebook_product(x_fp8: torch.Tensor, w_fp8: torch.Tensor, c: torch.Tensor, r: torch.Tensor) -> bool:
    """True iff c is the codebook product of x_fp8 [M,K] and w_fp8 [N,K] per the check (host sync)."""
    return int(mismatch_rows_codebook(x_fp8, w_fp8, c, r).item()) == 0

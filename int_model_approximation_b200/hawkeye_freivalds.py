"""Exact Hawkeye replay from class-count products, B200 edition.

Drop-in for the reference's hawkeye_freivalds.py: same constants (:13-19), the
same HawkeyeFreivaldsStats (:22-33), the same exact_hawkeye_fp8_sum signature and
parameter validation (:1017-1050, :878-886), bit-identical bf16 output and
identical stats.

How the B200 path works.  The reference materialises one packed count product per
(activation-class chunk, weight-class chunk) pair of every pack and replays the
Hawkeye accumulator from those counts.  Summing count(a, b) * aligned(a, b, maxe)
over class pairs is a regrouping of the per-k sum the direct replay computes, so the
output is produced by the direct replay engine (csrc/hawkeye.cu) without
materialising any counts.  The class bookkeeping that defines the checkable products
(one class-presence kernel over all packs, one host read instead of one
torch.unique sync per group) yields the same product count and class maxima as the
reference; each checkable product bumps the active int32 probe once, exactly as the
reference's raw_matmul calls do.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch

from . import _native as nat
from .hawkeye import HawkeyeOperand, _validate_params, hawkeye_replay, stage_weight

FP32_SIGNIFICAND_WIDTH = 24
FP32_MIN_NONZERO_EXPONENT = -126
SIGNED_SIG_BUCKETS = 31
SIGNED_SIG_OFFSET = 15
PACKED_COUNT_BASE_LOG2 = 6
PACKED_COUNT_BASE = 1 << PACKED_COUNT_BASE_LOG2
MAX_PACKED_COUNT_LANES = 6
CLASS_MASK_WORDS = 16  # presence bitmask words per pack (class ids < 512)


@dataclass(frozen=True)
class HawkeyeFreivaldsStats:
    products_per_group: int
    groups: int
    packed_group_lanes: int
    class_products_first_pass: int
    class_products_replay_pass: int
    total_checkable_products: int
    max_activation_classes_per_group: int
    max_weight_classes_per_group: int
    class_chunk: int
    packed_count_lanes: int


RawIntMatmul = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


def class_presence(fp8: torch.Tensor, pack_width: int) -> torch.Tensor:
    """int32 [packs, 16] bitmasks of the classes present in each pack (device tensor)."""
    raw = fp8.contiguous().view(torch.uint8)
    rows, k = raw.shape
    packs = (k + pack_width - 1) // pack_width
    masks = torch.empty((max(packs, 1), CLASS_MASK_WORDS), dtype=torch.int32, device=raw.device)
    with torch.cuda.device(raw.device):
        nat.call(
            "ima_class_presence", raw.data_ptr(), rows, k, k, pack_width, masks.data_ptr(), nat.stream_of(raw.device)
        )
    return masks[:packs]


def _popcounts(masks: torch.Tensor) -> list[int]:
    """Number of set bits per pack (host side, one D2H copy)."""
    words = masks.to("cpu", torch.int64) & 0xFFFFFFFF
    out = []
    for row in words.tolist():
        out.append(sum(int(w).bit_count() for w in row))
    return out


def _ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def class_count_stats(
    a_classes_per_pack: list[int],
    b_classes_per_pack: list[int],
    k_size: int,
    *,
    products_per_group: int,
    class_chunk: int,
    packed_count_lanes: int,
    packed_group_lanes: int,
) -> HawkeyeFreivaldsStats:
    """Stats of exact_hawkeye_fp8_sum given the class counts of every pack.

    Follows the reference's control flow: per pack, ceil(n_a / class_chunk) activation
    chunks times ceil(n_b / b_chunk) weight chunks checkable products, with b_chunk =
    class_chunk * packed_count_lanes // packed_group_lanes lanes (class_chunk alone when
    unpacked) (hawkeye_freivalds.py:910-913, :1114-1116)."""
    groups = 0
    products = 0
    if packed_group_lanes > 1:
        pack_width = products_per_group * packed_group_lanes
        b_chunk = class_chunk * (packed_count_lanes // packed_group_lanes)
        for p, (na, nb) in enumerate(zip(a_classes_per_pack, b_classes_per_pack)):
            k0 = p * pack_width
            k1 = min(k0 + pack_width, k_size)
            groups += _ceil_div(k1 - k0, products_per_group)
            products += _ceil_div(na, class_chunk) * _ceil_div(nb, b_chunk)
    else:
        b_chunk = class_chunk if packed_count_lanes == 1 else class_chunk * packed_count_lanes
        for na, nb in zip(a_classes_per_pack, b_classes_per_pack):
            groups += 1
            products += _ceil_div(na, class_chunk) * _ceil_div(nb, b_chunk)
    return HawkeyeFreivaldsStats(
        products_per_group=products_per_group,
        groups=groups,
        packed_group_lanes=packed_group_lanes,
        class_products_first_pass=0,
        class_products_replay_pass=products,
        total_checkable_products=products,
        max_activation_classes_per_group=max(a_classes_per_pack, default=0),
        max_weight_classes_per_group=max(b_classes_per_pack, default=0),
        class_chunk=class_chunk,
        packed_count_lanes=packed_count_lanes,
    )


def _bump_probe(count: int) -> None:
    # The reference bumps __main__._ACTIVE_INT32_PROBE once per raw_matmul launch
    # (__main__.py:239-240); the students module owns the probe here.
    from . import students

    probe = students._ACTIVE_INT32_PROBE
    if probe is not None:
        probe.count += count


def exact_hawkeye_fp8_sum(
    x_fp8: torch.Tensor,
    x_scale: torch.Tensor,
    w_fp8: torch.Tensor,
    w_scale: torch.Tensor,
    raw_matmul: RawIntMatmul | None = None,
    *,
    products_per_group: int = 32,
    internal_width: int = 14,
    zero_exponent: int = -139,
    class_chunk: int = 32,
    packed_count_lanes: int = 1,
    packed_group_lanes: int = 1,
    fused_replay: bool = False,
    cache_weight_chunks: bool = False,
    count_dtype: torch.dtype = torch.int32,
) -> tuple[torch.Tensor, HawkeyeFreivaldsStats]:
    """Replay Hawkeye exactly from Freivalds-checkable class-count products.

    ref: hawkeye_freivalds.py:1017-1246.  `raw_matmul` is accepted for signature
    compatibility: the B200 engine forms the count products itself (fused), so the
    callable is not invoked; every checkable product is still counted on the active
    int32 probe.
    """
    if count_dtype not in {torch.int8, torch.int32}:
        raise ValueError(f"count_dtype must be torch.int8 or torch.int32, got {count_dtype}")
    if count_dtype == torch.int8 and (packed_count_lanes != 1 or fused_replay):
        raise ValueError("int8 count products are only supported for unpacked non-fused replay")
    if packed_count_lanes < 1 or packed_count_lanes > MAX_PACKED_COUNT_LANES:
        raise ValueError(
            f"packed_count_lanes must be in [1, {MAX_PACKED_COUNT_LANES}], got {packed_count_lanes}"
        )
    if packed_group_lanes < 1 or packed_group_lanes > packed_count_lanes:
        raise ValueError("packed_group_lanes must fit inside packed_count_lanes")
    if packed_group_lanes > 1 and (count_dtype != torch.int32 or fused_replay or cache_weight_chunks):
        raise ValueError(
            "packed_group_lanes > 1 currently requires int32 count products without "
            "fused_replay or cache_weight_chunks"
        )
    if packed_group_lanes > 1:
        if packed_count_lanes // packed_group_lanes < 1:
            raise ValueError("packed_group_lanes leaves no lanes for weight classes")
        if products_per_group > PACKED_COUNT_BASE:
            raise ValueError(
                "packed group counts require products_per_group <= PACKED_COUNT_BASE "
                "to avoid cross-lane carries"
            )
    if x_fp8.device.type != "cuda" or w_fp8.device.type != "cuda":
        raise RuntimeError("Hawkeye class-count replay is CUDA-only")
    if x_fp8.dtype != torch.float8_e4m3fn or w_fp8.dtype != torch.float8_e4m3fn:
        raise RuntimeError("Hawkeye class-count replay requires float8_e4m3fn operands")
    if x_fp8.ndim != 2 or w_fp8.ndim != 2 or x_fp8.shape[1] != w_fp8.shape[1]:
        raise RuntimeError(f"Hawkeye shape mismatch: {x_fp8.shape} vs {w_fp8.shape}")
    if class_chunk <= 0:
        raise ValueError("class_chunk must be positive")
    _validate_params(products_per_group, internal_width, zero_exponent)

    m_size, k_size = x_fp8.shape
    n_size = w_fp8.shape[0]
    # The reference scales with y * x_scale * w_scale.reshape(1, -1), x_scale being the
    # per-token [M, 1] scale; a scalar scale broadcasts the same way.
    if x_scale.numel() not in (1, m_size):
        raise RuntimeError(f"x_scale of shape {tuple(x_scale.shape)} does not broadcast as [M, 1] for M={m_size}")
    xs = x_scale.reshape(-1).to(torch.float32)
    if xs.numel() == 1 and m_size != 1:
        xs = xs.expand(m_size)

    pack_width = products_per_group * (packed_group_lanes if packed_group_lanes > 1 else 1)
    a_counts = _popcounts(class_presence(x_fp8, pack_width))
    b_counts = _popcounts(class_presence(w_fp8, pack_width))
    stats = class_count_stats(
        a_counts,
        b_counts,
        k_size,
        products_per_group=products_per_group,
        class_chunk=class_chunk,
        packed_count_lanes=packed_count_lanes,
        packed_group_lanes=packed_group_lanes,
    )
    _bump_probe(stats.total_checkable_products)

    x_op = HawkeyeOperand(x_fp8)
    w_op = stage_weight(w_fp8)
    out = hawkeye_replay(x_op, w_op, xs.contiguous(), w_scale)
    return out, stats

"""Exact Hawkeye replay from class-count products, B200 edition.

Drop-in for the reference's hawkeye_freivalds.py: same constants (:13-19), the
same HawkeyeFreivaldsStats (:22-33), the same exact_hawkeye_fp8_sum signature and
parameter validation (:1017-1050, :878-886), bit-identical bf16 output and
identical stats.

How the B200 path works.  The reference forms one packed count product per
(activation-class chunk, weight-class chunk) pair of every pack and replays the
Hawkeye accumulator from those counts.  Here the class-count engine
(csrc/class_count_engine.cu) forms the counts on the tcgen05 tensor cores -- for each
group of 32 k, the counts of every (activation class, weight class) pair of every
output, i.e. every row and column of the reference's product that can be nonzero --
checks each count tile with a Freivalds fingerprint, and replays the accumulator from
the counts in the same kernel; the counts never reach HBM.  The class bookkeeping that
defines the reference's checkable products (one class-presence kernel over all packs,
one host read instead of one torch.unique sync per group) yields the same product count
and class maxima as the reference.

raw_matmul.  With raw_matmul None (what HawkeyeClassCountsLinear passes) the engine
forms the products and the active int32 probe is bumped once per product the reference
would have sent through its _int32_raw_matmul.  Any callable instead receives the
reference's products themselves -- the same one-hot / lane-packed operands in the same
order, one call per checkable product (as the reference calls it; _int32_raw_matmul
bumps the probe per call) -- and every product it returns is Freivalds-checked on the
GPU (a wrong one raises); the output is the engine's.  The count-product helpers keep
the reference's names and layouts (hawkeye_freivalds.py:39-57, :147-213, :593-704,
:840-841), so code written against them runs unchanged.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch

from . import _native as nat
from .hawkeye import _validate_params

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


# ---------------------------------------------------------------------------
# Class ids and count-product operands (the reference's layouts; any device)
# ---------------------------------------------------------------------------
def _decode_fp8_fields(x_fp8: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(effective exponent, signed 4-bit significand, present) of every e4m3 element, int64.
    ref: hawkeye_freivalds.py:39-48."""
    b = x_fp8.contiguous().view(torch.uint8).to(torch.int64)
    field = (b >> 3) & 0xF
    mag = torch.where(field != 0, (b & 7) | 8, b & 7)
    exp = torch.clamp(field, min=1)
    sig = torch.where((b & 0x80) != 0, -mag, mag)
    return exp, sig, mag != 0


def _class_ids(exp_eff: torch.Tensor, signed_sig: torch.Tensor, nonzero: torch.Tensor) -> torch.Tensor:
    """class = (e - 1) * 31 + (s + 15) for present elements, -1 otherwise.  ref: :51-57."""
    ids = (exp_eff - 1) * SIGNED_SIG_BUCKETS + signed_sig + SIGNED_SIG_OFFSET
    return ids.masked_fill(~nonzero, -1)


def _iter_class_chunks(classes: torch.Tensor, chunk_size: int) -> list[torch.Tensor]:
    """Consecutive slices of at most chunk_size classes.  ref: :840-841."""
    return [classes[i:i + chunk_size] for i in range(0, int(classes.numel()), chunk_size)]


def _one_hot_rows(class_group: torch.Tensor, classes: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """[len(classes) * rows, k]: row (c, r) marks the k where class_group[r, k] == classes[c]."""
    rows, k = class_group.shape
    hit = class_group.unsqueeze(0) == classes.reshape(-1, 1, 1)
    return hit.to(dtype).reshape(int(classes.numel()) * rows, k).contiguous()


def _weight_chunk_flat(
    b_class_group: torch.Tensor, b_classes: torch.Tensor, *, count_dtype: torch.dtype = torch.int32
) -> torch.Tensor:
    """[k, len(b_classes) * N]: column (c, n) marks the k where b_class_group[n, k] == b_classes[c].
    ref: :188-199."""
    return _one_hot_rows(b_class_group, b_classes, count_dtype).t().contiguous()


def _class_chunk_product_raw_with_b_flat(
    a_class_group: torch.Tensor, a_classes: torch.Tensor, b_flat: torch.Tensor, b_size: int, raw_matmul: RawIntMatmul
) -> tuple[torch.Tensor, int, int]:
    """raw_matmul(one-hot A, b_flat) -> ([a_size * M, b_size * N], a_size, b_size).  ref: :202-213."""
    a_flat = _one_hot_rows(a_class_group, a_classes, b_flat.dtype)
    return raw_matmul(a_flat, b_flat), int(a_classes.numel()), b_size


def _class_chunk_product_raw(
    a_class_group: torch.Tensor,
    b_class_group: torch.Tensor,
    a_classes: torch.Tensor,
    b_classes: torch.Tensor,
    raw_matmul: RawIntMatmul,
    *,
    count_dtype: torch.dtype = torch.int32,
) -> tuple[torch.Tensor, int, int]:
    """The unpacked count product, flat.  ref: :166-185."""
    b_flat = _weight_chunk_flat(b_class_group, b_classes, count_dtype=count_dtype)
    return _class_chunk_product_raw_with_b_flat(a_class_group, a_classes, b_flat, int(b_classes.numel()), raw_matmul)


def _class_chunk_product(
    a_class_group: torch.Tensor,
    b_class_group: torch.Tensor,
    a_classes: torch.Tensor,
    b_classes: torch.Tensor,
    raw_matmul: RawIntMatmul,
    *,
    count_dtype: torch.dtype = torch.int32,
) -> torch.Tensor:
    """counts[a, b, m, n] = #k with class a at (m, k) and class b at (n, k).  ref: :147-163."""
    flat, a_size, b_size = _class_chunk_product_raw(
        a_class_group, b_class_group, a_classes, b_classes, raw_matmul, count_dtype=count_dtype
    )
    m, n = a_class_group.shape[0], b_class_group.shape[0]
    return flat.reshape(a_size, m, b_size, n).permute(0, 2, 1, 3)


def _lane_packed_classes(b_classes: torch.Tensor, lanes: int) -> torch.Tensor:
    """b_classes laid out [ceil(nb / lanes), lanes], unused lanes -2 (never a class)."""
    groups = -(-int(b_classes.numel()) // lanes)
    out = torch.full((groups, lanes), -2, dtype=b_classes.dtype, device=b_classes.device)
    out.view(-1)[: b_classes.numel()] = b_classes
    return out


def _lane_packed_b_flat(
    b_class_pack: torch.Tensor, packed: torch.Tensor, lane_of_k: torch.Tensor, lanes_per_group: int
) -> torch.Tensor:
    """[k, groups * N] int32: 64^lane summed over the lane whose class matches (n, k); the lane of
    class slot j at k is lane_of_k[k] * lanes_per_group + j."""
    groups, slots = packed.shape
    n, k = b_class_pack.shape
    hit = b_class_pack.unsqueeze(0).unsqueeze(0) == packed.reshape(groups, slots, 1, 1)   # [G, S, N, K]
    lane = lane_of_k.reshape(1, 1, 1, k) * lanes_per_group + torch.arange(slots, device=packed.device).reshape(1, slots, 1, 1)
    weight = torch.bitwise_left_shift(torch.ones_like(lane), PACKED_COUNT_BASE_LOG2 * lane)
    value = (hit.to(torch.int64) * weight).sum(dim=1)                                      # [G, N, K]
    return value.permute(2, 0, 1).reshape(k, groups * n).to(torch.int32).contiguous()


def _packed_class_chunk_product(
    a_class_group: torch.Tensor,
    b_class_group: torch.Tensor,
    a_classes: torch.Tensor,
    b_classes: torch.Tensor,
    raw_matmul: RawIntMatmul,
    packed_count_lanes: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Counts of up to packed_count_lanes weight classes per int64, base 64.
    Returns (counts [a, packed group, m, n], packed_b_classes [groups, lanes]).  ref: :593-631."""
    packed = _lane_packed_classes(b_classes, packed_count_lanes)
    k = a_class_group.shape[1]
    b_flat = _lane_packed_b_flat(b_class_group, packed, torch.zeros(k, dtype=torch.int64, device=packed.device),
                                 packed_count_lanes)
    a_flat = _one_hot_rows(a_class_group, a_classes, torch.int32)
    flat = raw_matmul(a_flat, b_flat)
    m, n = a_class_group.shape[0], b_class_group.shape[0]
    return flat.reshape(int(a_classes.numel()), m, packed.shape[0], n).permute(0, 2, 1, 3), packed


def _packed_group_class_chunk_product(
    a_class_pack: torch.Tensor,
    b_class_pack: torch.Tensor,
    a_classes: torch.Tensor,
    b_classes: torch.Tensor,
    raw_matmul: RawIntMatmul,
    *,
    products_per_group: int,
    packed_group_lanes: int,
    packed_count_lanes: int,
) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Counts of a pack of groups: lane = group * (lanes // group lanes) + weight-class slot.
    Returns (counts [a, packed group, m, n], packed_b_classes, weight lanes per group).  ref: :634-704."""
    k = a_class_pack.shape[1]
    groups_in_pack = -(-k // products_per_group)
    if groups_in_pack > packed_group_lanes:
        raise RuntimeError("group pack contains more groups than packed_group_lanes")
    if packed_group_lanes < 1 or packed_group_lanes > packed_count_lanes:
        raise ValueError("packed_group_lanes must fit inside packed_count_lanes")
    b_lanes = packed_count_lanes // packed_group_lanes
    if b_lanes < 1:
        raise ValueError("packed_group_lanes leaves no lanes for weight classes")
    if packed_group_lanes * b_lanes > MAX_PACKED_COUNT_LANES:
        raise ValueError("too many packed count lanes")
    packed = _lane_packed_classes(b_classes, b_lanes)
    lane_of_k = torch.arange(k, device=packed.device) // products_per_group
    b_flat = _lane_packed_b_flat(b_class_pack, packed, lane_of_k, b_lanes)
    a_flat = _one_hot_rows(a_class_pack, a_classes, torch.int32)
    flat = raw_matmul(a_flat, b_flat)
    m, n = a_class_pack.shape[0], b_class_pack.shape[0]
    return flat.reshape(int(a_classes.numel()), m, packed.shape[0], n).permute(0, 2, 1, 3), packed, b_lanes


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


_SEED_COUNTER = [0x5EED]


class ClassCountOperand:
    """An e4m3 matrix [rows, K] staged for the class-count engine: per row and group of 32 k,
    the slot of each element's class among the row's classes in the group, the classes'
    codes, exponent pairs and present/sign masks (ima_class_count_prepare).  A weight
    (weight=True) is also expanded into its tile records (ima_class_count_weight_tiles): the
    one-hot weight slot rows, class magnitudes and the fingerprint weights, drawn from `seed`
    (a fresh one per staging when None)."""

    def __init__(self, fp8: torch.Tensor, *, weight: bool = False, seed: int | None = None):
        if fp8.device.type != "cuda":
            raise RuntimeError("Hawkeye class-count replay is CUDA-only")
        raw = fp8.contiguous().view(torch.uint8)
        self.rows, self.k = int(raw.shape[0]), int(raw.shape[1])
        self.device = raw.device
        nbytes = int(nat.lib().ima_class_count_operand_bytes(self.rows, self.k))
        self.buffer = torch.empty((max(nbytes, 16),), dtype=torch.uint8, device=raw.device)
        with torch.cuda.device(raw.device):
            nat.call("ima_class_count_prepare", raw.data_ptr(), self.rows, self.k, self.k, self.buffer.data_ptr(),
                     nat.stream_of(raw.device))
        self.tiles = None
        if weight:
            if seed is None:
                _SEED_COUNTER[0] += 1
                seed = _SEED_COUNTER[0] * 0x9E3779B97F4A7C15 % (1 << 64)
            tbytes = int(nat.lib().ima_class_count_weight_tiles_bytes(self.rows, self.k))
            self.tiles = torch.empty((max(tbytes, 16),), dtype=torch.uint8, device=raw.device)
            with torch.cuda.device(raw.device):
                nat.call("ima_class_count_weight_tiles", self.buffer.data_ptr(), self.rows, self.k,
                         int(seed) % (1 << 64), self.tiles.data_ptr(), nat.stream_of(raw.device))
        self._source = fp8
        self._version = nat.tensor_version(fp8)
        self._data_ptr = fp8.data_ptr()

    def matches(self, fp8: torch.Tensor) -> bool:
        """True while `fp8` is the staged tensor and unchanged since staging (never for
        inference tensors, whose in-place edits leave no trace)."""
        return (fp8 is self._source and self._version is not None and nat.tensor_version(fp8) == self._version
                and fp8.data_ptr() == self._data_ptr)

    def tables(self) -> dict[str, torch.Tensor]:
        """The staged tables as tensors (views of the buffer): slots [G, P, 32] uint8, codes
        [G, P, 32] uint8 (rows padded to the pitch P)."""
        pitch = -(-max(self.rows, 1) // 64) * 64
        groups = -(-self.k // 32)
        recs = pitch * groups
        return {"slots": self.buffer[: recs * 32].view(groups, pitch, 32),
                "codes": self.buffer[recs * 32: recs * 64].view(groups, pitch, 32)}


def stage_class_count_weight(w_fp8: torch.Tensor) -> ClassCountOperand:
    """Stage a weight for the class-count engine once and cache the staging on the tensor."""
    cached = getattr(w_fp8, "_ima_class_count_operand", None)
    if cached is not None and cached.matches(w_fp8):
        return cached
    op = ClassCountOperand(w_fp8, weight=True)
    try:
        w_fp8._ima_class_count_operand = op
    except (AttributeError, RuntimeError):
        pass
    return op


def class_count_replay(
    x_op: ClassCountOperand,
    w_op: ClassCountOperand,
    x_scale: torch.Tensor,
    w_scale: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    out_f32: torch.Tensor | None = None,
    mismatch: torch.Tensor | None = None,
    tiles_out: torch.Tensor | None = None,
    tiles_in: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """The engine on staged operands: returns (bf16 [M, N] or the given outputs, the device
    int32 count of slot rows whose count tile failed the fingerprint).  No host sync.
    tiles_out / tiles_in: int32 [ima_class_count_tile_entries(M, N, K)] count tiles as the
    tensor cores formed them / counts to replay instead (layout in include/ima_b200.h)."""
    m, n, k = x_op.rows, w_op.rows, x_op.k
    if w_op.k != k:
        raise RuntimeError(f"Hawkeye shape mismatch: K={k} vs K={w_op.k}")
    if w_op.tiles is None:
        raise RuntimeError("the weight operand was staged without its tile records (ClassCountOperand(w, weight=True))")
    dev = x_op.device
    xs = x_scale.reshape(-1).to(torch.float32).contiguous()
    ws = w_scale.reshape(-1).to(torch.float32).contiguous()
    if xs.numel() != m or ws.numel() != n:
        raise RuntimeError(f"Hawkeye scales have {xs.numel()} and {ws.numel()} entries, expected {m} and {n}")
    if out is None and out_f32 is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    if mismatch is None:
        mismatch = torch.zeros((1,), dtype=torch.int32, device=dev)
    entries = int(nat.lib().ima_class_count_tile_entries(m, n, k))
    for label, t in (("tiles_out", tiles_out), ("tiles_in", tiles_in)):
        if t is not None and (t.dtype != torch.int32 or t.numel() < entries or not t.is_contiguous()):
            raise RuntimeError(f"{label} must be a contiguous int32 tensor of at least {entries} entries")
    nat.require_device(dev, ("weight operand", w_op.buffer), ("weight tiles", w_op.tiles), ("x_scale", xs),
                       ("w_scale", ws), ("output", out),
                       ("fp32 output", out_f32), ("mismatch counter", mismatch), ("tiles_out", tiles_out),
                       ("tiles_in", tiles_in))
    with torch.cuda.device(dev):
        nat.call(
            "ima_class_count_replay", x_op.buffer.data_ptr(), w_op.buffer.data_ptr(), w_op.tiles.data_ptr(),
            xs.data_ptr(), ws.data_ptr(), m, n, k, nat.ptr(out), out.stride(0) if out is not None else n,
            nat.ptr(out_f32),
            out_f32.stride(0) if out_f32 is not None else n, mismatch.data_ptr(), nat.ptr(tiles_out),
            nat.ptr(tiles_in), nat.stream_of(dev),
        )
    return (out if out is not None else out_f32), mismatch


def count_tile_entries(m: int, n: int, k: int) -> int:
    """int32 entries of the engine's count-tile layout for an [m, k] x [n, k] product."""
    return int(nat.lib().ima_class_count_tile_entries(m, n, k))


class _CheckedMatmul:
    """Wraps an injected raw_matmul: every product it returns is Freivalds-checked on the GPU
    against its operands before use, and calls are counted."""

    def __init__(self, inner: RawIntMatmul):
        self.inner = inner
        self.calls = 0

    def __call__(self, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        from .freivalds import freivalds_vector, mismatch_rows_int32

        c = self.inner(a, b)
        self.calls += 1
        m, n = int(a.shape[0]), int(b.shape[1])
        if not isinstance(c, torch.Tensor) or tuple(c.shape) != (m, n) or c.dtype not in (torch.int32, torch.int64):
            raise RuntimeError(
                f"raw_matmul returned {getattr(c, 'dtype', type(c))} {tuple(getattr(c, 'shape', ()))} "
                f"for a ({m}, {int(a.shape[1])}) x ({int(b.shape[0])}, {n}) integer count product"
            )
        dev = c.device
        r = freivalds_vector(n, 0x5EED + self.calls, device=dev)
        bad = mismatch_rows_int32(a.to(device=dev, dtype=torch.int32), b.to(device=dev, dtype=torch.int32),
                                  c.to(torch.int64), r)
        if int(bad.item()) != 0:
            raise RuntimeError(
                f"raw_matmul returned a class-count product ({m} x {n}) that fails the Freivalds check "
                f"on {int(bad.item())} rows"
            )
        return c


def _materialise_count_products(
    x_fp8: torch.Tensor,
    w_fp8: torch.Tensor,
    raw_matmul: RawIntMatmul,
    *,
    products_per_group: int,
    class_chunk: int,
    packed_count_lanes: int,
    packed_group_lanes: int,
    fused_replay: bool,
    cache_weight_chunks: bool,
    count_dtype: torch.dtype,
) -> int:
    """Form every checkable count product the way the reference does (same operands, same
    order: hawkeye_freivalds.py:900-932 for packed groups, :1086-1207 otherwise), each
    through a Freivalds-checked call of raw_matmul.  Returns the number of calls."""
    checked = _CheckedMatmul(raw_matmul)
    a_class = _class_ids(*_decode_fp8_fields(x_fp8))
    b_class = _class_ids(*_decode_fp8_fields(w_fp8))
    k_size = a_class.shape[1]
    if packed_group_lanes > 1:
        width = products_per_group * packed_group_lanes
        b_lanes = packed_count_lanes // packed_group_lanes
        for k0 in range(0, k_size, width):
            a_pack, b_pack = a_class[:, k0:k0 + width], b_class[:, k0:k0 + width]
            a_classes = torch.unique(a_pack[a_pack >= 0])
            b_classes = torch.unique(b_pack[b_pack >= 0])
            for a_chunk in _iter_class_chunks(a_classes, class_chunk):
                for b_chunk in _iter_class_chunks(b_classes, class_chunk * b_lanes):
                    _packed_group_class_chunk_product(
                        a_pack, b_pack, a_chunk, b_chunk, checked, products_per_group=products_per_group,
                        packed_group_lanes=packed_group_lanes, packed_count_lanes=packed_count_lanes,
                    )
        return checked.calls
    for k0 in range(0, k_size, products_per_group):
        a_group, b_group = a_class[:, k0:k0 + products_per_group], b_class[:, k0:k0 + products_per_group]
        a_classes = torch.unique(a_group[a_group >= 0])
        b_classes = torch.unique(b_group[b_group >= 0])
        b_chunk_size = class_chunk if packed_count_lanes == 1 else class_chunk * packed_count_lanes
        b_chunks = _iter_class_chunks(b_classes, b_chunk_size)
        cached = None
        if cache_weight_chunks and packed_count_lanes == 1 and not fused_replay:
            cached = [(int(c.numel()), _weight_chunk_flat(b_group, c, count_dtype=count_dtype)) for c in b_chunks]
        for a_chunk in _iter_class_chunks(a_classes, class_chunk):
            if cached is not None:
                for b_size, b_flat in cached:
                    _class_chunk_product_raw_with_b_flat(a_group, a_chunk, b_flat, b_size, checked)
                continue
            for b_chunk in b_chunks:
                if packed_count_lanes == 1:
                    if not fused_replay:   # the fused reference kernel forms these counts itself
                        _class_chunk_product(a_group, b_group, a_chunk, b_chunk, checked, count_dtype=count_dtype)
                else:
                    _packed_class_chunk_product(a_group, b_group, a_chunk, b_chunk, checked, packed_count_lanes)
    return checked.calls


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

    ref: hawkeye_freivalds.py:1017-1246.  The class-count engine forms the count products
    on the tensor cores, fingerprints every count tile and replays the accumulator from the
    counts (RuntimeError if a tile fails its check).  With raw_matmul None the active int32
    probe is bumped once per product the reference would have sent through
    _int32_raw_matmul; a callable receives the reference's products, one call each (each
    result Freivalds-checked, RuntimeError if one fails).
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
    reference_calls = 0 if (fused_replay and packed_count_lanes == 1) else stats.total_checkable_products
    if raw_matmul is None:
        # the engine forms these products; the probe counts them as the reference's
        # _int32_raw_matmul launches would have been counted
        _bump_probe(reference_calls)
    else:
        made = _materialise_count_products(
            x_fp8, w_fp8, raw_matmul, products_per_group=products_per_group, class_chunk=class_chunk,
            packed_count_lanes=packed_count_lanes, packed_group_lanes=packed_group_lanes,
            fused_replay=fused_replay, cache_weight_chunks=cache_weight_chunks, count_dtype=count_dtype,
        )
        if made != reference_calls:
            raise RuntimeError(f"internal: {made} count products formed, {reference_calls} expected")

    x_op = ClassCountOperand(x_fp8)
    w_op = stage_class_count_weight(w_fp8)
    out, bad = class_count_replay(x_op, w_op, xs.contiguous(), w_scale)
    failed = int(bad.item())   # one host read per call, like the reference's class-list syncs
    if failed:
        raise RuntimeError(f"class-count products failed the Freivalds fingerprint on {failed} rows")
    return out, stats

"""The class-count engine (csrc/class_count_engine.cu) on the GPU.

1. Its bf16 output equals the direct Hawkeye replay and the CPU oracle bit for bit, on
   ragged shapes, odd group counts, raw byte patterns (NaN codes, subnormals, zeros) and
   the config-3 shape.
2. The count tiles it forms on the tensor cores ARE the reference's count products: decoded
   through the staged class tables, every tile entry equals the reference-layout count
   product (hawkeye_freivalds._class_chunk_product, unpacked) and, repacked in base-64 lanes,
   the reference's packed-group product with config 3's lane settings.
3. Its Freivalds fingerprint rejects a count tile with a wrong count: the tiles are dumped,
   one count is changed on the host side (a tensor edit, not a kernel change), and the
   engine replays the supplied tiles; the fingerprint flags the edited row.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from int_model_approximation_b200 import codebook, hawkeye, hawkeye_freivalds, students, synthetic

pytestmark = pytest.mark.gpu


def _case(m, k, n, seed, outliers=0.01):
    x = synthetic.student_t_activations(m, k, seed=seed, outlier_fraction=outliers)
    xq, xs = oracle.per_token_fp8(x)
    w, ws = synthetic.normal_fp8_weights(n, k, seed=seed + 1)
    return xq, xs, w, ws


def _engine(xq, xs, w, ws, device, **kw):
    x_op = hawkeye_freivalds.ClassCountOperand(xq.to(device))
    w_op = hawkeye_freivalds.ClassCountOperand(w.to(device), weight=True)
    out, bad = hawkeye_freivalds.class_count_replay(x_op, w_op, xs.to(device), ws.to(device), **kw)
    torch.cuda.synchronize()
    return out, int(bad.item()), x_op, w_op


@pytest.mark.parametrize("m,k,n", [(1, 32, 1), (5, 31, 7), (13, 100, 70), (130, 257, 300), (16, 896, 4864),
                                   (9, 1, 65), (64, 96, 200)])
def test_engine_equals_direct_replay_and_oracle(cuda_device, m, k, n):
    xq, xs, w, ws = _case(m, k, n, seed=m * 7 + k + n)
    out, bad, _, _ = _engine(xq, xs, w, ws, cuda_device)
    assert bad == 0
    direct, _ = hawkeye.hawkeye_fp8_sum(xq.to(cuda_device), xs.to(cuda_device), w.to(cuda_device),
                                        ws.to(cuda_device))
    assert torch.equal(out.view(torch.int16), direct.view(torch.int16))
    ref = oracle.hawkeye(xq, xs, w, ws).to(torch.bfloat16)
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


def test_engine_raw_byte_patterns_against_oracle(cuda_device):
    g = torch.Generator().manual_seed(19)
    x = torch.randint(0, 256, (37, 224), generator=g, dtype=torch.int64).to(torch.uint8).view(torch.float8_e4m3fn)
    w = torch.randint(0, 256, (90, 224), generator=g, dtype=torch.int64).to(torch.uint8).view(torch.float8_e4m3fn)
    xs = torch.rand(37, 1, generator=g) + 0.25
    ws = torch.rand(90, generator=g) + 0.25
    out, bad, _, _ = _engine(x, xs, w, ws, cuda_device)
    assert bad == 0
    ref = oracle.hawkeye(x, xs, w, ws).to(torch.bfloat16)
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


def _engine_counts(tiles: np.ndarray, x_op, w_op, m: int, n: int, k: int) -> dict[int, dict]:
    """Decode dumped tiles into {group: {(m, n, class_a, class_b): signed count}} through the
    staged class tables (slot -> e4m3 code -> class id); entries of unused slots must be 0."""
    g_count = -(-k // 32)
    gp_count = -(-g_count // 2)
    sm_n, sn_n = -(-m // 4), -(-n // 64)
    t = tiles[: sm_n * sn_n * gp_count * 8 * 2 * 128 * 256].reshape(sn_n, sm_n, gp_count, 8, 2, 4, 32, 8, 32)
    codes_a = x_op.tables()["codes"].cpu()
    codes_b = w_op.tables()["codes"].cpu()
    cls_a = oracle.class_ids(codes_a.view(torch.float8_e4m3fn)).numpy()   # [G, P, 32]; 0 code -> -1
    cls_b = oracle.class_ids(codes_b.view(torch.float8_e4m3fn)).numpy()
    out: dict[int, dict] = {g: {} for g in range(g_count)}
    nz = np.argwhere(t != 0)
    for sn, sm, gp, tt, h, ml, sa, nl, sb in nz:
        g, mm, nn = 2 * gp + h, 4 * sm + ml, 64 * sn + 8 * tt + nl
        assert g < g_count and mm < m and nn < n, "count outside the product"
        a, b = int(cls_a[g, mm, sa]), int(cls_b[g, nn, sb])
        assert a >= 0 and b >= 0, "count in an unused slot"
        out[g][(int(mm), int(nn), a, b)] = int(t[sn, sm, gp, tt, h, ml, sa, nl, sb])
    return out


def _cpu_matmul(a, b):
    return a.to(torch.int64) @ b.to(torch.int64)


def test_engine_count_tiles_are_the_reference_count_products(cuda_device):
    m, k, n = 10, 100, 70          # 4 groups, 3 x 2 strips, a partial last tile
    xq, xs, w, ws = _case(m, k, n, seed=77, outliers=0.05)
    entries = hawkeye_freivalds.count_tile_entries(m, n, k)
    tiles = torch.zeros((entries,), dtype=torch.int32, device=cuda_device)
    out, bad, x_op, w_op = _engine(xq, xs, w, ws, cuda_device, tiles_out=tiles)
    assert bad == 0
    eng = _engine_counts(tiles.cpu().numpy(), x_op, w_op, m, n, k)
    a_class = oracle.class_ids(xq)
    b_class = oracle.class_ids(w)
    sign_b = {int(c): (-1 if ((int(c) % 31) - 15) < 0 else 1) for c in torch.unique(b_class[b_class >= 0])}
    for g in range(-(-k // 32)):
        ag, bg = a_class[:, 32 * g:32 * g + 32], b_class[:, 32 * g:32 * g + 32]
        a_classes = torch.unique(ag[ag >= 0])
        b_classes = torch.unique(bg[bg >= 0])
        ref = hawkeye_freivalds._class_chunk_product(ag, bg, a_classes, b_classes, _cpu_matmul)   # [a, b, m, n]
        dense = torch.zeros_like(ref)
        a_index = {int(c): i for i, c in enumerate(a_classes)}
        b_index = {int(c): i for i, c in enumerate(b_classes)}
        for (mm, nn, a, b), v in eng[g].items():
            assert v * sign_b[b] > 0
            dense[a_index[a], b_index[b], mm, nn] = abs(v)
        assert torch.equal(dense, ref), f"group {g}"
    # the reference's packed product with config 3's lanes (6 count lanes, 2 group lanes per pack)
    for p in range(-(-k // 64)):
        ap, bp = a_class[:, 64 * p:64 * p + 64], b_class[:, 64 * p:64 * p + 64]
        a_classes = torch.unique(ap[ap >= 0])
        b_classes = torch.unique(bp[bp >= 0])
        packed_ref, packed_b, lanes = hawkeye_freivalds._packed_group_class_chunk_product(
            ap, bp, a_classes, b_classes, _cpu_matmul, products_per_group=32, packed_group_lanes=2,
            packed_count_lanes=6)
        rebuilt = torch.zeros_like(packed_ref)
        a_index = {int(c): i for i, c in enumerate(a_classes)}
        slot_of = {int(c): (pg, j) for pg in range(packed_b.shape[0]) for j in range(packed_b.shape[1])
                   for c in [int(packed_b[pg, j])] if c >= 0}
        for gl in range(2):
            g = 2 * p + gl
            if g not in eng:
                continue
            for (mm, nn, a, b), v in eng[g].items():
                pg, j = slot_of[b]
                rebuilt[a_index[a], pg, mm, nn] += abs(v) << (6 * (gl * lanes + j))
        assert torch.equal(rebuilt, packed_ref), f"pack {p}"


def test_engine_fingerprint_rejects_a_wrong_count(cuda_device):
    m, k, n = 12, 96, 40
    xq, xs, w, ws = _case(m, k, n, seed=5)
    entries = hawkeye_freivalds.count_tile_entries(m, n, k)
    tiles = torch.zeros((entries,), dtype=torch.int32, device=cuda_device)
    out, bad, x_op, w_op = _engine(xq, xs, w, ws, cuda_device, tiles_out=tiles)
    assert bad == 0
    # replaying the tiles as formed gives the same output and passes the check
    again, bad2 = hawkeye_freivalds.class_count_replay(x_op, w_op, xs.to(cuda_device), ws.to(cuda_device),
                                                       tiles_in=tiles)
    torch.cuda.synchronize()
    assert int(bad2.item()) == 0 and torch.equal(again.view(torch.int16), out.view(torch.int16))
    # one count changed on the host side: a live entry, then an entry of an unused slot row
    live = torch.nonzero(tiles).reshape(-1)
    for idx in (int(live[len(live) // 3]), int(live[-1]) - 1):
        bad_tiles = tiles.clone()
        bad_tiles[idx] += 1
        _, bad3 = hawkeye_freivalds.class_count_replay(x_op, w_op, xs.to(cuda_device), ws.to(cuda_device),
                                                       tiles_in=bad_tiles)
        torch.cuda.synchronize()
        assert int(bad3.item()) == 1, idx


def test_c3_class_counts_through_the_engine(cuda_device):
    """Config 3: down_proj M=4096, K=4864, N=896, class_chunk 512, 6 count lanes, 2 group
    lanes: the engine's output equals the direct replay and sampled oracle rows; stats equal
    the reference's control flow; the probe counts the 76 products the engine formed."""
    x, w, ws = synthetic.make_linear_inputs(3, 0, synthetic.LinearShape("down_proj", 896, 4864), device=cuda_device)
    xq, xs, *_ = codebook.per_token_fp8(x)
    with students._Int32KernelProbe() as probe:
        y, stats = hawkeye_freivalds.exact_hawkeye_fp8_sum(xq, xs, w, ws, None, class_chunk=512,
                                                           packed_count_lanes=6, packed_group_lanes=2)
    direct, _ = hawkeye.hawkeye_fp8_sum(xq, xs, w, ws)
    assert torch.equal(y.view(torch.int16), direct.view(torch.int16))
    rows = np.arange(0, 4096, 331)
    ref = oracle.hawkeye(xq.cpu(), xs.cpu(), w.cpu(), ws.cpu(), rows=rows).to(torch.bfloat16)
    assert torch.equal(y[torch.from_numpy(rows).to(cuda_device)].cpu().view(torch.int16), ref.view(torch.int16))
    assert stats.__dict__ == oracle.class_count_stats(xq.cpu(), w.cpu(), class_chunk=512, packed_count_lanes=6,
                                                       packed_group_lanes=2)
    assert stats.groups == 152 and probe.count == stats.total_checkable_products == 76


def test_class_counts_linear_runs_the_engine(cuda_device, monkeypatch):
    """HawkeyeClassCountsLinear forms its products with the engine: _int32_raw_matmul is not
    called, the probe still counts the reference's products, the output is the direct replay."""
    w, ws = synthetic.normal_fp8_weights(48, 160, seed=4)
    layer = students.HawkeyeClassCountsLinear(w.to(cuda_device), ws.to(cuda_device), None)
    x = synthetic.student_t_activations(6, 160, seed=8).to(cuda_device)

    def fail(*_a, **_k):
        raise AssertionError("the engine forms the count products itself")

    monkeypatch.setattr(students, "_int32_raw_matmul", fail)
    with students._Int32KernelProbe() as probe:
        y = layer(x)
    xq, xsc = students._per_token_fp8(x)
    direct, _ = hawkeye.hawkeye_fp8_sum(xq, xsc, layer.weight, layer.weight_scale)
    assert torch.equal(y.view(torch.int16), direct.to(y.dtype).view(torch.int16))
    stats = oracle.class_count_stats(xq.cpu(), w, class_chunk=students.HAWKEYE_CLASS_CHUNK,
                                     packed_count_lanes=students.HAWKEYE_PACKED_COUNT_LANES,
                                     packed_group_lanes=students.HAWKEYE_PACKED_GROUP_LANES)
    assert probe.count == stats["total_checkable_products"] > 0

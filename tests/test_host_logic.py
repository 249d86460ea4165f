"""Host-side behaviour of the plugin surface that needs no GPU: the reference's own
CPU tests (tests/test_real_integer_gemms.py, test_hawkeye.py, test_single_entrypoint.py)
restated against int_model_approximation_b200, plus the class-count bookkeeping."""

from __future__ import annotations

import pytest
import torch
import torch.nn as nn

import oracle
from int_model_approximation_b200 import hawkeye, hawkeye_freivalds, students


class TinyLinearModel(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.in_proj = nn.Linear(3, 5, bias=False)
        self.block = nn.Sequential(nn.GELU(), nn.Linear(5, 2, bias=True))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.block(self.in_proj(x))


def _disable_cuda_requirement(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(students, "_require_cuda_tensor", lambda _x, _label: None)


def _patch_non_int_gemm_fallbacks(monkeypatch: pytest.MonkeyPatch) -> None:
    def fail(*_args: object, **_kwargs: object) -> None:
        raise AssertionError("integerized model used a non-int GEMM fallback")

    for attr in ("mm", "matmul", "addmm", "bmm"):
        monkeypatch.setattr(torch, attr, fail)
    monkeypatch.setattr(torch.nn.functional, "linear", fail)
    if hasattr(torch, "_scaled_mm"):
        monkeypatch.setattr(torch, "_scaled_mm", fail)


def test_hawkeye_rejects_cpu_operands():
    x = torch.zeros((1, 32), dtype=torch.float8_e4m3fn)
    w = torch.zeros((1, 32), dtype=torch.float8_e4m3fn)
    with pytest.raises(RuntimeError, match="CUDA-only"):
        hawkeye.hawkeye_fp8_sum(x, torch.ones((1, 1)), w, torch.ones(1))


def test_exact_hawkeye_rejects_bad_parameters_before_any_launch():
    x = torch.zeros((1, 32), dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="count_dtype"):
        hawkeye_freivalds.exact_hawkeye_fp8_sum(x, torch.ones(1, 1), x, torch.ones(1), None, count_dtype=torch.int64)
    with pytest.raises(ValueError, match="packed_count_lanes"):
        hawkeye_freivalds.exact_hawkeye_fp8_sum(x, torch.ones(1, 1), x, torch.ones(1), None, packed_count_lanes=7)
    with pytest.raises(ValueError, match="packed_group_lanes"):
        hawkeye_freivalds.exact_hawkeye_fp8_sum(
            x, torch.ones(1, 1), x, torch.ones(1), None, packed_count_lanes=2, packed_group_lanes=3
        )
    with pytest.raises(ValueError, match="cross-lane carries"):
        hawkeye_freivalds.exact_hawkeye_fp8_sum(
            x, torch.ones(1, 1), x, torch.ones(1), None, products_per_group=65, packed_count_lanes=6,
            packed_group_lanes=2,
        )
    with pytest.raises(RuntimeError, match="CUDA-only"):
        hawkeye_freivalds.exact_hawkeye_fp8_sum(x, torch.ones(1, 1), x, torch.ones(1), None)


def test_int32_linear_rejects_cpu_weights():
    with pytest.raises(RuntimeError, match="CUDA"):
        students.Int32Linear(torch.randn(4, 4), None)


def test_int32_matmul_rejects_non_int_operands_before_launch(monkeypatch):
    _disable_cuda_requirement(monkeypatch)
    x_scale = torch.ones(2, 1)
    w_scale = torch.ones(1, 4)
    cases = [
        (torch.ones(2, 3, dtype=torch.float32), torch.ones(3, 4, dtype=torch.int32)),
        (torch.ones(2, 3, dtype=torch.int32), torch.ones(3, 4, dtype=torch.float32)),
    ]
    for activations, weight_t in cases:
        with pytest.raises(RuntimeError, match="non-int32 operands"):
            students._int32_matmul(activations, weight_t, x_scale, w_scale)
        with pytest.raises(RuntimeError, match="non-int32 operands"):
            students._int32_raw_matmul(activations, weight_t)
    with pytest.raises(RuntimeError, match="shape mismatch"):
        students._int32_matmul(torch.ones(2, 3, dtype=torch.int32), torch.ones(4, 4, dtype=torch.int32),
                               x_scale, w_scale)


def test_int32_linear_keeps_only_int32_weight_matrix(monkeypatch):
    _disable_cuda_requirement(monkeypatch)
    layer = students.Int32Linear(torch.randn(4, 3), bias=None)
    assert layer.weight_t.dtype == torch.int32
    assert not layer.weight_t.is_floating_point()
    assert layer.weight_t.shape == (3, 4)
    assert layer.weight_scale.dtype == torch.float32


def test_integerized_replacement_removes_all_linear_modules(monkeypatch):
    _disable_cuda_requirement(monkeypatch)
    model = TinyLinearModel()
    replaced = students._replace_int32_linears(model)
    assert replaced == ["in_proj", "block.1"]
    assert all(not isinstance(module, nn.Linear) for module in model.modules())
    assert isinstance(model.in_proj, students.Int32Linear)
    assert isinstance(model.block[1], students.Int32Linear)


def test_int32_linear_forward_uses_the_int32_matmul_path(monkeypatch):
    _disable_cuda_requirement(monkeypatch)
    layer = students.Int32Linear(torch.randn(4, 3), bias=torch.randn(4))
    calls = []

    def fake_int32_matmul(activations, weight_t, x_scale, w_scale):
        calls.append((activations, weight_t, x_scale, w_scale))
        assert activations.dtype == torch.int32
        assert weight_t.dtype == torch.int32
        return torch.zeros((activations.shape[0], weight_t.shape[1]), dtype=torch.float32)

    monkeypatch.setattr(students, "_int32_matmul", fake_int32_matmul)
    _patch_non_int_gemm_fallbacks(monkeypatch)
    y = layer(torch.randn(2, 3))
    assert len(calls) == 1
    assert y.shape == (2, 4)


def test_unknown_student_kernel_is_rejected(monkeypatch):
    monkeypatch.setattr(students, "STUDENT_KERNEL", "nope")
    with pytest.raises(RuntimeError, match="unknown IMA_STUDENT_KERNEL"):
        students._replace_int32_linears(TinyLinearModel())


def test_probe_context_manager():
    assert students._ACTIVE_INT32_PROBE is None
    with students._Int32KernelProbe() as probe:
        assert students._ACTIVE_INT32_PROBE is probe
        hawkeye_freivalds._bump_probe(3)
    assert probe.count == 3
    assert students._ACTIVE_INT32_PROBE is None


@pytest.mark.parametrize(
    "params",
    [
        dict(class_chunk=32, packed_count_lanes=6, packed_group_lanes=1),
        dict(class_chunk=512, packed_count_lanes=6, packed_group_lanes=2),
        dict(class_chunk=8, packed_count_lanes=3, packed_group_lanes=1),
        dict(class_chunk=16, packed_count_lanes=6, packed_group_lanes=3),
        dict(class_chunk=4, packed_count_lanes=1, packed_group_lanes=1),
        dict(class_chunk=7, packed_count_lanes=4, packed_group_lanes=4),
    ],
)
def test_class_count_stats_bookkeeping_matches_reference_loops(params):
    """class_count_stats (what the B200 path computes from presence masks) against the
    oracle's restatement of the reference's per-pack torch.unique loops."""
    g = torch.Generator().manual_seed(params["class_chunk"])
    x = torch.randn((20, 100), generator=g).to(torch.float8_e4m3fn)
    w = torch.randn((13, 100), generator=g).to(torch.float8_e4m3fn)
    x.view(torch.uint8)[:, 40:50] = 0
    expected = oracle.class_count_stats(x, w, **params)
    width = 32 * (params["packed_group_lanes"] if params["packed_group_lanes"] > 1 else 1)
    a_cls, b_cls = oracle.class_ids(x), oracle.class_ids(w)
    na, nb = [], []
    for k0 in range(0, 100, width):
        a = a_cls[:, k0:k0 + width]
        b = b_cls[:, k0:k0 + width]
        na.append(int(torch.unique(a[a >= 0]).numel()))
        nb.append(int(torch.unique(b[b >= 0]).numel()))
    got = hawkeye_freivalds.class_count_stats(na, nb, 100, products_per_group=32, **params)
    assert got.__dict__ == expected


# ---------------------------------------------------------------------------
# Count-product helpers (reference layouts), on CPU with an int64 matmul
# ---------------------------------------------------------------------------
def _cpu_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return a.to(torch.int64) @ b.to(torch.int64)


def _brute_counts(a_cls, b_cls, a_classes, b_classes):
    m, k = a_cls.shape
    n = b_cls.shape[0]
    out = torch.zeros((len(a_classes), len(b_classes), m, n), dtype=torch.int64)
    for ai, a in enumerate(a_classes.tolist()):
        for bi, b in enumerate(b_classes.tolist()):
            out[ai, bi] = ((a_cls == a).to(torch.int64) @ (b_cls == b).to(torch.int64).t())
    return out


def test_class_ids_of_every_e4m3_byte_match_the_oracle():
    codes = torch.arange(256, dtype=torch.int64).to(torch.uint8).view(torch.float8_e4m3fn).reshape(16, 16)
    ids = hawkeye_freivalds._class_ids(*hawkeye_freivalds._decode_fp8_fields(codes))
    assert torch.equal(ids, oracle.class_ids(codes))
    assert int(ids.max()) < 15 * 31 and int((ids == -1).sum()) == 2   # +0 and -0


def test_unpacked_class_count_product_counts_every_class_pair():
    g = torch.Generator().manual_seed(5)
    a_cls = torch.randint(-1, 6, (7, 32), generator=g)
    b_cls = torch.randint(-1, 9, (5, 32), generator=g)
    a_classes, b_classes = torch.tensor([0, 2, 3, 5]), torch.tensor([1, 4, 6, 7, 8])
    counts = hawkeye_freivalds._class_chunk_product(a_cls, b_cls, a_classes, b_classes, _cpu_matmul)
    assert torch.equal(counts.to(torch.int64), _brute_counts(a_cls, b_cls, a_classes, b_classes))


@pytest.mark.parametrize("lanes", [2, 3, 6])
def test_lane_packed_counts_decode_to_the_unpacked_counts(lanes):
    g = torch.Generator().manual_seed(lanes)
    a_cls = torch.randint(-1, 5, (6, 32), generator=g)
    b_cls = torch.randint(-1, 11, (4, 32), generator=g)
    a_classes, b_classes = torch.arange(5), torch.arange(11)
    packed, packed_b = hawkeye_freivalds._packed_class_chunk_product(a_cls, b_cls, a_classes, b_classes,
                                                                       _cpu_matmul, lanes)
    assert packed_b.shape == ((11 + lanes - 1) // lanes, lanes)
    want = _brute_counts(a_cls, b_cls, a_classes, b_classes)
    for bi in range(11):
        grp, lane = divmod(bi, lanes)
        assert int(packed_b[grp, lane]) == bi
        got = (packed[:, grp] >> (hawkeye_freivalds.PACKED_COUNT_BASE_LOG2 * lane)) & (hawkeye_freivalds.PACKED_COUNT_BASE - 1)
        assert torch.equal(got, want[:, bi])
    assert int((packed_b == -2).sum()) == packed_b.numel() - 11


def test_group_packed_counts_decode_to_each_group():
    g = torch.Generator().manual_seed(11)
    ppg, group_lanes, lanes = 8, 2, 6
    a_cls = torch.randint(-1, 4, (3, 2 * ppg), generator=g)
    b_cls = torch.randint(-1, 5, (4, 2 * ppg), generator=g)
    a_classes, b_classes = torch.arange(4), torch.arange(5)
    packed, packed_b, b_lanes = hawkeye_freivalds._packed_group_class_chunk_product(
        a_cls, b_cls, a_classes, b_classes, _cpu_matmul,
        products_per_group=ppg, packed_group_lanes=group_lanes, packed_count_lanes=lanes,
    )
    assert b_lanes == lanes // group_lanes
    for grp_lane in range(group_lanes):
        sl = slice(grp_lane * ppg, (grp_lane + 1) * ppg)
        want = _brute_counts(a_cls[:, sl], b_cls[:, sl], a_classes, b_classes)
        for bi in range(5):
            pg, slot = divmod(bi, b_lanes)
            lane = grp_lane * b_lanes + slot
            got = (packed[:, pg] >> (hawkeye_freivalds.PACKED_COUNT_BASE_LOG2 * lane)) & 63
            assert torch.equal(got, want[:, bi])
    with pytest.raises(RuntimeError, match="more groups than packed_group_lanes"):
        hawkeye_freivalds._packed_group_class_chunk_product(
            torch.zeros((1, 3 * ppg), dtype=torch.int64), torch.zeros((1, 3 * ppg), dtype=torch.int64),
            a_classes, b_classes, _cpu_matmul, products_per_group=ppg, packed_group_lanes=2, packed_count_lanes=6)
    with pytest.raises(ValueError, match="must fit inside packed_count_lanes"):
        hawkeye_freivalds._packed_group_class_chunk_product(
            a_cls, b_cls, a_classes, b_classes, _cpu_matmul, products_per_group=ppg, packed_group_lanes=7,
            packed_count_lanes=6)


def test_cached_weight_chunk_product_equals_the_plain_product():
    g = torch.Generator().manual_seed(3)
    a_cls = torch.randint(-1, 6, (5, 32), generator=g)
    b_cls = torch.randint(-1, 6, (3, 32), generator=g)
    a_classes, b_classes = torch.arange(6), torch.tensor([0, 1, 5])
    b_flat = hawkeye_freivalds._weight_chunk_flat(b_cls, b_classes)
    flat, a_size, b_size = hawkeye_freivalds._class_chunk_product_raw_with_b_flat(a_cls, a_classes, b_flat, 3,
                                                                                  _cpu_matmul)
    plain, _, _ = hawkeye_freivalds._class_chunk_product_raw(a_cls, b_cls, a_classes, b_classes, _cpu_matmul)
    assert (a_size, b_size) == (6, 3) and torch.equal(flat, plain)


def test_codebook_stack_batches_balance_cost_within_the_launch_limit():
    """Problems are dealt to ceil(n / GEMM_BATCH) launches, each at most GEMM_BATCH problems,
    every problem exactly once, launch costs within one largest problem of each other."""
    from types import SimpleNamespace

    from int_model_approximation_b200.pipeline import CodebookStack

    stack = CodebookStack.__new__(CodebookStack)
    shapes = [(896, 896), (128, 896), (128, 896), (896, 896), (4864, 896), (4864, 896), (896, 4864)] * 24
    stack.linears = [SimpleNamespace(n=n, k=k) for n, k in shapes]
    batches = stack._batches()
    assert len(batches) == -(-len(shapes) // CodebookStack.GEMM_BATCH)
    assert sorted(i for b in batches for i in b) == list(range(len(shapes)))
    assert all(len(b) <= CodebookStack.GEMM_BATCH for b in batches)
    costs = [sum(shapes[i][0] * shapes[i][1] for i in b) for b in batches]
    assert max(costs) - min(costs) <= max(n * k for n, k in shapes)


@pytest.mark.parametrize("k", [1, 300, 896, 4864, 18944])
def test_int32_linear_oracle_uses_the_plugin_qmax_and_tracks_the_float_product(k):
    """The CPU restatement of Int32Linear quantises with the same qmax as the plugin's
    `_int32_qmax` (every int32 product sum stays below 2^62), and its output is the float
    product up to the per-token / per-row quantisation error."""
    qmax = students._int32_qmax(k)
    assert qmax * qmax * k <= (1 << 62) - 1
    g = torch.Generator().manual_seed(k)
    x = torch.randn(4, k, generator=g)
    w = torch.randn(6, k, generator=g) * 0.05
    y = oracle.int32_linear(x, w)
    exact = x.double() @ w.double().t()
    bound = (x.abs().amax(dim=1, keepdim=True).double() * w.abs().sum(dim=1).double()[None, :] / qmax
             + w.abs().amax(dim=1).double()[None, :] * x.abs().sum(dim=1, keepdim=True).double() / qmax)
    assert bool(((y.double() - exact).abs() <= bound + 1e-5 * exact.abs() + 1e-30).all())


def _call_name(node) -> str | None:
    import ast

    if isinstance(node, ast.Name):
        return node.id
    if isinstance(node, ast.Attribute):
        base = _call_name(node.value)
        return f"{base}.{node.attr}" if base else node.attr
    return None


def _named_source(module, name: str) -> str:
    import ast
    import inspect

    source = inspect.getsource(module)
    for node in ast.parse(source).body:
        if isinstance(node, (ast.ClassDef, ast.FunctionDef)) and node.name == name:
            return ast.get_source_segment(source, node) or ""
    raise AssertionError(f"{name} not found in {module.__name__}")


def test_int32_path_source_has_no_float_gemm_or_cpu_fallbacks():
    """The integer students and the GEMM wrapper they call use no float GEMM, no CPU copy and
    no fake-quantisation path (the reference's own source check of its int32 path), and the
    product reaches the native library."""
    import ast

    from int_model_approximation_b200 import codebook

    source = "\n".join([
        _named_source(students, "Int32Linear"),
        _named_source(students, "CodebookLinear"),
        _named_source(students, "_int32_raw_matmul"),
        _named_source(students, "_int32_matmul"),
        _named_source(students, "_operand_planes"),
        _named_source(codebook, "int_gemm"),
    ])
    calls = {name for node in ast.walk(ast.parse(source)) if isinstance(node, ast.Call)
             for name in [_call_name(node.func)] if name}
    forbidden_calls = {"torch._scaled_mm", "torch.addmm", "torch.baddbmm", "torch.bmm", "torch.matmul", "torch.mm",
                       "torch.nn.functional.linear", "F.linear", "torch._int_mm"}
    assert calls.isdisjoint(forbidden_calls), calls & forbidden_calls
    code_only = "\n".join(line.split("#", 1)[0] for line in source.splitlines())
    for text in (".cpu(", "device='cpu'", 'device="cpu"', "fake_quant", "FakeQuantize", "QuantStub",
                 "DeQuantStub", "torch.ops.quantized"):
        assert text not in code_only, text
    assert not any(isinstance(node, ast.BinOp) and isinstance(node.op, ast.MatMult)
                   for node in ast.walk(ast.parse(source)))   # no `a @ b` on the path
    assert "ima_int_gemm" in _named_source(codebook, "int_gemm")


def test_plane_cache_keys_on_the_version_counter():
    """Cached digit planes are used only while the tensor is unchanged: an in-place edit
    (also under inference mode, on the normal tensors this package creates) drops them,
    and nothing is cached on inference tensors, which have no version counter."""
    from int_model_approximation_b200.codebook import DigitPlanes

    planes = DigitPlanes(torch.zeros((3, 4, 16), dtype=torch.int8), 4, 8, 3)
    t = torch.zeros((4, 8), dtype=torch.int32)
    students._attach_planes(t, planes)
    assert students._attached_planes(t) is planes
    t[1, 2] += 1
    assert students._attached_planes(t) is None
    with torch.inference_mode():
        with torch.inference_mode(False):
            u = torch.zeros((4, 8), dtype=torch.int32)
        students._attach_planes(u, planes)
        assert students._attached_planes(u) is planes
        u.add_(3)
        assert students._attached_planes(u) is None
        inf = torch.zeros((4, 8), dtype=torch.int32)
        students._attach_planes(inf, planes)
        assert students._attached_planes(inf) is None


def test_codebook_stack_passes_y_copies_to_the_gemm_descriptors():
    """bufs["y_copies"] (per linear, up to 8 device addresses) lands in the ima_gemm_y_copies
    array handed to ima_int_gemm_grouped_copies, slot by slot in each launch's problem order;
    without it the plain grouped launch is used; more than 8 copies are refused."""
    from types import SimpleNamespace

    from int_model_approximation_b200 import _native as nat
    from int_model_approximation_b200.pipeline import CodebookStack

    stack = CodebookStack.__new__(CodebookStack)
    shapes = [(64, 32), (16, 32), (48, 32)]
    t = lambda *s, dt=torch.float32: torch.zeros(s, dtype=dt)   # noqa: E731
    stack.linears = [SimpleNamespace(n=n, k=k, w_planes=SimpleNamespace(planes=t(3, n, 32, dt=torch.int8), ld=32),
                                     w_code_scale=t(n), bias=None, t=t(k, dt=torch.int64), r=t(n, dt=torch.int64))
                     for n, k in shapes]
    m = 8
    bufs = {key: [] for key in ("q", "scale", "code_scale", "planes", "c", "y")}
    for n, k in shapes:
        bufs["q"].append(t(m, k, dt=torch.uint8))
        bufs["scale"].append(t(m))
        bufs["code_scale"].append(t(m))
        bufs["planes"].append(SimpleNamespace(planes=t(3, m, 32, dt=torch.int8), ld=32))
        bufs["c"].append(t(m, n, dt=torch.int64))
        bufs["y"].append(t(m, n, dt=torch.bfloat16))
    bufs["mismatch"] = t(1, dt=torch.int32)
    xs = [t(m, k, dt=torch.bfloat16) for _n, k in shapes]
    _q, batches, _f = stack._descriptors(xs, bufs)
    assert all(c_arr is None for _g, _n, c_arr in batches)
    copies = [[0x1000, 0x2000], [], [0x3000 + 0x100 * d for d in range(8)]]
    bufs["y_copies"] = copies
    _q, batches, _f = stack._descriptors(xs, bufs)
    members = stack._batches()
    for (g_arr, count, c_arr), mem in zip(batches, members):
        assert count == len(mem) and c_arr is not None
        for slot, i in enumerate(mem):
            got = [c_arr[slot].y[d] or 0 for d in range(8)]
            assert got == copies[i] + [0] * (8 - len(copies[i]))
            assert g_arr[slot].y == bufs["y"][i].data_ptr()
    bufs["y_copies"] = [[1] * 9, [], []]
    with pytest.raises(ValueError):
        stack._descriptors(xs, bufs)
    import ctypes

    assert ctypes.sizeof(nat.GemmYCopies) == 8 * ctypes.sizeof(ctypes.c_void_p)   # ima_gemm_y_copies

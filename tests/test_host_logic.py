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

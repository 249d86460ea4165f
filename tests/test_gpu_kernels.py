"""GPU parity: every kernel of libima_b200.so against the CPU oracle and the
reference's own fixtures.  Integer and bf16 outputs are compared bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from int_model_approximation_b200 import _native as nat
from int_model_approximation_b200 import codebook, freivalds, hawkeye, hawkeye_freivalds, students, synthetic
from tests.conftest import golden_cases, json_field, load_golden

pytestmark = pytest.mark.gpu


def _fp8(b: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b)).to(device).view(torch.float8_e4m3fn)


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy()
    return t.numpy()


def _assert_status_clean(device):
    code, where, detail = nat.device_status(device.index or 0)
    assert code == 0, f"device status {code} at {where}/{detail}"


# ---------------------------------------------------------------------------
# quantiser
# ---------------------------------------------------------------------------
def test_quantiser_matches_reference_fixture(cuda_device):
    g = load_golden("quantize")
    x = torch.from_numpy(g["x_bf16"].view(np.int16)).view(torch.bfloat16).to(cuda_device)
    q, scale, cb, cs, planes = codebook.per_token_fp8(x, codebook=True, planes=True)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), g["q"])
    assert np.array_equal(_bits(scale), g["scale"].view(np.int32))
    assert np.array_equal(cb.cpu().numpy(), g["codebook"])
    assert np.array_equal(_bits(cs), g["code_scale"].view(np.int32))
    x32 = torch.from_numpy(g["x_f32"]).to(cuda_device)
    q32, s32, *_ = codebook.per_token_fp8(x32)
    assert np.array_equal(q32.view(torch.uint8).cpu().numpy(), g["q_f32"])
    assert np.array_equal(_bits(s32), g["scale_f32"].view(np.int32))


def test_e4m3_conversion_sweep(cuda_device):
    """Rows whose amax is exactly 448 have scale 1, so the kernel's cast of every
    in-range fixture value is compared with torch's cast directly."""
    g = load_golden("e4m3_cast")
    f = g["f32"]
    f = f[np.abs(f) <= 448.0]
    pad = (-len(f)) % 255
    f = np.concatenate([f, np.zeros(pad, dtype=np.float32)]).reshape(-1, 255)
    rows = np.concatenate([np.full((f.shape[0], 1), 448.0, dtype=np.float32), f], axis=1)
    x = torch.from_numpy(rows).to(cuda_device)
    q, scale, *_ = codebook.per_token_fp8(x)
    assert torch.all(scale == 1.0)
    expect = torch.from_numpy(rows).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), expect)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quantiser_random_rows_against_oracle(cuda_device, dtype):
    x = synthetic.student_t_activations(37, 1000, seed=3, outlier_fraction=0.01, dtype=dtype)
    x[5] = 0
    q, scale, cb, _cs, _ = codebook.per_token_fp8(x.to(cuda_device), codebook=True)
    q_ref, s_ref = oracle.per_token_fp8(x)
    assert torch.equal(q.view(torch.uint8).cpu(), q_ref.view(torch.uint8))
    assert torch.equal(scale.cpu(), s_ref)
    assert torch.equal(cb.cpu(), oracle.fp8_codebook(q_ref))


@pytest.mark.parametrize("kind", [0, 1, 2, 3, 4])
def test_quantiser_fast_path_selftest(cuda_device, kind):
    """Exhaustive on-device check of the quantiser's fast path against the torch-shaped
    software cast and IEEE division: the hardware e4m3 cast on every fp32 value below 464
    in magnitude (kind 0); the e4m3 codes (kinds 1, 2) and the normal fp32 quotients
    (kinds 3, 4) of the corrected-reciprocal division on every (amax, element) pair a
    bf16 / fp16 row can hold."""
    bad = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    nat.call("ima_quant_fast_selftest", kind, bad.data_ptr(), nat.stream_of(cuda_device))
    assert int(bad.item()) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_row_scale_is_torch_cuda_division_for_every_amax(cuda_device, dtype):
    """The reference forms the row scale as `amax / 448.0` on CUDA tensors, where torch
    multiplies by the fp32 reciprocal.  One row per positive finite value of the dtype (the
    row's amax) plus smaller elements: the kernel's scale equals torch's CUDA expression, and
    the oracle's CPU emulation of that rule, bit for bit."""
    bits = torch.arange(1, 0x7C00 if dtype == torch.float16 else 0x7F80, dtype=torch.int32).to(torch.int16)
    amax = bits.view(dtype)
    x = torch.stack([amax, -amax * 0.5, amax * 0.25, torch.zeros_like(amax)], dim=1).repeat(1, 4)
    xd = x.to(cuda_device)
    _q, scale, *_ = codebook.per_token_fp8(xd)
    expect = (xd.abs().amax(dim=1, keepdim=True).to(torch.float32) / 448.0).clamp_min(1e-12)
    assert torch.equal(scale.reshape(-1).view(torch.int32), expect.reshape(-1).view(torch.int32))
    _q_ref, s_ref = oracle.per_token_fp8(x)
    assert torch.equal(s_ref.reshape(-1).view(torch.int32), expect.reshape(-1).cpu().view(torch.int32))
    assert int((expect.reshape(-1).cpu() != x.abs().amax(dim=1).float() / 448.0).sum()) > 0   # the rules differ


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quantiser_special_rows_and_planes(cuda_device, dtype):
    """Rows with NaN, +-inf, all zeros, tiny (subnormal) values and a ragged K.  Codes are
    compared bit for bit with the reference's expression (__main__.py:148-154) evaluated by
    torch on CUDA, the platform the reference quantises on, and with the CPU oracle up to
    the sign of NaN codes: an invalid division (inf / inf) yields x86's negative default
    NaN on the CPU but CUDA's positive canonical NaN on the GPU.  The digit planes rebuild
    the codebook and are zero beyond K."""
    m, k = 12, 903
    x = synthetic.student_t_activations(m, k, seed=9, outlier_fraction=0.02, dtype=torch.float32)
    x[1, 17] = float("nan")
    x[2, 5] = float("inf")
    x[3, 100] = float("-inf")
    x[4] = 0.0
    x[5] = x[5] * 1e-38
    x[6, :3] = torch.tensor([65504.0, -1e-7, 3e-8])
    x = x.to(dtype)
    xd = x.to(cuda_device)
    q, scale, cb, _cs, dp = codebook.per_token_fp8(xd, codebook=True, planes=True)
    s_cuda = (xd.float().abs().amax(dim=1, keepdim=True) / 448.0).clamp_min(1e-12)
    q_cuda = (xd.float() / s_cuda).to(torch.float8_e4m3fn)
    assert torch.equal(q.view(torch.uint8), q_cuda.view(torch.uint8))
    finite = torch.isfinite(s_cuda.reshape(-1))
    assert torch.equal(scale.reshape(-1)[finite].view(torch.int32), s_cuda.reshape(-1)[finite].view(torch.int32))
    q_ref, s_ref = oracle.per_token_fp8(x)
    unsigned_nan = (q.view(torch.uint8).cpu() & 0x7F) == 0x7F
    assert torch.equal(unsigned_nan, (q_ref.view(torch.uint8) & 0x7F) == 0x7F)
    same = (q.view(torch.uint8).cpu() == q_ref.view(torch.uint8)) | unsigned_nan
    assert bool(same.all())
    nan = torch.isnan(scale.cpu().reshape(-1))
    assert torch.equal(nan, torch.isnan(s_ref.reshape(-1)))   # NaN payloads are platform-defined
    assert np.array_equal(_bits(scale.reshape(-1))[~nan.numpy()], _bits(s_ref.reshape(-1))[~nan.numpy()])
    assert torch.equal(cb.cpu(), oracle.fp8_codebook(q_ref))
    p = dp.planes.cpu().to(torch.int64)
    assert p.shape[0] == 3 and p.shape[1] == m and p.shape[2] >= k
    assert torch.equal(p[0, :, :k] + 128 * p[1, :, :k] + 16384 * p[2, :, :k], cb.cpu().to(torch.int64))
    assert int(p[:2].min()) >= -64 and int(p[:2].max()) <= 63
    assert not p[:, :, k:].any()


# ---------------------------------------------------------------------------
# Hawkeye replay
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", sorted(golden_cases(load_golden("hawkeye")).keys()))
def test_hawkeye_matches_reference_fixture(cuda_device, case):
    d = golden_cases(load_golden("hawkeye"))[case]
    x, w = _fp8(d["x"], cuda_device), _fp8(d["w"], cuda_device)
    xs = torch.from_numpy(d["x_scale"]).to(cuda_device)
    ws = torch.from_numpy(d["w_scale"]).to(cuda_device)
    out, stats = hawkeye.hawkeye_fp8_sum(x, xs, w, ws)
    assert np.array_equal(_bits(out), d["exact_bf16"].view(np.int16))
    f32 = torch.empty(out.shape, dtype=torch.float32, device=cuda_device)
    hawkeye.hawkeye_replay(hawkeye.HawkeyeOperand(x), hawkeye.HawkeyeOperand(w), xs, ws, out_f32=f32)
    assert np.array_equal(_bits(f32), d["y_f32"].view(np.int32))
    assert stats.total_checkable_products == 0
    assert stats.groups == (x.shape[1] + 31) // 32
    _assert_status_clean(cuda_device)


@pytest.mark.parametrize("m,k,n", [(1, 32, 1), (5, 31, 7), (65, 100, 129), (130, 257, 300), (16, 896, 4864)])
def test_hawkeye_random_shapes_against_oracle(cuda_device, m, k, n):
    x = synthetic.student_t_activations(m, k, seed=m + k, outlier_fraction=0.01)
    xq, xs = oracle.per_token_fp8(x)
    w, ws = synthetic.normal_fp8_weights(n, k, seed=n + k)
    out, _ = hawkeye.hawkeye_fp8_sum(xq.to(cuda_device), xs.to(cuda_device), w.to(cuda_device), ws.to(cuda_device))
    ref = oracle.hawkeye(xq, xs, w, ws).to(torch.bfloat16)
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


def test_hawkeye_stack_matches_single_launches(cuda_device):
    """HawkeyeStack (quantise + stage per linear, replays spread over side streams) gives
    the same bits as hawkeye_fp8_sum on every linear."""
    from int_model_approximation_b200.pipeline import HawkeyeStack

    weights, xs = [], []
    for i in range(9):
        m, n, k = 40 + 17 * i, 30 + 45 * i, 64 + 90 * i
        w, ws = synthetic.normal_fp8_weights(n, k, seed=2900 + i)
        weights.append((w.to(cuda_device), ws.to(cuda_device), None))
        xs.append(synthetic.student_t_activations(m, k, seed=3900 + i, outlier_fraction=0.02).to(cuda_device))
    stack = HawkeyeStack(weights)
    bufs = {"q": [], "scale": [], "xop": [], "y": []}
    lib = nat.lib()
    for (w, _ws, _b), x in zip(weights, xs):
        m, k = x.shape
        bufs["q"].append(torch.empty((m, k), dtype=torch.uint8, device=cuda_device))
        bufs["scale"].append(torch.empty((m,), dtype=torch.float32, device=cuda_device))
        bufs["xop"].append(torch.empty((int(lib.ima_hawkeye_operand_bytes(m, k)),), dtype=torch.uint8,
                                       device=cuda_device))
        bufs["y"].append(torch.empty((m, w.shape[0]), dtype=torch.bfloat16, device=cuda_device))
    stack.forward(xs, bufs)
    torch.cuda.synchronize()
    for i, ((w, ws, _b), x) in enumerate(zip(weights, xs)):
        xq, xsc, *_ = codebook.per_token_fp8(x)
        ref, _ = hawkeye.hawkeye_fp8_sum(xq, xsc, w, ws)
        assert torch.equal(bufs["y"][i].view(torch.int16), ref.view(torch.int16)), f"linear {i}"


def test_hawkeye_raw_byte_patterns_against_oracle(cuda_device):
    g = torch.Generator().manual_seed(9)
    x = torch.randint(0, 256, (70, 160), generator=g, dtype=torch.int64).to(torch.uint8).view(torch.float8_e4m3fn)
    w = torch.randint(0, 256, (90, 160), generator=g, dtype=torch.int64).to(torch.uint8).view(torch.float8_e4m3fn)
    xs = torch.rand(70, 1, generator=g) + 0.25
    ws = torch.rand(90, generator=g) + 0.25
    out, _ = hawkeye.hawkeye_fp8_sum(x.to(cuda_device), xs.to(cuda_device), w.to(cuda_device), ws.to(cuda_device))
    ref = oracle.hawkeye(x, xs, w, ws).to(torch.bfloat16)
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


def test_hawkeye_c2_shape_sampled_rows(cuda_device):
    """Config-2 shape (M = 16384 tokens, gate_proj) with 0.1% outliers: sampled rows are
    exact checks because every output row is independent."""
    x, w, ws = synthetic.make_linear_inputs(2, 4, synthetic.LinearShape("gate_proj", 4864, 896), device=cuda_device)
    xq, xs, *_ = codebook.per_token_fp8(x)
    out, _ = hawkeye.hawkeye_fp8_sum(xq, xs, w, ws)
    rows = torch.randperm(x.shape[0], generator=torch.Generator().manual_seed(0))[:24].numpy()
    ref = oracle.hawkeye(xq.cpu(), xs.cpu(), w.cpu(), ws.cpu(), rows=rows).to(torch.bfloat16)
    assert torch.equal(out[torch.from_numpy(rows).to(cuda_device)].cpu().view(torch.int16), ref.view(torch.int16))


# ---------------------------------------------------------------------------
# exact int GEMM (tcgen05)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["ref_test_4x3", "c16x96x40", "c7x200x33", "c3x32x17"])
def test_codebook_linear_matches_reference_fixture(cuda_device, case):
    d = golden_cases(load_golden("codebook"))[case]
    x = torch.from_numpy(d["x"]).to(cuda_device)
    if bool(d["x_is_bf16"]):
        x = x.to(torch.bfloat16)
    w = _fp8(d["w"], cuda_device)
    ws = torch.from_numpy(d["w_scale"]).to(cuda_device)
    bias = None
    if "bias_bf16" in d:
        bias = torch.from_numpy(d["bias_bf16"].view(np.int16)).view(torch.bfloat16).to(cuda_device)
    layer = students.CodebookLinear(w, ws, bias)
    x_i32, x_scale = students._per_token_fp8_int32(x)
    with students._Int32KernelProbe() as probe:
        c = students._int32_raw_matmul(x_i32, layer.weight_t)
        y = students._int32_matmul(x_i32, layer.weight_t, x_scale, layer.weight_scale)
        out = layer(x)
    assert probe.count == 3
    assert np.array_equal(c.cpu().numpy(), d["c"])
    assert np.array_equal(_bits(y), d["y"].view(np.int32))
    assert np.array_equal(_bits(out.to(torch.float32)), d["out_f32"].view(np.int32))
    _assert_status_clean(cuda_device)


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (3, 17, 5), (128, 128, 64), (129, 300, 65), (512, 896, 4864),
                                   (200, 4864, 896), (77, 18944, 40)])
def test_int_gemm_codebook_against_oracle(cuda_device, m, k, n):
    x = synthetic.student_t_activations(m, k, seed=m * 7 + k)
    w, ws = synthetic.normal_fp8_weights(n, k, seed=n * 3 + k)
    xq, xs, *_ = codebook.per_token_fp8(x.to(cuda_device), planes=True)
    _, _, _, _, a = codebook.per_token_fp8(x.to(cuda_device), planes=True)
    b, _ = codebook.codebook_planes_from_fp8(w.to(cuda_device))
    c, y = codebook.int_gemm(a, b, x_scale=xs / 512.0, w_scale=ws.to(cuda_device) / 512.0, y_dtype=torch.float32)
    rows = np.arange(m) if m <= 256 else np.random.default_rng(0).choice(m, 96, replace=False)
    a_ref = oracle.fp8_codebook(xq.cpu())[torch.from_numpy(rows)]
    b_ref = oracle.fp8_codebook(w)
    c_ref = oracle.int_gemm(a_ref, b_ref, b_is_nk=True)
    assert torch.equal(c.cpu()[torch.from_numpy(rows)], c_ref)
    y_ref = oracle.rescale(c_ref, (xs.cpu() / 512.0)[torch.from_numpy(rows)], ws / 512.0)
    assert torch.equal(y.cpu()[torch.from_numpy(rows)].view(torch.int32), y_ref.view(torch.int32))
    _assert_status_clean(cuda_device)


def test_int_gemm_extreme_codebook_values(cuda_device):
    """All operands at the largest codebook magnitude (0x7E = 448 -> 229376): the
    largest possible |C| for this K, exact in int64."""
    k = 4864
    x = torch.full((130, k), 0x7E, dtype=torch.uint8)
    x[::2] = 0xFE
    w = torch.full((70, k), 0x7E, dtype=torch.uint8)
    w[:, ::3] = 0xFE
    a, _ = codebook.codebook_planes_from_fp8(x.view(torch.float8_e4m3fn).to(cuda_device))
    b, _ = codebook.codebook_planes_from_fp8(w.view(torch.float8_e4m3fn).to(cuda_device))
    c, _ = codebook.int_gemm(a, b)
    ref = oracle.int_gemm(oracle.fp8_codebook(x.view(torch.float8_e4m3fn)), oracle.fp8_codebook(w.view(torch.float8_e4m3fn)),
                          b_is_nk=True)
    assert torch.equal(c.cpu(), ref)


@pytest.mark.parametrize("lo,hi", [(-(2**31), 2**31), (-1000, 1000)])
def test_int32_raw_matmul_generic_int32(cuda_device, lo, hi):
    g = torch.Generator().manual_seed(hi % 1000)
    a = torch.randint(lo, hi, (70, 200), generator=g, dtype=torch.int64).to(torch.int32)
    b = torch.randint(lo, hi, (200, 45), generator=g, dtype=torch.int64).to(torch.int32)
    a[0, :] = -(2**31) if lo < -1000 else lo
    c = students._int32_raw_matmul(a.to(cuda_device), b.to(cuda_device))
    assert torch.equal(c.cpu(), oracle.int_gemm(a, b))


@pytest.mark.parametrize("dtype,k", [(torch.bfloat16, 896), (torch.float32, 300), (torch.float16, 4864), (torch.float32, 1)])
def test_int32_linear_matches_reference_forward(cuda_device, dtype, k):
    """Int32Linear (the student the replacement pass puts on non-FP8 linears) against the CPU
    restatement of the reference's forward: per-row / per-token int32 quantisation with
    qmax = floor(sqrt((2^62 - 1) / K)), the exact int64 product (full-range operands, so the
    five-plane GEMM scheme), the fp32 rescale and bias, bit for bit; one probe bump.  K = 1
    makes qmax = 2^31 - 1, which rounds to 2^31 in fp32: the row maxima then go through
    CUDA's saturating float -> int32 cast."""
    g = torch.Generator().manual_seed(k)
    n = 70
    weight = (torch.randn(n, k, generator=g) * 0.05).to(torch.float32)
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.float32)
    x = synthetic.student_t_activations(2 * 9, k, seed=k + 3, outlier_fraction=0.01, dtype=dtype).reshape(2, 9, k)
    layer = students.Int32Linear(weight.to(cuda_device), bias.to(cuda_device))
    with torch.inference_mode(), students._Int32KernelProbe() as probe:
        y = layer(x.to(cuda_device))
        torch.cuda.synchronize()
    assert probe.count == 1
    assert y.shape == (2, 9, n) and y.dtype == dtype
    ref = oracle.int32_linear(x, weight, bias)
    assert torch.equal(_bits_any(y.cpu()), _bits_any(ref))
    _assert_status_clean(cuda_device)


@pytest.mark.parametrize("case", sorted(golden_cases(load_golden("int32_linear")).keys()))
def test_int32_linear_matches_reference_fixture(cuda_device, case):
    """Int32Linear against the reference's own Int32Linear run (tests/golden/int32_linear.npz):
    the quantised weight and activations, the exact int64 product through _int32_raw_matmul
    and the module output, bit for bit."""
    d = golden_cases(load_golden("int32_linear"))[case]
    dtype = getattr(torch, str(d["x_dtype"]))
    x = torch.from_numpy(d["x_f32"]).to(dtype).to(cuda_device)
    weight = torch.from_numpy(d["weight"]).to(cuda_device)
    bias = torch.from_numpy(d["bias"]).to(cuda_device) if "bias" in d else None
    layer = students.Int32Linear(weight, bias)
    assert layer.qmax == float(d["qmax"])
    assert torch.equal(layer.weight_t.cpu(), torch.from_numpy(d["weight_t"]))
    assert torch.equal(layer.weight_scale.cpu(), torch.from_numpy(d["weight_scale"]))
    x_i32, x_scale = students._per_token_int32(x, layer.qmax)
    assert torch.equal(x_i32.cpu(), torch.from_numpy(d["x_i32"]))
    assert torch.equal(x_scale.cpu(), torch.from_numpy(d["x_scale"]))
    with students._Int32KernelProbe() as probe:
        c = students._int32_raw_matmul(x_i32, layer.weight_t)
        y = layer(x)
    assert probe.count == 2
    assert torch.equal(c.cpu(), torch.from_numpy(d["c"]))
    assert y.dtype == dtype
    assert torch.equal(_bits_any(y.cpu()), _bits_any(torch.from_numpy(d["y_f32"]).to(dtype)))
    _assert_status_clean(cuda_device)


def _bits_any(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int32 if t.dtype == torch.float32 else torch.int16)


def _ref_test_fp8_weight(device) -> torch.Tensor:
    """The hand-written FP8 weight of the reference's integer-GEMM tests."""
    return torch.tensor([[0.125, -0.5, 1.0], [-1.5, 0.25, 2.0], [3.0, -0.75, 0.5], [-2.5, 1.5, -0.125]],
                        dtype=torch.float32, device=device).to(torch.float8_e4m3fn)


def test_codebook_linear_uses_one_int32_matmul_path(cuda_device, monkeypatch):
    """CodebookLinear.forward makes exactly one int32 x int32 matmul call and no float GEMM."""
    layer = students.CodebookLinear(_ref_test_fp8_weight(cuda_device), torch.ones(4, 1, device=cuda_device), None)
    calls = []

    def fake_int32_matmul(activations, weight_t, x_scale, w_scale):
        calls.append((activations, weight_t, x_scale, w_scale))
        assert activations.dtype == torch.int32 and weight_t.dtype == torch.int32
        return torch.zeros((activations.shape[0], weight_t.shape[1]), dtype=torch.float32, device=activations.device)

    monkeypatch.setattr(students, "_int32_matmul", fake_int32_matmul)

    def fail(*_args, **_kwargs):
        raise AssertionError("the codebook student used a float GEMM")

    for attr in ("mm", "matmul", "addmm", "bmm", "_scaled_mm"):
        monkeypatch.setattr(torch, attr, fail)
    monkeypatch.setattr(torch.nn.functional, "linear", fail)
    y = layer(torch.randn(2, 3, device=cuda_device))
    assert len(calls) == 1
    assert y.shape == (2, 4)


def test_forward_integer_gemms_are_freivalds_verifiable(cuda_device, monkeypatch):
    """Every integer product of an integerised forward, captured at the matmul boundary, is
    exact (against the oracle) and passes the Freivalds check with the reference test's
    vectors; a corrupted product fails it."""
    linear = torch.nn.Linear(3, 4, bias=False, device=cuda_device)
    linear.weight = torch.nn.Parameter(_ref_test_fp8_weight(cuda_device), requires_grad=False)
    linear.weight_scale = torch.ones(4, 1, device=cuda_device)
    model = torch.nn.Sequential(linear)
    monkeypatch.setattr(students, "STUDENT_KERNEL", "codebook")
    students._replace_int32_linears(model)
    assert isinstance(model[0], students.CodebookLinear)
    captured = []
    original = students._int32_matmul

    def wrapped(activations, weight_t, x_scale, w_scale):
        captured.append((activations.detach().clone(), weight_t.detach().clone()))
        return original(activations, weight_t, x_scale, w_scale)

    monkeypatch.setattr(students, "_int32_matmul", wrapped)
    x = torch.tensor([[0.25, -1.5, 2.0], [3.0, -0.75, 0.125]], device=cuda_device)
    with torch.inference_mode():
        y = model(x)
        torch.cuda.synchronize()
    assert y.device.type == "cuda" and len(captured) == 1
    for a, b in captured:
        c = students._int32_raw_matmul(a, b)
        assert torch.equal(c.cpu(), oracle.int_gemm(a.cpu(), b.cpu()))
        n = b.shape[1]
        for vec in ([1] + [0] * (n - 1), [1 if i % 2 == 0 else -1 for i in range(n)],
                    [0 if i % 3 == 0 else 1 for i in range(n)]):
            r = torch.tensor(vec, dtype=torch.int64, device=cuda_device)
            assert freivalds.verify_int32_product(a, b, c, r)
        bad = c.clone()
        bad[1, 0] += 1
        assert not freivalds.verify_int32_product(a, b, bad, torch.ones(n, dtype=torch.int64, device=cuda_device))


def test_raw_int32_matmul_is_freivalds_verifiable(cuda_device):
    """The reference's prime-matrix test (tests/test_real_integer_gemms.py:252-278)."""
    g = load_golden("freivalds")
    a = torch.from_numpy(g["prime_a"]).to(cuda_device)
    b = torch.from_numpy(g["prime_b"]).to(cuda_device)
    c = students._int32_raw_matmul(a, b)
    assert c.dtype == torch.int64 and c.device.type == "cuda"
    assert np.array_equal(c.cpu().numpy(), g["prime_c"])
    for r in g["prime_vectors"]:
        rt = torch.from_numpy(r).to(cuda_device)
        assert freivalds.verify_int32_product(a, b, c, rt)
        assert oracle.exact_matvec(a.cpu().tolist(), oracle.exact_matvec(b.cpu().tolist(), r.tolist())) == \
            oracle.exact_matvec(c.cpu().tolist(), r.tolist())
    bad = c.clone()
    bad[0, 0] += 1
    assert not freivalds.verify_int32_product(a, b, bad, torch.from_numpy(g["prime_vectors"][0]).to(cuda_device))


# ---------------------------------------------------------------------------
# Freivalds
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("m,k,n", [(1, 5, 3), (33, 300, 70), (512, 896, 4864), (64, 4864, 896)])
def test_freivalds_codebook_accepts_and_rejects(cuda_device, m, k, n):
    x = synthetic.student_t_activations(m, k, seed=k + 1)
    w, ws = synthetic.normal_fp8_weights(n, k, seed=k + 2)
    xq, xs, *_ = codebook.per_token_fp8(x.to(cuda_device))
    a = codebook.per_token_fp8(x.to(cuda_device), planes=True)[4]
    b, _ = codebook.codebook_planes_from_fp8(w.to(cuda_device))
    c, _ = codebook.int_gemm(a, b)
    r = freivalds.freivalds_vector(n, seed=k + 7, device=cuda_device)
    wd = w.to(cuda_device)
    assert freivalds.verify_codebook_product(xq, wd, c, r)
    bad = c.clone()
    bad[m // 2, n // 3] += 1
    assert int(r[n // 3]) != 0
    assert int(freivalds.mismatch_rows_codebook(xq, wd, bad, r).item()) == 1
    # oracle agrees on the verdicts
    a_ref = oracle.fp8_codebook(xq.cpu())
    b_ref = oracle.fp8_codebook(w).t().contiguous()
    assert oracle.freivalds_mismatch_rows(a_ref, b_ref, c.cpu(), r.cpu()) == 0
    assert oracle.freivalds_mismatch_rows(a_ref, b_ref, bad.cpu(), r.cpu()) == 1


# ---------------------------------------------------------------------------
# class counts
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", [c for c in sorted(golden_cases(load_golden("class_counts")).keys()) if c != "packing"])
def test_class_counts_match_reference_fixture(cuda_device, case):
    d = golden_cases(load_golden("class_counts"))[case]
    params = json_field(d["params"])
    x, w = _fp8(d["x"], cuda_device), _fp8(d["w"], cuda_device)
    with students._Int32KernelProbe() as probe:
        y, stats = hawkeye_freivalds.exact_hawkeye_fp8_sum(
            x, torch.ones((x.shape[0], 1), device=cuda_device), w, torch.ones((w.shape[0],), device=cuda_device),
            students._int32_raw_matmul, **params,
        )
    assert np.array_equal(_bits(y), d["y_bf16"].view(np.int16))
    assert stats.__dict__ == json_field(d["stats"])
    assert probe.count == stats.total_checkable_products


def _small_class_count_case(device):
    x = synthetic.student_t_activations(24, 200, seed=21, outlier_fraction=0.02)
    xq, xs = oracle.per_token_fp8(x)
    w, ws = synthetic.normal_fp8_weights(40, 200, seed=22)
    return xq.to(device), xs.to(device), w.to(device), ws.to(device)


@pytest.mark.parametrize(
    "params",
    [
        dict(class_chunk=32),
        dict(class_chunk=8, packed_count_lanes=6),
        dict(class_chunk=16, packed_count_lanes=6, packed_group_lanes=2),
        dict(class_chunk=32, cache_weight_chunks=True),
        dict(class_chunk=8, count_dtype=torch.int8),
        dict(class_chunk=8, packed_count_lanes=6, packed_group_lanes=3),
        dict(class_chunk=4, packed_count_lanes=6, packed_group_lanes=6),
    ],
)
def test_class_counts_with_an_injected_raw_matmul(cuda_device, params):
    """An injected raw_matmul receives the reference's count products, one call per
    checkable product, each Freivalds-checked; the output equals the engine-only call's
    (raw_matmul None) and the oracle's bit for bit."""
    xq, xs, w, ws = _small_class_count_case(cuda_device)
    shapes = []

    def logging_matmul(a, b):
        shapes.append((tuple(a.shape), tuple(b.shape)))
        return students._int32_raw_matmul(a.to(torch.int32), b.to(torch.int32))

    y, stats = hawkeye_freivalds.exact_hawkeye_fp8_sum(xq, xs, w, ws, logging_matmul, **params)
    fused, fused_stats = hawkeye_freivalds.exact_hawkeye_fp8_sum(xq, xs, w, ws, None, **params)
    assert len(shapes) == stats.total_checkable_products == fused_stats.total_checkable_products > 0
    assert all(a[1] == b[0] and a[0] % 24 == 0 and b[1] % 40 == 0 for a, b in shapes)
    assert torch.equal(y.view(torch.int16), fused.view(torch.int16))
    ref = oracle.hawkeye(xq.cpu(), xs.cpu(), w.cpu(), ws.cpu()).to(torch.bfloat16)
    assert torch.equal(y.cpu().view(torch.int16), ref.view(torch.int16))


def test_class_counts_reject_a_wrong_injected_product(cuda_device):
    xq, xs, w, ws = _small_class_count_case(cuda_device)

    def tampered(a, b):
        c = students._int32_raw_matmul(a, b)
        c[3, 1] += 1
        return c

    with pytest.raises(RuntimeError, match="fails the Freivalds check"):
        hawkeye_freivalds.exact_hawkeye_fp8_sum(xq, xs, w, ws, tampered)


def test_class_count_probe_counts_only_products_the_reference_sends_through_raw_matmul(cuda_device):
    xq, xs, w, ws = _small_class_count_case(cuda_device)
    with students._Int32KernelProbe() as probe:
        _, stats = hawkeye_freivalds.exact_hawkeye_fp8_sum(xq, xs, w, ws, students._int32_raw_matmul)
    assert probe.count == stats.total_checkable_products > 0
    with students._Int32KernelProbe() as probe:
        _, stats = hawkeye_freivalds.exact_hawkeye_fp8_sum(xq, xs, w, ws, students._int32_raw_matmul,
                                                           fused_replay=True)
    assert probe.count == 0 and stats.total_checkable_products > 0


# ---------------------------------------------------------------------------
# the plugin surface end to end
# ---------------------------------------------------------------------------
def _fp8_model(device):
    model = torch.nn.Sequential(torch.nn.Linear(96, 64, bias=True), torch.nn.GELU(), torch.nn.Linear(64, 40))
    model = model.to(device)
    for i, lin in enumerate((model[0], model[2])):
        w, ws = synthetic.normal_fp8_weights(lin.out_features, lin.in_features, seed=90 + i)
        lin.weight = torch.nn.Parameter(w.to(device), requires_grad=False)
        lin.weight_scale = ws.to(device)   # a plain attribute, as compressed-tensors checkpoints expose it
    return model


def test_host_tensors_are_refused_before_launch(cuda_device):
    w, ws = synthetic.normal_fp8_weights(40, 64, seed=1)
    layer = students.CodebookLinear(w.to(cuda_device), ws, None)   # scale left on the host
    x = synthetic.student_t_activations(3, 64, seed=2).to(cuda_device)
    with pytest.raises(RuntimeError, match="must be on CUDA"):
        layer(x)
    torch.cuda.synchronize()


def test_inference_mode_keeps_the_codebook_scheme(cuda_device):
    w, ws = synthetic.normal_fp8_weights(40, 64, seed=1)
    layer = students.CodebookLinear(w.to(cuda_device), ws.to(cuda_device), None)
    x = synthetic.student_t_activations(3, 64, seed=2).to(cuda_device)
    with torch.inference_mode():
        x_i32, _ = students._per_token_fp8_int32(x)
        a, b = students._operand_planes(x_i32, layer.weight_t)
    assert a.scheme == b.scheme == nat.IMA_SCHEME_DIGITS3


def test_in_place_edits_under_inference_mode_give_the_edited_product(cuda_device):
    """int32 operands edited in place under torch.inference_mode() (the reference's driver
    runs the student there) give the product of the edited values: the cached digit planes
    of the package's own operands are dropped by the edit, and an inference tensor (no
    version counter) is never served from a cache."""
    w, ws = synthetic.normal_fp8_weights(48, 96, seed=31)
    x = synthetic.student_t_activations(5, 96, seed=32).to(cuda_device)
    with torch.inference_mode():
        layer = students.CodebookLinear(w.to(cuda_device), ws.to(cuda_device), None)
        x_i32, _ = students._per_token_fp8_int32(x)
        first = students._int32_raw_matmul(x_i32, layer.weight_t)
        x_i32[1, 3] += 7
        layer.weight_t[5, 2] -= 11
        edited = students._int32_raw_matmul(x_i32, layer.weight_t)
        inf = torch.randint(-50, 50, (5, 96), dtype=torch.int32, device=cuda_device)
        assert inf.is_inference()
        c_inf = students._int32_raw_matmul(inf, layer.weight_t)
        inf.add_(1)
        c_inf_edited = students._int32_raw_matmul(inf, layer.weight_t)
        a_cpu, b_cpu, inf_cpu = x_i32.cpu(), layer.weight_t.cpu(), inf.cpu()
    assert not torch.equal(first, edited)
    assert torch.equal(edited.cpu(), oracle.int_gemm(a_cpu, b_cpu))
    assert torch.equal(c_inf_edited.cpu(), oracle.int_gemm(inf_cpu, b_cpu))
    assert torch.equal(c_inf.cpu(), oracle.int_gemm(inf_cpu - 1, b_cpu))

    # a Hawkeye student's staged weight follows an in-place edit of its weight buffer
    xb = synthetic.student_t_activations(7, 96, seed=33).to(cuda_device)
    with torch.inference_mode():
        hl = students.HawkeyeLinear(w.to(cuda_device), ws.to(cuda_device), None)
        hl(xb)
        hl.weight[3].copy_(hl.weight[4])
        y = hl(xb)
        xq, xs = students._per_token_fp8(xb)
        w_now = hl.weight.cpu()
    ref = oracle.hawkeye(xq.cpu(), xs.cpu(), w_now, ws).to(torch.bfloat16)
    assert torch.equal(y.cpu().view(torch.int16), ref.view(torch.int16))
    _assert_status_clean(cuda_device)


@pytest.mark.parametrize("kernel", ["codebook", "hawkeye", "hawkeye-class-counts"])
def test_student_model_end_to_end(cuda_device, monkeypatch, kernel):
    monkeypatch.setattr(students, "STUDENT_KERNEL", kernel)
    model = _fp8_model(cuda_device)
    w0 = model[0].weight.detach().cpu().clone()
    ws0 = model[0].weight_scale.detach().cpu().clone()
    b0 = model[0].bias.detach().cpu().clone()
    replaced = students._replace_int32_linears(model)
    assert replaced == ["0", "2"]
    x = synthetic.student_t_activations(9, 96, seed=5).to(cuda_device)
    with torch.inference_mode(), students._Int32KernelProbe() as probe:
        y = model(x)
        torch.cuda.synchronize()
    assert y.shape == (9, 40)
    if kernel == "codebook":
        assert probe.count == 2
    elif kernel == "hawkeye":
        assert probe.count == 0
    else:
        assert probe.count > 0
    with torch.inference_mode():
        h = model[0](x)
    if kernel == "codebook":
        ref = oracle.codebook_linear(x.cpu(), w0, ws0, b0)[2]
    else:
        xq, xs = oracle.per_token_fp8(x.cpu())
        ref = oracle.hawkeye(xq, xs, w0, ws0).to(torch.bfloat16)
        ref = (ref + b0.to(torch.bfloat16)).to(x.dtype)
    assert torch.equal(h.cpu().view(torch.int16), ref.view(torch.int16))


# ---------------------------------------------------------------------------
# grouped launches (many linears per launch) and the prepared pipeline
# ---------------------------------------------------------------------------
def test_grouped_pipeline_matches_oracle_and_flags_corruption(cuda_device):
    from int_model_approximation_b200.pipeline import CodebookStack

    shapes = [(40, 96), (300, 128), (17, 4864), (896, 896), (64, 200)]
    tokens = 150
    weights, xs = [], []
    for i, (n, k) in enumerate(shapes):
        w, ws = synthetic.normal_fp8_weights(n, k, seed=200 + i)
        bias = (torch.randn(n, generator=torch.Generator().manual_seed(i)) * 0.1).to(torch.bfloat16)
        weights.append((w.to(cuda_device), ws.to(cuda_device), bias.to(cuda_device)))
        xs.append(synthetic.student_t_activations(tokens, k, seed=300 + i).to(cuda_device))
    stack = CodebookStack(weights)
    bufs = stack.allocate(tokens)
    stack.forward(xs, bufs)
    torch.cuda.synchronize()
    assert int(bufs["mismatch"].item()) == 0
    for i, (w, ws, bias) in enumerate(weights):
        c_ref, _y, out_ref = oracle.codebook_linear(xs[i].cpu(), w.cpu(), ws.cpu(), bias.cpu())
        assert torch.equal(bufs["c"][i].cpu(), c_ref), f"linear {i}"
        assert torch.equal(bufs["y"][i].cpu().view(torch.int16), out_ref.view(torch.int16)), f"linear {i}"
    # corrupt one entry in two products: exactly two rows must be flagged
    bufs["mismatch"].zero_()
    bufs["c"][1][7, 3] += 1
    bufs["c"][3][149, 895] -= 5
    stack.verify(xs, bufs)
    torch.cuda.synchronize()
    expected = int(stack.linears[1].r[3].item() != 0) + int(stack.linears[3].r[895].item() != 0)
    assert int(bufs["mismatch"].item()) == expected == 2
    _assert_status_clean(cuda_device)


def test_grouped_check_aligned_path_flags_every_position(cuda_device):
    """Products whose check takes the unrolled aligned row pass (K % 4 == 0, N even, aligned
    rows): a correct forward passes, and one corrupted entry is flagged wherever it sits --
    inside the unrolled part of a row, in the remainder loop, at either end -- and so is a
    corrupted activation code."""
    from int_model_approximation_b200.pipeline import CodebookStack

    shapes = [(128, 896), (896, 4864), (4864, 896), (70, 300), (2, 4)]
    tokens = 40
    weights, xs = [], []
    for i, (n, k) in enumerate(shapes):
        w, ws = synthetic.normal_fp8_weights(n, k, seed=700 + i)
        weights.append((w.to(cuda_device), ws.to(cuda_device), None))
        xs.append(synthetic.student_t_activations(tokens, k, seed=800 + i).to(cuda_device))
    stack = CodebookStack(weights, seed=3)
    bufs = stack.allocate(tokens)
    stack.forward(xs, bufs)
    torch.cuda.synchronize()
    assert int(bufs["mismatch"].item()) == 0
    for i, (w, ws, _b) in enumerate(weights):
        c_ref, _y, _out = oracle.codebook_linear(xs[i].cpu(), w.cpu(), ws.cpu())
        assert torch.equal(bufs["c"][i].cpu(), c_ref), f"linear {i}"
    for i, (n, k) in enumerate(shapes):
        r = stack.linears[i].r.cpu()
        cols = sorted({0, 1, 63, 64, 127, 128, 255, 256, 511, 512, n // 2, n - 2, n - 1} & set(range(n)))
        for j, col in enumerate(cols):
            row = (j * 7) % tokens
            bufs["mismatch"].zero_()
            bufs["c"][i][row, col] += 1 + j
            stack.verify(xs, bufs)
            torch.cuda.synchronize()
            bufs["c"][i][row, col] -= 1 + j
            assert int(bufs["mismatch"].item()) == int(int(r[col]) * (1 + j) % 2**64 != 0), (i, row, col)
        # a corrupted activation code (raise the magnitude of a nonzero code by one step)
        q = bufs["q"][i]
        t = stack.linears[i].t.cpu()
        for col in sorted({0, 3, k // 2, k - 1}):
            row = (col * 5) % tokens
            old = int(q[row, col].item())
            if (old & 0x7F) in (0, 0x7E, 0x7F):
                continue
            bufs["mismatch"].zero_()
            q[row, col] = old + 1
            stack.verify(xs, bufs)
            torch.cuda.synchronize()
            q[row, col] = old
            delta = oracle.fp8_codebook(torch.tensor([old + 1], dtype=torch.uint8).view(torch.float8_e4m3fn)) - \
                oracle.fp8_codebook(torch.tensor([old], dtype=torch.uint8).view(torch.float8_e4m3fn))
            expect = int(int(delta[0]) * int(t[col]) % 2**64 != 0)
            assert int(bufs["mismatch"].item()) == expect, (i, row, col)
    _assert_status_clean(cuda_device)


def test_grouped_gemm_many_problems_fp32_outputs(cuda_device):
    """More problems than one launch holds (40), fp32 and bf16 outputs, ragged N."""
    import ctypes

    probs, refs, keep = [], [], []
    for i in range(45):
        m, n, k = 1 + (i * 37) % 200, 8 + (i * 53) % 300, 16 + (i * 29) % 700
        x = synthetic.student_t_activations(m, k, seed=i)
        w, ws = synthetic.normal_fp8_weights(n, k, seed=1000 + i)
        _q, xs, _cb, cs, a = codebook.per_token_fp8(x.to(cuda_device), codebook=True, planes=True)
        b, _ = codebook.codebook_planes_from_fp8(w.to(cuda_device))
        wsc = (ws.reshape(-1) / 512.0).to(cuda_device)
        y_dtype = torch.float32 if i % 2 else torch.bfloat16
        c = torch.empty((m, n), dtype=torch.int64, device=cuda_device)
        y = torch.empty((m, n), dtype=y_dtype, device=cuda_device)
        g = nat.GemmProblem()
        g.a_planes, g.lda, g.b_planes, g.ldb = a.planes.data_ptr(), a.ld, b.planes.data_ptr(), b.ld
        g.M, g.N, g.K, g.c, g.ldc = m, n, k, c.data_ptr(), n
        g.x_scale, g.w_scale, g.bias = cs.reshape(-1).data_ptr(), wsc.data_ptr(), None
        g.y, g.y_dtype, g.ldy = y.data_ptr(), nat.dtype_code(y_dtype), n
        probs.append(g)
        keep += [a, b, c, y, cs, wsc]
        refs.append((x, w, ws, c, y))
    arr = (nat.GemmProblem * len(probs))(*probs)
    nat.check("grouped", nat.lib().ima_int_gemm_grouped(ctypes.byref(arr), len(probs), nat.IMA_SCHEME_DIGITS3,
                                                       nat.stream_of(cuda_device)))
    torch.cuda.synchronize()
    for x, w, ws, c, y in refs:
        c_ref, y_ref, _ = oracle.codebook_linear(x, w, ws)
        assert torch.equal(c.cpu(), c_ref)
        assert torch.equal(y.cpu().to(torch.float32).view(torch.int32), y_ref.to(y.dtype).to(torch.float32).view(torch.int32))
    _assert_status_clean(cuda_device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m,k", [(1, 1), (12, 903), (33, 64), (130, 257), (300, 896)])
def test_fused_quantise_and_stage_equals_two_launches(cuda_device, dtype, m, k):
    """ima_hawkeye_quantize_prepare writes the same scale, codes and staged operand bytes as
    ima_quantize_per_token followed by ima_hawkeye_prepare, including rows with NaN, +-inf,
    all zeros and subnormal values, a ragged K, padding rows up to the operand pitch and a
    row stride wider than K."""
    x = synthetic.student_t_activations(m, k + 5, seed=41 + m + k, outlier_fraction=0.02, dtype=torch.float32)
    if m >= 8:
        x[1, k // 2] = float("nan")
        x[2, 0] = float("inf")
        x[3, k - 1] = float("-inf")
        x[4] = 0.0
        x[5] = x[5] * 1e-38
    xd = x.to(dtype).to(cuda_device)[:, :k]            # row stride k + 5
    q_ref, s_ref, *_ = codebook.per_token_fp8(xd)
    ref_op = hawkeye.HawkeyeOperand(q_ref)
    op, scale, q = hawkeye.quantize_and_stage(xd, codes=True)
    torch.cuda.synchronize()
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
    assert torch.equal(scale.view(torch.int32), s_ref.view(torch.int32))
    assert torch.equal(op.buffer, ref_op.buffer)
    op2, scale2, none = hawkeye.quantize_and_stage(xd)
    assert none is None and torch.equal(op2.buffer, ref_op.buffer)
    assert torch.equal(scale2.view(torch.int32), scale.view(torch.int32))


def test_hawkeye_linear_forward_uses_the_fused_staging(cuda_device):
    """HawkeyeLinear.forward (fused quantise + stage, then the replay) equals the reference
    composition _fp8_per_token -> hawkeye_fp8_sum on 3-D input with a bias."""
    w, ws = synthetic.normal_fp8_weights(70, 300, seed=77)
    bias = torch.randn(70, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    lin = students.HawkeyeLinear(w.to(cuda_device), ws.to(cuda_device), bias.to(cuda_device))
    x = synthetic.student_t_activations(2 * 19, 300, seed=5, outlier_fraction=0.02).reshape(2, 19, 300).to(cuda_device)
    y = lin(x)
    xq, xsc, *_ = codebook.per_token_fp8(x)
    ref, _ = hawkeye.hawkeye_fp8_sum(xq, xsc, w.to(cuda_device), ws.to(cuda_device))
    ref = (ref + bias.to(cuda_device).to(ref.dtype)).to(x.dtype).reshape(2, 19, 70)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


def test_grouped_gemm_writes_every_copy_of_y(cuda_device):
    """ima_int_gemm_grouped_copies stores each problem's y into every further destination it
    is given (here local buffers standing in for other GPUs' gathered buffers): 16-byte
    aligned copies through the staged vector path, a copy at an odd element offset through
    the element path, problems without copies unchanged; c and y equal the plain grouped
    launch bit for bit, and the copies equal y."""
    import ctypes

    probs, copies, keep, outs = [], [], [], []
    for i in range(5):
        m, n, k = 40 + 70 * i, 24 + 56 * i, 64 + 200 * i
        x = synthetic.student_t_activations(m, k, seed=70 + i)
        w, ws = synthetic.normal_fp8_weights(n, k, seed=170 + i)
        _q, _xs, _cb, cs, a = codebook.per_token_fp8(x.to(cuda_device), codebook=True, planes=True)
        b, _ = codebook.codebook_planes_from_fp8(w.to(cuda_device))
        wsc = (ws.reshape(-1) / 512.0).to(cuda_device)
        c = torch.empty((m, n), dtype=torch.int64, device=cuda_device)
        y = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
        g = nat.GemmProblem()
        g.a_planes, g.lda, g.b_planes, g.ldb = a.planes.data_ptr(), a.ld, b.planes.data_ptr(), b.ld
        g.M, g.N, g.K, g.c, g.ldc = m, n, k, c.data_ptr(), n
        g.x_scale, g.w_scale, g.bias = cs.reshape(-1).data_ptr(), wsc.data_ptr(), None
        g.y, g.y_dtype, g.ldy = y.data_ptr(), nat.IMA_DTYPE_BF16, n
        cp = nat.GemmYCopies()
        dests = []
        for d in range((0, 1, 2, 3, 8)[i]):
            buf = torch.full((m * n + 8,), -1, dtype=torch.int16, device=cuda_device)
            off = 1 if (i == 3 and d == 1) else 0           # odd element offset: not 16-byte aligned
            cp.y[d] = buf.data_ptr() + 2 * off
            dests.append((buf, off))
        probs.append(g)
        copies.append(cp)
        keep += [a, b, cs, wsc]
        outs.append((c, y, dests, m, n))
    arr = (nat.GemmProblem * len(probs))(*probs)
    carr = (nat.GemmYCopies * len(copies))(*copies)
    lib = nat.lib()
    nat.check("copies", lib.ima_int_gemm_grouped_copies(ctypes.byref(arr), ctypes.byref(carr), len(probs),
                                                       nat.IMA_SCHEME_DIGITS3, nat.stream_of(cuda_device)))
    torch.cuda.synchronize()
    first = [(c.clone(), y.clone()) for c, y, _d, _m, _n in outs]
    nat.check("plain", lib.ima_int_gemm_grouped(ctypes.byref(arr), len(probs), nat.IMA_SCHEME_DIGITS3,
                                               nat.stream_of(cuda_device)))
    torch.cuda.synchronize()
    for (c0, y0), (c, y, dests, m, n) in zip(first, outs):
        assert torch.equal(c0, c) and torch.equal(y0.view(torch.int16), y.view(torch.int16))
        for buf, off in dests:
            assert torch.equal(buf[off:off + m * n].view(m, n), y.view(torch.int16))
            assert bool((buf[:off] == -1).all()) and bool((buf[off + m * n:] == -1).all())
    _assert_status_clean(cuda_device)
    # copies of a y that is not written are refused
    arr[1].y = None
    assert lib.ima_int_gemm_grouped_copies(ctypes.byref(arr), ctypes.byref(carr), len(probs),
                                           nat.IMA_SCHEME_DIGITS3, nat.stream_of(cuda_device)) != 0


def test_copy_many_moves_every_byte(cuda_device):
    """ima_copy_many: many copies of ragged sizes (tails shorter than a 16-byte lane and
    than a 512-byte unit) in one launch on a few blocks; every destination equals its
    source and nothing around it is touched; misaligned pointers are refused."""
    import ctypes

    g = torch.Generator().manual_seed(5)
    sizes = [0, 1, 15, 16, 17, 511, 512, 513, 4096 + 48, 100_000 + 7, 3 * 1024 * 1024 + 16]
    srcs, dsts = [], []
    descs = (nat.CopyDesc * len(sizes))()
    for i, nbytes in enumerate(sizes):
        src = torch.randint(0, 256, (nbytes + 16,), generator=g, dtype=torch.int64).to(torch.uint8).to(cuda_device)
        dst = torch.full((nbytes + 32,), 0xA5, dtype=torch.uint8, device=cuda_device)
        descs[i].dst, descs[i].src, descs[i].bytes = dst.data_ptr() + 16, src.data_ptr(), nbytes
        srcs.append(src)
        dsts.append(dst)
    lib = nat.lib()
    for ctas in (1, 3, 16):
        for d in dsts:
            d.fill_(0xA5)
        nat.check("copy_many", lib.ima_copy_many(ctypes.byref(descs), len(sizes), ctas, nat.stream_of(cuda_device)))
        torch.cuda.synchronize()
        for nbytes, src, dst in zip(sizes, srcs, dsts):
            assert torch.equal(dst[16:16 + nbytes], src[:nbytes])
            assert bool((dst[:16] == 0xA5).all()) and bool((dst[16 + nbytes:] == 0xA5).all())
    descs[3].dst = dsts[3].data_ptr() + 8
    assert lib.ima_copy_many(ctypes.byref(descs), len(sizes), 4, nat.stream_of(cuda_device)) != 0

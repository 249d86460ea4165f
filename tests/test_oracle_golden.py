"""The CPU oracle against fixtures produced by the reference itself (tests/golden/).

These pin the oracle before it is trusted as the checker of the CUDA kernels.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import golden_cases, json_field, load_golden


def _bf16_from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def _fp8(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b)).view(torch.float8_e4m3fn)


def test_quantiser_matches_reference():
    g = load_golden("quantize")
    x = _bf16_from_bits(g["x_bf16"])
    q, scale = oracle.per_token_fp8(x)
    assert np.array_equal(q.view(torch.uint8).numpy(), g["q"])
    assert np.array_equal(scale.numpy().view(np.uint32), g["scale"].view(np.uint32))
    assert np.array_equal(oracle.fp8_codebook(q).numpy(), g["codebook"])
    q32, s32 = oracle.per_token_fp8(torch.from_numpy(g["x_f32"]))
    assert np.array_equal(q32.view(torch.uint8).numpy(), g["q_f32"])
    assert np.array_equal(s32.numpy().view(np.uint32), g["scale_f32"].view(np.uint32))


def e4m3_rne_bits(f: np.ndarray) -> np.ndarray:
    """Restatement (numpy) of the quantiser kernel's fp32 -> e4m3fn conversion
    (csrc/ima_common.cuh ima_f32_to_e4m3), checked here against torch's cast."""
    bits = f.astype(np.float32).view(np.uint32)
    sign = (bits >> 24) & 0x80
    a = bits & 0x7FFFFFFF
    out = np.zeros_like(a)
    big = a >= 0x43F00000
    small = (~big) & (a < 0x3C800000)
    normal = ~(big | small)
    out[big] = 0x7F
    v = a[small].view(np.float32) * np.float32(512.0)
    out[small] = np.rint(v).astype(np.uint32)  # rint is round-half-even
    an = a[normal]
    e = (an >> 23) - 120
    m = an & 0x7FFFFF
    q = (e << 3) | (m >> 20)
    rem = m & 0xFFFFF
    q = q + ((rem > 0x80000) | ((rem == 0x80000) & ((q & 1) == 1))).astype(np.uint32)
    out[normal] = q
    return (out | sign).astype(np.uint8)


def test_e4m3_cast_restatement_matches_torch():
    g = load_golden("e4m3_cast")
    assert np.array_equal(e4m3_rne_bits(g["f32"]), g["e4m3"])


def test_e4m3_cast_restatement_random_bits():
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2**32, size=400_000, dtype=np.uint64).astype(np.uint32)
    f = bits.view(np.float32)
    f = f[np.isfinite(f)]
    mine = e4m3_rne_bits(f)
    ref = torch.from_numpy(f.copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    nan_code = (ref & 0x7F) == 0x7F
    assert np.array_equal(mine[~nan_code], ref[~nan_code])
    assert np.all((mine[nan_code] & 0x7F) == 0x7F)


@pytest.mark.parametrize("case", ["ref_test_4x3", "c16x96x40", "c7x200x33", "c3x32x17"])
def test_codebook_linear_matches_reference(case):
    d = golden_cases(load_golden("codebook"))[case]
    x = torch.from_numpy(d["x"])
    if bool(d["x_is_bf16"]):
        x = x.to(torch.bfloat16)
    bias = _bf16_from_bits(d["bias_bf16"]) if "bias_bf16" in d else None
    c, y, out = oracle.codebook_linear(x, _fp8(d["w"]), torch.from_numpy(d["w_scale"]), bias)
    assert np.array_equal(c.numpy(), d["c"])
    assert np.array_equal(y.numpy().view(np.uint32), d["y"].view(np.uint32))
    assert np.array_equal(out.to(torch.float32).numpy().view(np.uint32), d["out_f32"].view(np.uint32))


HAWKEYE_CASES = sorted(golden_cases(load_golden("hawkeye")).keys())


@pytest.mark.parametrize("case", HAWKEYE_CASES)
def test_hawkeye_oracle_matches_reference(case):
    d = golden_cases(load_golden("hawkeye"))[case]
    y = oracle.hawkeye(_fp8(d["x"]), torch.from_numpy(d["x_scale"]), _fp8(d["w"]), torch.from_numpy(d["w_scale"]))
    assert np.array_equal(y.numpy().view(np.uint32), d["y_f32"].view(np.uint32))
    assert np.array_equal(y.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16), d["exact_bf16"])
    stats = json_field(d["exact_stats"])
    mine = oracle.class_count_stats(_fp8(d["x"]), _fp8(d["w"]), class_chunk=32, packed_count_lanes=1)
    assert mine == stats


def test_hawkeye_oracle_row_subset():
    d = golden_cases(load_golden("hawkeye"))["c0like8x896x32"]
    rows = np.array([5, 0, 7], dtype=np.int64)
    y = oracle.hawkeye(_fp8(d["x"]), torch.from_numpy(d["x_scale"]), _fp8(d["w"]), torch.from_numpy(d["w_scale"]),
                       rows=rows)
    assert np.array_equal(y.numpy().view(np.uint32), d["y_f32"][rows].view(np.uint32))


def _class_count_cases():
    try:
        return sorted(golden_cases(load_golden("class_counts")).keys())
    except FileNotFoundError:
        return []


@pytest.mark.parametrize("case", [c for c in _class_count_cases() if c != "packing"])
def test_class_count_stats_and_output_match_reference(case):
    d = golden_cases(load_golden("class_counts"))[case]
    params = json_field(d["params"])
    x, w = _fp8(d["x"]), _fp8(d["w"])
    assert oracle.class_count_stats(x, w, **params) == json_field(d["stats"])
    y = oracle.hawkeye(x, torch.ones(x.shape[0], 1), w, torch.ones(w.shape[0]))
    assert np.array_equal(y.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16), d["y_bf16"])


def test_freivalds_oracle_on_reference_test_matrices():
    g = load_golden("freivalds")
    a, b, c = (torch.from_numpy(g[k]) for k in ("prime_a", "prime_b", "prime_c"))
    assert np.array_equal(oracle.int_gemm(a, b).numpy(), g["prime_c"])
    for r in g["prime_vectors"]:
        rt = torch.from_numpy(r)
        assert oracle.freivalds_mismatch_rows(a, b, c, rt) == 0
        # the reference's exact big-integer identity holds as well
        assert oracle.exact_matvec(a.tolist(), oracle.exact_matvec(b.tolist(), r.tolist())) == \
            oracle.exact_matvec(c.tolist(), r.tolist())
    bad = c.clone()
    bad[0, 0] += 1
    assert oracle.freivalds_mismatch_rows(a, b, bad, torch.from_numpy(g["prime_vectors"][0])) == 1
    a2, b2, c2 = (torch.from_numpy(g[k]) for k in ("cb_a", "cb_b", "cb_c"))
    assert np.array_equal(oracle.int_gemm(a2, b2).numpy(), g["cb_c"])
    r = torch.randint(0, 1 << 20, (b2.shape[1],), generator=torch.Generator().manual_seed(1))
    assert oracle.freivalds_mismatch_rows(a2, b2, c2, r) == 0
    bad = c2.clone()
    bad[3, 5] -= 7
    assert oracle.freivalds_mismatch_rows(a2, b2, bad, r) == (1 if int(r[5]) != 0 else 0)


def _balanced_digits(v: np.ndarray, count: int) -> list[np.ndarray]:
    """Balanced base-128 digits as the plane kernels write them (csrc/quantize.cu)."""
    out = []
    w = v.astype(np.int64)
    for _ in range(count - 1):
        d = ((w + 64) & 127) - 64
        out.append(d)
        w = (w - d) >> 7
    out.append(w)
    return out


@pytest.mark.parametrize("count,lo,hi", [(3, -1_064_960, 1_064_961), (5, -(2**31), 2**31)])
def test_digit_shift_recombination_is_exact(count, lo, hi):
    """C = sum_s 2^(7 s) sum_{i+j=s} A_i B_j^T, the GEMM epilogue's recombination,
    checked in exact integers; every digit fits int8."""
    rng = np.random.default_rng(count)
    a = rng.integers(lo, hi, size=(7, 50), dtype=np.int64)
    b = rng.integers(lo, hi, size=(9, 50), dtype=np.int64)
    a[0, :3] = [lo, hi - 1, 0]
    da, db = _balanced_digits(a, count), _balanced_digits(b, count)
    assert all(np.all((d >= -128) & (d <= 127)) for d in da + db)
    c = np.zeros((7, 9), dtype=object)
    for i in range(count):
        for j in range(count):
            c = c + (da[i].astype(object) @ db[j].T.astype(object)) * (2 ** (7 * (i + j)))
    assert np.array_equal(c, a.astype(object) @ b.T.astype(object))


def test_gfloat_known_answers_of_the_reference_tests():
    """tests/test_hawkeye_freivalds.py:28-46 of the reference, against the oracle's gfloat
    conversion: a zero significand is +0, and the smallest nonzero one at the zero exponent
    stays a tiny finite value instead of wrapping to a large one."""
    zero = oracle.gfloat_to_float32(torch.tensor([False]), torch.tensor([-139]), torch.tensor([0]))
    assert zero.item() == 0.0
    tiny = oracle.gfloat_to_float32(torch.tensor([False]), torch.tensor([-139]), torch.tensor([1]))
    assert torch.isfinite(tiny).all() and tiny.abs().item() < 1e-35


def test_gfloat_conversion_matches_reference_sweep():
    """The oracle's gfloat -> fp32 conversion equals the reference's on every exponent from
    -170 to 149, both signs, structured and random significands (fixture made by the
    reference's own function)."""
    g = load_golden("gfloat")
    y = oracle.gfloat_to_float32(torch.from_numpy(g["sign"].astype(np.int32)), torch.from_numpy(g["exponent"]),
                                 torch.from_numpy(g["significand"]))
    assert np.array_equal(y.numpy().view(np.int32), g["f32_bits"])


def _int32_linear_case(d):
    dtype = getattr(torch, str(d["x_dtype"]))
    x = torch.from_numpy(d["x_f32"]).to(dtype)
    weight = torch.from_numpy(d["weight"])
    bias = torch.from_numpy(d["bias"]) if "bias" in d else None
    return x, weight, bias


@pytest.mark.parametrize("case", sorted(golden_cases(load_golden("int32_linear")).keys()))
def test_int32_linear_oracle_matches_the_reference_run(case):
    """oracle.int32_linear against the reference's own Int32Linear (its Triton kernels run
    by the interpreter on full-range int32 operands): quantised operands, the int64 product
    and the module output, bit for bit."""
    d = golden_cases(load_golden("int32_linear"))[case]
    x, weight, bias = _int32_linear_case(d)
    out = oracle.int32_linear(x, weight, bias)
    assert out.dtype == x.dtype
    assert torch.equal(out.to(torch.float32), torch.from_numpy(d["y_f32"]))
    k = weight.shape[1]
    qmax = float(min((1 << 31) - 1, int(math.sqrt(((1 << 62) - 1) / k))))
    assert qmax == float(d["qmax"])
    c = oracle.int_gemm(torch.from_numpy(d["x_i32"]), torch.from_numpy(d["weight_t"]))
    assert torch.equal(c, torch.from_numpy(d["c"]))

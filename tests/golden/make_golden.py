"""Generate the golden fixtures of tests/golden/ by running the reference itself.

Run in a container that has the reference checkout (read-only is fine):
    python tests/golden/make_golden.py /path/to/int-model-approximation [section ...]

It imports the reference package from <checkout>/src with TRITON_INTERPRET=1, so the
reference's own Triton kernels execute on CPU tensors, and with
`_require_cuda_tensor` patched out exactly as the reference's tests do
(tests/test_real_integer_gemms.py:45-46).  The reference only runs on CUDA tensors, where
torch evaluates a tensor divided by a Python number as the tensor times the number's fp32
reciprocal; torch on the CPU divides, which changes the last bit of about a third of the
per-token scales `amax / 448.0`.  The generator therefore runs each section under
`_CudaScalarDivision`, which applies the CUDA rule to exactly that operation (a floating
tensor divided by a Python number) and leaves every other op to the CPU; the synthetic
inputs drawn inside a section are stored beside the outputs, so the rule changes only which
inputs were drawn.  Hawkeye kernels are launched directly
with an fp32 output tensor (the interpreter truncates bf16 stores; the bf16 result is
the RNE cast of that fp32 value, which is what a CUDA bf16 store does).  The packed
class-count replay kernels are launched the same way (their wrappers only refuse
non-CUDA tensors before launching).  Nothing here runs on the GPU box; the fixtures
it writes are plain .npz files read by the tests.
"""

from __future__ import annotations

import ast
import json
import os
import sys
import time

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from int_model_approximation_b200 import synthetic  # noqa: E402


class _CudaScalarDivision(torch.overrides.TorchFunctionMode):
    """tensor / python_number as torch computes it on CUDA tensors: RN(t * RN(1 / number)) in
    fp32 (the op math type of fp32, bf16 and fp16), cast back to the tensor's dtype."""

    DIVS = {torch.Tensor.__truediv__, torch.Tensor.div, torch.div, torch.true_divide}

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if (func in self.DIVS and len(args) == 2 and not kwargs and isinstance(args[0], torch.Tensor)
                and isinstance(args[1], (int, float)) and not isinstance(args[1], bool)
                and args[0].dtype in (torch.float32, torch.bfloat16, torch.float16)):
            t = args[0]
            inv = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(float(args[1]), dtype=torch.float32)
            return (t.to(torch.float32) * inv).to(t.dtype)
        return func(*args, **kwargs)


def _load_reference(checkout: str):
    sys.path.insert(0, os.path.join(checkout, "src"))
    import int_model_approximation.__main__ as entry  # noqa: E402
    import int_model_approximation.hawkeye as hk  # noqa: E402
    import int_model_approximation.hawkeye_freivalds as hf  # noqa: E402

    entry._require_cuda_tensor = lambda _x, _label: None  # the reference tests' own idiom
    return entry, hk, hf


def _bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


def _u8(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().view(torch.uint8).numpy()


def _cpu_raw_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return a.to(torch.int64) @ b.to(torch.int64)


# ---------------------------------------------------------------------------
def gen_quantize(entry) -> dict:
    rows = []
    x = synthetic.student_t_activations(12, 96, seed=11)
    rows.append(x)
    special = torch.zeros((6, 96), dtype=torch.float32)
    special[1] = 1e-30                                  # scale clamps to 1e-12
    special[2] = torch.linspace(-3e4, 3e4, 96)          # large values
    special[3, ::3] = 1.0                               # sparse row
    special[4] = torch.linspace(-1, 1, 96) * 448.0      # exactly the e4m3 range
    g = torch.Generator().manual_seed(5)
    special[5] = torch.randn(96, generator=g) * 1e-3
    rows.append(special.to(torch.bfloat16))
    x = torch.cat(rows, 0)
    q, scale = entry._per_token_fp8(x)
    cb = entry._fp8_e4m3_to_int32(q)
    cb2, code_scale = entry._per_token_fp8_int32(x)
    assert torch.equal(cb, cb2)
    x32 = synthetic.student_t_activations(8, 64, seed=12, dtype=torch.float32)
    q32, s32 = entry._per_token_fp8(x32)
    return dict(
        x_bf16=_bf16_bits(x), q=_u8(q), scale=scale.numpy(), codebook=cb.numpy(), code_scale=code_scale.numpy(),
        x_f32=x32.numpy(), q_f32=_u8(q32), scale_f32=s32.numpy(),
    )


def gen_e4m3_cast() -> dict:
    """torch's fp32 -> e4m3fn cast on boundary and random bit patterns."""
    vals = []
    # every e4m3 magnitude and the midpoints around it
    grid = torch.arange(0, 127, dtype=torch.uint8).view(torch.float8_e4m3fn).to(torch.float32)
    mids = (grid[1:] + grid[:-1]) / 2
    vals += [grid, mids, torch.nextafter(mids, torch.full_like(mids, 1e9)),
             torch.nextafter(mids, torch.full_like(mids, -1e9))]
    vals.append(torch.tensor([448.0, 456.0, 464.0, 463.99997, 464.00003, 472.0, 479.99997, 480.0, 1e9,
                              float("inf"), 2 ** -6, 2 ** -7, 2 ** -9, 2 ** -10, 2 ** -10 * 1.0000001,
                              3 * 2 ** -11, 1e-40, 0.0]))
    g = torch.Generator().manual_seed(7)
    vals.append(torch.randn(20000, generator=g) * 100)
    vals.append(torch.randn(20000, generator=g) * 0.01)
    v = torch.cat(vals)
    v = torch.cat([v, -v])
    return dict(f32=v.numpy(), e4m3=_u8(v.to(torch.float8_e4m3fn)))


def gen_codebook(entry) -> dict:
    out = {}
    # the reference test's hand-written FP8 weight (tests/test_real_integer_gemms.py:288-321)
    w = torch.tensor([[0.125, -0.5, 1.0], [-1.5, 0.25, 2.0], [3.0, -0.75, 0.5], [-2.5, 1.5, -0.125]],
                     dtype=torch.float32).to(torch.float8_e4m3fn)
    x = torch.tensor([[0.25, -1.5, 2.0], [3.0, -0.75, 0.125]], dtype=torch.float32)
    cases = [("ref_test_4x3", x, w, torch.ones(4, 1), None)]
    for name, (m, k, n, seed) in {"c16x96x40": (16, 96, 40, 21), "c7x200x33": (7, 200, 33, 22),
                                  "c3x32x17": (3, 32, 17, 23)}.items():
        xx = synthetic.student_t_activations(m, k, seed=seed)
        ww, ws = synthetic.normal_fp8_weights(n, k, seed=seed + 1)
        bias = torch.randn(n, generator=torch.Generator().manual_seed(seed + 2)).to(torch.bfloat16)
        cases.append((name, xx, ww, ws, bias))
    for name, xx, ww, ws, bias in cases:
        layer = entry.CodebookLinear(ww, ws, bias)
        x_i32, x_scale = entry._per_token_fp8_int32(xx)
        c = entry._int32_raw_matmul(x_i32, layer.weight_t)
        y = entry._int32_matmul(x_i32, layer.weight_t, x_scale, layer.weight_scale)
        mod_out = layer(xx)
        out[f"{name}/x"] = xx.to(torch.float32).numpy()
        out[f"{name}/x_is_bf16"] = np.array(xx.dtype == torch.bfloat16)
        out[f"{name}/w"] = _u8(ww)
        out[f"{name}/w_scale"] = ws.numpy()
        if bias is not None:
            out[f"{name}/bias_bf16"] = _bf16_bits(bias)
        out[f"{name}/c"] = c.numpy()
        out[f"{name}/y"] = y.numpy()
        out[f"{name}/out_f32"] = mod_out.to(torch.float32).numpy()
    return out


def gen_int32_linear(entry) -> dict:
    """The reference's Int32Linear (__main__.py:390-418: per-row / per-token int32 quantisers
    with qmax = floor(sqrt((2^62 - 1) / K)), _int32_raw_matmul / _int32_matmul through the
    Triton kernels, fp32 bias, cast back to x.dtype) on full-range int32 operands."""
    out = {}
    cases = {
        "k300_bf16": (2 * 3, 300, 40, torch.bfloat16, True, 41),
        "k37_f32": (5, 37, 24, torch.float32, False, 42),
        "k2_f16": (4, 2, 5, torch.float16, True, 43),
        "k896_bf16": (3, 896, 17, torch.bfloat16, True, 44),
    }
    for name, (m, k, n, dtype, with_bias, seed) in cases.items():
        g = torch.Generator().manual_seed(seed)
        weight = (torch.randn(n, k, generator=g) * 0.05).to(torch.float32)
        bias = (torch.randn(n, generator=g) * 0.1).to(torch.float32) if with_bias else None
        x = synthetic.student_t_activations(m, k, seed=seed + 1, outlier_fraction=0.02, dtype=dtype)
        if name == "k300_bf16":
            x = x.reshape(2, 3, k)
        layer = entry.Int32Linear(weight, bias)
        x_i32, x_scale = entry._per_token_int32(x, layer.qmax)
        c = entry._int32_raw_matmul(x_i32, layer.weight_t)
        y = layer(x)
        out[f"{name}/x_f32"] = x.to(torch.float32).numpy()
        out[f"{name}/x_dtype"] = np.array(str(dtype).replace("torch.", ""))
        out[f"{name}/weight"] = weight.numpy()
        if bias is not None:
            out[f"{name}/bias"] = bias.numpy()
        out[f"{name}/qmax"] = np.array(layer.qmax)
        out[f"{name}/weight_t"] = layer.weight_t.numpy()
        out[f"{name}/weight_scale"] = layer.weight_scale.numpy()
        out[f"{name}/x_i32"] = x_i32.numpy()
        out[f"{name}/x_scale"] = x_scale.numpy()
        out[f"{name}/c"] = c.numpy()
        out[f"{name}/y_f32"] = y.to(torch.float32).numpy()
    return out


def _hawkeye_kernel_fp32(hk, x_fp8, x_scale, w_fp8, w_scale, block_m=4, block_n=32):
    import triton

    m, k = x_fp8.shape
    n = w_fp8.shape[0]
    out = torch.empty((m, n), dtype=torch.float32)
    hk._hawkeye_fp8_sum_kernel[(triton.cdiv(m, block_m), triton.cdiv(n, block_n))](
        x_fp8.contiguous().view(torch.uint8), x_scale.reshape(-1).contiguous(),
        w_fp8.contiguous().view(torch.uint8), w_scale.reshape(-1).contiguous(), out,
        m, n, k, 32, 14, -139, block_m=block_m, block_n=block_n, num_warps=4,
    )
    return out


def _special_bytes(rows: int, k: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    b = torch.randint(0, 256, (rows, k), generator=g, dtype=torch.int64).to(torch.uint8)
    # sprinkle zeros, negative zeros, subnormals, NaN codes and extremes
    specials = torch.tensor([0x00, 0x80, 0x01, 0x81, 0x07, 0x87, 0x7F, 0xFF, 0x7E, 0xFE, 0x08, 0x88],
                            dtype=torch.uint8)
    idx = torch.randint(0, rows * k, (rows * k // 4,), generator=g)
    b.view(-1)[idx] = specials[torch.randint(0, specials.numel(), (idx.numel(),), generator=g)]
    return b.view(torch.float8_e4m3fn)


def hawkeye_cases() -> list:
    cases = []
    g = torch.Generator().manual_seed(1)
    x = torch.randn((64, 32), generator=g).to(torch.float8_e4m3fn)
    w = torch.randn((128, 32), generator=g).to(torch.float8_e4m3fn)
    cases.append(("tile64x32x128", x, torch.ones(64, 1), w, torch.ones(128)))
    g = torch.Generator().manual_seed(4)
    x = torch.randn((64, 64), generator=g).to(torch.float8_e4m3fn)
    w = torch.randn((128, 64), generator=g).to(torch.float8_e4m3fn)
    cases.append(("tile64x64x128", x, torch.ones(64, 1), w, torch.ones(128)))
    xq, xs = synthetic.quantize_rows_e4m3(synthetic.student_t_activations(16, 80, seed=31).float())
    wq, ws = synthetic.normal_fp8_weights(24, 80, seed=32)
    cases.append(("ragged16x80x24", xq, xs, wq, ws))
    cases.append(("special12x96x40", _special_bytes(12, 96, 33), torch.rand(12, 1) + 0.5,
                  _special_bytes(40, 96, 34), torch.rand(40) + 0.5))
    xq, xs = synthetic.quantize_rows_e4m3(synthetic.student_t_activations(8, 896, seed=35).float())
    wq, ws = synthetic.normal_fp8_weights(32, 896, seed=36)
    cases.append(("c0like8x896x32", xq, xs, wq, ws))
    xq = torch.zeros((4, 33), dtype=torch.float8_e4m3fn)
    wq, ws = synthetic.normal_fp8_weights(8, 33, seed=37)
    cases.append(("zeros4x33x8", xq, torch.ones(4, 1), wq, ws))
    return cases


def gen_hawkeye(hk, hf) -> dict:
    out = {}
    for name, x, xs, w, ws in hawkeye_cases():
        t0 = time.time()
        y32 = _hawkeye_kernel_fp32(hk, x, xs, w, ws)
        exact, stats = hf.exact_hawkeye_fp8_sum(x, xs, w, ws, _cpu_raw_matmul, class_chunk=32, packed_count_lanes=1)
        # the reference's two Hawkeye paths agree bit for bit
        assert torch.equal(y32.to(torch.bfloat16).view(torch.int16), exact.view(torch.int16)), name
        out[f"{name}/x"] = _u8(x)
        out[f"{name}/x_scale"] = xs.to(torch.float32).numpy()
        out[f"{name}/w"] = _u8(w)
        out[f"{name}/w_scale"] = ws.to(torch.float32).numpy()
        out[f"{name}/y_f32"] = y32.numpy()
        out[f"{name}/exact_bf16"] = _bf16_bits(exact)
        out[f"{name}/exact_stats"] = np.array(json.dumps(stats.__dict__))
        print(f"  hawkeye {name}: {time.time() - t0:.1f}s", flush=True)
    return out


def _aligned_values(hf, a_exp, a_sig, b_class, max_exp, internal_width):
    """aligned(a, b, max_exp) of hawkeye_freivalds.py:517-530 for a [A] x b [G] grid -> [A, G, M, N]."""
    b_exp = torch.div(b_class, hf.SIGNED_SIG_BUCKETS, rounding_mode="floor") + 1
    b_sig = torch.remainder(b_class, hf.SIGNED_SIG_BUCKETS) - hf.SIGNED_SIG_OFFSET
    prod_exp = a_exp[:, None] + b_exp[None, :] - 14
    signed = a_sig[:, None] * b_sig[None, :]
    scaled = signed << (internal_width - 7)
    shift = (max_exp[None, None] - prod_exp[:, :, None, None]).clamp(0, 62)
    mag = torch.bitwise_right_shift(scaled.abs()[:, :, None, None], shift)
    aligned = torch.where(scaled[:, :, None, None] < 0, -mag, mag)
    return torch.where((b_class >= 0)[None, :, None, None], aligned, torch.zeros_like(aligned))


def _patch_packed_wrappers(hf):
    """The reference's packed replay kernels (K6 hawkeye_freivalds.py:464-545, K7 :707-790)
    refuse CPU tensors and are far too slow under the Triton interpreter; this torch
    restatement of their arithmetic is plugged into the reference's own control flow
    (class lists, chunking, packing and raw products all stay the reference's)."""

    def packed(contribution, packed_counts, packed_b_classes, a_chunk_exp, a_chunk_sig, max_exp, *, a_size,
               internal_width, class_chunk):
        lanes = int(packed_b_classes.shape[1])
        for lane in range(lanes):
            count = torch.bitwise_and(torch.bitwise_right_shift(packed_counts.to(torch.int64), lane * 6), 63)
            for a0 in range(0, a_size, 8):
                al = _aligned_values(hf, a_chunk_exp[a0:a0 + 8], a_chunk_sig[a0:a0 + 8], packed_b_classes[:, lane],
                                     max_exp, internal_width)
                contribution += (count[a0:a0 + 8] * al).sum(dim=(0, 1))

    def packed_group(contribution, packed_counts, packed_b_classes, a_chunk_exp, a_chunk_sig, max_exp, *,
                     group_lane, b_class_lanes, a_size, internal_width, class_chunk):
        for b_lane in range(b_class_lanes):
            lane = group_lane * b_class_lanes + b_lane
            count = torch.bitwise_and(torch.bitwise_right_shift(packed_counts.to(torch.int64), lane * 6), 63)
            for a0 in range(0, a_size, 8):
                al = _aligned_values(hf, a_chunk_exp[a0:a0 + 8], a_chunk_sig[a0:a0 + 8], packed_b_classes[:, b_lane],
                                     max_exp, internal_width)
                contribution += (count[a0:a0 + 8] * al).sum(dim=(0, 1))

    hf._add_packed_contribution_fused = packed
    hf._add_packed_group_contribution_fused = packed_group


def gen_class_counts(hf) -> dict:
    _patch_packed_wrappers(hf)
    out = {}
    cases = [
        ("lanes6_chunk32", 1, 64, 32, 128, dict(class_chunk=32, packed_count_lanes=6, packed_group_lanes=1)),
        ("lanes6_chunk512_g2", 4, 64, 64, 128, dict(class_chunk=512, packed_count_lanes=6, packed_group_lanes=2)),
        ("lanes3_chunk8", 41, 16, 80, 24, dict(class_chunk=8, packed_count_lanes=3, packed_group_lanes=1)),
        ("lanes6_chunk16_g3", 42, 12, 96, 20, dict(class_chunk=16, packed_count_lanes=6, packed_group_lanes=3)),
        ("unpacked_chunk4", 43, 10, 64, 12, dict(class_chunk=4, packed_count_lanes=1, packed_group_lanes=1)),
    ]
    for name, seed, m, k, n, params in cases:
        t0 = time.time()
        g = torch.Generator().manual_seed(seed)
        x = torch.randn((m, k), generator=g).to(torch.float8_e4m3fn)
        w = torch.randn((n, k), generator=g).to(torch.float8_e4m3fn)
        xs = torch.ones((m, 1))
        ws = torch.ones((n,))
        y, stats = hf.exact_hawkeye_fp8_sum(x, xs, w, ws, _cpu_raw_matmul, **params)
        out[f"{name}/x"] = _u8(x)
        out[f"{name}/w"] = _u8(w)
        out[f"{name}/y_bf16"] = _bf16_bits(y)
        out[f"{name}/stats"] = np.array(json.dumps(stats.__dict__))
        out[f"{name}/params"] = np.array(json.dumps(params))
        print(f"  class counts {name}: {time.time() - t0:.1f}s", flush=True)
    # count products of the packing helpers on small class matrices
    g = torch.Generator().manual_seed(50)
    a_cls = torch.randint(-1, 40, (6, 64), generator=g)
    b_cls = torch.randint(-1, 40, (9, 64), generator=g)
    a_classes = torch.unique(a_cls[a_cls >= 0])
    b_classes = torch.unique(b_cls[b_cls >= 0])
    packed, packed_b, lanes = hf._packed_group_class_chunk_product(
        a_cls, b_cls, a_classes, b_classes, _cpu_raw_matmul, products_per_group=32, packed_group_lanes=2,
        packed_count_lanes=6)
    out["packing/a_cls"] = a_cls.numpy()
    out["packing/b_cls"] = b_cls.numpy()
    out["packing/group2_counts"] = packed.contiguous().numpy()
    out["packing/group2_b_classes"] = packed_b.numpy()
    packed1, packed_b1 = hf._packed_class_chunk_product(a_cls[:, :32], b_cls[:, :32], a_classes, b_classes,
                                                        _cpu_raw_matmul, packed_count_lanes=3)
    out["packing/lanes3_counts"] = packed1.contiguous().numpy()
    out["packing/lanes3_b_classes"] = packed_b1.numpy()
    return out


def gen_gfloat(hf) -> dict:
    """The reference's gfloat -> fp32 conversion (hawkeye_freivalds.py:120-144) over every
    exponent from -170 to 149, both signs, and structured plus random significands."""
    sigs = [0, 1, 2, 3, 0x3FFF, 0x4000, 0x2000 << 10, 0x3FFF << 10, 0x7FFFFF, 0x800000, 0x800001, 0xFFFFFF,
            0x1000000, 0x1FFFFFF, 1 << 40, (1 << 62) - 1]
    g = torch.Generator().manual_seed(71)
    sigs += torch.randint(0, 1 << 24, (24,), generator=g).tolist()
    sign, exp, sig = torch.meshgrid(torch.tensor([0, 1]), torch.arange(-170, 150), torch.tensor(sigs, dtype=torch.int64),
                                    indexing="ij")
    sign, exp, sig = sign.reshape(-1), exp.reshape(-1).to(torch.int64), sig.reshape(-1)
    y = hf._gfloat_to_float32(sign.to(torch.bool), exp, sig)
    return dict(sign=sign.to(torch.int8).numpy(), exponent=exp.numpy(), significand=sig.numpy(),
                f32_bits=y.to(torch.float32).view(torch.int32).numpy())


def _test_matrices(checkout: str) -> tuple[list, list]:
    """The prime matrices of the reference's Freivalds test, read from its source."""
    path = os.path.join(checkout, "tests", "test_real_integer_gemms.py")
    tree = ast.parse(open(path).read())
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == "test_raw_int32_matmul_is_freivalds_verifiable":
            lists = [n for n in ast.walk(node) if isinstance(n, ast.Call) and getattr(n.func, "attr", "") == "tensor"]
            a = ast.literal_eval(lists[0].args[0])
            b = ast.literal_eval(lists[1].args[0])
            return a, b
    raise RuntimeError("reference Freivalds test not found")


def gen_freivalds(entry, checkout: str) -> dict:
    a, b = _test_matrices(checkout)
    at = torch.tensor(a, dtype=torch.int32)
    bt = torch.tensor(b, dtype=torch.int32)
    c = entry._int32_raw_matmul(at, bt)
    out = dict(prime_a=at.numpy(), prime_b=bt.numpy(), prime_c=c.numpy())
    # the test's three vectors over the output columns (tests/test_real_integer_gemms.py:83-87)
    n = bt.shape[1]
    vecs = [[1] + [0] * (n - 1), [1 if i % 2 == 0 else -1 for i in range(n)], [0 if i % 3 == 0 else 1 for i in range(n)]]
    out["prime_vectors"] = np.array(vecs, dtype=np.int64)
    # a larger codebook product at the edge of the codebook range
    x = synthetic.student_t_activations(9, 300, seed=61)
    w, ws = synthetic.normal_fp8_weights(14, 300, seed=62)
    x_i32, _ = entry._per_token_fp8_int32(x)
    w_i32 = entry._fp8_e4m3_to_int32(w).t().contiguous()
    out["cb_a"] = x_i32.numpy()
    out["cb_b"] = w_i32.numpy()
    out["cb_c"] = entry._int32_raw_matmul(x_i32, w_i32).numpy()
    return out


def main() -> None:
    checkout = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("IMA_REFERENCE_CHECKOUT", "")
    if not checkout or not os.path.isdir(checkout):
        raise SystemExit("usage: make_golden.py <reference checkout>")
    entry, hk, hf = _load_reference(checkout)
    sections = set(sys.argv[2:]) or {"quantize", "e4m3_cast", "codebook", "int32_linear", "freivalds", "hawkeye",
                                     "class_counts", "gfloat"}
    gens = {
        "quantize": lambda: gen_quantize(entry),
        "e4m3_cast": gen_e4m3_cast,
        "codebook": lambda: gen_codebook(entry),
        "int32_linear": lambda: gen_int32_linear(entry),
        "freivalds": lambda: gen_freivalds(entry, checkout),
        "hawkeye": lambda: gen_hawkeye(hk, hf),
        "class_counts": lambda: gen_class_counts(hf),
        "gfloat": lambda: gen_gfloat(hf),
    }
    t0 = time.time()
    for name, fn in gens.items():
        if name in sections:
            with _CudaScalarDivision():
                data = fn()
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **data)
            print(f"{name}.npz written", flush=True)
    print(f"fixtures written in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()

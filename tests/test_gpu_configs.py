"""Parity at the benchmark configurations' own shapes (2 and 4).

Every output row of the codebook GEMM and of the Hawkeye replay depends only on its own
token row (the per-token quantiser included), so a seeded sample of rows checked against
the CPU oracle is an exact check of those rows at the full shape; the GPU computes every
row.  Hawkeye at K = 18944 (the 7B down_proj) runs 592 groups through one accumulator,
the longest carried exponent range of any config.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from int_model_approximation_b200 import codebook, hawkeye, synthetic
from int_model_approximation_b200.pipeline import CodebookStack

pytestmark = pytest.mark.gpu

QWEN05B = synthetic.qwen_layer_shapes(896, 128, 4864)
QWEN7B = synthetic.qwen_layer_shapes(3584, 512, 18944)


def _rows(m: int, count: int, seed: int) -> np.ndarray:
    return np.sort(torch.randperm(m, generator=torch.Generator().manual_seed(seed))[:count].numpy())


def _hawkeye_rows_match(x_bf16, w, ws, rows):
    xq, xs, *_ = codebook.per_token_fp8(x_bf16)
    out, stats = hawkeye.hawkeye_fp8_sum(xq, xs, w, ws)
    ref = oracle.hawkeye(xq.cpu(), xs.cpu(), w.cpu(), ws.cpu(), rows=rows).to(torch.bfloat16)
    got = out[torch.from_numpy(rows).to(out.device)].cpu()
    assert stats.groups == (x_bf16.shape[1] + 31) // 32
    return torch.equal(got.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("index", range(7), ids=[s.name for s in QWEN05B])
def test_c2_hawkeye_every_linear_shape_sampled_rows(cuda_device, index):
    """Config 2: each of the seven 0.5B linear shapes at 16384 tokens with 0.1 % x50
    outliers; 16 sampled rows per shape against the oracle, bit for bit."""
    shape = QWEN05B[index]
    x, w, ws = synthetic.make_linear_inputs(2, index, shape, device=cuda_device)
    assert x.shape == (16384, shape.k)
    assert _hawkeye_rows_match(x, w, ws, _rows(16384, 16, index))


C4_CASES = [(s.name, 2048, s.n, s.k) for s in QWEN7B] + [("gate_proj_colshard", 16384, 18944 // 8, 3584)]


@pytest.mark.parametrize("name,m,n,k", C4_CASES, ids=[c[0] for c in C4_CASES])
def test_c4_hawkeye_every_linear_shape_sampled_rows(cuda_device, name, m, n, k):
    """Config 4: the seven 7B linear shapes at the per-GPU row count of an 8-GPU split
    (2048 tokens), plus the gate/up column shard (all 16384 tokens, 2368 columns); 8
    sampled rows per shape against the oracle.  down_proj has K = 18944 (592 groups)."""
    index = [c[0] for c in C4_CASES].index(name)
    shape = synthetic.LinearShape(name, n, k)
    x, w, ws = synthetic.make_linear_inputs(4, index, shape, tokens=m, device=cuda_device)
    assert _hawkeye_rows_match(x, w, ws, _rows(m, 8, 40 + index))


def _stack_parity(weights, xs, rows_per_linear: int, seed: int):
    """CodebookStack forward of every linear, then per linear: sampled rows of the int64
    product and of the bf16 output (bias added) against the oracle, and the Freivalds check
    passing; then one corrupted entry per product must be flagged."""
    tokens = xs[0].shape[0]
    stack = CodebookStack(weights, seed=seed)
    bufs = stack.allocate(tokens)
    stack.forward(xs, bufs)
    torch.cuda.synchronize()
    assert int(bufs["mismatch"].item()) == 0
    for i, (w, ws, bias) in enumerate(weights):
        rows = _rows(xs[i].shape[0], rows_per_linear, seed + i)
        sel = torch.from_numpy(rows)
        c_ref, _y, out_ref = oracle.codebook_linear(xs[i].cpu()[sel], w.cpu(), ws.cpu(),
                                                    None if bias is None else bias.cpu())
        dev_sel = sel.to(xs[i].device)
        assert torch.equal(bufs["c"][i][dev_sel].cpu(), c_ref), f"linear {i}: int64 product"
        assert torch.equal(bufs["y"][i][dev_sel].cpu().view(torch.int16), out_ref.view(torch.int16)), \
            f"linear {i}: bf16 output"
    expected = 0
    for i, lin in enumerate(stack.linears):
        row, col = (i * 37) % tokens, (i * 101) % lin.n
        bufs["c"][i][row, col] += 1
        expected += int(int(lin.r[col].item()) != 0)
    bufs["mismatch"].zero_()
    stack.verify(xs, bufs)
    torch.cuda.synchronize()
    assert int(bufs["mismatch"].item()) == expected > 0


def _bias(n: int, seed: int, device) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).to(device)


def test_c1_whole_stack_against_oracle(cuda_device):
    """Config 1: all 168 linears of the 0.5B shapes at 512 tokens through the grouped
    pipeline (one quantiser launch, three GEMM launches, one check launch), with biases;
    8 sampled rows of every linear's int64 product and bf16 output against the oracle."""
    shapes = synthetic.config_linears(1)
    assert len(shapes) == 168
    weights, xs = [], []
    for i, s in enumerate(shapes):
        x, w, ws = synthetic.make_linear_inputs(1, i, s, device=cuda_device)
        weights.append((w, ws, _bias(s.n, 5000 + i, cuda_device)))
        xs.append(x)
    _stack_parity(weights, xs, rows_per_linear=8, seed=11)


def test_c4_codebook_and_freivalds_every_linear_shape(cuda_device):
    """Config 4: the seven 7B linear shapes at the per-GPU shapes of an 8-GPU split (2048
    token rows, full N; gate/up also as the column shard: 16384 rows, 2368 columns) through
    the grouped pipeline: int64 products, bf16 outputs and the Freivalds check."""
    weights, xs = [], []
    for i, (name, m, n, k) in enumerate(C4_CASES):
        x, w, ws = synthetic.make_linear_inputs(4, i, synthetic.LinearShape(name, n, k), tokens=m, device=cuda_device)
        weights.append((w, ws, _bias(n, 6000 + i, cuda_device)))
        xs.append(x)
    # the stack runs every linear at one token count: the 2048-row shapes first, then the shard
    _stack_parity(weights[:7], xs[:7], rows_per_linear=6, seed=21)
    _stack_parity(weights[7:], xs[7:], rows_per_linear=6, seed=31)

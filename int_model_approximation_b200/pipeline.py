"""A model's worth of student linears prepared for repeated forwards.

`CodebookStack` holds every linear of a model in the codebook student form
(weights prepacked once into digit planes, a Freivalds vector per linear) and runs
one forward of all of them -- per-token quantisation, the exact int64 GEMM with the
fused rescale/bias/bf16 epilogue, and the Freivalds check of each int64 product --
entirely on the device, with no host synchronisation.  The sequence of launches can
be captured once into a CUDA graph and replayed.

`HawkeyeStack` does the same for the direct Hawkeye replay student.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat
from .codebook import DigitPlanes, codebook_planes_from_fp8, int_gemm
from .freivalds import freivalds_vector
from .hawkeye import HawkeyeOperand, hawkeye_replay


@dataclass
class PreparedLinear:
    n: int
    k: int
    w_fp8: torch.Tensor          # [N, K] e4m3
    w_planes: DigitPlanes        # Karatsuba planes of codebook(w)
    w_code_scale: torch.Tensor   # [N] fp32 = weight_scale / 512
    bias: torch.Tensor | None    # [N] fp32
    r: torch.Tensor              # [N] int64 Freivalds vector


class CodebookStack:
    def __init__(self, weights: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]], *, seed: int = 0):
        self.linears: list[PreparedLinear] = []
        for i, (w, ws, bias) in enumerate(weights):
            planes, _ = codebook_planes_from_fp8(w)
            self.linears.append(
                PreparedLinear(
                    n=int(w.shape[0]),
                    k=int(w.shape[1]),
                    w_fp8=w.contiguous(),
                    w_planes=planes,
                    w_code_scale=(ws.reshape(-1).to(torch.float32) / 512.0).contiguous(),
                    bias=None if bias is None else bias.reshape(-1).to(torch.float32).contiguous(),
                    r=freivalds_vector(int(w.shape[0]), seed * 100_003 + i + 7, device=w.device),
                )
            )
        self.device = weights[0][0].device

    def allocate(self, tokens: int) -> dict:
        """Per-forward buffers for `tokens` rows (reused by every forward / graph replay)."""
        dev = self.device
        bufs = dict(q=[], scale=[], planes=[], c=[], y=[], ws=[])
        for lin in self.linears:
            bufs["q"].append(torch.empty((tokens, lin.k), dtype=torch.uint8, device=dev))
            bufs["scale"].append(torch.empty((tokens,), dtype=torch.float32, device=dev))
            bufs["planes"].append(DigitPlanes.empty(tokens, lin.k, nat.IMA_SCHEME_KARATSUBA3, dev))
            bufs["c"].append(torch.empty((tokens, lin.n), dtype=torch.int64, device=dev))
            bufs["y"].append(torch.empty((tokens, lin.n), dtype=torch.bfloat16, device=dev))
            bufs["ws"].append(torch.empty((int(nat.lib().ima_freivalds_workspace_bytes(lin.k)) // 8,),
                                          dtype=torch.int64, device=dev))
        bufs["mismatch"] = torch.zeros((1,), dtype=torch.int32, device=dev)
        bufs["code_scale"] = [torch.empty((tokens,), dtype=torch.float32, device=dev) for _ in self.linears]
        return bufs

    def forward(self, xs: list[torch.Tensor], bufs: dict, *, check: bool = True) -> None:
        """One forward of every linear on activations xs[i] [tokens, K_i] (bf16).

        Writes bufs["c"][i] (exact int64 products), bufs["y"][i] (bf16 outputs) and
        accumulates failed Freivalds rows into bufs["mismatch"].  Launches only."""
        lib = nat.lib()
        dev = self.device
        stream = nat.stream_of(dev)
        for i, lin in enumerate(self.linears):
            x = xs[i]
            m = int(x.shape[0])
            q, scale, cs = bufs["q"][i], bufs["scale"][i], bufs["code_scale"][i]
            planes = bufs["planes"][i]
            nat.check("ima_quantize_per_token", lib.ima_quantize_per_token(
                x.data_ptr(), nat.dtype_code(x.dtype), m, lin.k, x.stride(0), q.data_ptr(), lin.k,
                scale.data_ptr(), None, lin.k, cs.data_ptr(), planes.planes.data_ptr(), planes.ld, stream))
            c, y = bufs["c"][i], bufs["y"][i]
            nat.check("ima_int_gemm", lib.ima_int_gemm(
                planes.planes.data_ptr(), planes.ld, lin.w_planes.planes.data_ptr(), lin.w_planes.ld, m, lin.n, lin.k,
                nat.IMA_SCHEME_KARATSUBA3, c.data_ptr(), lin.n, cs.data_ptr(), lin.w_code_scale.data_ptr(),
                nat.ptr(lin.bias), y.data_ptr(), nat.IMA_DTYPE_BF16, lin.n, stream))
            if check:
                nat.check("ima_freivalds_fp8", lib.ima_freivalds_fp8(
                    q.data_ptr(), lin.k, lin.w_fp8.data_ptr(), lin.k, c.data_ptr(), lin.n, lin.r.data_ptr(), m, lin.n,
                    lin.k, bufs["ws"][i].data_ptr(), bufs["mismatch"].data_ptr(), stream))

    @staticmethod
    def kernels_per_linear(check: bool = True) -> int:
        return 4 if check else 2   # quantise, GEMM (+ Freivalds: B r pass, row pass)


class HawkeyeStack:
    def __init__(self, weights: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]]):
        self.weights = [(w.contiguous(), ws.reshape(-1).to(torch.float32).contiguous()) for w, ws, _b in weights]
        self.w_ops = [HawkeyeOperand(w) for w, _ in self.weights]
        self.device = weights[0][0].device

    def allocate(self, tokens: int) -> dict:
        dev = self.device
        bufs = dict(q=[], scale=[], xop=[], y=[])
        lib = nat.lib()
        for w, _ in self.weights:
            n, k = w.shape
            bufs["q"].append(torch.empty((tokens, k), dtype=torch.uint8, device=dev))
            bufs["scale"].append(torch.empty((tokens,), dtype=torch.float32, device=dev))
            bufs["xop"].append(torch.empty((int(lib.ima_hawkeye_operand_bytes(tokens, k)),), dtype=torch.uint8,
                                           device=dev))
            bufs["y"].append(torch.empty((tokens, n), dtype=torch.bfloat16, device=dev))
        return bufs

    def forward(self, xs: list[torch.Tensor], bufs: dict) -> None:
        lib = nat.lib()
        stream = nat.stream_of(self.device)
        for i, ((w, ws), wop) in enumerate(zip(self.weights, self.w_ops)):
            x = xs[i]
            m, k = int(x.shape[0]), int(x.shape[1])
            n = int(w.shape[0])
            q, scale, xop, y = bufs["q"][i], bufs["scale"][i], bufs["xop"][i], bufs["y"][i]
            nat.check("ima_quantize_per_token", lib.ima_quantize_per_token(
                x.data_ptr(), nat.dtype_code(x.dtype), m, k, x.stride(0), q.data_ptr(), k, scale.data_ptr(), None,
                k, None, None, 16, stream))
            nat.check("ima_hawkeye_prepare", lib.ima_hawkeye_prepare(q.data_ptr(), m, k, k, xop.data_ptr(), stream))
            nat.check("ima_hawkeye_replay", lib.ima_hawkeye_replay(
                xop.data_ptr(), wop.buffer.data_ptr(), scale.data_ptr(), ws.data_ptr(), m, n, k, 32, 14, -139,
                y.data_ptr(), n, None, n, stream))

    @staticmethod
    def kernels_per_linear() -> int:
        return 3


__all__ = ["CodebookStack", "HawkeyeStack", "PreparedLinear", "hawkeye_replay", "int_gemm"]

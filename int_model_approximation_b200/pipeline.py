"""A model's worth of student linears prepared for repeated forwards.

`CodebookStack` holds every linear of a model in the codebook student form
(weights prepacked once into digit planes; per linear a Freivalds vector r and the
weight half of the check t = codebook(W)^T r, both fixed) and runs one forward of all
of them -- per-token quantisation, the exact int64 GEMM with the fused
rescale/bias/bf16 epilogue, and the Freivalds row check of every int64 product -- as
grouped launches (one quantiser launch, one GEMM launch per 64 linears, one Freivalds
launch for all products), entirely on the device and without host synchronisation.  The
three phases can be run (and captured into CUDA graphs) separately or together.

`HawkeyeStack` does the same for the direct Hawkeye replay student (quantise and stage,
then replays spread over side streams).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native as nat
from .codebook import DigitPlanes, codebook_planes_from_fp8
from .freivalds import freivalds_vector, weight_vector
from .hawkeye import HawkeyeOperand


@dataclass
class PreparedLinear:
    n: int
    k: int
    w_fp8: torch.Tensor          # [N, K] e4m3
    w_planes: DigitPlanes        # digit planes of codebook(w)
    w_code_scale: torch.Tensor   # [N] fp32 = weight_scale / 512
    bias: torch.Tensor | None    # [N] fp32
    r: torch.Tensor              # [N] int64 Freivalds vector
    t: torch.Tensor              # [K] int64 = codebook(w)^T r


class CodebookStack:
    GEMM_BATCH = 64    # problems per GEMM launch (kernel-parameter budget of the C side)
    CHECK_BATCH = 192  # products per Freivalds row-pass launch (kernel-parameter budget of the C side)

    def __init__(self, weights: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]], *, seed: int = 0):
        self.linears: list[PreparedLinear] = []
        for i, (w, ws, bias) in enumerate(weights):
            planes, _ = codebook_planes_from_fp8(w)
            r = freivalds_vector(int(w.shape[0]), seed * 100_003 + i + 7, device=w.device)
            self.linears.append(
                PreparedLinear(
                    n=int(w.shape[0]),
                    k=int(w.shape[1]),
                    w_fp8=w.contiguous(),
                    w_planes=planes,
                    w_code_scale=(ws.reshape(-1).to(torch.float32) / 512.0).contiguous(),
                    bias=None if bias is None else bias.reshape(-1).to(torch.float32).contiguous(),
                    r=r,
                    t=weight_vector(w, r),
                )
            )
        self.device = weights[0][0].device

    def allocate(self, tokens: int) -> dict:
        """Per-forward buffers for `tokens` rows (reused by every forward / graph replay)."""
        dev = self.device
        bufs = dict(q=[], scale=[], code_scale=[], planes=[], c=[], y=[])
        for lin in self.linears:
            bufs["q"].append(torch.empty((tokens, lin.k), dtype=torch.uint8, device=dev))
            bufs["scale"].append(torch.empty((tokens,), dtype=torch.float32, device=dev))
            bufs["code_scale"].append(torch.empty((tokens,), dtype=torch.float32, device=dev))
            bufs["planes"].append(DigitPlanes.empty(tokens, lin.k, nat.IMA_SCHEME_DIGITS3, dev))
            bufs["c"].append(torch.empty((tokens, lin.n), dtype=torch.int64, device=dev))
            bufs["y"].append(torch.empty((tokens, lin.n), dtype=torch.bfloat16, device=dev))
        bufs["mismatch"] = torch.zeros((1,), dtype=torch.int32, device=dev)
        bufs["tokens"] = tokens
        return bufs

    def _descriptors(self, xs: list[torch.Tensor], bufs: dict) -> tuple:
        n = len(self.linears)
        quant = (nat.QuantizeProblem * n)()
        gemm = (nat.GemmProblem * n)()
        rows = (nat.FreivaldsRowsProblem * n)()
        for i, lin in enumerate(self.linears):
            x = xs[i]
            m = int(x.shape[0])
            planes = bufs["planes"][i]
            q = quant[i]
            q.x, q.x_dtype, q.M, q.K, q.ldx = x.data_ptr(), nat.dtype_code(x.dtype), m, lin.k, x.stride(0)
            q.q_fp8, q.ldq, q.scale = bufs["q"][i].data_ptr(), lin.k, bufs["scale"][i].data_ptr()
            q.codebook, q.ldc, q.code_scale = None, lin.k, bufs["code_scale"][i].data_ptr()
            q.planes, q.ldp = planes.planes.data_ptr(), planes.ld
            g = gemm[i]
            g.a_planes, g.lda, g.b_planes, g.ldb = planes.planes.data_ptr(), planes.ld, \
                lin.w_planes.planes.data_ptr(), lin.w_planes.ld
            g.M, g.N, g.K = m, lin.n, lin.k
            g.c, g.ldc = bufs["c"][i].data_ptr(), lin.n
            g.x_scale, g.w_scale = bufs["code_scale"][i].data_ptr(), lin.w_code_scale.data_ptr()
            g.bias = nat.ptr(lin.bias)
            g.y, g.y_dtype, g.ldy = bufs["y"][i].data_ptr(), nat.IMA_DTYPE_BF16, lin.n
            f = rows[i]
            f.a, f.lda, f.t = bufs["q"][i].data_ptr(), lin.k, lin.t.data_ptr()
            f.c, f.ldc, f.r = bufs["c"][i].data_ptr(), lin.n, lin.r.data_ptr()
            f.M, f.N, f.K, f.a_kind = m, lin.n, lin.k, nat.IMA_FREIVALDS_A_FP8
            f.mismatch_rows = bufs["mismatch"].data_ptr()
        copies = bufs.get("y_copies")
        gemm_batches = []
        for members in self._batches():
            g_arr = (nat.GemmProblem * len(members))(*[gemm[i] for i in members])
            c_arr = None
            if copies:
                c_arr = (nat.GemmYCopies * len(members))()
                for slot, i in enumerate(members):
                    dests = list(copies[i])
                    if len(dests) > 8:
                        raise ValueError("at most 8 further copies of a linear's output")
                    for d, ptr in enumerate(dests):
                        c_arr[slot].y[d] = ptr
            gemm_batches.append((g_arr, len(members), c_arr))
        return quant, gemm_batches, rows

    def _prepared(self, xs: list[torch.Tensor], bufs: dict) -> tuple:
        """Launch descriptors for these activations and buffers (built once, then reused)."""
        key = tuple(x.data_ptr() for x in xs)
        if bufs.get("_key") != key:
            bufs["_desc"] = self._descriptors(xs, bufs)
            bufs["_key"] = key
        return bufs["_desc"]

    def _batches(self) -> list[list[int]]:
        """Problems dealt to ceil(n / GEMM_BATCH) GEMM launches, largest first onto the least
        loaded launch (cost N * K; every linear has the same token count), so the launches
        take about the same time."""
        n = len(self.linears)
        count = -(-n // self.GEMM_BATCH)
        loads, members = [0] * count, [[] for _ in range(count)]
        for i in sorted(range(n), key=lambda j: -self.linears[j].n * self.linears[j].k):
            b = min((b for b in range(count) if len(members[b]) < self.GEMM_BATCH), key=lambda b: loads[b])
            members[b].append(i)
            loads[b] += self.linears[i].n * self.linears[i].k
        return [sorted(m) for m in members if m]

    def quantize(self, xs: list[torch.Tensor], bufs: dict) -> None:
        """Per-token quantisation of every activation xs[i] [tokens, K_i] (bf16) into its
        e4m3 codes, scales and digit planes: one launch."""
        quant, _g, _f = self._prepared(xs, bufs)
        main = torch.cuda.current_stream(self.device)
        nat.check("ima_quantize_grouped",
                  nat.lib().ima_quantize_grouped(ctypes.byref(quant), len(self.linears), main.cuda_stream))

    def multiply(self, xs: list[torch.Tensor], bufs: dict) -> None:
        """The exact int64 GEMM with the fused rescale/bias/bf16 epilogue of every linear
        (reads the planes that quantize() wrote): a few cost-balanced grouped launches.

        With bufs["y_copies"] (per linear, up to 8 device addresses with the layout of
        bufs["y"][i], e.g. other GPUs' gathered-output buffers opened through CUDA IPC) the
        epilogue also stores every bf16 output to each of them: the gather of the outputs is
        done when the launch is."""
        _q, gemm_batches, _f = self._prepared(xs, bufs)
        main = torch.cuda.current_stream(self.device)
        for g_arr, count, c_arr in gemm_batches:
            if c_arr is None:
                nat.check("ima_int_gemm_grouped", nat.lib().ima_int_gemm_grouped(
                    ctypes.byref(g_arr), count, nat.IMA_SCHEME_DIGITS3, main.cuda_stream))
            else:
                nat.check("ima_int_gemm_grouped_copies", nat.lib().ima_int_gemm_grouped_copies(
                    ctypes.byref(g_arr), ctypes.byref(c_arr), count, nat.IMA_SCHEME_DIGITS3, main.cuda_stream))

    def verify(self, xs: list[torch.Tensor], bufs: dict) -> None:
        """The Freivalds row check of every int64 product that multiply() wrote, failed rows
        accumulated into bufs["mismatch"]: one row-pass launch over all products (the C side
        splits it when there are more than CHECK_BATCH)."""
        _q, _g, rows = self._prepared(xs, bufs)
        main = torch.cuda.current_stream(self.device)
        nat.check("ima_freivalds_rows_grouped",
                  nat.lib().ima_freivalds_rows_grouped(ctypes.byref(rows), len(self.linears), main.cuda_stream))

    def forward(self, xs: list[torch.Tensor], bufs: dict, *, check: bool = True) -> None:
        """One forward of every linear on activations xs[i] [tokens, K_i] (bf16).

        Writes bufs["c"][i] (exact int64 products), bufs["y"][i] (bf16 outputs) and
        accumulates failed Freivalds rows into bufs["mismatch"].  Launches only, all on the
        current stream: quantize(), multiply(), then verify().  The check runs after the
        last GEMM launch with the whole GPU to itself; overlapping it with the GEMMs on a
        side stream was measured slower, because its warps then get only the registers
        that the persistent GEMM CTAs leave on each SM."""
        self.quantize(xs, bufs)
        self.multiply(xs, bufs)
        if check:
            self.verify(xs, bufs)

    def launches_per_forward(self, check: bool = True) -> int:
        checks = -(-len(self.linears) // self.CHECK_BATCH)
        return 1 + len(self._batches()) + (checks if check else 0)


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

    REPLAY_STREAMS = 4

    def prepare(self, xs: list[torch.Tensor], bufs: dict) -> None:
        """Quantise and stage every activation xs[i] [tokens, K_i]: one fused launch per
        linear (ima_hawkeye_quantize_prepare), which also writes the e4m3 codes to bufs["q"]."""
        lib = nat.lib()
        main = torch.cuda.current_stream(self.device)
        for i in range(len(self.weights)):
            x = xs[i]
            m, k = int(x.shape[0]), int(x.shape[1])
            q, scale, xop = bufs["q"][i], bufs["scale"][i], bufs["xop"][i]
            nat.check("ima_hawkeye_quantize_prepare", lib.ima_hawkeye_quantize_prepare(
                x.data_ptr(), nat.dtype_code(x.dtype), m, k, x.stride(0), scale.data_ptr(), q.data_ptr(), q.stride(0),
                xop.data_ptr(), main.cuda_stream))

    def replay(self, xs: list[torch.Tensor], bufs: dict) -> None:
        """Replay every linear on the operands prepare() staged, round-robin on
        REPLAY_STREAMS side streams that fork from and join back to the current stream: the
        last partial wave of one linear's grid overlaps the next linear's first (measured
        15 % faster than one stream at the c2 shapes).  xs gives the token counts only."""
        lib = nat.lib()
        main = torch.cuda.current_stream(self.device)
        side = self._side_streams()
        for st in side:
            st.wait_stream(main)
        for i, ((w, ws), wop) in enumerate(zip(self.weights, self.w_ops)):
            m, k, n = int(xs[i].shape[0]), int(xs[i].shape[1]), int(w.shape[0])
            nat.check("ima_hawkeye_replay", lib.ima_hawkeye_replay(
                bufs["xop"][i].data_ptr(), wop.buffer.data_ptr(), bufs["scale"][i].data_ptr(), ws.data_ptr(), m, n, k,
                32, 14, -139, bufs["y"][i].data_ptr(), n, None, n, side[i % len(side)].cuda_stream))
        for st in side:
            main.wait_stream(st)

    def forward(self, xs: list[torch.Tensor], bufs: dict) -> None:
        """prepare() then replay(): bf16 outputs of every linear in bufs["y"].  Launches only."""
        self.prepare(xs, bufs)
        self.replay(xs, bufs)

    def _side_streams(self) -> list[torch.cuda.Stream]:
        s = getattr(self, "_side", None)
        if s is None:
            s = self._side = [torch.cuda.Stream(self.device) for _ in range(self.REPLAY_STREAMS)]
        return s

    def launches_per_forward(self) -> int:
        return 2 * len(self.weights)

    @staticmethod
    def kernels_per_linear() -> int:
        return 2

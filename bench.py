"""Benchmark of the B200 student-linear hot path (prints ONE JSON line on rank 0).

Headline workload, at every GPU count (python bench.py --gpus N, one process per GPU under
torchrun for N > 1): configuration 4 -- the 196 FP8 linears of a random-init
Qwen2.5-7B-shaped model at 16384 tokens, codebook student: per-token e4m3 quantisation, the
exact int64 GEMM (tcgen05 kind::i8, fused rescale/bias/bf16 epilogue) with full int64
outputs, a Freivalds check of every product, and the bf16 outputs gathered to every GPU.
The tokens are split over the GPUs by rows, gate/up by output columns (strong scaling).  A
"step" is one forward of all 196 linears.  Metric: exact int GEMM TOPS = sum over linears of
2*M*N*K / step time (whole job, max over ranks).  Every N also reports config 4 through the
direct Hawkeye replay ("c4_hawkeye").

At N = 1 the line also carries "c1" (the 168 Qwen2.5-0.5B-shaped linears at 512 tokens, with
its pipelined and per-linear-plugin end-to-end loops), "hawkeye_c2" (the 0.5B linears at 16384
tokens through the Hawkeye replay) and "class_counts_c3" (the class-count engine on the
down_proj shape).  --c1-only, --hawkeye-only and --class-counts-only run one of those alone;
--profile-step / --profile-c4 run two eager forwards for ncu captures.

--impl reference times the reference's CPU formulation of the codebook path (its torch
quantiser expressions, torch int64 matmul, fp32 rescale) on the host cores over a bounded
sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TOKENS = 512
# the metric both arms report (the driver compares the lines)
METRIC = ("exact int GEMM TOPS (bit-exact codebook int64 GEMM + fused rescale + Freivalds check of every "
          "product; config 4: 196 Qwen2.5-7B-shaped linears, 16384 tokens)")


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_int8_peak(device) -> float:
    """Dense int8 tensor throughput of a library GEMM (torch._int_mm, 8192^3), TOPS."""
    n = 8192
    a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=device)
    b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=device).t().contiguous().t()
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    return 2 * n**3 / (best * 1e-3) / 1e12


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def ncu_figure(kernel: str) -> dict | None:
    """One kernel's figures from an ncu capture, as recorded in profiles/ncu_figures.json
    (DRAM bytes per launch, instructions per unit of work, the capture command), plus
    "current": whether the kernel's source files still hash to what was captured (False
    means the figure predates the code being measured)."""
    import hashlib

    try:
        with open(os.path.join(ROOT, "profiles", "ncu_figures.json")) as f:
            rec = dict(json.load(f)[kernel])
    except (OSError, ValueError, KeyError):
        return None
    h = hashlib.sha256()
    try:
        for src in rec.get("sources", []):
            with open(os.path.join(ROOT, src), "rb") as f:
                h.update(f.read())
    except OSError:
        rec["current"] = False
        return rec
    rec["current"] = h.hexdigest()[:16] == rec.get("sources_sha256_16")
    return rec


def int8_tensor_peak() -> tuple[float | None, str]:
    """Dense int8 tensor peak for the GEMM roofline: twice the measured dense bf16 GEMM rate
    (the int8 tensor path issues twice the bf16 MACs per cycle; MEASURED_PEAKS.json has no
    int8 figure of its own)."""
    peaks = measured_peaks()
    if peaks.get("bf16_tflops"):
        return 2.0 * float(peaks["bf16_tflops"]), "2 x MEASURED_PEAKS.json bf16_tflops (dense, burst)"
    return None, "MEASURED_PEAKS.json absent"


def build_workload(config: int, tokens: int, device, rank: int):
    from int_model_approximation_b200 import synthetic

    shapes = synthetic.config_linears(config)
    weights, xs = [], []
    for i, s in enumerate(shapes):
        seed = synthetic.linear_seed(config, i)
        w, ws = synthetic.normal_fp8_weights(s.n, s.k, seed + 500_000, device=device)
        g = torch.Generator(device=device).manual_seed(seed + 77)
        bias = (torch.randn(s.n, generator=g, device=device) * 0.01).to(torch.bfloat16)
        weights.append((w, ws, bias))
        xs.append(synthetic.student_t_activations(tokens, s.k, seed + 1_000_003 * rank, device=device,
                                                  outlier_fraction=synthetic.CONFIGS[config]["outliers"]))
    return shapes, weights, xs


def measured_int32_issue_rate(device) -> float:
    """Integer-ALU instruction throughput of the device (G ops/s) from ima_int32_issue_probe."""
    from int_model_approximation_b200 import _native as nat

    sink = torch.zeros((256,), dtype=torch.int32, device=device)
    blocks = 148 * 8
    iters = 1 << 14
    stream = torch.cuda.current_stream(device)
    for _ in range(2):
        nat.call("ima_int32_issue_probe", iters, blocks, sink.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        nat.call("ima_int32_issue_probe", iters, blocks, sink.data_ptr(), stream.cuda_stream)
        e.record(stream)
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    return blocks * 256 * iters * 16 / (best * 1e-3) / 1e9


def run_hawkeye(args, emit: bool = True) -> dict:
    """Config 2: direct Hawkeye replay of all 168 linears of the 0.5B shapes at
    `--hawkeye-tokens` tokens (0.1 % x50 outliers).  One step = quantise and stage every
    linear, then replay every linear, the replays spread over four side streams (each phase
    captured once in a CUDA graph).  Metric: Hawkeye outputs per second."""
    from int_model_approximation_b200 import _native as nat
    from int_model_approximation_b200.pipeline import HawkeyeStack

    world, rank, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    nat.lib()
    tokens = args.hawkeye_tokens
    shapes, weights, xs = build_workload(2, tokens, device, rank)
    stack = HawkeyeStack(weights)
    bufs = stack.allocate(tokens)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        stack.forward(xs, bufs)
    torch.cuda.synchronize()
    # the two phases as CUDA graphs replayed back to back; events between them time the
    # replay inside the timed steps
    graphs = {name: torch.cuda.CUDAGraph() for name in ("prepare", "replay")}
    with torch.cuda.stream(stream):
        for name, g in graphs.items():
            with torch.cuda.graph(g, stream=stream):
                getattr(stack, name)(xs, bufs)
    steps = max(2, args.hawkeye_steps)
    with torch.cuda.stream(stream):
        for _ in range(2):
            for g in graphs.values():
                g.replay()
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps + 1)]
        marks[0].record(stream)
        for i in range(steps):
            graphs["prepare"].replay()
            marks[2 * i + 1].record(stream)
            graphs["replay"].replay()
            marks[2 * i + 2].record(stream)
    marks[-1].synchronize()
    times = {
        "step": marks[0].elapsed_time(marks[-1]) / steps,
        "replay": sum(marks[2 * i + 1].elapsed_time(marks[2 * i + 2]) for i in range(steps)) / steps,
    }
    outputs = sum(tokens * s.n for s in shapes)
    products = sum(tokens * s.n * s.k for s in shapes)
    int_peak = measured_int32_issue_rate(device)
    replay_terms = products / (times["replay"] * 1e-3)
    fig = ncu_figure("hawkeye_replay_kernel") or {}
    inst = fig.get("thread_instructions_per_product")
    res = {
        "workload": f"c2: 168 linears of Qwen2.5-0.5B shape, {tokens} tokens, direct Hawkeye K=32 replay",
        "outputs_per_s": outputs / (times["step"] * 1e-3),
        "ms_per_step": times["step"],
        "replay_ms_per_step": times["replay"],
        "products_per_s": products / (times["step"] * 1e-3),
        "roofline": {
            "kernel": "hawkeye_replay_kernel",
            "bound": "instruction issue (integer ALU and FMA pipes)",
            "achieved": round(inst * replay_terms / 1e9, 1) if inst else None,
            "peak": round(int_peak, 1),
            "unit": "G thread-instructions/s issued",
            "frac": round(inst * replay_terms / 1e9 / int_peak, 4) if inst else None,
            "instructions_per_product": inst,
            "instructions_source": f"ncu inst_executed x 32 / products of one launch ({fig.get('command')}); "
                                   f"capture matches the current source: {fig.get('current')}",
            "peak_source": "ima_int32_issue_probe (XOR+ADD chains on every SM: the full issue rate) measured in "
                           "this run",
            "products_per_s_replay_phase": replay_terms,
            "reference_op_count": "the reference kernel's 10 integer ops per product would be "
                                  f"{round(10.0 * replay_terms / 1e9, 1)} G ops/s equivalent",
        },
        "launches_per_step": stack.launches_per_forward(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = hawkeye_cpu_baseline(shapes, stack, bufs, budget_s=args.hawkeye_cpu_seconds)
    if emit and rank == 0:
        print(json.dumps({"hawkeye": res}), flush=True)
    return res


def run_class_counts_c3(args) -> dict:
    """Config 3: the hawkeye-class-counts student on the down_proj shape (M = 4096, K = 4864,
    N = 896) with class_chunk 512, 6 packed count lanes and 2 packed group lanes, through
    exact_hawkeye_fp8_sum with raw_matmul None (what HawkeyeClassCountsLinear passes): the
    per-pack class presence for the stats, then the class-count engine -- count products
    formed on the tensor cores, every count tile fingerprinted, the accumulator replayed from
    the counts.  Each call reads the stats and the fingerprint verdict back to the host (as
    the reference reads its class lists), so each timed call is bracketed by CUDA events on
    an otherwise idle stream.  The engine kernel alone (operands staged) is timed the same
    way for its tensor-pipe fraction."""
    from int_model_approximation_b200 import codebook, hawkeye, hawkeye_freivalds, synthetic

    device = torch.device("cuda", 0)
    shape = synthetic.LinearShape("down_proj", 896, 4864)
    x, w, ws = synthetic.make_linear_inputs(3, 0, shape, tokens=args.c3_tokens, device=device)
    xq, xs, *_ = codebook.per_token_fp8(x)
    params = dict(class_chunk=512, packed_count_lanes=6, packed_group_lanes=2)

    def call():
        return hawkeye_freivalds.exact_hawkeye_fp8_sum(xq, xs, w, ws, None, **params)

    y, stats = call()
    direct, _ = hawkeye.hawkeye_fp8_sum(xq, xs, w, ws)
    equal = bool(torch.equal(y.view(torch.int16), direct.view(torch.int16)))
    for _ in range(2):
        call()
    torch.cuda.synchronize()
    steps = 5
    stream = torch.cuda.current_stream(device)

    def timed(fn) -> float:
        total = 0.0
        for _ in range(steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            b.synchronize()
            total += a.elapsed_time(b)
        return total / steps

    ms = timed(call)
    # the engine kernel alone on staged operands
    x_op = hawkeye_freivalds.ClassCountOperand(xq)
    w_op = hawkeye_freivalds.stage_class_count_weight(w)
    mism = torch.zeros((1,), dtype=torch.int32, device=device)
    out = torch.empty_like(y)
    xs32 = xs.reshape(-1).to(torch.float32).contiguous()
    ws32 = ws.reshape(-1).to(torch.float32).contiguous()

    def engine():
        hawkeye_freivalds.class_count_replay(x_op, w_op, xs32, ws32, out=out, mismatch=mism)

    engine()
    torch.cuda.synchronize()
    mism.zero_()
    kernel_ms = timed(engine)
    fingerprint_failures = int(mism.item())
    m, n, k = int(x.shape[0]), shape.n, shape.k
    groups = -(-k // 32)
    tiles = -(-m // 4) * sum(min(8, -(-(n - n0) // 8)) for n0 in range(0, n, 64)) * 2 * (-(-groups // 2))
    count_macs = tiles * 128 * 256 * 32          # MACs the engine's MMAs perform (one 128x256x32 MMA per tile)
    peak, peak_source = int8_tensor_peak()
    # the reference's count products for the same stats: per pack (n_a M) x 64 x (ceil(n_b / 3) N)
    a_cnt = hawkeye_freivalds._popcounts(hawkeye_freivalds.class_presence(xq, 64))
    b_cnt = hawkeye_freivalds._popcounts(hawkeye_freivalds.class_presence(w, 64))
    ref_macs = sum(na * m * 64 * (-(-nb // 3)) * n for na, nb in zip(a_cnt, b_cnt))
    res = {
        "workload": "c3: down_proj 4096 x 4864 -> 896, hawkeye-class-counts, class_chunk 512, "
                    "6 count lanes, 2 group lanes",
        "outputs_per_s": m * n / (ms * 1e-3),
        "products_per_s": m * n * k / (ms * 1e-3),
        "ms_per_call": round(ms, 4),
        "engine_kernel_ms": round(kernel_ms, 4),
        "steps": steps,
        "equals_direct_replay": equal,
        "fingerprint_failed_rows": fingerprint_failures,
        "stats": {key: val for key, val in stats.__dict__.items()},
        "count_products": {
            "formed_by": "class_count_replay_kernel: one tcgen05.mma kind::i8 (128 x 256 x 32) per tile of 4 "
                         "tokens x 8 weight rows x 32 class slots each, per group of 32 k",
            "mma_tiles_per_call": tiles,
            "count_macs_per_call": count_macs,
            "count_macs_per_s": count_macs / (kernel_ms * 1e-3),
            "count_entries_replayed_per_call": tiles * 128 * 256,
            "reference_count_macs_per_call": ref_macs,
            "reference_products_per_call": stats.total_checkable_products,
        },
        "roofline": {
            "kernel": "class_count_replay_kernel",
            "bound": "epilogue instruction issue (every count entry is replayed: FFMA.RZ + 2 IMAD); "
                     "the tensor pipe forms the counts",
            "achieved": round(2.0 * count_macs / (kernel_ms * 1e-3) / 1e12, 2),
            "peak": round(peak, 1) if peak else None,
            "unit": "TOPS (int8 tensor ops of the count MMAs)",
            "frac": round(2.0 * count_macs / (kernel_ms * 1e-3) / 1e12 / peak, 4) if peak else None,
            "peak_source": peak_source,
        },
    }
    if not args.no_cpu_baseline:
        import oracle

        rows = 128
        t0 = time.perf_counter()
        ref = oracle.hawkeye(xq[:rows].cpu(), xs[:rows].cpu(), w.cpu(), ws.cpu())
        t = time.perf_counter() - t0
        res["cpu_baseline"] = {
            "value": rows * n * k / t, "unit": "products/s", "cores": max(1, min(32, os.cpu_count() or 1)),
            "kind": "port",
            "sample": f"{rows} token rows through the oracle's C restatement of the replay (the output equals "
                      f"the direct replay), {t:.1f} s",
            "parity": {"rows_checked": rows, "ok": bool(torch.equal(y[:rows].cpu().view(torch.int16),
                                                                    ref.to(torch.bfloat16).view(torch.int16))),
                       "what": "the engine's bf16 rows vs the CPU replay, bit for bit"},
        }
    return res


def hawkeye_cpu_baseline(shapes, stack, bufs, budget_s: float) -> dict:
    """The replay on the host cores: the oracle's scalar C restatement of the reference's
    Hawkeye kernel (hawkeye.py:127-219; the reference's own CPU form, exact_hawkeye_fp8_sum
    with a CPU raw_matmul, needs about 160 s per K = 32 group of one c0 row block), its rows
    split over the host threads.  Bounded sample: 64 token rows of each linear in turn,
    quantised by the GPU step above, until the budget is used."""
    import oracle

    rows = 64
    done_products, done_outputs, t_used, linears = 0.0, 0.0, 0.0, 0
    parity_ok = True
    while t_used < budget_s and linears < len(shapes):
        i = linears
        s = shapes[i]
        w, ws = stack.weights[i]
        xq = bufs["q"][i][:rows].cpu().view(torch.float8_e4m3fn)
        xs = bufs["scale"][i][:rows].cpu()
        wq, wsc = w.cpu(), ws.cpu()
        t0 = time.perf_counter()
        ref = oracle.hawkeye(xq, xs, wq, wsc)
        t_used += time.perf_counter() - t0
        # the CPU rows double as the parity check of the GPU replay (same operands)
        parity_ok = parity_ok and torch.equal(bufs["y"][i][:rows].cpu().view(torch.int16),
                                              ref.to(torch.bfloat16).view(torch.int16))
        done_products += float(rows) * s.n * s.k
        done_outputs += float(rows) * s.n
        linears += 1
    threads = max(1, min(32, os.cpu_count() or 1))
    return {
        "value": done_products / t_used,
        "unit": "products/s",
        "outputs_per_s": done_outputs / t_used,
        "cores": threads,
        "kind": "port",
        "sample": f"{rows} token rows of each of the first {linears} linears, {t_used:.1f} s",
        "parity": {"rows_checked": rows * linears, "linears_checked": linears, "ok": parity_ok,
                   "what": "GPU bf16 outputs of the timed steps vs the CPU replay, bit for bit"},
    }


def run_profile_step(args) -> None:
    """Two eager forwards of the c1 workload and nothing else: the command profiled by
    ncu for the per-kernel launch list (the second forward is the one summarised)."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    from int_model_approximation_b200.pipeline import CodebookStack

    tokens = args.profile_tokens
    _shapes, weights, xs = build_workload(1, tokens, device, 0)
    stack = CodebookStack(weights)
    bufs = stack.allocate(tokens)
    for _ in range(2):
        stack.forward(xs, bufs)
        torch.cuda.synchronize()
    print(json.dumps({"profile_step": "done", "mismatch": int(bufs["mismatch"].item())}))


def run_profile_c4(args) -> None:
    """Two eager forwards of the first `--c4-layers` layers of config 4 at N = 1 (one grouped
    quantiser, GEMM and check launch per layer): the command profiled by ncu for the c4 GEMM's
    DRAM traffic (its second forward's launches are the captured ones)."""
    from int_model_approximation_b200.codebook import DigitPlanes  # noqa: F401
    from int_model_approximation_b200.pipeline import CodebookStack

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    specs = c4_specs(args.c4_tokens, 1, 0)
    xs = c4_inputs(specs, args.c4_tokens, device)
    stacks = [CodebookStack([c4_weights(sp, layer, p, device) for p, sp in enumerate(specs)], seed=layer)
              for layer in range(args.c4_layers)]
    bufs = stacks[0].allocate(args.c4_tokens)
    views = [dict(bufs) for _ in stacks]
    # this stack mixes token counts per linear (gate/up keep all tokens), so allocate per linear
    for v in views:
        for key in ("q", "scale", "code_scale", "planes", "c", "y"):
            v[key] = list(bufs[key])
    for _ in range(2):
        for st, v in zip(stacks, views):
            st.forward(xs, v)
        torch.cuda.synchronize()
    print(json.dumps({"profile_c4": "done", "layers": args.c4_layers, "mismatch": int(bufs["mismatch"].item())}))


def run_c1(args) -> dict:
    """Config 1 on one GPU (returned as the "c1" object of the default line): all 168 linears of
    the 0.5B shapes at 512 tokens, codebook student with int64 outputs and a Freivalds check of
    every product; exact TOPS, the GEMM roofline, the pipelined end-to-end loop, the per-linear
    plugin loop and the CPU baseline with parity of the timed outputs."""
    world, rank, local = 1, 0, 0
    device = torch.device("cuda", local)
    from int_model_approximation_b200 import _native as nat
    from int_model_approximation_b200.pipeline import CodebookStack

    nat.lib()
    int8_peak = measured_int8_peak(device)
    shapes, weights, xs = build_workload(1, TOKENS, device, rank)
    stack = CodebookStack(weights, seed=rank)

    def packed_views(store: torch.Tensor, like: list[torch.Tensor]) -> list[torch.Tensor]:
        out, off = [], 0
        for t in like:
            out.append(store[off:off + t.numel()].view(t.shape))
            off += t.numel()
        return out

    def contiguous_set() -> tuple[list[torch.Tensor], dict]:
        """Activations and bf16 outputs of all linears as views of one allocation each, so
        that a step's host transfers are one copy per direction."""
        x_store = torch.empty((sum(x.numel() for x in xs),), dtype=torch.bfloat16, device=device)
        xv = packed_views(x_store, xs)
        b = stack.allocate(TOKENS)
        y_store = torch.empty((sum(y.numel() for y in b["y"]),), dtype=torch.bfloat16, device=device)
        b["y"] = packed_views(y_store, b["y"])
        b["x_store"], b["y_store"] = x_store, y_store
        return xv, b

    xs_gen = xs
    xs, bufs = contiguous_set()
    for dst, src in zip(xs, xs_gen):
        dst.copy_(src)
    del xs_gen
    flops = sum(2.0 * TOKENS * s.n * s.k for s in shapes)

    # eager warm-up (initialises kernel attributes, tensor-map entry points)
    stack.forward(xs, bufs)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    # The step's three phases, each captured once into its own CUDA graph and replayed back
    # to back on one stream, so that CUDA events between them time each kernel inside the
    # timed region (the whole forward, one graph, serves the end-to-end loop below).
    graph = torch.cuda.CUDAGraph()
    phase_graphs = {name: torch.cuda.CUDAGraph() for name in ("quantize", "multiply", "verify")}
    with torch.cuda.stream(stream):
        stack.forward(xs, bufs)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            stack.forward(xs, bufs)
        for name, g in phase_graphs.items():
            with torch.cuda.graph(g, stream=stream):
                getattr(stack, name)(xs, bufs)
    torch.cuda.synchronize()
    phase_ms = {name: 0.0 for name in phase_graphs}

    def step(marks: list | None = None):
        for k, g in enumerate(phase_graphs.values()):
            g.replay()
            if marks is not None:
                marks[k].record(stream)
        if world > 1:
            torch.distributed.all_reduce(bufs["mismatch"])

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    bufs["mismatch"].zero_()

    # ---- timed region (device resident inputs; inputs 2.4 GB per step > L2) ----
    marks = [[torch.cuda.Event(enable_timing=True) for _ in phase_graphs] for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        s_ev.record(stream)
        for i in range(args.steps):
            step(marks[i])
        e_ev.record(stream)
    e_ev.synchronize()
    clocks = sampler.stop()
    ms = s_ev.elapsed_time(e_ev) / args.steps
    # per-phase device time: from the end of the previous mark (the step's start for the
    # quantiser, which includes the previous step's mismatch all-reduce when world > 1)
    for i in range(args.steps):
        prev = s_ev if i == 0 else marks[i - 1][-1]
        for k, name in enumerate(phase_graphs):
            phase_ms[name] += prev.elapsed_time(marks[i][k]) / args.steps
            prev = marks[i][k]
    if world > 1:
        t = torch.tensor([ms] + list(phase_ms.values()), device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t[0].item())
        phase_ms = dict(zip(phase_ms, (float(v) for v in t[1:].tolist())))
        torch.distributed.barrier()
    mismatches = int(bufs["mismatch"].item())
    gemm_ms_per_step = phase_ms["multiply"]
    gemm_launches = len(stack._batches())
    # algorithmic bytes of the Freivalds row pass: fp8 codes of A, int64 C, int64 r and t
    check_bytes = sum(TOKENS * s.k + 8 * TOKENS * s.n + 8 * s.n + 8 * s.k for s in shapes)
    # quantiser: bf16 activations in; e4m3 codes and three digit-plane bytes out per element
    quant_bytes = sum(TOKENS * s.k * (2 + 1 + 3) + 8 * TOKENS for s in shapes)

    # ---- end to end through the public API: host buffers in, host results out ----
    # Every step copies its activations in from pinned host memory and its bf16 outputs and
    # Freivalds verdict back out.  The three are pipelined across steps as a serving loop
    # would run them: the inputs of step i + 1 stream in and the outputs of step i - 1 stream
    # out while step i computes (copy-in, compute and copy-out streams, two device buffer
    # sets, each forward captured once per set).
    host_x = bufs["x_store"].cpu().pin_memory()
    host_y = torch.empty(bufs["y_store"].shape, dtype=torch.bfloat16).pin_memory()
    host_mm = torch.empty((1,), dtype=torch.int32).pin_memory()
    h2d = host_x.numel() * host_x.element_size()
    d2h = host_y.numel() * host_y.element_size() + 4
    xs1, bufs1 = contiguous_set()
    xs_sets = [xs, xs1]
    bufs_sets = [bufs, bufs1]
    e2e_graphs = [graph]
    with torch.cuda.stream(stream):
        stack.forward(xs_sets[1], bufs_sets[1])
        torch.cuda.synchronize()
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1, stream=stream):
            stack.forward(xs_sets[1], bufs_sets[1])
        e2e_graphs.append(g1)
    torch.cuda.synchronize()
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i: int) -> None:
        j = i % 2
        s_in.wait_event(ev_done[j])            # step i - 2 has finished reading set j's inputs
        with torch.cuda.stream(s_in):
            bufs_sets[j]["x_store"].copy_(host_x, non_blocking=True)
        ev_in[j].record(s_in)
        stream.wait_event(ev_in[j])
        stream.wait_event(ev_out[j])           # step i - 2's outputs of set j are on the host
        with torch.cuda.stream(stream):
            e2e_graphs[j].replay()
            if world > 1:
                torch.distributed.all_reduce(bufs_sets[j]["mismatch"])
        ev_done[j].record(stream)
        s_out.wait_event(ev_done[j])
        with torch.cuda.stream(s_out):
            host_y.copy_(bufs_sets[j]["y_store"], non_blocking=True)
            host_mm.copy_(bufs_sets[j]["mismatch"], non_blocking=True)
        ev_out[j].record(s_out)

    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    s_in.wait_event(x0)
    for i in range(args.steps):
        e2e_step(i)
    for j in range(2):
        stream.wait_event(ev_out[j])
    x1.record(stream)
    x1.synchronize()
    e2e_ms = x0.elapsed_time(x1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    del e2e_graphs
    plugin = None
    if world == 1:
        plugin = plugin_e2e(weights, xs, min(args.steps, 10), device)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(shapes, weights, xs, budget_s=args.cpu_seconds, gpu_c=bufs["c"],
                                  gpu_y=bufs["y"])

    if rank == 0:
        peaks = measured_peaks()
        total_ops = flops * world
        value = total_ops / (ms * 1e-3) / 1e12
        # DIGITS3: nine int8 digit products (3 x 3 planes) per exact product
        gemm_tc_ops = 9.0 * flops / (gemm_ms_per_step * 1e-3) / 1e12
        fig = ncu_figure("int_gemm_kernel<DIGITS3>") or {}
        peak, peak_source = int8_tensor_peak()
        if peak is None:
            peak, peak_source = int8_peak, "torch._int_mm 8192^3 measured in this run (MEASURED_PEAKS.json absent)"
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "TOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int8 digit planes -> int32 TMEM -> int64",
            "data": "synthetic (seeded Student-t activations, N(0,0.02) e4m3 weights; no checkpoint)",
            "config": {
                "workload": "c1: 168 FP8 linears of Qwen2.5-0.5B shape, 512 tokens per GPU, codebook student, "
                            "int64 outputs + per-linear Freivalds",
                "linears": len(shapes),
                "tokens_per_gpu": TOKENS,
                "exact_int_ops_per_step_per_gpu": flops,
                "l2": "inputs larger than L2 (about 2.4 GB of weight planes and activations per step)",
                "launch": "three CUDA graphs per step on one stream: grouped quantiser, grouped GEMM (up to "
                          "64 linears per launch), Freivalds row check of every product (one launch)",
                "parallelism": f"replicas x{world} (token batches per rank)",
            },
            "freivalds_mismatch_rows": mismatches,
            "gpu_launches": stack.launches_per_forward() * args.steps,
            "roofline": {
                "kernel": "int_gemm_kernel<DIGITS3>",
                "bound": "tensor",
                "achieved": round(gemm_tc_ops, 2),
                "peak": round(peak, 1),
                "unit": "TOPS (int8 tensor ops, 9 digit products per exact product)",
                "limb_adjusted_peak_exact_tops": round(peak / 9.0, 1),
                "frac": round(gemm_tc_ops / peak, 4),
                "peak_source": peak_source,
                "library_int8_gemm_tops": round(int8_peak, 1),
                "library_int8_gemm": "torch._int_mm 8192^3 best-of-10 measured in this run (context: a library "
                                     "int8 GEMM on this device)",
                "traffic": fig.get("dram_bytes_per_launch"),
                "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one grouped launch "
                                   f"({fig.get('command')}); capture matches the current source: "
                                   f"{fig.get('current')}") if fig else None,
                "gemm_ms_per_step": round(gemm_ms_per_step, 4),
                "gemm_launches_per_step": gemm_launches,
                "exact_tops_gemm_only": round(flops / (gemm_ms_per_step * 1e-3) / 1e12, 3),
                "timing": "CUDA events around the GEMM launches inside the timed steps",
            },
            "phases_ms_per_step": {k: round(v, 4) for k, v in phase_ms.items()},
            "freivalds_roofline": {
                "kernel": "fv_rows_aligned_kernel",
                "bound": "hbm",
                "achieved": round(check_bytes / (phase_ms["verify"] * 1e-3) / 1e9, 1),
                "peak": peaks.get("hbm_gbs"),
                "unit": "GB/s",
                "frac": round(check_bytes / (phase_ms["verify"] * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)
                if peaks.get("hbm_gbs") else None,
                "bytes_per_step": check_bytes,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (copy bandwidth)",
            },
            "quantizer_roofline": {
                "kernel": "quantize_rows_kernel",
                "bound": "hbm",
                "achieved": round(quant_bytes / (phase_ms["quantize"] * 1e-3) / 1e9, 1),
                "peak": peaks.get("hbm_gbs"),
                "unit": "GB/s",
                "frac": round(quant_bytes / (phase_ms["quantize"] * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)
                if peaks.get("hbm_gbs") else None,
                "bytes_per_step": quant_bytes,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (copy bandwidth)",
            },
            "e2e": {
                "value": round(total_ops / (e2e_ms * 1e-3) / 1e12, 3),
                "unit": "TOPS",
                "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "CodebookStack.forward (bf16 activations from pinned host memory, bf16 outputs + "
                       "Freivalds verdict back to host)",
                "pipelining": "inputs of step i+1 in and outputs of step i-1 out while step i computes "
                              "(copy-in, compute and copy-out streams; two device buffer sets)",
            },
            "e2e_plugin": plugin,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "measured_peaks": {k: peaks.get(k) for k in ("hbm_gbs", "bf16_tflops")},
        }
        return line
    return {}


def plugin_e2e(weights, xs, steps: int, device) -> dict:
    """End to end through the reference-facing plugin: one students.CodebookLinear per
    linear (built once, as the replacement pass builds them), called once per linear per
    step on activations copied in from pinned host memory, its bf16 output copied back to
    pinned host memory.  This is the per-call path the reference's driver takes (one module
    forward per linear, __main__.py:754-773), so each call's ctypes, allocation and launch
    overhead is inside the timed region; CUDA events on the launching stream time the
    device timeline, host gaps included."""
    from int_model_approximation_b200 import students

    layers = [students.CodebookLinear(w, ws, b) for w, ws, b in weights]
    host_x = [x.cpu().pin_memory() for x in xs]
    host_y = [torch.empty((x.shape[0], lay.out_features), dtype=torch.bfloat16).pin_memory()
              for x, lay in zip(xs, layers)]
    ops = sum(2.0 * x.shape[0] * lay.out_features * lay.in_features for x, lay in zip(xs, layers))
    stream = torch.cuda.current_stream(device)

    def one_step() -> None:
        for lay, hx, hy in zip(layers, host_x, host_y):
            xd = hx.to(device, non_blocking=True)
            hy.copy_(lay(xd), non_blocking=True)

    for _ in range(2):
        one_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        one_step()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {
        "value": round(ops / (ms * 1e-3) / 1e12, 3),
        "unit": "TOPS",
        "ms_per_step": round(ms, 3),
        "steps": steps,
        "h2d_bytes_per_step": sum(x.numel() * 2 for x in host_x),
        "d2h_bytes_per_step": sum(y.numel() * 2 for y in host_y),
        "api": "students.CodebookLinear.forward, once per linear (168 calls per step), host bf16 activations "
               "in, host bf16 outputs out; no Freivalds check (the reference's plugin has none)",
    }


def cpu_baseline_sample(shapes, weights, xs, budget_s: float = 15.0, gpu_c=None, gpu_y=None) -> dict:
    """The reference's CPU path (oracle port: torch quantiser, torch int64 matmul,
    fp32 rescale) on a bounded sample of the same workload: whole linears, cycling
    through the model, until the time budget is used.  torch's int64 matmul is
    single-threaded, so each linear's token rows are split over all host threads; the
    weight codes are prepared once per linear outside the timed region, as the
    reference's CodebookLinear.__init__ does.  The CPU results double as the parity check
    of the GPU step: gpu_c / gpu_y (the int64 products and bf16 outputs the timed steps
    wrote for the same inputs) are compared with them bit for bit, outside the CPU timing."""
    import oracle

    threads = os.cpu_count() or 1
    prev_threads = torch.get_num_threads()
    torch.set_num_threads(1)   # one row part per host thread instead of intra-op threads
    done_ops, t_used, linears = 0.0, 0.0, 0
    rows_checked, parity_ok = 0, True
    i = 0
    try:
        while t_used < budget_s and linears < len(shapes):
            s = shapes[i]
            w, ws, bias = weights[i]
            wc, wsc, bc = w.cpu(), ws.cpu(), bias.cpu()
            codes = oracle.fp8_codebook(wc).to(torch.int64)
            x = xs[i].cpu()
            t0 = time.perf_counter()
            c_ref, out_ref = oracle.torch_cpu_codebook_linear(x, wc, wsc, bc, threads=threads, w_codes=codes)
            t_used += time.perf_counter() - t0
            if gpu_c is not None and gpu_y is not None:
                same = torch.equal(gpu_c[i].cpu(), c_ref) and torch.equal(
                    gpu_y[i].cpu().view(torch.int16), out_ref.view(torch.int16))
                parity_ok = parity_ok and same
                rows_checked += int(x.shape[0])
            done_ops += 2.0 * x.shape[0] * s.n * s.k
            linears += 1
            i += 1
    finally:
        torch.set_num_threads(prev_threads)
    out = {
        "value": round(done_ops / t_used / 1e12, 6),
        "unit": "TOPS",
        "cores": threads,
        "kind": "port",
        "sample": f"{linears} whole linears of the c1 workload ({TOKENS} tokens each, rows split over "
                  f"{threads} threads), {t_used:.1f} s",
    }
    if gpu_c is not None:
        out["parity"] = {"rows_checked": rows_checked, "linears_checked": linears, "ok": parity_ok,
                         "what": "GPU int64 products and bf16 outputs of the timed steps vs the CPU results, "
                                 "bit for bit"}
    return out


def run_reference(args) -> None:
    """The reference arm: the reference's own CPU formulation of the codebook path (its torch
    quantiser expressions, torch int64 matmul in place of its Triton kernel, fp32 rescale, bias;
    oracle.torch_cpu_codebook_linear) on the host cores, on the B200 arm's workload (config 4),
    each step one linear of the 7B-shaped model with `--reference-rows` token rows, cycling
    through the seven shapes of successive layers; rows split over every host thread.  Under
    torchrun only rank 0 runs it."""
    world, rank, _local = _dist()
    if rank != 0:
        return
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(1)   # one row part per host thread (torch's int64 matmul is single-threaded)
    specs = c4_specs(args.c4_tokens, 1, 0)
    rows = args.reference_rows

    def sample(i):
        layer, p = (i // 7) % args.c4_layers, i % 7
        sp = specs[p]
        from int_model_approximation_b200 import synthetic

        x = synthetic.student_t_activations(rows, sp["k"], synthetic.linear_seed(4, p))
        w, ws, bias = c4_weights(sp, layer, p, "cpu")
        return sp, x, w, ws, bias, oracle.fp8_codebook(w).to(torch.int64)   # weight prepack: once per linear

    for i in range(args.warmup):
        sp, x, w, ws, bias, codes = sample(i)
        oracle.torch_cpu_codebook_linear(x, w, ws, bias, threads=threads, w_codes=codes)
    total_t, total_ops = 0.0, 0.0
    for i in range(args.steps):
        sp, x, w, ws, bias, codes = sample(args.warmup + i)
        t0 = time.perf_counter()
        oracle.torch_cpu_codebook_linear(x, w, ws, bias, threads=threads, w_codes=codes)
        total_t += time.perf_counter() - t0
        total_ops += 2.0 * rows * sp["n"] * sp["k"]
    value = total_ops / total_t / 1e12
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 6),
        "unit": "TOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_t / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int64",
        "data": "synthetic",
        "config": {"workload": "c4: 196 FP8 linears of Qwen2.5-7B shape, codebook student (the reference's CPU "
                               "formulation)",
                   "sample_rows_per_step": rows,
                   "freivalds": "not timed: the reference checks its products only in its tests"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TOPS", "cores": threads, "kind": "port",
                         "sample": f"one linear per step ({rows} token rows split over {threads} threads), cycling "
                                   f"through the seven 7B shapes of successive layers"},
        "e2e": {"value": round(value, 6), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


C4_METRIC = METRIC


def c4_specs(tokens: int, world: int, rank: int) -> list[dict]:
    """This rank's share of each of the seven linears of a layer: token rows for q/k/v/o/down,
    output columns (all tokens) for gate/up."""
    from int_model_approximation_b200 import sharding, synthetic

    specs = []
    for s in synthetic.qwen_layer_shapes(3584, 512, 18944):
        if s.name in ("gate_proj", "up_proj"):
            c0, c1 = sharding.col_shard(s.n, world, rank)
            if (c1 - c0) * world != s.n:
                raise SystemExit(f"{s.name}: {s.n} columns do not split evenly over {world} GPUs")
            specs.append(dict(name=s.name, k=s.k, n=c1 - c0, n_full=s.n, rows=tokens, col=True, col0=c0))
        else:
            r0, r1 = sharding.row_shard(tokens, world, rank)
            specs.append(dict(name=s.name, k=s.k, n=s.n, n_full=s.n, rows=r1 - r0, col=False, row0=r0))
    return specs


def c4_weight_seed(layer: int, p: int) -> int:
    from int_model_approximation_b200 import synthetic

    return synthetic.linear_seed(4, 7 * layer + p) + 500_000


def c4_weights(spec: dict, layer: int, p: int, device):
    """(w_fp8 [n, K], w_scale [n, 1], bias bf16 [n]) of this rank's share of linear (layer, p): the
    full weight is drawn from its seed and the rank keeps its output columns (gate/up), so
    every rank computes exactly its part of the same model."""
    from int_model_approximation_b200 import synthetic

    w, ws = synthetic.normal_fp8_weights(spec["n_full"], spec["k"], c4_weight_seed(layer, p), device=device)
    g = torch.Generator(device=device).manual_seed(c4_weight_seed(layer, p) + 77)
    bias = (torch.randn(spec["n_full"], generator=g, device=device) * 0.01).to(torch.bfloat16)
    if spec["col"]:
        c0, c1 = spec["col0"], spec["col0"] + spec["n"]
        return w[c0:c1].contiguous(), ws[c0:c1].contiguous(), bias[c0:c1].contiguous()
    return w, ws, bias


def c4_inputs(specs: list[dict], tokens: int, device) -> list[torch.Tensor]:
    """The seven activation matrices of a layer (shared by the 28 layers: synthetic inputs of
    the right shapes; the work per layer is unchanged), this rank's rows of each."""
    from int_model_approximation_b200 import synthetic

    xs = []
    for p, sp in enumerate(specs):
        x = synthetic.student_t_activations(tokens, sp["k"], synthetic.linear_seed(4, p), device=device)
        xs.append(x if sp["col"] else x[sp["row0"]:sp["row0"] + sp["rows"]].contiguous())
    return xs


def run_headline(args) -> None:
    """The default measurement: config 4 -- the 196 FP8 linears of a Qwen2.5-7B-shaped model at
    16384 tokens -- on N GPUs (one process per GPU under torchrun), partitioned as BASELINE's
    north star says: token rows over the ranks with the weights replicated, gate/up split by
    output columns (every rank holds all tokens for them), and the bf16 outputs gathered to
    every rank.  A step is one forward of all 196 linears: per layer the grouped quantiser,
    the exact int64 GEMM with the fused rescale (one grouped launch), the gathers of its
    outputs (peer-to-peer copies on the copy engines, started as soon as the GEMM has written
    them; `--c4-gather sm`: one copy kernel per layer on SMs kept from the GEMM; `--c4-gather
    epilogue`: stores from the GEMM epilogue) and the Freivalds row check of every local
    int64 product.  Strong scaling: the
    16384 tokens are fixed.  value = exact int ops of the whole model / step time (max over
    ranks).  At N = 1 the line also carries config 1 (the 0.5B codebook stack), config 2
    (Hawkeye replay) and config 3 (class counts); at every N it carries config 4's Hawkeye
    replay phase."""
    import ctypes
    import datetime

    world, rank, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = torch.distributed
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=600))
    from int_model_approximation_b200 import _native as nat
    from int_model_approximation_b200 import synthetic
    from int_model_approximation_b200.codebook import DigitPlanes
    from int_model_approximation_b200.pipeline import CodebookStack

    lib = nat.lib()
    tokens, layers = args.c4_tokens, args.c4_layers
    if tokens % world:
        raise SystemExit("--c4-tokens must be a multiple of the number of GPUs")
    specs = c4_specs(tokens, world, rank)
    xs = c4_inputs(specs, tokens, device)
    stacks = []
    for layer in range(layers):
        stacks.append(CodebookStack([c4_weights(sp, layer, p, device) for p, sp in enumerate(specs)], seed=layer))
    torch.cuda.synchronize()
    mismatch = torch.zeros((1,), dtype=torch.int32, device=device)

    def buffer_set():
        b = dict(q=[], scale=[], code_scale=[], planes=[], c=[], y=[], mismatch=mismatch)
        for sp in specs:
            rows, k, n = sp["rows"], sp["k"], sp["n"]
            b["q"].append(torch.empty((rows, k), dtype=torch.uint8, device=device))
            b["scale"].append(torch.empty((rows,), dtype=torch.float32, device=device))
            b["code_scale"].append(torch.empty((rows,), dtype=torch.float32, device=device))
            b["planes"].append(DigitPlanes.empty(rows, k, nat.IMA_SCHEME_DIGITS3, device))
            b["c"].append(torch.empty((rows, n), dtype=torch.int64, device=device))
            b["y"].append(torch.empty((rows, n), dtype=torch.bfloat16, device=device))
        return b

    sets = [buffer_set(), buffer_set()]
    views = [[dict(sets[s]) for s in range(2)] for _ in range(layers)]   # own descriptor caches per layer
    cs = torch.cuda.Stream(device)                    # compute
    ms = torch.cuda.Stream(device, priority=-1)       # gather bookkeeping
    gs_copy = torch.cuda.Stream(device, priority=-1)  # copy kernels of the SM gather
    # copy streams: `--c4-ce-split` per destination rank
    ce_streams = [torch.cuda.Stream(device, priority=-1) for _ in range(world * args.c4_ce_split)]
    ce_done = [[torch.cuda.Event() for _ in range(world * args.c4_ce_split)] for _ in range(2)]
    computed = [torch.cuda.Event(), torch.cuda.Event()]
    drained = [torch.cuda.Event(), torch.cuda.Event()]

    # Gather buffers: every rank allocates two sets of gathered outputs (one per buffer set, so
    # that the copies of layer L and L + 1 never share a destination) and shares them through
    # CUDA IPC; each rank copies its shard of every output into every rank's buffer.  After its
    # copies of a buffer set a rank records an interprocess event, on which every receiver waits
    # before the timed region ends (receiver-side completion).
    own_bufs, peer_bufs, sent, peer_sent = [], [], [], []
    if world > 1:
        hb = int(lib.ima_ipc_handle_bytes())
        handles = []
        for s in range(2):
            for sp in specs:
                ptr, h = ctypes.c_void_p(), (ctypes.c_char * hb)()
                rows_full = tokens if not sp["col"] else tokens
                nat.call("ima_ipc_alloc", world * sp["rows"] * sp["n"] * 2, ctypes.byref(ptr), h)
                own_bufs.append(ptr.value)
                handles.append(bytes(h))
                del rows_full
        sent = [torch.cuda.Event(interprocess=True, blocking=False) for _ in range(2)]
        ev_handles = [e.ipc_handle() for e in sent]
        everyone = [None] * world
        dist.all_gather_object(everyone, (handles, ev_handles))
        for q in range(world):
            row, evs = [], []
            for i in range(2 * len(specs)):
                if q == rank:
                    row.append(own_bufs[i])
                else:
                    ptr = ctypes.c_void_p()
                    h = (ctypes.c_char * hb).from_buffer_copy(everyone[q][0][i])
                    nat.call("ima_ipc_open", h, ctypes.byref(ptr))
                    row.append(ptr.value)
            peer_bufs.append(row)
            peer_sent.append([None if q == rank else torch.cuda.Event.from_ipc_handle(device, everyone[q][1][s])
                              for s in range(2)])

    fused = world > 1 and args.c4_gather == "epilogue"
    sm_gather = world > 1 and args.c4_gather == "sm"
    copy_descs = []
    if sm_gather:
        # one copy launch per layer: every output shard to every rank's gathered buffer, the
        # destinations in the order rank, rank + 1, ... (the ranks write to different GPUs)
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        nat.call("ima_set_gemm_sm_limit", max(1, sms - args.c4_gather_sms))
        for s in range(2):
            descs = (nat.CopyDesc * (world * len(specs)))()
            i = 0
            for q in range(world):
                for p, sp in enumerate(specs):
                    shard = sp["rows"] * sp["n"] * 2
                    descs[i].dst = peer_bufs[(rank + q) % world][s * len(specs) + p] + rank * shard
                    descs[i].src = sets[s]["y"][p].data_ptr()
                    descs[i].bytes = shard
                    i += 1
            copy_descs.append(descs)
    if fused:
        # the GEMM epilogue stores every output chunk into every rank's gathered buffer
        for layer in range(layers):
            for s in range(2):
                # destinations in the order rank, rank + 1, ...: at any moment the ranks store
                # into different GPUs
                views[layer][s]["y_copies"] = [
                    [peer_bufs[(rank + q) % world][s * len(specs) + p] + rank * sp["rows"] * sp["n"] * 2
                     for q in range(world)]
                    for p, sp in enumerate(specs)]

    def gather(s: int) -> None:
        """Copies of this rank's output shards of buffer set s into every rank's gathered
        buffers (ordered after the GEMM that wrote them); with the fused gather the GEMM has
        written them already, and only the completion events are recorded."""
        computed[s].record(cs)
        if sm_gather:
            gs_copy.wait_event(computed[s])
            nat.check("ima_copy_many", lib.ima_copy_many(ctypes.byref(copy_descs[s]), len(copy_descs[s]),
                                                         2 * args.c4_gather_sms, gs_copy.cuda_stream))
            drained[s].record(gs_copy)
            sent[s].record(gs_copy)
            return
        if world == 1 or fused:
            drained[s].record(cs)
            if fused:
                sent[s].record(cs)
            return
        split = args.c4_ce_split
        for q in range(world):
            dst = (rank + q) % world                  # start at different peers on different ranks
            for part in range(split):                 # each copy in `split` pieces on as many streams
                st = ce_streams[dst * split + part]
                st.wait_event(computed[s])
                for p, sp in enumerate(specs):
                    shard = sp["rows"] * sp["n"] * 2
                    piece = -(-shard // (16 * split)) * 16
                    lo = part * piece
                    nbytes = max(0, min(piece, shard - lo))
                    if nbytes:
                        nat.call("ima_copy_async", peer_bufs[dst][s * len(specs) + p] + rank * shard + lo,
                                 sets[s]["y"][p].data_ptr() + lo, nbytes, st.cuda_stream)
                ce_done[s][q * split + part].record(st)
        for e in ce_done[s][:world * split]:
            ms.wait_event(e)
        drained[s].record(ms)
        sent[s].record(ms)

    gemm_marks: list | None = None

    def forward_layers() -> None:
        """One step: every layer, each on the buffer set it alternates with the previous one."""
        for layer in range(layers):
            s = layer % 2
            cs.wait_event(drained[s])        # the gathers of two layers ago have read this set
            v = views[layer][s]
            with torch.cuda.stream(cs):
                stacks[layer].quantize(xs, v)
                if gemm_marks is not None:
                    gemm_marks.append(torch.cuda.Event(enable_timing=True))
                    gemm_marks[-1].record(cs)
                stacks[layer].multiply(xs, v)
                if gemm_marks is not None:
                    gemm_marks.append(torch.cuda.Event(enable_timing=True))
                    gemm_marks[-1].record(cs)
                gather(s)
                stacks[layer].verify(xs, v)

    def finish_gathers() -> None:
        """The end of a timed region: this rank's copies are done and every peer's copies into
        this rank's buffers have landed."""
        for s in range(2):
            cs.wait_event(drained[s])
        if world > 1:
            dist.barrier()                   # every rank has enqueued its last copies and events
            for q in range(world):
                if q != rank:
                    for s in range(2):
                        cs.wait_event(peer_sent[q][s])

    def timed(fn, steps: int, warmup: int) -> float:
        for _ in range(warmup):
            fn()
        finish_gathers()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cs)
        for _ in range(steps):
            fn()
        finish_gathers()
        e1.record(cs)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    shapes_full = synthetic.qwen_layer_shapes(3584, 512, 18944)
    ops = sum(2.0 * tokens * s.n * s.k for s in shapes_full) * layers
    local_ops = sum(2.0 * sp["rows"] * sp["n"] * sp["k"] for sp in specs) * layers
    gather_bytes = sum(2 * (world - 1) * sp["rows"] * sp["n"] for sp in specs) * layers if world > 1 else 0
    int8_peak, peak_source = int8_tensor_peak()

    # ---- timed region: device-resident inputs (2.7 GB of digit planes per layer > L2) ----
    clock = ClockSampler(local)
    clock.start()
    time.sleep(0.3)
    mismatch.zero_()
    ms_step = timed(forward_layers, args.steps, args.warmup)
    clocks = clock.stop()
    bad = mismatch.clone()
    if world > 1:
        dist.all_reduce(bad)
    # the GEMM's share of the step: CUDA events around each layer's GEMM launch inside one more
    # step, so the roofline is taken inside the real step
    gemm_marks = []
    timed(forward_layers, 1, 0)
    gemm_ms = sum(gemm_marks[2 * i].elapsed_time(gemm_marks[2 * i + 1]) for i in range(layers))
    gemm_marks = None
    gt = torch.tensor([gemm_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
    gemm_ms = float(gt.item())
    gather_check = None
    if world > 1:
        # every rank's gathered buffers hold, for each buffer set, the outputs of the last layer
        # that used it on every rank: compare them with an NCCL all-gather of the local outputs
        ok, nbytes = True, 0
        with torch.cuda.stream(cs):
            for s in range(2):
                for p, sp in enumerate(specs):
                    shard = sp["rows"] * sp["n"]
                    mine = torch.empty((world * shard,), dtype=torch.bfloat16, device=device)
                    nat.call("ima_copy_async", mine.data_ptr(), own_bufs[s * len(specs) + p], world * shard * 2,
                             cs.cuda_stream)
                    ref = torch.empty_like(mine)
                    dist.all_gather_into_tensor(ref, sets[s]["y"][p].reshape(-1).contiguous())
                    ok = ok and bool(torch.equal(mine.view(torch.int16), ref.view(torch.int16)))
                    nbytes += world * shard * 2
        flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=device)
        dist.all_reduce(flag)
        gather_check = {"ok": int(flag.item()) == 0, "bytes_checked_per_gpu": nbytes,
                        "what": "each GPU's gathered buffers of both buffer sets vs an NCCL all-gather of the "
                                "ranks' local outputs, bit for bit"}

    # ---- end to end through the public API: host inputs in, the step's result out ----
    host_x = [x.cpu().pin_memory() for x in xs]
    last = len(specs) - 1                              # the final layer's down_proj
    host_out = torch.empty(sets[(layers - 1) % 2]["y"][last].shape, dtype=torch.bfloat16).pin_memory()
    host_bad = torch.empty((1,), dtype=torch.int32).pin_memory()
    cin = torch.cuda.Stream(device)

    def e2e_step() -> None:
        cin.wait_stream(cs)                            # the previous step no longer reads the inputs
        with torch.cuda.stream(cin):
            for x, hx in zip(xs, host_x):
                x.copy_(hx, non_blocking=True)
        cs.wait_stream(cin)
        forward_layers()
        with torch.cuda.stream(cs):
            host_out.copy_(sets[(layers - 1) % 2]["y"][last], non_blocking=True)
            host_bad.copy_(mismatch, non_blocking=True)

    e2e_ms = timed(e2e_step, max(2, min(args.steps, 5)), 1)
    h2d = sum(x.numel() * 2 for x in xs)
    d2h = host_out.numel() * 2 + 4

    # ---- CPU baseline (rank 0 of a 1-GPU run): the reference's CPU path on sampled rows of the
    # last two layers' linears, compared with the outputs the timed steps left in the buffers ----
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = c4_cpu_baseline(specs, stacks, xs, sets, layers, args.cpu_seconds)

    fig = ncu_figure("int_gemm_kernel<DIGITS3> c4") or {}
    gemm_tc = 9.0 * local_ops / (gemm_ms * 1e-3) / 1e12
    line = {
        "metric": C4_METRIC,
        "value": round(ops / (ms_step * 1e-3) / 1e12, 3),
        "unit": "TOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 digit planes -> int32 TMEM -> int64",
        "data": "synthetic (seeded Student-t activations, N(0,0.02) e4m3 weights; no checkpoint)",
        "config": {
            "workload": "c4: 196 FP8 linears of Qwen2.5-7B shape (28 layers), 16384 tokens in total, codebook "
                        "student, int64 outputs + per-product Freivalds check, bf16 outputs gathered to every GPU",
            "linears": 7 * layers,
            "tokens": tokens,
            "exact_int_ops_per_step": ops,
            "parallelism": f"token rows over {world} GPU(s), gate/up output columns over {world} GPU(s)",
            "gather": (None if world == 1 else
                       "fused into the GEMM epilogue: every output chunk stored into every GPU's gathered buffer "
                       "(CUDA-IPC peer memory, plain NVLink stores), receiver-side completion by interprocess "
                       "events" if fused else
                       f"one copy kernel per layer (512-byte warp stores into CUDA-IPC peer memory) on "
                       f"{args.c4_gather_sms} SMs kept from the GEMM, receiver-side completion by interprocess "
                       f"events" if sm_gather else
                       "copy engines: peer-to-peer copies into CUDA-IPC-shared buffers, receiver-side completion by "
                       "interprocess events"),
            "nvlink_bytes_received_per_gpu_per_step": gather_bytes,
            "l2": "inputs larger than L2 (0.70 GB of weight and 2.0 GB of activation digit planes per layer)",
            "activations": "the seven activation matrices of a layer are shared by the 28 layers (the work per "
                           "layer is unchanged)",
        },
        "freivalds_mismatch_rows": int(bad.item()),
        "gather_check": gather_check,
        "gpu_launches": sum(st.launches_per_forward() for st in stacks) * args.steps,
        "roofline": {
            "kernel": "int_gemm_kernel<DIGITS3>",
            "bound": "tensor",
            "achieved": round(gemm_tc, 2),
            "peak": round(int8_peak, 1) if int8_peak else None,
            "unit": "TOPS (int8 tensor ops, 9 digit products per exact product)",
            "frac": round(gemm_tc / int8_peak, 4) if int8_peak else None,
            "peak_source": peak_source,
            "gemm_ms_per_step": round(gemm_ms, 3),
            "exact_tops_gemm_only": round(local_ops / (gemm_ms * 1e-3) / 1e12, 2),
            "traffic": fig.get("dram_bytes_per_launch"),
            "traffic_algorithmic": fig.get("algorithmic_bytes_per_launch"),
            "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one layer's grouped GEMM launch "
                               f"at N = 1 ({fig.get('command')}); capture matches the current source: "
                               f"{fig.get('current')}") if fig else None,
            "timing": "CUDA events around each layer's GEMM launch inside one step (max over ranks)",
        },
        "e2e": {
            "value": round(ops / (e2e_ms * 1e-3) / 1e12, 3),
            "unit": "TOPS",
            "ms_per_step": round(e2e_ms, 3),
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "CodebookStack (quantize / multiply / verify per layer) with the activations copied in from "
                   "pinned host memory each step and the step's result (the last layer's down_proj output rows "
                   "of this GPU and the Freivalds verdict) copied back",
        },
        "clocks": clocks,
        "cpu_baseline": cpu,
        "measured_peaks": {k: measured_peaks().get(k) for k in ("hbm_gbs", "bf16_tflops")},
    }
    if sm_gather:
        nat.call("ima_set_gemm_sm_limit", 0)
    del stacks, sets, views
    torch.cuda.empty_cache()
    # ---- config 4, Hawkeye replay phase (same partition and gathers) ----
    if not args.no_hawkeye:
        try:
            line["c4_hawkeye"] = c4_hawkeye_phase(args, specs, xs, world, rank, device)
        except Exception as exc:  # noqa: BLE001
            line["c4_hawkeye"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()   # every rank's copies into the shared buffers are done
        for q in range(len(peer_bufs)):
            if q != rank:
                for ptr in peer_bufs[q]:
                    nat.call("ima_ipc_close", ptr)
        dist.barrier()   # every peer has unmapped this rank's buffers
        for ptr in own_bufs:
            nat.call("ima_ipc_free", ptr)
    if world == 1 and rank == 0:
        for key, fn in (("c1", run_c1), ("hawkeye_c2", lambda a: run_hawkeye(a, emit=False)),
                        ("class_counts_c3", run_class_counts_c3)):
            if (key == "hawkeye_c2" and args.no_hawkeye) or (key == "class_counts_c3" and args.no_class_counts):
                continue
            try:
                line[key] = fn(args)
            except Exception as exc:  # noqa: BLE001
                line[key] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def c4_cpu_baseline(specs, stacks, xs, sets, layers: int, budget_s: float) -> dict:
    """The reference's CPU path (torch quantiser expressions, torch int64 matmul, fp32 rescale)
    on sampled token rows of the last two layers' linears, whose outputs the timed steps left in
    the two buffer sets; rows split over all host threads.  The CPU results double as the
    parity check of those GPU outputs (int64 products and bf16 outputs, bit for bit)."""
    import oracle

    threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(1)
    rows = 64
    done_ops, t_used, checked, ok = 0.0, 0.0, 0, True
    try:
        for layer in (layers - 1, layers - 2):
            s = layer % 2
            for p, sp in enumerate(specs):
                if t_used >= budget_s:
                    break
                lin = stacks[layer].linears[p]
                x = xs[p][:rows].cpu()
                w, ws = lin.w_fp8.cpu(), lin.w_code_scale.cpu() * 512.0
                bias = lin.bias.cpu() if lin.bias is not None else None
                codes = oracle.fp8_codebook(w).to(torch.int64)
                t0 = time.perf_counter()
                c_ref, out_ref = oracle.torch_cpu_codebook_linear(x, w, ws.reshape(-1, 1), bias, threads=threads,
                                                                  w_codes=codes)
                t_used += time.perf_counter() - t0
                done_ops += 2.0 * rows * sp["n"] * sp["k"]
                same = torch.equal(sets[s]["c"][p][:rows].cpu(), c_ref) and torch.equal(
                    sets[s]["y"][p][:rows].cpu().view(torch.int16), out_ref.to(torch.bfloat16).view(torch.int16))
                ok = ok and same
                checked += rows
    finally:
        torch.set_num_threads(prev)
    return {
        "value": round(done_ops / t_used / 1e12, 6),
        "unit": "TOPS",
        "cores": threads,
        "kind": "port",
        "sample": f"{rows} token rows of each linear of the last two layers (rows split over {threads} threads), "
                  f"{t_used:.1f} s",
        "parity": {"rows_checked": checked, "ok": ok,
                   "what": "GPU int64 products and bf16 outputs of the timed steps vs the CPU results, bit for bit"},
    }


def c4_hawkeye_phase(args, specs, xs, world: int, rank: int, device) -> dict:
    """Config 4 through the direct Hawkeye replay: per layer, quantise and stage the seven
    activations (one fused launch each), replay the seven linears (round-robin on four side streams), gather the bf16
    outputs (NCCL all-gather per linear at N > 1).  Timed on the device, max over ranks."""
    from int_model_approximation_b200 import _native as nat
    from int_model_approximation_b200 import synthetic
    from int_model_approximation_b200.hawkeye import HawkeyeOperand

    dist = torch.distributed
    lib = nat.lib()
    tokens, layers = args.c4_tokens, args.c4_layers
    w_ops, w_scales = [], []
    for layer in range(layers):
        row_ops, row_ws = [], []
        for p, sp in enumerate(specs):
            w, ws, _b = c4_weights(sp, layer, p, device)
            row_ops.append(HawkeyeOperand(w))
            row_ws.append(ws.reshape(-1).to(torch.float32).contiguous())
            del w
        w_ops.append(row_ops)
        w_scales.append(row_ws)
    q = [torch.empty((sp["rows"], sp["k"]), dtype=torch.uint8, device=device) for sp in specs]
    scale = [torch.empty((sp["rows"],), dtype=torch.float32, device=device) for sp in specs]
    xop = [torch.empty((int(lib.ima_hawkeye_operand_bytes(sp["rows"], sp["k"])),), dtype=torch.uint8, device=device)
           for sp in specs]
    ys = [[torch.empty((sp["rows"], sp["n"]), dtype=torch.bfloat16, device=device) for sp in specs] for _ in range(2)]
    gathered = [torch.empty((world * sp["rows"], sp["n"]), dtype=torch.bfloat16, device=device) for sp in specs] \
        if world > 1 else []
    cs = torch.cuda.Stream(device)
    side = [torch.cuda.Stream(device) for _ in range(4)]
    gs = torch.cuda.Stream(device)
    done = [torch.cuda.Event(), torch.cuda.Event()]

    def step() -> None:
        for layer in range(layers):
            s = layer % 2
            cs.wait_event(done[s])
            sp_ = cs.cuda_stream
            for p, sp in enumerate(specs):
                rows, k = sp["rows"], sp["k"]
                nat.check("qp", lib.ima_hawkeye_quantize_prepare(xs[p].data_ptr(), nat.IMA_DTYPE_BF16, rows, k, k,
                                                                 scale[p].data_ptr(), q[p].data_ptr(), k,
                                                                 xop[p].data_ptr(), sp_))
            for st in side:
                st.wait_stream(cs)
            for p, sp in enumerate(specs):
                nat.check("r", lib.ima_hawkeye_replay(xop[p].data_ptr(), w_ops[layer][p].buffer.data_ptr(),
                                                      scale[p].data_ptr(), w_scales[layer][p].data_ptr(), sp["rows"],
                                                      sp["n"], sp["k"], 32, 14, -139, ys[s][p].data_ptr(), sp["n"],
                                                      None, sp["n"], side[p % len(side)].cuda_stream))
            for st in side:
                cs.wait_stream(st)
            if world > 1:
                gs.wait_stream(cs)
                with torch.cuda.stream(gs):
                    for p in range(len(specs)):
                        dist.all_gather_into_tensor(gathered[p], ys[s][p])
                done[s].record(gs)
            else:
                done[s].record(cs)
        for s in range(2):
            cs.wait_event(done[s])

    step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, args.c4_hawkeye_steps)
    e0.record(cs)
    for _ in range(steps):
        step()
    e1.record(cs)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    shapes_full = synthetic.qwen_layer_shapes(3584, 512, 18944)
    outputs = sum(tokens * s.n for s in shapes_full) * layers
    products = sum(tokens * s.n * s.k for s in shapes_full) * layers
    res = {"outputs_per_s": outputs / (ms * 1e-3), "products_per_s": products / (ms * 1e-3), "ms_per_step": ms,
           "steps": steps, "warmup": 1, "gather": "NCCL all_gather_into_tensor per linear" if world > 1 else None}
    if world == 1 and not args.no_cpu_baseline:
        import oracle

        rows = 8
        t_used, ok, checked = 0.0, True, 0
        s = (layers - 1) % 2
        for p, sp in enumerate(specs):
            w, ws, _b = c4_weights(sp, layers - 1, p, device)
            t0 = time.perf_counter()
            ref = oracle.hawkeye(q[p][:rows].cpu().view(torch.float8_e4m3fn), scale[p][:rows].cpu(), w.cpu(), ws.cpu())
            t_used += time.perf_counter() - t0
            ok = ok and torch.equal(ys[s][p][:rows].cpu().view(torch.int16), ref.to(torch.bfloat16).view(torch.int16))
            checked += rows
        res["cpu_baseline"] = {
            "value": sum(rows * sp["n"] * sp["k"] for sp in specs) / t_used, "unit": "products/s",
            "cores": max(1, min(32, os.cpu_count() or 1)), "kind": "port",
            "sample": f"{rows} token rows of each linear of the last layer through the oracle's C restatement of "
                      f"the replay, {t_used:.1f} s",
            "parity": {"rows_checked": checked, "ok": ok,
                       "what": "GPU bf16 outputs of the timed step vs the CPU replay, bit for bit"}}
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--hawkeye-cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-class-counts", action="store_true")
    ap.add_argument("--class-counts-only", action="store_true", help="only the config-3 class-count measurement")
    ap.add_argument("--c3-tokens", type=int, default=4096, help="token rows of config 3 (4096; fewer for ncu only)")
    ap.add_argument("--reference-rows", type=int, default=256)
    ap.add_argument("--profile-step", action="store_true", help="two eager forwards only (for ncu)")
    ap.add_argument("--profile-tokens", type=int, default=TOKENS)
    ap.add_argument("--hawkeye-only", action="store_true", help="only the config-2 Hawkeye measurement")
    ap.add_argument("--hawkeye-tokens", type=int, default=16384)
    ap.add_argument("--hawkeye-steps", type=int, default=3)
    ap.add_argument("--no-hawkeye", action="store_true", help="skip the config-2 Hawkeye object of the default line")
    ap.add_argument("--c4-tokens", type=int, default=16384)
    ap.add_argument("--c4-layers", type=int, default=28)
    ap.add_argument("--c4-hawkeye-steps", type=int, default=1)
    ap.add_argument("--c4-gather", choices=["ce", "sm", "epilogue"], default="ce",
                    help="N > 1: gather the outputs by copy-engine copies (default), by a copy kernel on "
                         "--c4-gather-sms SMs kept from the GEMM, or from the GEMM epilogue")
    ap.add_argument("--c4-gather-sms", type=int, default=8)
    ap.add_argument("--c4-ce-split", type=int, default=1,
                    help="copy-engine gather: streams per destination rank (each copy split into as many pieces)")
    ap.add_argument("--c1-only", action="store_true", help="only the config-1 measurement (one GPU)")
    ap.add_argument("--profile-c4", action="store_true", help="two eager forwards of --c4-layers layers (for ncu)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.c1_only:
        print(json.dumps({"c1": run_c1(args)}), flush=True)
    elif args.hawkeye_only:
        run_hawkeye(args)
    elif args.class_counts_only:
        print(json.dumps({"class_counts_c3": run_class_counts_c3(args)}), flush=True)
    elif args.profile_step:
        run_profile_step(args)
    elif args.profile_c4:
        run_profile_c4(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        # compute, gather bookkeeping, input and per-peer copy streams: more than the default 8
        # hardware queues, which would serialise unrelated streams (set before CUDA starts)
        os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
        run_headline(args)


if __name__ == "__main__":
    main()

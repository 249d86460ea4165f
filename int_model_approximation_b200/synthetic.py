"""Seeded synthetic inputs for the five workloads (no checkpoint or dataset is used).

Activations: Student-t(nu=4) * 0.5, drawn as z / sqrt(chi2_4 / 4) with
chi2_4 = -2 log(u1 u2), optionally with a fraction of entries scaled by 50 as
outliers, rounded to bf16.  Weights: N(0, 0.02) quantised per output channel to
e4m3 with scale = max(amax / 448, 1e-12) (the activation quantiser's formula applied
per row, evaluated by torch on the generator's device: on CUDA the division by 448 is a
multiplication by its fp32 reciprocal), weight_scale [N, 1] fp32.  Every tensor is drawn from its own
torch.Generator seeded with `seed`, on the device the generator lives on; the GPU
kernels and the CPU oracle are always fed the same materialised bytes.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

FP8_E4M3_MAX = 448.0


def _gen(seed: int, device: torch.device | str) -> torch.Generator:
    dev = torch.device(device)
    g = torch.Generator(device=dev.type if dev.type == "cpu" else dev)
    g.manual_seed(int(seed))
    return g


def student_t_activations(
    m: int,
    k: int,
    seed: int,
    *,
    device: torch.device | str = "cpu",
    outlier_fraction: float = 0.0,
    outlier_scale: float = 50.0,
    scale: float = 0.5,
    dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    g = _gen(seed, device)
    z = torch.randn((m, k), generator=g, device=device, dtype=torch.float32)
    u1 = torch.rand((m, k), generator=g, device=device, dtype=torch.float32).clamp_min_(1e-30)
    u2 = torch.rand((m, k), generator=g, device=device, dtype=torch.float32).clamp_min_(1e-30)
    chi2 = -2.0 * torch.log(u1 * u2)
    x = scale * z / torch.sqrt(chi2 / 4.0)
    if outlier_fraction > 0.0:
        count = int(m * k * outlier_fraction)
        idx = torch.randperm(m * k, generator=g, device=device)[:count]
        x.view(-1)[idx] *= outlier_scale
    return x.to(dtype)


def quantize_rows_e4m3(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row e4m3 quantisation (same formula as the per-token activation quantiser)."""
    w32 = w.to(torch.float32)
    s = (w32.abs().amax(dim=1, keepdim=True) / FP8_E4M3_MAX).clamp_min(1e-12)
    return (w32 / s).to(torch.float8_e4m3fn), s


def normal_fp8_weights(
    n: int, k: int, seed: int, *, device: torch.device | str = "cpu", std: float = 0.02
) -> tuple[torch.Tensor, torch.Tensor]:
    g = _gen(seed, device)
    w = torch.randn((n, k), generator=g, device=device, dtype=torch.float32) * std
    return quantize_rows_e4m3(w)


@dataclass(frozen=True)
class LinearShape:
    name: str
    n: int  # out_features
    k: int  # in_features


def qwen_layer_shapes(hidden: int, kv: int, inter: int) -> list[LinearShape]:
    return [
        LinearShape("q_proj", hidden, hidden),
        LinearShape("k_proj", kv, hidden),
        LinearShape("v_proj", kv, hidden),
        LinearShape("o_proj", hidden, hidden),
        LinearShape("gate_proj", inter, hidden),
        LinearShape("up_proj", inter, hidden),
        LinearShape("down_proj", hidden, inter),
    ]


def qwen05b_linears() -> list[LinearShape]:
    """The 168 FP8 linears of a Qwen2.5-0.5B-shaped model (24 layers)."""
    out = []
    for layer in range(24):
        for s in qwen_layer_shapes(896, 128, 4864):
            out.append(LinearShape(f"layers.{layer}.{s.name}", s.n, s.k))
    return out


def qwen7b_linears() -> list[LinearShape]:
    """The 196 FP8 linears of a Qwen2.5-7B-shaped model (28 layers)."""
    out = []
    for layer in range(28):
        for s in qwen_layer_shapes(3584, 512, 18944):
            out.append(LinearShape(f"layers.{layer}.{s.name}", s.n, s.k))
    return out


# The five benchmark configurations (0: one gate_proj linear at 16 tokens; 1-2: the 0.5B
# shapes, codebook at 512 tokens and Hawkeye at 16384; 3: down_proj class counts; 4: the 7B
# shapes at 16384 tokens).
CONFIGS = {
    0: dict(name="c0-gate-16tok", linears=[LinearShape("gate_proj", 4864, 896)], tokens=16, outliers=0.0),
    1: dict(name="c1-qwen0.5b-codebook-512tok", linears=None, tokens=512, outliers=0.0),
    2: dict(name="c2-qwen0.5b-hawkeye-16384tok", linears=None, tokens=16384, outliers=0.001),
    3: dict(name="c3-down-classcounts-4096tok", linears=[LinearShape("down_proj", 896, 4864)], tokens=4096, outliers=0.0),
    4: dict(name="c4-qwen7b-16384tok", linears=None, tokens=16384, outliers=0.0),
}


def config_linears(config: int) -> list[LinearShape]:
    c = CONFIGS[config]
    if c["linears"] is not None:
        return list(c["linears"])
    return qwen7b_linears() if config == 4 else qwen05b_linears()


def linear_seed(config: int, index: int) -> int:
    return 1000 * config + index


def make_linear_inputs(
    config: int,
    index: int,
    shape: LinearShape,
    *,
    tokens: int | None = None,
    device: torch.device | str = "cpu",
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(x bf16 [tokens, K], w_fp8 [N, K], w_scale [N, 1]) for one linear of a config."""
    c = CONFIGS[config]
    t = c["tokens"] if tokens is None else tokens
    seed = linear_seed(config, index)
    x = student_t_activations(t, shape.k, seed, device=device, outlier_fraction=c["outliers"])
    w, ws = normal_fp8_weights(shape.n, shape.k, seed + 500_000, device=device)
    return x, w, ws

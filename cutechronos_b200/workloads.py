"""Seeded synthetic workloads and the deterministic weight initialisation.

The reference quotes its numbers on private CSV price data that is not part
of the project; these generators stand in for it with the shapes, lengths,
NaN rates and group structure of the five benchmark configurations.  The
weight initialisation re-initialises every parameter of a module that has
the reference's parameter names and registration order
(cutechronos/model.py:419-468), so the reference module, the CPU oracle and
this package all see bit-identical weights for a given seed.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


@torch.no_grad()
def seeded_init_(module: torch.nn.Module, seed: int = 0, std: float = 0.02) -> torch.nn.Module:
    """N(0, std) for every weight, bias and the ``shared`` embedding; 1.0 for
    every RMS-norm weight; parameters visited in ``named_parameters`` order
    under ``torch.manual_seed(seed)`` (drawn on the CPU, then copied)."""
    torch.manual_seed(seed)
    for name, p in module.named_parameters():
        if name.endswith("layer_norm_weight"):
            p.fill_(1.0)
        else:
            t = torch.empty(p.shape, dtype=torch.float32)
            t.normal_(0.0, std)
            p.copy_(t.to(p.dtype))
    return module


def seeded_state_dict(names_shapes, seed: int = 0, std: float = 0.02) -> dict:
    """Same values as :func:`seeded_init_` for an ordered list of
    (name, shape) pairs, as fp32 CPU tensors."""
    torch.manual_seed(seed)
    out = {}
    for name, shape in names_shapes:
        t = torch.empty(shape, dtype=torch.float32)
        if name.endswith("layer_norm_weight"):
            t.fill_(1.0)
        else:
            t.normal_(0.0, std)
        out[name] = t
    return out


def _nan_mask(gen: torch.Generator, shape, frac: float) -> torch.Tensor:
    return torch.rand(shape, generator=gen) < frac


@dataclass
class Workload:
    name: str
    context: torch.Tensor          # (B, L) float32 CPU, NaN = missing
    group_ids: torch.Tensor | None  # (B,) int64 or None (each series its own group)
    prediction_length: int
    dtype: str                     # "f32" or "bf16"

    @property
    def num_output_patches(self) -> int:
        return math.ceil(self.prediction_length / 16)


def config0() -> Workload:
    """B=1, ctx 512, pred 64, fp32: random walk + period-24 sinusoid, 5% NaN."""
    g = torch.Generator().manual_seed(0)
    L = 512
    t = torch.arange(L, dtype=torch.float32)
    x = torch.cumsum(torch.randn(1, L, generator=g), -1) + 10 * torch.sin(2 * math.pi * t / 24)
    x[_nan_mask(g, x.shape, 0.05)] = float("nan")
    return Workload("cfg0_b1_ctx512_f32", x, None, 64, "f32")


def series_cfg1(B: int, L: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    t = torch.arange(L, dtype=torch.float32)
    x = (torch.cumsum(torch.randn(B, L, generator=g), -1)
         + 5 * torch.sin(2 * math.pi * t / 24) + 3 * torch.sin(2 * math.pi * t / 168)
         + 0.1 * torch.randn(B, L, generator=g))
    x[_nan_mask(g, x.shape, 0.02)] = float("nan")
    return x


def config1(B: int = 256, L: int = 2048) -> Workload:
    """B=256 univariate, ctx 2048, pred 64, bf16; 2% NaN."""
    return Workload("cfg1_b256_ctx2048_bf16", series_cfg1(B, L, 1), None, 64, "bf16")


def config2(groups: int = 64, variates: int = 8, L: int = 2048) -> Workload:
    """64 groups x 8 correlated variates (rho 0.7), ctx 2048, pred 64, bf16."""
    g = torch.Generator().manual_seed(2)
    z = torch.cumsum(torch.randn(groups, 1, L, generator=g), -1)
    e = torch.cumsum(torch.randn(groups, variates, L, generator=g), -1)
    x = (0.7 * z + math.sqrt(1 - 0.49) * e).reshape(groups * variates, L)
    x[_nan_mask(g, x.shape, 0.02)] = float("nan")
    gid = torch.arange(groups).repeat_interleave(variates)
    return Workload("cfg2_g64x8_ctx2048_bf16", x, gid, 64, "bf16")


def config3(B: int = 32, L: int = 8192) -> Workload:
    """B=32, ctx 8192, pred 128, bf16: AR(2)+trend, 25% left-padded to a
    valid length drawn from U[4096, 8192]."""
    rng = np.random.default_rng(3)
    eps = rng.standard_normal((B, L)).astype(np.float64)
    x = np.zeros((B, L))
    for t in range(L):
        a1 = x[:, t - 1] if t >= 1 else 0.0
        a2 = x[:, t - 2] if t >= 2 else 0.0
        x[:, t] = 0.6 * a1 + 0.3 * a2 + eps[:, t]
    x = x + 0.01 * np.arange(L)[None, :]
    padded = rng.random(B) < 0.25
    lengths = rng.integers(4096, 8193, size=B)
    for b in range(B):
        if padded[b]:
            x[b, : L - lengths[b]] = np.nan
    return Workload("cfg3_b32_ctx8192_bf16", torch.from_numpy(x.astype(np.float32)), None, 128, "bf16")


def config4(B: int = 4096, L: int = 512) -> Workload:
    """4096 univariate series, ctx 512, pred 64, bf16 (sharding sweep)."""
    return Workload("cfg4_b4096_ctx512_bf16", series_cfg1(B, L, 4), None, 64, "bf16")


CONFIGS = {0: config0, 1: config1, 2: config2, 3: config3, 4: config4}

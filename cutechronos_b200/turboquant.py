"""TurboQuant-style K/V quantisation hook of the time attention: host side.

``CuteChronos2Model.enable_turboquant_kv`` (cutechronos/model.py:615-667 of
lee101/cutedsl) fake-quantises the time-attention K and V vectors (64 values
each, after RoPE) before the attention, as the reference's ``TurboQuantizer``
does (tubroquant/quantizer.py:41-178):

  unit = x / ||x||, rotated by a random orthogonal rotation (Hadamard with
  random signs and permutation, or a dense QR matrix), each coordinate
  replaced by its Lloyd-Max centroid for the coordinate distribution of a
  uniform point on the 64-sphere (``mse`` mode: ``bits`` per coordinate), and
  in ``prod`` mode (``bits - 1`` for the centroids) the residual's 1-bit QJL
  sketch (signs of a Gaussian projection) added back; the result is rotated
  back and scaled by the norm stored in ``norm_dtype``.

This module builds each quantiser's parameters on the host - the rotation
from the same seeded torch generators as the reference, the codebook by a
Lloyd-Max iteration of its own (same problem and stopping rule as
tubroquant/codebooks.py:20-58) - and hands them to the device kernel
``cc2_kv_quant`` (csrc/kvquant.cu), which the forward runs between the QKV
GEMM and the time attention.  The device path has no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import functools
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as nat

MODES = {"mse": 0, "prod": 1}
ROTATIONS = {"hadamard": 0, "qr": 1}
NORM_DTYPES = {"float16": 0, "bfloat16": 1, "float32": 2}
NORM_BYTES = {"float16": 2, "bfloat16": 2, "float32": 4}


@functools.lru_cache(maxsize=None)
def lloyd_max_codebook(dim: int, bits: int, grid: int = 32769) -> tuple[np.ndarray, np.ndarray]:
    """Centroids (2**bits, ascending) and the inner bucket boundaries
    (2**bits - 1) of the MSE-optimal scalar quantiser for one coordinate of a
    uniform point on the unit sphere in ``dim`` dimensions, whose density on
    [-1, 1] is proportional to (1 - x^2)^((dim - 3) / 2).

    Lloyd-Max on a uniform grid of ``grid`` points: centroids start at the
    density's quantiles (k + 1/2) / 2**bits, then alternate "boundaries =
    midpoints of neighbouring centroids" and "centroid = mean of its bucket"
    until no centroid moves by 1e-8 (at most 256 rounds)."""
    if bits <= 0:
        return np.zeros(1, np.float32), np.zeros(0, np.float32)
    n = 1 << bits
    xs = np.linspace(-1.0, 1.0, grid)
    log_c = math.lgamma(dim / 2) - 0.5 * math.log(math.pi) - math.lgamma((dim - 1) / 2)
    dens = math.exp(log_c) * np.power(np.clip(1.0 - xs * xs, 0.0, None), max((dim - 3) / 2, 0.0))
    w = dens / max(dens.sum(), 1e-12)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    cent = np.sort(np.interp((np.arange(n) + 0.5) / n, cdf, xs))
    for _ in range(256):
        cuts = 0.5 * (cent[:-1] + cent[1:])
        bucket = np.searchsorted(cuts, xs, side="right")
        new = cent.copy()
        for k in range(n):
            sel = bucket == k
            mass = w[sel].sum()
            if mass > 0:
                new[k] = float((w[sel] * xs[sel]).sum() / mass)
        done = np.max(np.abs(new - cent)) < 1e-8
        cent = new
        if done:
            break
    cuts = 0.5 * (cent[:-1] + cent[1:])
    return cent.astype(np.float32), cuts.astype(np.float32)


def hadamard_params(dim: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Random signs (+-1) and permutation of the structured rotation, drawn
    from torch's CPU generator in the reference's order (rotation.py:31-45)."""
    g = torch.Generator().manual_seed(seed)
    signs = torch.where(torch.rand(dim, generator=g) > 0.5, 1.0, -1.0)
    perm = torch.randperm(dim, generator=g)
    return signs.float(), perm


def dense_rotation(dim: int, seed: int) -> torch.Tensor:
    """Q of the QR factorisation of a seeded Gaussian matrix (rotation.py:57-70)."""
    g = torch.Generator().manual_seed(seed)
    q, _ = torch.linalg.qr(torch.randn(dim, dim, generator=g))
    return q.float().contiguous()


def qjl_projection(dim: int, seed: int) -> torch.Tensor:
    """Gaussian projection of the QJL residual sketch (quantizer.py:72-75)."""
    g = torch.Generator().manual_seed(seed + 1729)
    return torch.randn(dim, dim, generator=g).float().contiguous()


class KVQ(C.Structure):
    """Mirror of ``cc2_kvq`` (include/cc2.h)."""

    _fields_ = [("mode", C.c_int), ("bits", C.c_int), ("rotation", C.c_int), ("norm_dtype", C.c_int),
                ("signs", C.c_void_p), ("perm", C.c_void_p), ("inv_perm", C.c_void_p), ("matrix", C.c_void_p),
                ("codebook", C.c_void_p), ("boundaries", C.c_void_p), ("proj", C.c_void_p)]


@dataclass
class TurboQuantParams:
    """One quantiser (one layer's K or V): its settings and device tensors."""

    dim: int
    bits: int
    mode: str
    rotation: str
    seed: int
    norm_dtype: str
    tensors: dict

    @property
    def mse_bits(self) -> int:
        return self.bits if self.mode == "mse" else max(self.bits - 1, 0)

    @classmethod
    def build(cls, dim: int = 64, bits: int = 4, *, mode: str = "mse", rotation: str = "hadamard", seed: int = 0,
              norm_dtype: str = "float16", device="cuda") -> "TurboQuantParams":
        if bits < 0:
            raise ValueError(f"bits must be >= 0, got {bits}")
        if mode not in MODES:
            raise ValueError(f"mode must be 'mse' or 'prod', got {mode}")
        if rotation not in ROTATIONS:
            raise ValueError(f"Unknown rotation kind: {rotation}")
        if norm_dtype not in NORM_DTYPES:
            raise ValueError(f"norm_dtype must be one of {sorted(NORM_DTYPES)}, got {norm_dtype}")
        if dim != 64:
            raise ValueError(f"the device quantiser works on 64-value vectors (d_kv), got {dim}")
        mse_bits = bits if mode == "mse" else max(bits - 1, 0)
        if mse_bits > 8:
            raise ValueError(f"at most 8 bits per coordinate for the centroids, got {mse_bits}")
        t = {}
        if rotation == "hadamard":
            signs, perm = hadamard_params(dim, seed)
            inv = torch.empty_like(perm)
            inv[perm] = torch.arange(dim)
            t["signs"], t["perm"], t["inv_perm"] = signs, perm.to(torch.int32), inv.to(torch.int32)
        else:
            t["matrix"] = dense_rotation(dim, seed)
        cb, cuts = lloyd_max_codebook(dim, mse_bits)
        t["codebook"] = torch.from_numpy(cb)
        t["boundaries"] = torch.from_numpy(cuts) if cuts.size else torch.zeros(1)
        if mode == "prod":
            t["proj"] = qjl_projection(dim, seed)
        t = {k: v.contiguous().to(device) for k, v in t.items()}
        return cls(dim, bits, mode, rotation, seed, norm_dtype, t)

    def native(self) -> KVQ:
        p = lambda k: self.tensors[k].data_ptr() if k in self.tensors else None  # noqa: E731
        return KVQ(MODES[self.mode], self.bits, ROTATIONS[self.rotation], NORM_DTYPES[self.norm_dtype],
                   p("signs"), p("perm"), p("inv_perm"), p("matrix"), p("codebook"), p("boundaries"), p("proj"))

    def quantized_bytes_per_vector(self) -> int:
        """Packed payload of one vector as the reference counts it
        (quantizer.py:31-38): the bit-packed centroid indices and the norm, and
        in prod mode the packed QJL signs and the residual norm."""
        n = (self.dim * self.mse_bits + 7) // 8 + NORM_BYTES[self.norm_dtype]
        if self.mode == "prod":
            n += (self.dim + 7) // 8 + NORM_BYTES[self.norm_dtype]
        return n


def kv_quant(qkv: torch.Tensor, rows: int, heads: int, key: TurboQuantParams | None,
             value: TurboQuantParams | None, *, q_col: int, k_col: int, v_col: int,
             rope_cs: torch.Tensor | None = None, rope_period: int = 0, stats: torch.Tensor | None = None) -> None:
    """In place on the packed [Q|K|V] rows: RoPE on Q and K (when ``rope_cs``),
    then K and V replaced by their quantised reconstructions.  ``stats``
    (float32 (4,), device) accumulates K squared error, K max |error|, V
    squared error, V max |error|."""
    if not qkv.is_cuda:
        raise RuntimeError("cutechronos_b200 kernels take CUDA tensors only (no CPU path)")
    code = {torch.bfloat16: nat.CC2_BF16, torch.float32: nat.CC2_F32}[qkv.dtype]
    kq = key.native() if key is not None else None
    vq = value.native() if value is not None else None
    nat.check(nat.load().cc2_kv_quant(
        code, qkv.data_ptr(), qkv.stride(0), rows, q_col, k_col, v_col, heads,
        C.byref(kq) if kq is not None else None, C.byref(vq) if vq is not None else None,
        rope_cs.data_ptr() if rope_cs is not None else None, rope_period,
        stats.data_ptr() if stats is not None else None, torch.cuda.current_stream(qkv.device).cuda_stream),
        "cc2_kv_quant")

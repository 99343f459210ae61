"""CPU oracle of the TurboQuant K/V fake-quantiser of the time attention.

TEST INFRASTRUCTURE ONLY (only ``tests/`` may import it).  Restates, in plain
torch on the CPU, ``TurboQuantizer.forward`` of the reference
(tubroquant/quantizer.py:119-178: encode then decode) with the rotations of
tubroquant/rotation.py:11-70.  The quantiser's parameters (rotation signs and
permutation or dense matrix, codebook, boundaries, projection) are inputs, so
the same parameters drive this oracle, the reference and the CUDA kernel.

Parity pin: ``tests/golden/make_turboquant_golden.py`` runs the reference's
own quantiser on seeded inputs and commits its parameters and outputs;
``tests/test_turboquant.py`` checks this restatement against them.
"""

from __future__ import annotations

import math

import torch


def fwht(x: torch.Tensor) -> torch.Tensor:
    """Fast Walsh-Hadamard transform on the last dimension, butterflies of
    width 1, 2, 4, ... (rotation.py:11-25)."""
    dim = x.shape[-1]
    y, h = x, 1
    while h < dim:
        y = y.reshape(*y.shape[:-1], -1, 2 * h)
        a, b = y[..., :h], y[..., h:]
        y = torch.cat((a + b, a - b), dim=-1).reshape(*x.shape[:-1], dim)
        h *= 2
    return y


def rotate(x, signs=None, perm=None, matrix=None):
    """Forward rotation (rotation.py:47-49 Hadamard, 66-67 dense)."""
    if matrix is not None:
        return x @ matrix.t()
    return fwht(x[..., perm.long()] * signs) * (x.shape[-1] ** -0.5)


def rotate_inverse(x, signs=None, inv_perm=None, matrix=None):
    """Inverse rotation (rotation.py:51-54 Hadamard, 69-70 dense)."""
    if matrix is not None:
        return x @ matrix
    y = fwht(x) * (x.shape[-1] ** -0.5)
    return (y * signs)[..., inv_perm.long()]


def fake_quant(x: torch.Tensor, *, mode: str, bits: int, codebook, boundaries, signs=None, perm=None,
               inv_perm=None, matrix=None, proj=None, norm_dtype=torch.float16, idx_override=None,
               sign_override=None, internals=None):
    """-> (decoded float32, stats dict) as TurboQuantizer.forward
    (quantizer.py:119-178) computes them; x (..., 64) any float dtype.

    Test hooks (not in the reference): ``idx_override`` / ``sign_override``
    replace the bucket indices / QJL signs (for re-running a vector with one
    decision at a bucket edge taken the other way); a dict passed as
    ``internals`` receives the rotated unit vector ``y``, the indices ``idx``,
    the QJL projections ``sr`` and the signs ``sgn``."""
    dim = x.shape[-1]
    mse_bits = bits if mode == "mse" else max(bits - 1, 0)
    xf = x.float()
    norms = xf.norm(dim=-1, keepdim=True)
    unit = torch.where(norms > 0, xf / norms.clamp_min(1e-12), torch.zeros_like(xf))
    if mse_bits == 0:
        mse_unit = torch.zeros_like(unit)
    else:
        y = rotate(unit, signs, perm, matrix)
        idx = torch.bucketize(y, boundaries) if idx_override is None else idx_override
        if internals is not None:
            internals.update(y=y, idx=idx)
        mse_unit = rotate_inverse(codebook[idx].float(), signs, inv_perm, matrix)
    recon = mse_unit
    if mode == "prod":
        residual = unit - mse_unit
        rnorm = residual.norm(dim=-1, keepdim=True).to(norm_dtype).float()
        if bits == 0:
            sgn = torch.ones_like(residual)
        else:
            sr = torch.einsum("...d,ed->...e", residual, proj.float())
            sgn = torch.where(sr >= 0, 1.0, -1.0) if sign_override is None else sign_override
            if internals is not None:
                internals.update(sr=sr, sgn=sgn)
        coeff = math.sqrt(math.pi / 2.0) / dim
        recon = mse_unit + coeff * rnorm * torch.einsum("...e,ed->...d", sgn, proj.float())
    out = recon * norms.to(norm_dtype).float()
    stats = {"sse": float(((out - xf) ** 2).sum().item()), "max_abs_error": float((out - xf).abs().max().item()),
             "count": xf.numel()}
    return out, stats

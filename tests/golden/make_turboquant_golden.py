"""Generate tests/golden/turboquant.npz from the reference's TurboQuantizer.

Runs ``tubroquant.quantizer.TurboQuantizer`` (lee101/cutedsl) on seeded
64-value vectors for each (mode, bits, rotation) case and stores the
quantiser's parameters (rotation signs/permutation or matrix, codebook,
boundaries, QJL projection), the inputs, the decoded outputs and the stats.
The reference checkout is needed only to regenerate.

Usage:  python tests/golden/make_turboquant_golden.py --reference <path to reference checkout>
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
CASES = [("mse", 4, "hadamard", 3), ("prod", 4, "hadamard", 4), ("mse", 2, "hadamard", 5), ("prod", 3, "qr", 6),
         ("mse", 1, "qr", 7), ("prod", 1, "hadamard", 8), ("mse", 8, "hadamard", 9)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from tubroquant.codebooks import get_codebook
    from tubroquant.quantizer import TurboQuantizer

    out, meta = {}, []
    for i, (mode, bits, rot, seed) in enumerate(CASES):
        q = TurboQuantizer(dim=64, bits=bits, mode=mode, rotation=rot, seed=seed)
        g = torch.Generator().manual_seed(100 + i)
        x = (torch.randn(96, 64, generator=g) * 2.0).to(torch.bfloat16)
        x[7] = 0  # a zero vector
        y = q(x)
        dec = q.decode(q.encode(x))
        p = f"c{i}_"
        out[p + "x"] = x.float().numpy()
        out[p + "decoded"] = dec.float().numpy()
        out[p + "codebook"] = q.codebook.numpy()
        out[p + "boundaries"] = q.boundaries.numpy()
        if rot == "hadamard":
            out[p + "signs"] = q.rotation.signs.numpy()
            out[p + "perm"] = q.rotation.perm.numpy()
        else:
            out[p + "matrix"] = q.rotation.matrix.numpy()
        if mode == "prod":
            out[p + "proj"] = q.proj.numpy()
        meta.append({"mode": mode, "bits": bits, "rotation": rot, "seed": seed, **q.last_stats})
    for bits in range(0, 9):
        cb, cuts = get_codebook(64, bits)
        out[f"codebook64_{bits}"] = cb.numpy()
        out[f"boundaries64_{bits}"] = cuts.numpy()
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "turboquant.npz", **out)
    print("wrote", HERE / "turboquant.npz")


if __name__ == "__main__":
    main()

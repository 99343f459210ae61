"""Generate tests/golden/pipeline_host.npz from the reference pipeline itself.

Calls the reference's ``cutechronos.pipeline._select_quantiles``
(pipeline.py:24-58) and ``CuteChronos2Pipeline._left_pad_and_stack_rows`` +
the ``_finalize_context_batch`` truncation (pipeline.py:221-243) on seeded
inputs and stores inputs and outputs.  The reference checkout is only needed
when (re)generating; the tests read the committed ``.npz``.

Usage:  python tests/golden/make_pipeline_golden.py --reference <path to reference checkout>
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

TRAINED = [0.01, 0.05, 0.1, 0.15, 0.2, 0.25, 0.3, 0.35, 0.4, 0.45, 0.5,
           0.55, 0.6, 0.65, 0.7, 0.75, 0.8, 0.85, 0.9, 0.95, 0.99]
LEVEL_SETS = {
    "default": [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9],
    "mixed": [0.5, 0.33, 0.025, 0.999, 0.001, 0.875, 0.01, 0.99],
    "median": [0.5],
    "all": TRAINED,
}
# (row lengths, context_length) of the stacking cases; 0 = an empty series
STACK_CASES = [([5, 3, 8], 512), ([700, 20, 513, 1], 512), ([0, 4], 16), ([31, 32, 33], 32)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from cutechronos.pipeline import CuteChronos2Pipeline, _select_quantiles

    out = {}
    g = torch.Generator().manual_seed(7)
    # fp32 forecasts, and fp32 values that are exactly bf16 (what a bf16 model returns)
    p32 = torch.randn(6, 21, 40, generator=g) * 50 + 100
    pbf = (torch.randn(6, 21, 40, generator=g) * 3).to(torch.bfloat16).float()
    out["preds_f32"] = p32.numpy()
    out["preds_bf16_as_f32"] = pbf.numpy()
    for name, levels in LEVEL_SETS.items():
        out[f"levels_{name}"] = np.asarray(levels, dtype=np.float64)
        out[f"sel_f32_{name}"] = _select_quantiles(p32, TRAINED, levels).numpy()
        out[f"sel_bf16_{name}"] = _select_quantiles(pbf, TRAINED, levels).numpy()
    for ci, (lens, ctx_len) in enumerate(STACK_CASES):
        rows = [torch.randn(n, generator=g) for n in lens]
        rows[0][:1] = float("nan") if lens[0] else rows[0][:1]
        stacked = CuteChronos2Pipeline._left_pad_and_stack_rows(rows)
        if stacked.shape[-1] > ctx_len:
            stacked = stacked[..., -ctx_len:]
        out[f"stack{ci}_values"] = torch.cat(rows).numpy()
        out[f"stack{ci}_lens"] = np.asarray(lens, dtype=np.int64)
        out[f"stack{ci}_ctxlen"] = np.asarray(ctx_len)
        out[f"stack{ci}_out"] = stacked.numpy()
    np.savez_compressed(HERE / "pipeline_host.npz", **out)
    print("wrote", HERE / "pipeline_host.npz")


if __name__ == "__main__":
    main()

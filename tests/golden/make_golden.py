"""Generate the golden fixtures under tests/golden/ from the reference itself.

Runs the reference ``cutechronos.model.CuteChronos2Model`` (lee101/cutedsl)
on the CPU through its own public API, with weights re-initialised by
``cutechronos_b200.workloads.seeded_init_`` and seeded inputs, and stores the
inputs and outputs as small ``.npz`` files.  The reference checkout is only
needed when (re)generating; the tests read the committed ``.npz`` files.

Usage:  python tests/golden/make_golden.py --reference <path to reference checkout>
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from cutechronos_b200.workloads import config0, seeded_init_  # noqa: E402

SMALL = dict(d_model=128, d_kv=64, d_ff=256, num_layers=2, num_heads=2, dropout_rate=0.0,
             layer_norm_epsilon=1e-6, dense_act_fn="relu", rope_theta=10000.0, vocab_size=2,
             reg_token_id=1, context_length=512, input_patch_size=16, input_patch_stride=16,
             output_patch_size=16, use_reg_token=True, use_arcsinh=True, time_encoding_scale=512)


def _ctx(B, L, nan_frac, seed, scale=1.0, offset=0.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.cumsum(torch.randn(B, L, generator=g), -1) * scale + offset
    x[torch.rand(B, L, generator=g) < nan_frac] = float("nan")
    return x


def small_cases():
    cases = []
    cases.append(("ragged_nan", _ctx(3, 100, 0.1, 11), None, 2, None))
    gx = _ctx(4, 64, 0.05, 12)
    cases.append(("groups_2x2", gx, None, 1, torch.tensor([0, 0, 1, 1])))
    cases.append(("truncate_700", _ctx(2, 700, 0.0, 13), None, 4, None))
    x = _ctx(4, 48, 0.0, 14)
    x[0] = float("nan")          # all-NaN series
    x[1] = 3.5                   # constant series (scale 0 -> 1e-5)
    x[2, :20] = float("nan")     # left padding
    cases.append(("edge_rows", x, None, 1, None))
    x = _ctx(2, 40, 0.1, 15)
    m = (torch.rand(2, 40, generator=torch.Generator().manual_seed(16)) > 0.2).float()
    m[torch.isnan(x)] = 0.0
    cases.append(("explicit_mask", x, m, 2, None))
    x = _ctx(5, 33, 0.2, 17, scale=1e3, offset=1e6)
    cases.append(("large_scale_groups", x, None, 3, torch.tensor([2, 0, 2, 1, 0])))
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from cutechronos.model import CuteChronos2Config, CuteChronos2Model

    torch.set_num_threads(8)
    names = {}

    # ---- small config: full forward in fp32 and bf16 + preprocessing -------
    cfg = CuteChronos2Config(**SMALL)
    model = seeded_init_(CuteChronos2Model(cfg).eval(), seed=0)
    names["small"] = [n for n, _ in model.named_parameters()]
    out = {}
    for name, ctx, mask, N, gid in small_cases():
        with torch.no_grad():
            y32 = model(ctx.clone(), context_mask=mask, num_output_patches=N, group_ids=gid)
            pcx, amx, (locx, scx) = model._prepare_patched_context(ctx.clone(), mask)
        out[f"{name}/context"] = ctx.numpy()
        if mask is not None:
            out[f"{name}/context_mask"] = mask.numpy()
        if gid is not None:
            out[f"{name}/group_ids"] = gid.numpy()
        out[f"{name}/N"] = np.array(N)
        out[f"{name}/out_f32"] = y32.numpy()
        out[f"{name}/patched"] = pcx.numpy()
        out[f"{name}/attn"] = amx.numpy()
        out[f"{name}/loc"] = locx.numpy()
        out[f"{name}/scale"] = scx.numpy()
    mb = seeded_init_(CuteChronos2Model(cfg).eval(), seed=0).to(torch.bfloat16)
    for name, ctx, mask, N, gid in small_cases():
        with torch.no_grad():
            yb = mb(ctx.clone(), context_mask=mask, num_output_patches=N, group_ids=gid)
        out[f"{name}/out_bf16"] = yb.float().numpy()
    np.savez_compressed(HERE / "small_model.npz", **out)

    # ---- full Chronos-2-base config, configs[0] input ------------------------
    cfg = CuteChronos2Config()
    model = seeded_init_(CuteChronos2Model(cfg).eval(), seed=0)
    names["base"] = [n for n, _ in model.named_parameters()]
    w = config0()
    with torch.no_grad():
        y32 = model(w.context.clone(), num_output_patches=w.num_output_patches)
        model = model.to(torch.bfloat16)
        yb = model(w.context.clone(), num_output_patches=w.num_output_patches)
    np.savez_compressed(HERE / "base_cfg0.npz", context=w.context.numpy(), out_f32=y32.numpy(),
                        out_bf16=yb.float().numpy(), N=np.array(w.num_output_patches))
    (HERE / "param_names.json").write_text(json.dumps(names, indent=0))
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()

"""Shared fixtures.  Tests marked ``gpu`` need a B200 and the built library;
everything else runs on the CPU (oracle, host logic, C-ABI surface)."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))

SMALL = dict(d_model=128, d_kv=64, d_ff=256, num_layers=2, num_heads=2, context_length=512,
             time_encoding_scale=512)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the built native library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden_small():
    z = np.load(GOLDEN / "small_model.npz")
    cases = {}
    for key in z.files:
        name, field = key.split("/")
        cases.setdefault(name, {})[field] = z[key]
    return cases


@pytest.fixture(scope="session")
def golden_base():
    return dict(np.load(GOLDEN / "base_cfg0.npz"))


@pytest.fixture(scope="session")
def param_names():
    return json.loads((GOLDEN / "param_names.json").read_text())


def small_config(**kw):
    from cutechronos_b200.model import CuteChronos2Config
    d = dict(SMALL)
    d.update(kw)
    return CuteChronos2Config(**d)


def oracle_config(**kw):
    from oracle.chronos2_oracle import OracleConfig
    d = dict(SMALL)
    d.update(kw)
    return OracleConfig(**d)


def case_inputs(c):
    ctx = torch.from_numpy(c["context"])
    mask = torch.from_numpy(c["context_mask"]) if "context_mask" in c else None
    gid = torch.from_numpy(c["group_ids"]) if "group_ids" in c else None
    return ctx, mask, int(c["N"]), gid


def hf_state_dict(model) -> dict:
    """The HuggingFace Chronos-2 key layout of a CuteChronos2Model's weights."""
    sd = {"shared.weight": model.shared.weight, "encoder.final_layer_norm.weight": model.final_layer_norm_weight}
    for name in ("input_patch_embedding", "output_patch_embedding"):
        for layer in ("hidden_layer", "output_layer", "residual_layer"):
            for prm in ("weight", "bias"):
                sd[f"{name}.{layer}.{prm}"] = getattr(getattr(getattr(model, name), layer), prm)
    for i, b in enumerate(model.blocks):
        pre = f"encoder.block.{i}.layer"
        for j, att in ((0, b.time_attn), (1, b.group_attn)):
            sd[f"{pre}.{j}.layer_norm.weight"] = att.layer_norm_weight
            for prj in "qkvo":
                sd[f"{pre}.{j}.self_attention.{prj}.weight"] = getattr(att, prj).weight
        sd[f"{pre}.2.layer_norm.weight"] = b.feed_forward.layer_norm_weight
        sd[f"{pre}.2.mlp.wi.weight"] = b.feed_forward.wi.weight
        sd[f"{pre}.2.mlp.wo.weight"] = b.feed_forward.wo.weight
    return {k: v.detach().contiguous() for k, v in sd.items()}


def write_checkpoint(model, path, dtype=torch.float32) -> None:
    """config.json + model.safetensors of a CuteChronos2Model, as a HF checkpoint directory."""
    from safetensors.torch import save_file
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    cfg = model.config
    save_file({k: v.to(dtype) for k, v in hf_state_dict(model).items()}, str(path / "model.safetensors"))
    (path / "config.json").write_text(json.dumps({
        "d_model": cfg.d_model, "d_kv": cfg.d_kv, "d_ff": cfg.d_ff, "num_layers": cfg.num_layers,
        "num_heads": cfg.num_heads, "layer_norm_epsilon": cfg.layer_norm_epsilon, "rope_theta": cfg.rope_theta,
        "dense_act_fn": "relu", "vocab_size": cfg.vocab_size, "reg_token_id": cfg.reg_token_id,
        "chronos_config": {"context_length": cfg.context_length, "input_patch_size": cfg.input_patch_size,
                           "input_patch_stride": cfg.input_patch_stride,
                           "output_patch_size": cfg.output_patch_size, "quantiles": list(cfg.quantiles),
                           "use_reg_token": cfg.use_reg_token, "use_arcsinh": cfg.use_arcsinh,
                           "time_encoding_scale": cfg.time_encoding_scale,
                           "max_output_patches": cfg.max_output_patches}}, indent=1))

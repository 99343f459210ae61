"""The CPU oracle against fixtures produced by the reference module itself
(tests/golden/make_golden.py), and the parameter layout of the drop-in model."""

import numpy as np
import pytest
import torch

from conftest import GOLDEN, SMALL, case_inputs, oracle_config, small_config
from cutechronos_b200.model import CuteChronos2Config, CuteChronos2Model
from cutechronos_b200.workloads import seeded_init_, seeded_state_dict
from oracle import chronos2_oracle as orc
from oracle.chronos2_oracle import OracleConfig, forward, prepare_patched_context


def _small_weights():
    m = CuteChronos2Model(small_config())
    return seeded_state_dict([(n, tuple(p.shape)) for n, p in m.named_parameters()], seed=0)


def test_parameter_names_match_reference(param_names):
    assert [n for n, _ in CuteChronos2Model(small_config()).named_parameters()] == param_names["small"]
    assert [n for n, _ in CuteChronos2Model(CuteChronos2Config()).named_parameters()] == param_names["base"]


def test_seeded_init_equals_seeded_state_dict():
    m = seeded_init_(CuteChronos2Model(small_config()), seed=0)
    W = _small_weights()
    for n, p in m.named_parameters():
        assert torch.equal(p.detach(), W[n]), n


@pytest.mark.parametrize("case", ["ragged_nan", "groups_2x2", "truncate_700", "edge_rows", "explicit_mask",
                                  "large_scale_groups"])
def test_oracle_f32_matches_reference(golden_small, case):
    c = golden_small[case]
    ctx, mask, N, gid = case_inputs(c)
    y = forward(oracle_config(), _small_weights(), ctx, mask, N, gid, torch.float32)
    ref = torch.from_numpy(c["out_f32"])
    assert y.shape == ref.shape
    assert (y - ref).abs().max().item() <= 1e-5 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("case", ["ragged_nan", "groups_2x2", "truncate_700", "edge_rows", "explicit_mask",
                                  "large_scale_groups"])
def test_oracle_bf16_matches_reference(golden_small, case):
    c = golden_small[case]
    ctx, mask, N, gid = case_inputs(c)
    y = forward(oracle_config(), _small_weights(), ctx, mask, N, gid, torch.bfloat16).float()
    ref = torch.from_numpy(c["out_bf16"])
    # two bf16 ulps of the largest magnitude (reduction order of CPU bf16 matmuls)
    assert (y - ref).abs().max().item() <= 2 ** -6 * ref.abs().max().item()


@pytest.mark.parametrize("case", ["ragged_nan", "truncate_700", "edge_rows", "explicit_mask", "large_scale_groups"])
def test_oracle_preprocess_matches_reference(golden_small, case):
    c = golden_small[case]
    ctx, mask, _, _ = case_inputs(c)
    pc, attn, loc, scale = prepare_patched_context(oracle_config(), ctx, mask, torch.float32)
    ref = torch.from_numpy(c["patched"])
    assert torch.equal(torch.isnan(pc), torch.isnan(ref))
    assert torch.equal(attn, torch.from_numpy(c["attn"]))  # bit-exact mask
    assert torch.allclose(torch.nan_to_num(pc), torch.nan_to_num(ref), atol=1e-6, rtol=0)
    assert torch.allclose(loc, torch.from_numpy(c["loc"]), rtol=1e-6, atol=0)
    assert torch.allclose(scale, torch.from_numpy(c["scale"]), rtol=1e-6, atol=0)


def test_oracle_base_cfg0(golden_base):
    m = CuteChronos2Model(CuteChronos2Config())
    W = seeded_state_dict([(n, tuple(p.shape)) for n, p in m.named_parameters()], seed=0)
    ctx = torch.from_numpy(golden_base["context"])
    y = forward(OracleConfig(), W, ctx, None, int(golden_base["N"]))
    ref = torch.from_numpy(golden_base["out_f32"])
    assert (y - ref).abs().max().item() <= 2e-4


# ---- pipeline host steps (fixtures from the reference pipeline: make_pipeline_golden.py) -------
def _pipeline_golden():
    return dict(np.load(GOLDEN / "pipeline_host.npz"))


def test_oracle_select_quantiles_matches_reference():
    z = _pipeline_golden()
    tq = z["levels_all"].tolist()
    for kind in ("f32", "bf16"):
        preds = torch.from_numpy(z["preds_f32" if kind == "f32" else "preds_bf16_as_f32"])
        for name in ("default", "mixed", "median", "all"):
            got = orc.select_quantiles(preds, tq, z[f"levels_{name}"].tolist())
            assert np.array_equal(got.numpy(), z[f"sel_{kind}_{name}"]), (kind, name)


def test_oracle_left_pad_and_stack_matches_reference():
    z = _pipeline_golden()
    ci = 0
    while f"stack{ci}_out" in z:
        got = orc.left_pad_and_stack(torch.from_numpy(z[f"stack{ci}_values"]), z[f"stack{ci}_lens"],
                                     int(z[f"stack{ci}_ctxlen"]))
        assert np.array_equal(got.numpy(), z[f"stack{ci}_out"], equal_nan=True), ci
        ci += 1
    assert ci == 4

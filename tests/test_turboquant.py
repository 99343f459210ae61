"""TurboQuant K/V hook of the time attention (model.py:615-688,
tubroquant/quantizer.py:41-178 of the reference).

CPU: the host-side parameters (Lloyd-Max codebooks, Hadamard signs and
permutations, dense rotations, QJL projections) equal the reference's, and
the oracle's quantiser reproduces the reference's outputs and statistics
(fixtures: tests/golden/make_turboquant_golden.py).  GPU: cc2_kv_quant
against the oracle on the same parameters, and the model forward with the
hook against the oracle forward with the same quantisers."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN, oracle_config, small_config
from cutechronos_b200 import turboquant as tq
from oracle import turboquant_oracle as tqo

CASES = [("mse", 4, "hadamard", 3), ("prod", 4, "hadamard", 4), ("mse", 2, "hadamard", 5), ("prod", 3, "qr", 6),
         ("mse", 1, "qr", 7), ("prod", 1, "hadamard", 8), ("mse", 8, "hadamard", 9)]


@pytest.fixture(scope="module")
def gold():
    z = dict(np.load(GOLDEN / "turboquant.npz"))
    z["meta"] = json.loads(bytes(z["meta"]).decode())
    return z


def _params(case, device="cpu"):
    mode, bits, rot, seed = case
    return tq.TurboQuantParams.build(64, bits, mode=mode, rotation=rot, seed=seed, device=device)


@pytest.mark.parametrize("bits", range(0, 9))
def test_codebooks_match_reference(gold, bits):
    cb, cuts = tq.lloyd_max_codebook(64, bits)
    assert np.array_equal(cb, gold[f"codebook64_{bits}"])
    assert np.array_equal(cuts, gold[f"boundaries64_{bits}"])


@pytest.mark.parametrize("ci", range(len(CASES)))
def test_parameters_match_reference(gold, ci):
    p = _params(CASES[ci]).tensors
    pre = f"c{ci}_"
    assert np.array_equal(p["codebook"].numpy(), gold[pre + "codebook"])
    if CASES[ci][2] == "hadamard":
        assert np.array_equal(p["signs"].numpy(), gold[pre + "signs"])
        assert np.array_equal(p["perm"].numpy(), gold[pre + "perm"])
    else:
        assert np.allclose(p["matrix"].numpy(), gold[pre + "matrix"], atol=1e-6)
    if CASES[ci][0] == "prod":
        assert np.array_equal(p["proj"].numpy(), gold[pre + "proj"])


def _oracle(case, x, params):
    t = params.tensors
    return tqo.fake_quant(x, mode=case[0], bits=case[1], codebook=t["codebook"], boundaries=t["boundaries"][
        :max((1 << params.mse_bits) - 1, 0)], signs=t.get("signs"), perm=t.get("perm"), inv_perm=t.get("inv_perm"),
        matrix=t.get("matrix"), proj=t.get("proj"))


@pytest.mark.parametrize("ci", range(len(CASES)))
def test_oracle_matches_reference(gold, ci):
    case = CASES[ci]
    x = torch.from_numpy(gold[f"c{ci}_x"]).to(torch.bfloat16)
    out, st = _oracle(case, x, _params(case))
    ref = torch.from_numpy(gold[f"c{ci}_decoded"])
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-6), (out - ref).abs().max()
    meta = gold["meta"][ci]
    assert st["sse"] / st["count"] == pytest.approx(meta["mse"], rel=1e-4)
    assert st["max_abs_error"] == pytest.approx(meta["max_abs_error"], rel=1e-4)
    # packed payload as the reference counts it
    assert _params(case).quantized_bytes_per_vector() * x.shape[0] == meta["quantized_bytes"]
    assert x.numel() * 2 == meta["raw_bytes"]


def test_argument_errors():
    with pytest.raises(ValueError, match="mode must be"):
        tq.TurboQuantParams.build(64, 4, mode="fast", device="cpu")
    with pytest.raises(ValueError, match="Unknown rotation"):
        tq.TurboQuantParams.build(64, 4, rotation="givens", device="cpu")
    with pytest.raises(ValueError, match="bits must be"):
        tq.TurboQuantParams.build(64, -1, device="cpu")
    from cutechronos_b200.model import CuteChronos2Model
    m = CuteChronos2Model(small_config())
    with pytest.raises(ValueError):
        m.enable_turboquant_kv(bits=4, key_mode="nope")
    m.enable_turboquant_kv(bits=4)
    s = m.get_tubroquant_summary()
    assert s["enabled"] is True and s["layers"] == [] and s["config"]["key_mode"] == "prod"
    m.disable_turboquant_kv()
    s = m.get_tubroquant_summary()
    assert s["enabled"] is False and s["layers"] == []


# ---------------------------------------------------------------------------------------- GPU --
def _close_fraction(out, ref, scale):
    """Fraction of vectors whose reconstruction matches within 1e-4 of the
    vector's norm (the rest differ by a centroid or QJL-sign decision at a
    bucket edge, where the reduction order of the norm decides)."""
    err = (out - ref).abs().amax(dim=-1) / scale.clamp_min(1e-6)
    return (err <= 1e-4).float().mean().item(), err.max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("heads", [12, 3])  # 4 heads per warp / one vector per warp
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_kernel_matches_oracle(gold, ci, heads):
    case = CASES[ci]
    g = torch.Generator().manual_seed(ci)
    rows = 40
    qkv = (torch.randn(rows, 3 * heads * 64, generator=g) * 1.5).to(torch.bfloat16)
    qkv[3, heads * 64: heads * 64 + 64] = 0  # a zero K vector
    kp = _params(case, "cuda")
    vp = _params(("mse", 4, "hadamard", 100 + ci), "cuda")
    d = qkv.cuda()
    stats = torch.zeros(4, device="cuda")
    tq.kv_quant(d, rows, heads, kp, vp, q_col=0, k_col=heads * 64, v_col=2 * heads * 64, stats=stats)
    out = d.cpu()
    assert torch.equal(out[:, :heads * 64], qkv[:, :heads * 64])  # Q untouched without RoPE
    for col, case_, par in ((heads * 64, case, _params(case)), (2 * heads * 64, ("mse", 4, "hadamard", 100 + ci),
                                                                 _params(("mse", 4, "hadamard", 100 + ci)))):
        x = qkv[:, col:col + heads * 64].reshape(-1, 64)
        ref, st = _oracle(case_, x, par)
        got = out[:, col:col + heads * 64].reshape(-1, 64).float()
        frac, worst = _close_fraction(got, ref.to(torch.bfloat16).float(), x.float().norm(dim=-1))
        assert frac >= 0.99 and worst <= 0.5, (frac, worst)
    s = stats.cpu()
    x = qkv[:, heads * 64:2 * heads * 64].reshape(-1, 64)
    _, st = _oracle(case, x, _params(case))
    assert s[0].item() == pytest.approx(st["sse"], rel=2e-2)
    assert s[1].item() == pytest.approx(st["max_abs_error"], rel=2e-1)


@pytest.mark.gpu
def test_kernel_rope_then_quant_fp32():
    from cutechronos_b200.kernels import rope_table
    from oracle import chronos2_oracle as orc
    rows, heads, S = 2 * 37, 12, 37
    g = torch.Generator().manual_seed(7)
    qkv = torch.randn(rows, 3 * heads * 64, generator=g)
    kp, vp = _params(("prod", 4, "hadamard", 1), "cuda"), _params(("mse", 3, "qr", 2), "cuda")
    d = qkv.cuda()
    tq.kv_quant(d, rows, heads, kp, vp, q_col=0, k_col=heads * 64, v_col=2 * heads * 64,
                rope_cs=rope_table(S, 64, 10000.0, "cuda"), rope_period=S)
    out = d.cpu()
    cos, sin = orc.rope_cos_sin(orc.OracleConfig(), S, torch.float32)
    pos = torch.arange(rows) % S

    def rope(x):
        x = x.view(rows, heads, 64)
        c, s = cos[0, pos].unsqueeze(1), sin[0, pos].unsqueeze(1)
        return (x * c + orc._rotate_half(x) * s).reshape(rows, heads * 64)

    q_ref = rope(qkv[:, :heads * 64])
    assert torch.allclose(out[:, :heads * 64], q_ref, atol=1e-5)
    k_ref, _ = _oracle(("prod", 4, "hadamard", 1), rope(qkv[:, heads * 64:2 * heads * 64]).reshape(-1, 64),
                       _params(("prod", 4, "hadamard", 1)))
    frac, worst = _close_fraction(out[:, heads * 64:2 * heads * 64].reshape(-1, 64), k_ref,
                                  k_ref.norm(dim=-1))
    assert frac >= 0.99 and worst <= 0.5


@pytest.mark.gpu
def test_model_forward_with_hook_vs_oracle():
    from cutechronos_b200.model import CuteChronos2Model
    from cutechronos_b200.workloads import seeded_init_
    from oracle import chronos2_oracle as orc
    cfg = small_config()
    m = seeded_init_(CuteChronos2Model(cfg), seed=1).to("cuda", torch.float32).eval()
    W = {k: v.detach().cpu() for k, v in m.named_parameters()}
    g = torch.Generator().manual_seed(3)
    ctx = torch.cumsum(torch.randn(3, 200, generator=g), -1) + 10
    base = m(ctx.cuda(), num_output_patches=2).cpu()
    m.enable_turboquant_kv(bits=4, key_mode="prod", value_mode="mse", seed=11)
    y = m(ctx.cuda(), num_output_patches=2).cpu()
    hooks = []
    for l in range(cfg.num_layers):
        kp = tq.TurboQuantParams.build(64, 4, mode="prod", seed=11 + 2 * l, device="cpu")
        vp = tq.TurboQuantParams.build(64, 4, mode="mse", seed=11 + 2 * l + 1, device="cpu")

        def hook(k, v, kp=kp, vp=vp):
            kq, _ = _oracle(("prod", 4, "hadamard", 0), k, kp)
            vq, _ = _oracle(("mse", 4, "hadamard", 0), v, vp)
            return kq, vq
        hooks.append(hook)
    ref = orc.forward(oracle_config(), W, ctx, None, 2, kv_hooks=hooks)
    scale = ref.abs().max().item()
    assert (y - ref).abs().max().item() <= 2e-3 * scale
    assert (base - ref).abs().max().item() > 20 * (y - ref).abs().max().item()  # the hook changed the output
    s = m.get_tubroquant_summary()
    assert s["enabled"] and len(s["layers"]) == cfg.num_layers and s["compression_ratio"] > 1.0
    assert all(0 < layer["key_mse"] < 1 and 0 < layer["value_mse"] < 1 for layer in s["layers"])
    m.disable_turboquant_kv()
    assert torch.equal(m(ctx.cuda(), num_output_patches=2).cpu(), base)

"""Pipeline host path on the device: cc2_stack_series and
cc2_select_quantiles against the reference pipeline's own outputs
(tests/golden/pipeline_host.npz, made by make_pipeline_golden.py) and the
CPU oracle, bit for bit, and CuteChronos2Pipeline end to end against the
oracle's restatement of the same steps around the same forward."""

import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN, small_config
from oracle import chronos2_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"
TRAINED = orc.DEFAULT_QUANTILES


def K():
    from cutechronos_b200 import kernels
    return kernels


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN / "pipeline_host.npz"))


def _stack(values, lens, L):
    offs = torch.zeros(len(lens) + 1, dtype=torch.int64)
    offs[1:] = torch.cumsum(torch.as_tensor(lens, dtype=torch.int64), 0)
    return K().stack_series(values.to(DEV), offs.to(DEV), L).cpu()


def test_stack_series_vs_reference(golden):
    ci = 0
    while f"stack{ci}_out" in golden:
        lens = golden[f"stack{ci}_lens"].tolist()
        ref = golden[f"stack{ci}_out"]
        got = _stack(torch.from_numpy(golden[f"stack{ci}_values"]), lens, ref.shape[-1])
        assert np.array_equal(got.numpy(), ref, equal_nan=True), ci
        ci += 1


@pytest.mark.parametrize("B, maxlen, L", [(1000, 3000, 2048), (7, 9000, 8192), (300, 17, 512)])
def test_stack_series_vs_oracle_random(B, maxlen, L):
    g = torch.Generator().manual_seed(B)
    lens = torch.randint(0, maxlen + 1, (B,), generator=g).tolist()
    lens[0] = maxlen
    vals = torch.randn(sum(lens), generator=g)
    vals[torch.rand(vals.numel(), generator=g) < 0.02] = float("nan")
    Lout = min(max(lens), L)
    got = _stack(vals, lens, Lout)
    ref = orc.left_pad_and_stack(vals, lens, L)
    assert got.shape == ref.shape and torch.equal(got.isnan(), ref.isnan())
    assert torch.equal(torch.nan_to_num(got, nan=0.0), torch.nan_to_num(ref, nan=0.0))


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("name", ["default", "mixed", "median", "all"])
def test_select_quantiles_vs_reference(golden, kind, name):
    src = torch.from_numpy(golden["preds_f32" if kind == "f32" else "preds_bf16_as_f32"])
    preds = (src if kind == "f32" else src.to(torch.bfloat16)).to(DEV)
    levels = golden[f"levels_{name}"].tolist()
    ref = golden[f"sel_{kind}_{name}"]
    H = preds.shape[-1]
    got = K().select_quantiles(preds, H, TRAINED, levels, layout=1).cpu().numpy()
    assert np.array_equal(got, ref)
    got0 = K().select_quantiles(preds, H, TRAINED, levels, layout=0).cpu().numpy()
    assert np.array_equal(got0, ref.transpose(0, 2, 1))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_select_quantiles_large_with_median_and_short_horizon(dtype):
    g = torch.Generator().manual_seed(3)
    preds = (torch.randn(4096, 21, 64, generator=g) * 10).to(dtype)
    levels = [0.1, 0.2, 0.3, 0.33, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 0.005]
    H = 50  # fewer than the 64 forecast columns: the first H are used
    lv, med = K().select_quantiles(preds.to(DEV), H, TRAINED, levels, layout=1, median_level=10)
    ref = orc.select_quantiles(preds[..., :H].float(), TRAINED, levels)
    assert torch.equal(lv.cpu(), ref)
    assert torch.equal(med.cpu(), preds[:, 10, :H].float())


def test_select_quantiles_argument_errors():
    from cutechronos_b200._native import NativeError
    p = torch.zeros(2, 21, 16, device=DEV)
    with pytest.raises(NativeError, match="nq=65"):
        K().select_quantiles(p, 16, TRAINED, [0.5] * 65)
    with pytest.raises(NativeError, match="bad sizes"):
        K().select_quantiles(p, 17, TRAINED, [0.5])


@pytest.fixture(scope="module")
def small_pipe():
    from cutechronos_b200.model import CuteChronos2Model
    from cutechronos_b200.pipeline import CuteChronos2Pipeline
    from cutechronos_b200.workloads import seeded_init_
    m = seeded_init_(CuteChronos2Model(small_config()), seed=2).to(DEV, torch.bfloat16).eval()
    return CuteChronos2Pipeline(m, device=DEV)


def _oracle_steps(pipe, series, H, levels):
    """The reference pipeline's host steps (oracle restatement) around the
    same device forward: stack on the CPU, forward, select on the CPU."""
    rows = [s.float() for s in series]
    ctx = orc.left_pad_and_stack(torch.cat(rows), [r.numel() for r in rows], pipe.model_context_length)
    N = math.ceil(H / 16)
    preds = pipe.model(ctx.to(DEV), num_output_patches=N, group_ids=torch.arange(len(rows))).float().cpu()
    return preds[..., :H], orc.select_quantiles(preds[..., :H], TRAINED, levels)


def test_pipeline_ragged_list_end_to_end(small_pipe):
    g = torch.Generator().manual_seed(9)
    series = [torch.randn(n, generator=g).cumsum(0) + 20 for n in (700, 33, 512, 1, 250)]
    series[2][100:140] = float("nan")
    levels = [0.1, 0.25, 0.5, 0.62, 0.9]
    H = 40
    q, mean = small_pipe.predict_quantiles(series, prediction_length=H, quantile_levels=levels)
    preds_ref, sel_ref = _oracle_steps(small_pipe, series, H, levels)
    assert len(q) == 5 and q[0].shape == (1, H, 5) and mean[0].shape == (1, H)
    assert torch.equal(torch.cat(q), sel_ref)
    assert torch.equal(torch.cat(mean), preds_ref[:, TRAINED.index(0.5)])
    p = small_pipe.predict(series, prediction_length=H)
    assert torch.equal(torch.cat(p), preds_ref)


def test_predict_df_end_to_end(small_pipe):
    pd = pytest.importorskip("pandas")
    g = torch.Generator().manual_seed(4)
    lens = {"x": 90, "y": 600, "z": 17}
    frames = [pd.DataFrame({"item_id": k, "timestamp": np.arange(n)[::-1].copy(),
                            "target": torch.randn(n, generator=g).numpy()}) for k, n in lens.items()]
    df = pd.concat(frames, ignore_index=True)
    out = small_pipe.predict_df(df, prediction_length=24, quantile_levels=[0.1, 0.5, 0.77])
    order = list(dict.fromkeys(out["item_id"].tolist()))  # groups in order of first appearance
    assert sorted(order) == ["x", "y", "z"] and out.shape == (72, 5)
    assert out["item_id"].tolist() == [k for k in order for _ in range(24)]
    by_id = dict(zip(lens, frames))
    series = [torch.from_numpy(by_id[k].sort_values("timestamp")["target"].to_numpy().astype(np.float32))
              for k in order]
    _, sel_ref = _oracle_steps(small_pipe, series, 24, [0.1, 0.5, 0.77])
    got = torch.from_numpy(out[["0.1", "0.5", "0.77"]].to_numpy()).float().view(3, 24, 3)
    assert torch.equal(got, sel_ref)

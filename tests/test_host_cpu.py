"""Host-side logic on the CPU: pipeline input handling, quantile selection,
chunking, checkpoint and LoRA loading, workload generators, and the
series-group sharding + gather over 2 gloo ranks.  Mirrors the reference's
test_predict_df.py, test_pipeline_api.py and test_lora_loading.py."""

import json
import os

import pytest
import torch
import torch.multiprocessing as mp

from conftest import hf_state_dict, small_config
from cutechronos_b200.model import CuteChronos2Model
from cutechronos_b200.pipeline import CuteChronos2Pipeline, _select_quantiles
from cutechronos_b200.sharding import gather_forecasts, partition_groups
from cutechronos_b200.workloads import CONFIGS, config2, config3, seeded_init_
from oracle import chronos2_oracle as orc


class FakeModel:
    """Stands in for the CUDA model: forecasts are a deterministic function of
    each series alone (plus its group's mean, to expose group plumbing)."""

    def __init__(self):
        self.config = small_config()
        self.is_offloaded = False
        self.calls = []

    def __call__(self, ctx, num_output_patches=1, group_ids=None):
        self.calls.append((ctx.shape[0], group_ids.clone() if group_ids is not None else None))
        B = ctx.shape[0]
        last = torch.nan_to_num(ctx, nan=0.0).sum(-1)
        gid = (group_ids if group_ids is not None else torch.arange(B)).to(ctx.device)
        gmean = torch.stack([last[gid == g].mean() for g in gid])
        H = 16 * num_output_patches
        q = torch.arange(21, dtype=torch.float32, device=ctx.device).view(1, 21, 1)
        h = torch.arange(H, dtype=torch.float32, device=ctx.device).view(1, 1, H)
        return (last.view(B, 1, 1) + 0.01 * gmean.view(B, 1, 1) + q + 0.1 * h)


def pipe(device="cpu"):
    return CuteChronos2Pipeline(FakeModel(), device=device)


def test_plan_context_shapes_and_groups():
    p = pipe()
    rows, gid, rng = p._plan_context(torch.randn(5))
    assert rows.shape == (1, 5) and gid.tolist() == [0] and rng == [(0, 1)]
    rows, gid, rng = p._plan_context(torch.randn(3, 7))
    assert gid.tolist() == [0, 1, 2] and rng == [(0, 1), (1, 2), (2, 3)]
    rows, gid, rng = p._plan_context(torch.randn(2, 4, 9))
    assert rows.shape == (8, 9) and gid.tolist() == [0] * 4 + [1] * 4 and rng == [(0, 4), (4, 8)]
    a, b = torch.randn(3), torch.randn(2, 5)
    rows, gid, rng = p._plan_context([a, b])
    assert [r.shape[-1] for r in rows] == [3, 5, 5] and gid.tolist() == [0, 1, 1] and rng == [(0, 1), (1, 3)]
    assert torch.equal(rows[0], a) and torch.equal(rows[2], b[1])
    with pytest.raises(NotImplementedError):
        p._plan_context([{"target": torch.randn(4)}])
    with pytest.raises(ValueError):
        p._plan_context(torch.randn(2, 2, 2, 2))
    with pytest.raises(ValueError):
        p._plan_context([torch.randn(2, 2, 2)])


def test_truncation_to_model_context_length():
    rows, _, _ = pipe()._plan_context(torch.arange(600, dtype=torch.float32))
    assert rows.shape == (1, 512) and rows[0, 0].item() == 88.0


def test_prediction_length_limit():
    p = pipe()
    with pytest.raises(ValueError, match="Set limit_prediction_length=False"):
        p.predict(torch.randn(1, 30), prediction_length=64 * 16 + 1)
    with pytest.raises(ValueError, match="Set limit_prediction_length=False"):
        p.predict_quantiles(torch.randn(1, 30), prediction_length=64 * 16 + 1)


def test_oracle_select_quantiles_known_answers():
    tq = [0.1, 0.5, 0.9]
    preds = torch.tensor([[[1.0, 2.0], [3.0, 4.0], [5.0, 8.0]]])  # (1, Q=3, H=2)
    assert orc.select_quantiles(preds, tq, [0.5, 0.1]).tolist() == [[[3.0, 1.0], [4.0, 2.0]]]
    out = orc.select_quantiles(preds, tq, [0.3, 0.7])
    assert torch.allclose(out, torch.tensor([[[2.0, 4.0], [3.0, 6.0]]]))


# The same host logic through the device kernels (stack_series, select_quantiles).
@pytest.mark.gpu
def test_predict_chunking_equals_single_batch():
    x = torch.randn(10, 40)
    a = pipe("cuda").predict(x, prediction_length=20)
    b = pipe("cuda").predict(x, prediction_length=20, batch_size=3)
    assert len(a) == 10 and a[0].shape == (1, 21, 20) and a[0].device.type == "cpu"
    for u, v in zip(a, b):
        assert torch.allclose(u, v)


@pytest.mark.gpu
def test_cross_learning_uses_one_group_and_disables_chunking():
    p = pipe("cuda")
    p.predict(torch.randn(6, 30), prediction_length=16, cross_learning=True, batch_size=2)
    assert len(p.model.calls) == 1 and p.model.calls[0][1].tolist() == [0] * 6


@pytest.mark.gpu
def test_select_quantiles_gather_and_interpolate():
    tq = [0.1, 0.5, 0.9]
    preds = torch.tensor([[[1.0, 2.0], [3.0, 4.0], [5.0, 8.0]]])
    assert _select_quantiles(preds, tq, [0.5, 0.1]).tolist() == [[[3.0, 1.0], [4.0, 2.0]]]
    assert torch.allclose(_select_quantiles(preds, tq, [0.3, 0.7]), torch.tensor([[[2.0, 4.0], [3.0, 6.0]]]))


@pytest.mark.gpu
def test_predict_quantiles_and_df():
    pd = pytest.importorskip("pandas")
    p = pipe("cuda")
    q, mean = p.predict_quantiles(torch.randn(2, 32), prediction_length=16, quantile_levels=[0.1, 0.5])
    assert q[0].shape == (1, 16, 2) and mean[0].shape == (1, 16)
    assert torch.equal(mean[0], q[0][..., 1])
    df = pd.DataFrame({"item_id": ["a"] * 30 + ["b"] * 20, "timestamp": list(range(30)) + list(range(20)),
                       "target": torch.randn(50).tolist()})
    out = p.predict_df(df, prediction_length=16, quantile_levels=[0.5])
    assert list(out.columns) == ["item_id", "step", "0.5"] and len(out) == 32
    assert out["item_id"].tolist() == ["a"] * 16 + ["b"] * 16 and out["step"].tolist() == list(range(16)) * 2
    assert out["0.5"].dtype == "float64"


def test_checkpoint_and_lora_loading(tmp_path):
    sf = pytest.importorskip("safetensors.torch")
    cfg = small_config()
    src = seeded_init_(CuteChronos2Model(cfg), seed=3)
    sd = hf_state_dict(src)
    sf.save_file({k: v.detach().contiguous() for k, v in sd.items()}, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps({
        "d_model": cfg.d_model, "d_kv": cfg.d_kv, "d_ff": cfg.d_ff, "num_layers": cfg.num_layers,
        "num_heads": cfg.num_heads, "chronos_config": {"context_length": 512, "time_encoding_scale": 512}}))
    m = CuteChronos2Model.from_pretrained(tmp_path)
    for (n1, p1), (n2, p2) in zip(m.named_parameters(), src.named_parameters()):
        assert n1 == n2 and torch.equal(p1, p2), n1
    # LoRA: W += (alpha / r) * B @ A on the targeted projections
    r, alpha = 2, 4
    A = torch.randn(r, cfg.d_model)
    Bm = torch.randn(cfg.d_model, r)
    lora = {"base_model.model.encoder.block.1.layer.0.self_attention.q.lora_A.weight": A,
            "base_model.model.encoder.block.1.layer.0.self_attention.q.lora_B.weight": Bm}
    ad = tmp_path / "adapter"
    ad.mkdir()
    sf.save_file(lora, str(ad / "adapter_model.safetensors"))
    (ad / "adapter_config.json").write_text(json.dumps({"r": r, "lora_alpha": alpha, "target_modules": ["q"]}))
    before = m.blocks[1].time_attn.q.weight.detach().clone()
    m.load_lora_adapter(ad)
    assert torch.allclose(m.blocks[1].time_attn.q.weight, before + (alpha / r) * (Bm @ A), atol=1e-5)
    assert torch.equal(m.blocks[0].time_attn.q.weight, src.blocks[0].time_attn.q.weight)


def test_workload_generators():
    w2 = config2(groups=4, variates=8, L=256)
    assert w2.context.shape == (32, 256) and w2.group_ids.tolist()[:9] == [0] * 8 + [1]
    w3 = config3(B=8, L=512)
    assert w3.context.shape == (8, 512) and w3.prediction_length == 128 and w3.num_output_patches == 8
    nan = torch.isnan(CONFIGS[1](B=8, L=2048).context).float().mean().item()
    assert 0.01 < nan < 0.03


def test_partition_groups_keeps_groups_whole_and_balances():
    gid = torch.tensor([0] * 8 + [1] * 8 + [2] * 8 + [3] * 8 + [4] * 2)
    shards = partition_groups(gid, len(gid), 4)
    assert sorted(torch.cat(shards).tolist()) == list(range(len(gid)))
    for s in shards:
        groups = set(gid[s].tolist())
        for g in groups:  # whole groups only
            assert set(s.tolist()) >= set((gid == g).nonzero().view(-1).tolist())
    assert max(len(s) for s in shards) - min(len(s) for s in shards) <= 8
    assert [len(s) for s in partition_groups(None, 10, 3)] in ([4, 3, 3], [3, 4, 3], [3, 3, 4])


def _rank_main(rank, world, init_file, ctx, gid, result_q):
    import torch.distributed as dist
    # file rendezvous: no TCP port to race for while the ranks start up
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        shards = partition_groups(gid, ctx.shape[0], world)
        mine = shards[rank]
        local = FakeModel()(ctx[mine], num_output_patches=2, group_ids=gid[mine])
        full = gather_forecasts(local, shards)
        result_q.put((rank, full))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharding_and_gather(tmp_path):
    ctx = torch.randn(11, 40)
    gid = torch.tensor([0, 0, 1, 2, 2, 2, 3, 4, 4, 5, 6])
    expect = FakeModel()(ctx, num_output_patches=2, group_ids=gid)
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    init_file = str(tmp_path / "rendezvous")
    procs = [mpc.Process(target=_rank_main, args=(r, 2, init_file, ctx, gid, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert torch.allclose(results[r], expect)


def test_group_series_matches_groupby():
    pd = pytest.importorskip("pandas")
    from cutechronos_b200.pipeline import _group_series
    g = torch.Generator().manual_seed(0)
    n = 500
    ids = torch.randint(0, 7, (n,), generator=g).tolist()
    df = pd.DataFrame({"item_id": [f"s{i}" if i != 6 else None for i in ids],
                       "timestamp": torch.randperm(n, generator=g).tolist(),
                       "target": torch.randn(n, generator=g).tolist()})
    got_ids, rag = _group_series(df, "item_id", "timestamp", "target")
    groups = df.sort_values("timestamp").groupby("item_id", sort=False)
    assert got_ids == list(groups.groups.keys())
    ref = [torch.tensor(grp["target"].values, dtype=torch.float32) for _, grp in groups]
    assert rag.lens == [len(r) for r in ref]
    assert torch.equal(rag.values, torch.cat(ref))

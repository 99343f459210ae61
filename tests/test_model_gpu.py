"""Whole-forward parity on the GPU: CuteChronos2Model (native engine) against
fixtures from the reference module and against the CPU oracle.

Tolerances (the parity bar of this path): fp32 mode max-abs 1e-4 in absolute
terms on the Chronos-2-base configs[0] forward and on the reference's own test
input; on the small edge-case fixtures (inputs up to 1e6 in magnitude) the same
1e-4 in the model's normalised output space (|y - ref| / scale_b, scale_b = the
series' instance-norm scale).  bf16 mode 2e-2 relative per series:
max over series b of max|y_b - ref_b| / max|ref_b| <= 2e-2.
Each test prints its measured maximum (run with -s to see them).
"""

import pytest
import torch

from conftest import case_inputs, oracle_config, small_config
from cutechronos_b200.model import CuteChronos2Config, CuteChronos2Model
from cutechronos_b200.workloads import config1, config2, config3, config4, seeded_init_, seeded_state_dict
from oracle import chronos2_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"
CASES = ["ragged_nan", "groups_2x2", "truncate_700", "edge_rows", "explicit_mask", "large_scale_groups"]


def _model(cfg, dtype):
    return seeded_init_(CuteChronos2Model(cfg), seed=0).to(DEV, dtype).eval()


def _norm_err(y, ref, scale):
    return ((y.float() - ref.float()).abs() / scale.view(-1, 1, 1)).max().item()


def _rel_err(y, ref):
    """Per-series relative error, worst series: max_b max|y_b - ref_b| / max|ref_b|."""
    d = (y.float() - ref.float()).abs().flatten(1).amax(1)
    r = ref.float().abs().flatten(1).amax(1).clamp_min(1e-30)
    return (d / r).max().item()


def _report(name, value):
    print(f"PARITY {name} {value:.3e}")
    return value


@pytest.fixture(scope="module")
def small_f32():
    return _model(small_config(), torch.float32)


@pytest.fixture(scope="module")
def small_bf16():
    return _model(small_config(), torch.bfloat16)


@pytest.mark.parametrize("case", CASES)
def test_small_f32_vs_reference(golden_small, small_f32, case):
    c = golden_small[case]
    ctx, mask, N, gid = case_inputs(c)
    y = small_f32(ctx.to(DEV), mask.to(DEV) if mask is not None else None, N, gid).cpu()
    ref = torch.from_numpy(c["out_f32"])
    assert y.shape == ref.shape and y.dtype == torch.float32
    scale = torch.from_numpy(c["scale"]).view(-1)
    assert _report(f"small_{case}_f32_norm", _norm_err(y, ref, scale)) <= 1e-4


@pytest.mark.parametrize("case", CASES)
def test_small_bf16_vs_reference(golden_small, small_bf16, case):
    c = golden_small[case]
    ctx, mask, N, gid = case_inputs(c)
    y = small_bf16(ctx.to(DEV), mask.to(DEV) if mask is not None else None, N, gid).cpu()
    assert y.dtype == torch.bfloat16
    assert _report(f"small_{case}_bf16_rel_vs_f32", _rel_err(y, torch.from_numpy(c["out_f32"]))) <= 2e-2
    assert _report(f"small_{case}_bf16_rel_vs_bf16", _rel_err(y, torch.from_numpy(c["out_bf16"]))) <= 2e-2


@pytest.fixture(scope="module")
def base_weights():
    m = CuteChronos2Model(CuteChronos2Config())
    return seeded_state_dict([(n, tuple(p.shape)) for n, p in m.named_parameters()], seed=0)


@pytest.fixture(scope="module")
def base_f32():
    return _model(CuteChronos2Config(), torch.float32)


@pytest.fixture(scope="module")
def base_bf16():
    return _model(CuteChronos2Config(), torch.bfloat16)


def test_base_cfg0_f32(golden_base, base_f32):
    ctx = torch.from_numpy(golden_base["context"])
    y = base_f32(ctx.to(DEV), num_output_patches=int(golden_base["N"])).cpu()
    ref = torch.from_numpy(golden_base["out_f32"])
    assert _report("cfg0_base_f32_maxabs", (y - ref).abs().max().item()) <= 1e-4


def test_base_cfg0_reference_style_input_f32(base_f32, base_weights):
    # the reference's own parity input (test_model.py:31-55): randn*0.1 + 100, absolute max-abs 1e-4
    g = torch.Generator().manual_seed(42)
    ctx = torch.randn(2, 512, generator=g) * 0.1 + 100.0
    y = base_f32(ctx.to(DEV), num_output_patches=4).cpu()
    ref = orc.forward(orc.OracleConfig(), base_weights, ctx, None, 4)
    assert _report("reference_style_f32_maxabs", (y - ref).abs().max().item()) <= 1e-4


def test_base_cfg0_bf16(golden_base, base_bf16):
    ctx = torch.from_numpy(golden_base["context"])
    y = base_bf16(ctx.to(DEV), num_output_patches=int(golden_base["N"])).cpu()
    assert _report("cfg0_base_bf16_rel", _rel_err(y, torch.from_numpy(golden_base["out_f32"]))) <= 2e-2


def _subset_check(model, weights, ctx, gid, N, idx, dtype=torch.float32):
    """Forecasts of a subset (whole groups) from the full-batch GPU run vs the
    CPU oracle run on that subset alone."""
    y = model(ctx.to(DEV), num_output_patches=N, group_ids=gid).cpu()
    assert torch.isfinite(y.float()).all()
    sub_gid = gid[idx] if gid is not None else None
    ref = orc.forward(orc.OracleConfig(), weights, ctx[idx], None, N, sub_gid, torch.float32)
    return _rel_err(y[idx], ref)


def test_cfg1_full_batch_subset_vs_oracle(base_bf16, base_weights):
    w = config1()
    idx = torch.arange(0, 256, 8)  # 32 of the 256 series
    err = _subset_check(base_bf16, base_weights, w.context, None, w.num_output_patches, idx)
    assert _report("cfg1_bf16_rel_32series", err) <= 2e-2


def test_cfg2_groups_subset_vs_oracle(base_bf16, base_weights):
    w = config2()
    idx = torch.cat([torch.arange(8 * g, 8 * g + 8) for g in (1, 2, 30, 63)])  # 4 whole groups
    err = _subset_check(base_bf16, base_weights, w.context, w.group_ids, w.num_output_patches, idx)
    assert _report("cfg2_bf16_rel_4groups", err) <= 2e-2


def test_cfg3_left_padded_subset_vs_oracle(base_bf16, base_weights):
    w = config3()
    padded = torch.isnan(w.context[:, 0]).nonzero().view(-1)
    full = (~torch.isnan(w.context[:, 0])).nonzero().view(-1)
    assert padded.numel() >= 4
    idx = torch.cat([padded[:4], full[:4]]).sort().values  # 8 series, half of them left-padded
    err = _subset_check(base_bf16, base_weights, w.context, None, w.num_output_patches, idx)
    assert _report("cfg3_bf16_rel_8series", err) <= 2e-2


def test_cfg4_full_batch_subset_vs_oracle(base_bf16, base_weights):
    # 4096 series x ctx 512 (37 tokens per series: the short-set
    # attention path), whole batch on the GPU, 32 series against the oracle
    w = config4()
    idx = torch.arange(0, 4096, 128)
    err = _subset_check(base_bf16, base_weights, w.context, None, w.num_output_patches, idx)
    assert _report("cfg4_bf16_rel_32series", err) <= 2e-2


def test_batch_composition_invariance_and_determinism(base_bf16):
    # a series' forecast does not depend on the other (independent) series in
    # the batch, bit for bit: every reduction has a fixed order (no atomics)
    w = config1(B=300, L=2048)
    full = base_bf16(w.context.to(DEV), num_output_patches=4).cpu()
    again = base_bf16(w.context.to(DEV), num_output_patches=4).cpu()
    part = base_bf16(w.context[5:9].to(DEV), num_output_patches=4).cpu()
    assert torch.equal(full, again)
    assert torch.equal(part, full[5:9])


def test_group_ids_none_equals_arange(small_bf16):
    ctx = torch.randn(6, 100)
    a = small_bf16(ctx.to(DEV), num_output_patches=2)
    b = small_bf16(ctx.to(DEV), num_output_patches=2, group_ids=torch.arange(6))
    assert torch.equal(a, b)


def test_repack_after_weight_change(small_f32, golden_small):
    c = golden_small["ragged_nan"]
    ctx, mask, N, gid = case_inputs(c)
    y0 = small_f32(ctx.to(DEV), num_output_patches=N).clone()
    with torch.no_grad():
        small_f32.blocks[0].feed_forward.wo.weight.mul_(2.0)
    y1 = small_f32(ctx.to(DEV), num_output_patches=N)
    with torch.no_grad():
        small_f32.blocks[0].feed_forward.wo.weight.mul_(0.5)
    y2 = small_f32(ctx.to(DEV), num_output_patches=N)
    assert not torch.equal(y0, y1)
    assert torch.allclose(y0, y2, atol=1e-6)


def test_cpu_model_raises():
    m = CuteChronos2Model(small_config())
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 32))


def test_cuda_graph_replay_equals_eager(small_bf16):
    """enable_cuda_graphs: one graph per shape, replays equal eager runs,
    shape changes (workspace regrowth) recapture, outputs are copies."""
    g = torch.Generator().manual_seed(5)
    xs = [torch.randn(4, 300, generator=g), torch.randn(4, 300, generator=g), torch.randn(9, 700, generator=g),
          torch.randn(4, 300, generator=g)]
    eager = [small_bf16(x.to(DEV), num_output_patches=3).cpu() for x in xs]
    small_bf16.enable_cuda_graphs(True)
    try:
        outs = [small_bf16(x.to(DEV), num_output_patches=3) for x in xs]
        assert outs[0].data_ptr() != outs[1].data_ptr()
        for o, e in zip(outs, eager):
            assert torch.equal(o.cpu(), e)
        # series groups run eagerly under the same switch
        gid = torch.tensor([0, 0, 1, 1])
        assert torch.equal(small_bf16(xs[0].to(DEV), num_output_patches=3, group_ids=gid).cpu(),
                           small_bf16.__class__.forward(small_bf16, xs[0].to(DEV), num_output_patches=3,
                                                        group_ids=gid).cpu())
    finally:
        small_bf16.enable_cuda_graphs(False)



def test_batch1_equals_batched(base_bf16, base_weights):
    """A single series (batch-1 serving, 133 token rows) run kernel by kernel
    gives the same forecast, bit for bit, as inside a batch, and stays within
    the bf16 bar of the oracle."""
    from cutechronos_b200 import _native as nat
    lib = nat.load()
    w = config1(B=8, L=2048)
    old = lib.cc2_set_layer_chain(0)
    try:
        one = base_bf16(w.context[3:4].to(DEV), num_output_patches=4).cpu()
        batch = base_bf16(w.context.to(DEV), num_output_patches=4).cpu()[3:4]
    finally:
        lib.cc2_set_layer_chain(old)
    assert torch.equal(one, batch)
    ref = orc.forward(orc.OracleConfig(), base_weights, w.context[3:4], None, 4)
    assert _report("batch1_bf16_rel", _rel_err(one, ref)) <= 2e-2


def _chain_pair(model, ctx, N):
    """(layer-persistent forward with the whole-set attention arithmetic,
    kernel-by-kernel forward with the same attention kernel,
    layer-persistent forward in its default split-key mode), all eager."""
    from cutechronos_b200 import _native as nat
    lib = nat.load()
    old_v = lib.cc2_set_attention_variant(3)
    old_c = lib.cc2_set_layer_chain(2)
    try:
        a = model(ctx.to(DEV), num_output_patches=N).cpu()
        lib.cc2_set_layer_chain(0)
        b = model(ctx.to(DEV), num_output_patches=N).cpu()
        lib.cc2_set_layer_chain(1)
        c = model(ctx.to(DEV), num_output_patches=N).cpu()
        c2 = model(ctx.to(DEV), num_output_patches=N).cpu()
    finally:
        lib.cc2_set_layer_chain(old_c)
        lib.cc2_set_attention_variant(old_v)
    assert torch.equal(c, c2)  # deterministic
    return a, b, c


# (B, L): 133 token rows (ctx 2048), 2 x 37 rows (ctx 512), 3 x 81 rows with
# left padding and NaN gaps (token masks), 384 rows (the largest chained M)
@pytest.mark.parametrize("B,L", [(1, 2048), (2, 512), (3, 1200), (3, 1968)])
def test_layer_chain_equals_kernel_by_kernel(base_bf16, base_weights, B, L):
    """The layer-persistent forward (one cooperative launch for all encoder
    layers) computes the same forecasts, bit for bit, as the per-kernel
    forward with the same tile GEMMs and attention kernel, and stays within
    the bf16 bar of the oracle."""
    w = config1(B=B, L=L)
    ctx = w.context.clone()
    if B == 3:
        ctx[1, : L // 3] = float("nan")  # left padding
        ctx[2, 100:140] = float("nan")   # a gap inside the context
    a, b, c = _chain_pair(base_bf16, ctx, 4)
    assert torch.equal(a, b)
    ref = orc.forward(orc.OracleConfig(), base_weights, ctx, None, 4)
    assert _report(f"layer_chain_exact_B{B}_L{L}_bf16_rel", _rel_err(a, ref)) <= 2e-2
    assert _report(f"layer_chain_B{B}_L{L}_bf16_rel", _rel_err(c, ref)) <= 2e-2
    assert _rel_err(c, a) <= 2e-2


def test_layer_chain_small_model_and_graph(small_bf16):
    """Other model shapes (small config: different d_model / heads / layers),
    and replay of the cooperative launch from a CUDA graph."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 300, generator=g)
    a, b, c = _chain_pair(small_bf16, x, 3)
    assert torch.equal(a, b)
    assert _rel_err(c, a) <= 2e-2
    from cutechronos_b200 import _native as nat
    lib = nat.load()
    old_c = lib.cc2_set_layer_chain(1)
    small_bf16.enable_cuda_graphs(True)
    try:
        outs = [small_bf16(x.to(DEV), num_output_patches=3).cpu() for _ in range(3)]
        small_bf16.enable_cuda_graphs(False)
        eager = small_bf16(x.to(DEV), num_output_patches=3).cpu()
    finally:
        small_bf16.enable_cuda_graphs(False)
        lib.cc2_set_layer_chain(old_c)
    for o in outs:
        assert torch.equal(o, eager)

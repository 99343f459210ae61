"""Component kernels on the GPU (through the C ABI) against the CPU oracle /
fp32 torch references.  Mirrors the reference's kernel tests
(cutechronos/tests/test_preprocessing.py, test_output.py,
test_rms_layernorm.py, test_fused_mlp.py, test_attention.py,
test_group_attention.py)."""

import math

import pytest
import torch

from conftest import case_inputs, oracle_config
from oracle import chronos2_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"


def K():
    from cutechronos_b200 import kernels
    return kernels


def _ctx(B, L, nan_frac, seed, scale=1.0, offset=0.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.cumsum(torch.randn(B, L, generator=g), -1) * scale + offset
    x[torch.rand(B, L, generator=g) < nan_frac] = float("nan")
    return x


# ---------------------------------------------------------------------------
# preprocessing (instance norm + arcsinh + patching + time encoding)
# ---------------------------------------------------------------------------
PRE_CASES = [
    ("basic", _ctx(4, 512, 0.1, 1), 512),
    ("pad_500", _ctx(3, 500, 0.05, 2), 512),          # L not a multiple of 16
    ("truncate", _ctx(2, 1024, 0.0, 3), 512),          # L > context_length
    ("scale_1e6", _ctx(2, 256, 0.1, 4, 1e3, 1e6), 512),
    ("nan_90", _ctx(3, 128, 0.9, 5), 512),
    ("long_8192", _ctx(2, 8192, 0.02, 6), 8192),
]


def _edge_ctx():
    x = _ctx(5, 64, 0.0, 7)
    x[0] = float("nan")      # all-NaN -> loc 0, scale 1
    x[1] = 2.5               # constant -> scale 1e-5
    x[2, :40] = float("nan")  # left-padded
    x[3, 17] = float("nan")
    return x


@pytest.mark.parametrize("name,ctx,cl", PRE_CASES + [("edge", _edge_ctx(), 512)])
@pytest.mark.parametrize("arcsinh", [True, False])
def test_preprocess_f32(name, ctx, cl, arcsinh):
    cfg = orc.OracleConfig(context_length=cl, use_arcsinh=arcsinh)
    pc, attn, loc, scale = orc.prepare_patched_context(cfg, ctx, None, torch.float32)
    gpc, gattn, gloc, gscale = K().fused_preprocess(ctx.to(DEV), 16, cl, arcsinh)
    gpc = gpc.cpu()
    assert gpc.shape == pc.shape
    assert torch.equal(gattn.cpu().bool(), attn)                      # bit-exact patch mask
    assert torch.equal(gpc[..., 32:], pc[..., 32:])                    # bit-exact observed mask
    assert torch.equal(gpc[..., :16], pc[..., :16])                    # bit-exact time encoding
    assert torch.equal(torch.isnan(gpc), torch.isnan(pc))
    assert torch.allclose(gloc.cpu(), loc, rtol=2e-7, atol=0)
    assert torch.allclose(gscale.cpu(), scale, rtol=2e-6, atol=0)
    assert torch.allclose(torch.nan_to_num(gpc[..., 16:32]), torch.nan_to_num(pc[..., 16:32]), rtol=0, atol=2e-6)


def test_preprocess_bf16_and_explicit_mask(golden_small):
    c = golden_small["explicit_mask"]
    ctx, mask, _, _ = case_inputs(c)
    cfg = oracle_config()
    pc, attn, _, _ = orc.prepare_patched_context(cfg, ctx, mask, torch.bfloat16)
    gpc, gattn, _, _ = K().fused_preprocess(ctx.to(DEV), 16, 512, True, context_mask=mask.to(DEV), dtype=torch.bfloat16)
    assert torch.equal(gattn.cpu().bool(), attn)
    assert torch.equal(gpc.cpu()[..., :16], pc[..., :16])
    assert torch.equal(gpc.cpu()[..., 32:], pc[..., 32:])
    d = (gpc.cpu()[..., 16:32].float() - pc[..., 16:32].float()).abs()
    assert d.max().item() <= 2 ** -7 * max(1.0, pc[..., 16:32].float().abs().max().item())


# a caller's mask with fractional values and NaNs: the patched mask carries the
# values in the model dtype, NaN counts as 0 (model.py:481-499)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("L", [2048, 512])
def test_preprocess_fractional_mask(dtype, L):
    g = torch.Generator().manual_seed(L)
    ctx = torch.cumsum(torch.randn(3, L, generator=g), -1) + 50
    ctx[0, :100] = float("nan")
    mask = torch.rand(3, L, generator=g)
    mask[mask < 0.2] = 0.0
    mask[1, 5:40] = float("nan")
    mask[2, ::7] = 1.0 / 3.0
    cfg = oracle_config(context_length=8192, time_encoding_scale=8192)
    pc, attn, loc, scale = orc.prepare_patched_context(cfg, ctx, mask, dtype)
    gpc, gattn, gloc, gscale = K().fused_preprocess(ctx.to(DEV), 16, 8192, True, context_mask=mask.to(DEV),
                                                    dtype=dtype)
    gpc = gpc.cpu()
    assert torch.equal(gattn.cpu().bool(), attn)
    assert torch.equal(gpc[..., :16], pc[..., :16])
    assert torch.equal(gpc[..., 32:], pc[..., 32:])
    # a NaN value under a positive mask stays NaN, as in the reference
    a, r = gpc[..., 16:32].float(), pc[..., 16:32].float()
    assert torch.equal(torch.isnan(a), torch.isnan(r))
    a, r = torch.nan_to_num(a), torch.nan_to_num(r)
    tol = 2e-6 if dtype == torch.float32 else 2 ** -7 * max(1.0, r.abs().max().item())
    assert (a - r).abs().max().item() <= tol


def test_preprocess_patch_size_1():
    ctx = _ctx(2, 40, 0.2, 8)
    cfg = orc.OracleConfig(context_length=512, input_patch_size=1, output_patch_size=1)
    pc, attn, loc, scale = orc.prepare_patched_context(cfg, ctx, None, torch.float32)
    gpc, gattn, _, _ = K().fused_preprocess(ctx.to(DEV), 1, 512, True)
    assert torch.equal(gattn.cpu().bool(), attn)
    assert torch.allclose(torch.nan_to_num(gpc.cpu()), torch.nan_to_num(pc), atol=2e-6, rtol=0)


# ---------------------------------------------------------------------------
# output transform / RMSNorm
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,N", [(1, 1), (3, 4), (64, 8), (3001, 4), (2499, 8)])
def test_output_transform(dtype, B, N):
    g = torch.Generator().manual_seed(B * 10 + N)
    x = (torch.randn(B, N, 21 * 16, generator=g) * 2).to(dtype)
    loc, scale = torch.randn(B, 1, generator=g) * 100, torch.rand(B, 1, generator=g) * 10 + 0.1
    ref = orc.output_transform(x, loc, scale, 21, 16)
    out = K().fused_output_transform(x.to(DEV), loc.to(DEV), scale.to(DEV), 21, 16).cpu()
    assert out.shape == (B, 21, N * 16) and out.dtype == dtype
    tol = 1e-5 if dtype == torch.float32 else 2 ** -7
    assert ((out.float() - ref.float()).abs() <= tol * ref.float().abs() + 1e-5 * scale.max()).all()


# forecasts with a row pitch larger than Q * ps (the streaming path then
# copies each (series, patch) row on its own; the padding is never read)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B", [5, 3001])
def test_output_transform_row_pitch(dtype, B):
    from cutechronos_b200 import _native as nat
    g = torch.Generator().manual_seed(B + 7)
    N, ld = 4, 344
    xp = torch.full((B, N, ld), float("nan")).to(dtype)
    xp[..., :336] = (torch.randn(B, N, 336, generator=g) * 2).to(dtype)
    loc, scale = torch.randn(B, 1, generator=g) * 100, torch.rand(B, 1, generator=g) * 10 + 0.1
    ref = orc.output_transform(xp[..., :336].contiguous(), loc, scale, 21, 16)
    xd, lf, sf = xp.to(DEV), loc.view(B).to(DEV), scale.view(B).to(DEV)
    out = torch.empty(B, 21, N * 16, dtype=dtype, device=DEV)
    code = nat.CC2_BF16 if dtype == torch.bfloat16 else nat.CC2_F32
    nat.check(nat.load().cc2_output_transform(code, xd.data_ptr(), ld, lf.data_ptr(), sf.data_ptr(), out.data_ptr(),
                                              B, N, 21, 16, 1, torch.cuda.current_stream().cuda_stream),
              "cc2_output_transform")
    out = out.cpu()
    tol = 1e-5 if dtype == torch.float32 else 2 ** -7
    assert torch.isfinite(out.float()).all()
    assert ((out.float() - ref.float()).abs() <= tol * ref.float().abs() + 1e-5 * scale.max()).all()


@pytest.mark.parametrize("B", [5, 4000])
def test_output_transform_bf16_sinh_within_one_ulp(B):
    # the bf16 path computes sinh on the FMA pipe (range reduction + shared
    # even/odd polynomial); checked against a float64 sinh over |x| <= 60,
    # values near 0 included, one bf16 ulp of the exact result (the fp32
    # arithmetic adds ~3e-7 relative to the final rounding's 2^-9); where
    # sinh leaves the fp32 range the result is inf with the sign of x, and
    # NaN stays NaN
    g = torch.Generator().manual_seed(B)
    x = torch.randn(B, 4, 21 * 16, generator=g, dtype=torch.float64) * 12
    x[:, 0, :16] = torch.linspace(-1e-3, 1e-3, 16, dtype=torch.float64)
    x[0, 1, :8] = torch.tensor([0.0, -0.0, 1e-30, -60.0, 60.0, 88.5, -100.0, float("nan")], dtype=torch.float64)
    xb = x.to(torch.bfloat16)
    loc, scale = torch.zeros(B, 1), torch.ones(B, 1)
    out = K().fused_output_transform(xb.to(DEV), loc.to(DEV), scale.to(DEV), 21, 16).cpu().double()
    ref = torch.sinh(xb.double()).view(B, 4, 21, 16).permute(0, 2, 1, 3).reshape(B, 21, 64)
    fin = torch.isfinite(ref) & (ref.abs() < 3.0e38)
    assert ((out[fin] - ref[fin]).abs() <= 2.0 ** -8 * ref[fin].abs() + 1e-38).all()
    big = ref.abs() > 3.5e38
    assert big.sum() >= 1 and fin[0, 0, 16 + 5]  # -100 overflows; 88.5 (1.4e38) does not
    assert torch.isinf(out[big]).all() and (torch.sign(out[big]) == torch.sign(ref[big])).all()
    assert torch.isnan(out[0, 0, 16 + 7]) and torch.isnan(ref[0, 0, 16 + 7])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 34, 768), (4, 130, 768), (16, 514, 768)])
def test_rms_layernorm(dtype, shape):
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g).to(dtype)
    w = (torch.rand(shape[-1], generator=g) + 0.5).to(dtype)
    ref = orc.rms_norm(x, w, 1e-6).float()
    out = K().rms_layernorm(x.to(DEV), w.to(DEV), 1e-6).cpu().float()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert (out - ref).abs().max().item() <= tol * ref.abs().max().item()


# ---------------------------------------------------------------------------
# GEMM with fused epilogues (tcgen05 for bf16, FFMA for fp32)
# ---------------------------------------------------------------------------
GEMM_SHAPES = [(1, 16, 64), (37, 768, 768), (128, 2304, 768), (300, 336, 3840), (1000, 3072, 48),
               (4257, 768, 3072), (133, 768, 3136), (2048, 256, 128)]


def _gemm_ref(x, w, bias, relu, resid, ssq, dim, eps):
    acc = x.double() @ w.double().T
    if ssq is not None:
        acc = acc * torch.rsqrt(ssq.double() / dim + eps)[:, None]
    if bias is not None:
        acc = acc + bias.double()
    if relu:
        acc = acc.clamp_min(0)
    if resid is not None:
        acc = acc + resid.double()
    return acc


@pytest.mark.parametrize("M,N,Kd", GEMM_SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_linear_plain(M, N, Kd, dtype):
    g = torch.Generator().manual_seed(M + N + Kd)
    x = torch.randn(M, Kd, generator=g).to(dtype)
    w = (torch.randn(N, Kd, generator=g) / math.sqrt(Kd)).to(dtype)
    out = K().linear(x.to(DEV), w.to(DEV)).cpu().double()
    ref = _gemm_ref(x, w, None, False, None, None, 0, 0)
    tol = 1e-5 if dtype == torch.float32 else 8e-3
    assert (out - ref).abs().max().item() <= tol * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("M,N,Kd", [(37, 768, 768), (1000, 2304, 768), (257, 3072, 768), (4257, 768, 3072)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_linear_fused_epilogues(M, N, Kd, dtype):
    g = torch.Generator().manual_seed(7 * M + N)
    x = torch.randn(M, Kd, generator=g).to(dtype)
    w = (torch.randn(N, Kd, generator=g) / math.sqrt(Kd)).to(dtype)
    bias = torch.randn(N, generator=g)
    resid = torch.randn(M, N, generator=g).to(dtype)
    ssq = x.float().pow(2).sum(-1)
    kk = K()
    parts = kk.row_sumsq_parts(x)
    # row scale + bias + relu
    o1 = kk.linear(x.to(DEV), w.to(DEV), bias.to(DEV), relu=True, row_ssq=parts.to(DEV), norm_dim=Kd, eps=1e-6)
    r1 = _gemm_ref(x, w, bias, True, None, ssq, Kd, 1e-6)
    tol = 1e-5 if dtype == torch.float32 else 8e-3
    assert (o1.cpu().double() - r1).abs().max().item() <= tol * max(1.0, r1.abs().max().item())
    # residual (in place) + sum of squares of the stored result
    out = resid.to(DEV).clone()
    so = torch.full(((N + 63) // 64, M), float("nan"), device=DEV)
    kk.linear(x.to(DEV), w.to(DEV), residual=out, ssq_out=so, out=out)
    r2 = _gemm_ref(x, w, None, False, resid, None, 0, 0)
    assert (out.cpu().double() - r2).abs().max().item() <= tol * max(1.0, r2.abs().max().item())
    assert torch.allclose(so.cpu(), kk.row_sumsq_parts(out.cpu()), rtol=1e-4, atol=1e-3)


# (34048, 768) and (34048, 2304): the 2-SM kernel's last partial wave runs as
# 256 x 128 half units; (40000, 336): half units past N and a partial group
@pytest.mark.parametrize("M,N,Kd", [(129, 768, 768), (34048, 768, 768), (1000, 2304, 768), (777, 336, 3840),
                                    (34048, 2304, 768), (40000, 336, 256)])
def test_gemm_pair_vs_single_sm_tiles(M, N, Kd):
    # the 2-SM (cta_group::2) and 1-SM tile paths give the same result
    from cutechronos_b200 import _native as nat
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, Kd, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(N, Kd, generator=g) / math.sqrt(Kd)).to(torch.bfloat16).to(DEV)
    resid = torch.randn(M, N, generator=g).to(torch.bfloat16).to(DEV)
    lib = nat.load()
    outs = []
    try:
        for variant in (0, 1):
            lib.cc2_set_gemm_variant(variant)
            out = resid.clone()
            so = torch.zeros(((N + 63) // 64, M), device=DEV)
            K().linear(x, w, residual=out, ssq_out=so, out=out)
            outs.append((out.float().cpu(), so.cpu()))
    finally:
        lib.cc2_set_gemm_variant(0)
    assert (outs[0][0] - outs[1][0]).abs().max().item() <= 2 ** -7 * outs[1][0].abs().max().item()
    assert torch.allclose(outs[0][1], outs[1][1], rtol=1e-2, atol=1e-2)
    ref = _gemm_ref(x.cpu(), w.cpu(), None, False, resid.cpu(), None, 0, 0)
    assert (outs[0][0].double() - ref).abs().max().item() <= 8e-3 * ref.abs().max().item()


# few token rows (batch-1 serving): 128 x 64 single-SM tiles instead of the
# 256 x 256 pair tiles (at most 64 rows: 64-row A slots, 4 k-blocks per ring
# stage); the per-element accumulation is the same, so the results must be
# too, bit for bit
@pytest.mark.parametrize("M,N,Kd", [(4, 3072, 768), (37, 768, 3072), (64, 2304, 768), (65, 768, 768),
                                    (133, 768, 768), (133, 2304, 768), (133, 768, 3072),
                                    (266, 3072, 768), (532, 768, 768), (100, 336, 256)])
def test_gemm_small_m_tiles_bit_identical(M, N, Kd):
    from cutechronos_b200 import _native as nat
    g = torch.Generator().manual_seed(M + N)
    x = torch.randn(M, Kd, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(N, Kd, generator=g) / math.sqrt(Kd)).to(torch.bfloat16).to(DEV)
    resid = torch.randn(M, N, generator=g).to(torch.bfloat16).to(DEV)
    bias = torch.randn(N, generator=g).to(DEV)
    lib = nat.load()
    outs = []
    try:
        for variant in (0, 2):
            lib.cc2_set_gemm_variant(variant)
            out = resid.clone()
            so = torch.zeros(((N + 63) // 64, M), device=DEV)
            K().linear(x, w, residual=out, ssq_out=so, out=out)
            plain = K().linear(x, w)
            # hi + lo residual stream with the row scale (the engine's O / FFN-down form)
            hl, lo_buf = resid.clone(), K().rows_to_lo((resid.float() * 2 ** -9).to(torch.bfloat16))
            K().linear(x, w, residual=hl, residual_lo=lo_buf, lo_out=lo_buf, out=hl,
                       row_ssq=K().row_sumsq_parts(x.float()), norm_dim=Kd, eps=1e-6)
            # the QKV form (row scale + RoPE on the first 2/3 of the columns) and bias + ReLU
            rc = (2 * N // 3) // 64 * 64
            qkv = K().linear(x, w, row_ssq=K().row_sumsq_parts(x.float()), norm_dim=Kd, eps=1e-6,
                             rope_period=133, rope_cols=rc) if rc else plain
            br = K().linear(x, w, bias, relu=True)
            outs.append((out.cpu(), so.cpu(), plain.cpu(), hl.cpu(), lo_buf.cpu(), qkv.cpu(), br.cpu()))
    finally:
        lib.cc2_set_gemm_variant(0)
    for i, (a, b) in enumerate(zip(outs[0], outs[1])):
        assert torch.equal(a, b), i


# few two-tile sets (batch-1 serving): each query tile of a set runs as an
# item of its own on its own CTA; the per-tile arithmetic is the same as in a
# large batch (one CTA running both tiles), so the rows must match bit for bit
@pytest.mark.parametrize("S", [129, 133, 144])
@pytest.mark.parametrize("n_few", [1, 5])
def test_time_attention_split_tiles_bit_identical(S, n_few):
    g = torch.Generator().manual_seed(S + n_few)
    B, H = 300, 12
    qkv = (torch.randn(B * S, 3 * H * 64, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    tok = torch.ones(B * S, dtype=torch.uint8)
    tok[: S // 3] = 0  # a left-padded first series
    tok = tok.to(DEV)
    full = K().attention_rows(qkv, tok, B, S, H, False)
    few = K().attention_rows(qkv[: n_few * S].contiguous(), tok[: n_few * S].contiguous(), n_few, S, H, False)
    torch.cuda.synchronize()
    assert torch.isfinite(few[S // 3:].float()).all()
    assert torch.equal(few.cpu(), full[: n_few * S].cpu())


@pytest.mark.parametrize("M,S", [(133 * 3, 133), (37, 37), (521 * 2, 521)])
def test_qkv_epilogue_rope(M, S):
    # RoPE applied in the QKV GEMM epilogue (Q and K columns, position = row % S)
    g = torch.Generator().manual_seed(M + S)
    x = torch.randn(M, 768, generator=g).to(torch.bfloat16)
    w = (torch.randn(2304, 768, generator=g) / 28).to(torch.bfloat16)
    out = K().linear(x.to(DEV), w.to(DEV), rope_period=S, rope_cols=1536).float().cpu()
    y = (x.double() @ w.double().T).float()
    tab = K().rope_table(S, 64, 10000.0, "cpu").to(torch.bfloat16).float()  # bf16 cos/sin, as the engine
    pos = torch.arange(M) % S
    c, sn = tab[pos, :, 0], tab[pos, :, 1]
    ref = y.clone()
    for h in range(24):  # Q and K heads
        a, b = y[:, 64 * h:64 * h + 32], y[:, 64 * h + 32:64 * h + 64]
        ref[:, 64 * h:64 * h + 32] = a * c - b * sn
        ref[:, 64 * h + 32:64 * h + 64] = b * c + a * sn
    assert (out - ref).abs().max().item() <= 8e-3 * ref.abs().max().item()


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def _rope_ref(q, k, S):
    cos, sin = orc.rope_cos_sin(orc.OracleConfig(), S, torch.float32)
    c, s = cos.unsqueeze(1), sin.unsqueeze(1)
    return q * c + orc._rotate_half(q) * s, k * c + orc._rotate_half(k) * s


# (256, 37) and (24, 521): many items per CTA in the persistent kernel (buffer reloads,
# few query tiles per item; a single buffer for long sets)
@pytest.mark.parametrize("B,S", [(1, 37), (4, 133), (2, 521), (3, 64), (256, 37), (24, 521)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rope", [True, False])
def test_time_attention(B, S, dtype, rope):
    g = torch.Generator().manual_seed(B * 1000 + S)
    H = 12
    q, k, v = (torch.randn(B, H, S, 64, generator=g) * 0.5 for _ in range(3))
    q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    valid = torch.rand(B, S, generator=g) > 0.3
    valid[:, -1] = True
    qf, kf = q.float(), k.float()
    if rope:
        qf, kf = _rope_ref(qf, kf, S)
    mask = (1.0 - valid.float())[:, None, None, :] * torch.finfo(torch.float32).min
    ref = orc.unscaled_attention(qf, kf, v.float(), mask)
    out = K().unscaled_attention(q.to(DEV), k.to(DEV), v.to(DEV), valid.to(DEV), rope=rope).cpu().float()
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    assert (out - ref).abs().max().item() <= tol * max(1.0, ref.abs().max().item())


@pytest.fixture
def attn_variant():
    from cutechronos_b200 import _native as nat
    lib = nat.load()
    old = lib.cc2_set_attention_variant(0)
    yield lib.cc2_set_attention_variant
    lib.cc2_set_attention_variant(old)


# tcgen05 kernels (variant 2: wherever they run, 17..640 tokens), the default
# choice (0) and the mma.sync kernels (1) on bf16 sets: one or two query
# tiles, 64/128/144-key widths, one or two buffer stages, many items per CTA,
# a series whose keys are all masked; long sets of 2..5 key blocks with a
# ragged last block (145, 200, 257, 521) or full blocks (256, 640)
@pytest.mark.parametrize("B,S", [(1, 17), (3, 37), (2, 64), (5, 20), (9, 50), (4, 63), (5, 128), (4, 129), (7, 133), (2, 144), (3, 160),
                                 (2, 160), (2, 192), (300, 133), (700, 37), (3, 145), (4, 200), (2, 256),
                                 (3, 257), (5, 521), (3, 640), (30, 521)])
@pytest.mark.parametrize("variant", [0, 1, 2])
def test_time_attention_bf16_variants(attn_variant, B, S, variant):
    attn_variant(variant)
    g = torch.Generator().manual_seed(B * 7 + S)
    H = 12
    q, k, v = ((torch.randn(B, H, S, 64, generator=g) * 0.5).to(torch.bfloat16) for _ in range(3))
    valid = torch.rand(B, S, generator=g) > 0.3
    valid[:, -1] = True
    if B > 2:
        valid[1] = False  # every key of series 1 masked: its queries average V with equal weights
    mask = (1.0 - valid.float())[:, None, None, :] * torch.finfo(torch.float32).min
    ref = orc.unscaled_attention(q.float(), k.float(), v.float(), mask)
    if B > 2:
        ref[1] = v[1].float().mean(dim=1, keepdim=True).expand(H, S, 64)
    out = K().unscaled_attention(q.to(DEV), k.to(DEV), v.to(DEV), valid.to(DEV)).cpu().float()
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())


# long sets with large, rising scores: the running max of a row grows by more
# than 2^8 from one key block to the next, so O is rescaled in TMEM
@pytest.mark.parametrize("S", [300, 521])
@pytest.mark.parametrize("variant", [0, 2])
def test_time_attention_long_rescale(attn_variant, S, variant):
    attn_variant(variant)
    g = torch.Generator().manual_seed(S)
    B, H = 3, 12
    q, k, v = (torch.randn(B, H, S, 64, generator=g) for _ in range(3))
    k = k + torch.linspace(0, 3, S)[None, None, :, None] * q.mean(dim=2, keepdim=True).sign()
    q, k, v = (t.to(torch.bfloat16) for t in (q * 2, k * 2, v))
    valid = torch.rand(B, S, generator=g) > 0.1
    valid[:, -1] = True
    mask = (1.0 - valid.float())[:, None, None, :] * torch.finfo(torch.float32).min
    ref = orc.unscaled_attention(q.float(), k.float(), v.float(), mask)
    out = K().unscaled_attention(q.to(DEV), k.to(DEV), v.to(DEV), valid.to(DEV)).cpu().float()
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())


# key blocks without masked keys take a separate path (no bias, scale folded
# into the exponent): fully valid series, left padding that covers the first
# one or two blocks (as a shorter series in a batch has), and large scores
@pytest.mark.parametrize("S", [256, 521, 640])
@pytest.mark.parametrize("scale", [0.5, 2.0])
def test_time_attention_long_clean_blocks(attn_variant, S, scale):
    attn_variant(0)
    g = torch.Generator().manual_seed(S + int(scale * 10))
    B, H = 4, 12
    q, k, v = ((torch.randn(B, H, S, 64, generator=g) * s).to(torch.bfloat16) for s in (scale, scale, 1.0))
    valid = torch.ones(B, S, dtype=torch.bool)
    valid[1, :150] = False
    valid[2, :40] = False
    valid[3, torch.rand(S, generator=g) < 0.05] = False
    mask = (1.0 - valid.float())[:, None, None, :] * torch.finfo(torch.float32).min
    ref = orc.unscaled_attention(q.float(), k.float(), v.float(), mask)
    out = K().unscaled_attention(q.to(DEV), k.to(DEV), v.to(DEV), valid.to(DEV)).cpu().float()
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())


def test_attention_uniform_known_answer():
    # identical keys -> uniform weights -> output = mean of V (reference test_attention.py:199-213)
    B, H, S = 2, 12, 70
    q = torch.randn(B, H, S, 64)
    k = torch.ones(B, H, S, 64)
    v = torch.randn(B, H, S, 64)
    out = K().unscaled_attention(q.to(DEV), k.to(DEV), v.to(DEV)).cpu()
    assert torch.allclose(out, v.mean(dim=2, keepdim=True).expand_as(v), atol=1e-5)


@pytest.mark.parametrize("gids,S", [([0, 0, 1, 1, 1, 2, 3, 3], 19), ([5] * 40 + [1] * 3, 9), (list(range(6)), 7),
                                    ([0] * 100, 5), ([0] * 8 + [1] * 9 + [2] * 16 + [3], 7),
                                    ([i // 8 for i in range(64)], 133)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_group_attention(gids, S, dtype):
    B, H = len(gids), 12
    g = torch.Generator().manual_seed(B + S)
    qkv = (torch.randn(B, S, 3 * 768, generator=g) * 0.5).to(dtype)
    tok = torch.rand(B, S, generator=g) > 0.2
    gid = torch.tensor(gids)
    # oracle: (T, H, B, D) attention with the group-time mask (model.py:561-569)
    q, k, v = (qkv.float()[..., i * 768:(i + 1) * 768].transpose(0, 1).reshape(S, B, H, 64).permute(0, 2, 1, 3)
               for i in range(3))
    same = (gid[:, None] == gid[None, :]).float()
    gm = torch.einsum("qb,bt->qbt", same, tok.float()).permute(2, 0, 1).unsqueeze(1)
    ref = orc.unscaled_attention(q, k, v, (1.0 - gm) * torch.finfo(torch.float32).min)
    ref = ref.permute(0, 2, 1, 3).reshape(S, B, 768).transpose(0, 1)
    out = K().group_attention(qkv.to(DEV), tok.to(DEV), gid, H).cpu().float()
    # queries whose whole group is masked at that step are padding: compare the rest
    live = (same @ tok.float()) > 0
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    d = (out - ref).abs()[live]
    assert d.max().item() <= tol * max(1.0, ref.abs().max().item())
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("M,N,Kd,rowscale", [(37, 768, 768, False), (1000, 768, 768, True), (34048, 768, 3072, False),
                                             (300, 768, 3136, False)])
def test_linear_hi_lo_residual_stream(M, N, Kd, rowscale):
    """CC2_EPI_LO (bf16): out + lo_out carries the fp32 result
    v = x @ w^T [* rowscale] + (resid + resid_lo) to ~16 significant bits, in
    place as the engine updates its residual stream; the sums of squares are
    those of v.  1-SM (M <= 128) and 2-SM tiles."""
    g = torch.Generator().manual_seed(11 * M + Kd)
    x = torch.randn(M, Kd, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, Kd, generator=g) / math.sqrt(Kd)).to(torch.bfloat16)
    full = 4.0 * torch.randn(M, N, generator=g)
    hi = full.to(torch.bfloat16)
    lo = (full - hi.float()).to(torch.bfloat16)
    kk = K()
    kw = {}
    ssq = None
    if rowscale:
        kw = dict(row_ssq=kk.row_sumsq_parts(x).to(DEV), norm_dim=Kd, eps=1e-6)
        ssq = x.float().pow(2).sum(-1)
    out, out_lo_buf = hi.to(DEV).clone(), kk.rows_to_lo(lo.to(DEV))
    so = torch.full(((N + 63) // 64, M), float("nan"), device=DEV)
    kk.linear(x.to(DEV), w.to(DEV), residual=out, residual_lo=out_lo_buf, lo_out=out_lo_buf, ssq_out=so, out=out,
              **kw)
    out_lo = kk.lo_to_rows(out_lo_buf, M, N)
    ref = _gemm_ref(x, w, None, False, hi.double() + lo.double(), ssq, Kd if rowscale else 0, 1e-6)
    v = out.cpu().double() + out_lo.cpu().double()
    # fp32 accumulation order of the K-sum bounds the agreement, not the storage
    assert (v - ref).abs().max().item() <= 2e-6 * Kd ** 0.5 * ref.abs().max().item()
    assert (out.cpu().double() - ref).abs().max().item() <= 2 ** -8 * ref.abs().max().item()
    assert (out_lo.cpu().float().abs() <= out.cpu().float().abs() * 2 ** -8 + 1e-30).all()
    ref_parts = kk.row_sumsq_parts(ref.float())
    assert torch.allclose(so.cpu(), ref_parts, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("B,S,gsize", [(512, 133, 8), (64, 37, 2), (96, 20, 4), (128, 9, 16), (160, 5, 32), (200, 7, 8)])
def test_group_attention_tensor_core(B, S, gsize):
    """cc2_group_attention_tc (groups of gsize consecutive series on tcgen05)
    against the oracle's attention with the group-time mask; 20 % of tokens
    masked; B not a multiple of 128 for the last cases (a partial block)."""
    H = 12
    g = torch.Generator().manual_seed(B + S + gsize)
    qkv = (torch.randn(B, S, 3 * 768, generator=g) * 0.5).to(torch.bfloat16)
    tok = torch.rand(B, S, generator=g) > 0.2
    gid = torch.arange(B) // gsize
    q, k, v = (qkv.float()[..., i * 768:(i + 1) * 768].transpose(0, 1).reshape(S, B, H, 64).permute(0, 2, 1, 3)
               for i in range(3))
    same = (gid[:, None] == gid[None, :]).float()
    gm = torch.einsum("qb,bt->qbt", same, tok.float()).permute(2, 0, 1).unsqueeze(1)
    ref = orc.unscaled_attention(q, k, v, (1.0 - gm) * torch.finfo(torch.float32).min)
    ref = ref.permute(0, 2, 1, 3).reshape(S, B, 768).transpose(0, 1)
    out = K().group_attention_contig(qkv.to(DEV), tok.to(DEV), gsize, H).cpu().float()
    live = (same @ tok.float()) > 0
    d = (out - ref).abs()[live]
    assert d.max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
    assert torch.isfinite(out).all()
    # the same as the mma.sync group kernel on every live query, within bf16 rounding of P
    mma = K().group_attention(qkv.to(DEV), tok.to(DEV), gid, H).cpu().float()
    assert (out - mma).abs()[live].max().item() <= 2e-2 * max(1.0, ref.abs().max().item())

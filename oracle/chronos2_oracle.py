"""CPU oracle for the CuteChronos2 encoder forward pass.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA path:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product path
(``cutechronos_b200``) never calls it and has no CPU fallback.

It restates, in plain PyTorch on the CPU, the algorithm of the reference
``cutechronos`` package (lee101/cutedsl) for the path
``CuteChronos2Model.forward``.  Every function cites the reference lines it
follows (paths relative to the reference project root).  Weights are passed as
a ``state_dict``-style mapping that uses the reference's own parameter names
(``blocks.{i}.time_attn.q.weight`` ...), so the same dictionary drives the
reference module, this oracle and the CUDA engine.

Parity pin: ``tests/golden/make_golden.py`` runs the reference module itself
(imported from the reference checkout) on seeded inputs and commits its
outputs as fixtures; ``tests/test_oracle_golden.py`` checks this restatement
against them.

Precision model: every op runs in the dtype it runs in inside the reference's
CPU torch path (``dtype`` argument), including the reference's intermediate
roundings (RMSNorm cast before the weight multiply, bf16 scores, fp32
softmax, fp32 inverse instance norm).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

DEFAULT_QUANTILES = [
    0.01, 0.05, 0.1, 0.15, 0.2, 0.25, 0.3, 0.35, 0.4, 0.45,
    0.5, 0.55, 0.6, 0.65, 0.7, 0.75, 0.8, 0.85, 0.9, 0.95, 0.99,
]


@dataclass
class OracleConfig:
    """Mirror of ``CuteChronos2Config`` (cutechronos/model.py:59-91)."""

    d_model: int = 768
    d_kv: int = 64
    d_ff: int = 3072
    num_layers: int = 12
    num_heads: int = 12
    layer_norm_epsilon: float = 1e-6
    rope_theta: float = 10000.0
    reg_token_id: int = 1
    context_length: int = 8192
    input_patch_size: int = 16
    output_patch_size: int = 16
    quantiles: list = field(default_factory=lambda: list(DEFAULT_QUANTILES))
    use_reg_token: bool = True
    use_arcsinh: bool = True
    time_encoding_scale: int | None = None

    def __post_init__(self):
        if self.time_encoding_scale is None:  # model.py:90-91
            self.time_encoding_scale = self.context_length

    @property
    def num_quantiles(self) -> int:
        return len(self.quantiles)


# ---------------------------------------------------------------------------
# Preprocessing: InstanceNorm + Patch + time encoding
# ---------------------------------------------------------------------------

def instance_norm(x: torch.Tensor, eps: float = 1e-5, use_arcsinh: bool = True):
    """InstanceNorm.forward (cutechronos/model.py:369-385): nanmean / nan-std in
    fp32, scale==0 -> eps, all-NaN row -> (loc 0, scale 1), optional arcsinh."""
    orig = x.dtype
    x = x.to(torch.float32)
    loc = torch.nan_to_num(torch.nanmean(x, dim=-1, keepdim=True), nan=0.0)
    scale = torch.nan_to_num((x - loc).square().nanmean(dim=-1, keepdim=True).sqrt(), nan=1.0)
    scale = torch.where(scale == 0, torch.full_like(scale, eps), scale)
    y = (x - loc) / scale
    if use_arcsinh:
        y = torch.arcsinh(y)
    return y.to(orig), loc, scale


def instance_norm_inverse(x: torch.Tensor, loc, scale, use_arcsinh: bool = True):
    """InstanceNorm.inverse (cutechronos/model.py:387-394): fp32 sinh, x*scale+loc,
    cast back to the input dtype."""
    orig = x.dtype
    x = x.to(torch.float32)
    if use_arcsinh:
        x = torch.sinh(x)
    return (x * scale + loc).to(orig)


def patch(x: torch.Tensor, size: int) -> torch.Tensor:
    """Patch.forward (cutechronos/model.py:406-414): left-pad with NaN to a
    multiple of ``size`` and unfold into non-overlapping patches."""
    L = x.shape[-1]
    if L % size:
        pad = torch.full((*x.shape[:-1], size - L % size), float("nan"), dtype=x.dtype)
        x = torch.cat([pad, x], dim=-1)
    return x.unfold(-1, size, size)


def prepare_patched_context(cfg: OracleConfig, context: torch.Tensor,
                            context_mask: torch.Tensor | None, dtype: torch.dtype):
    """_prepare_patched_context (cutechronos/model.py:473-519).

    Returns (patched (B,P,3*ps) dtype, attention_mask (B,P) bool, loc, scale)."""
    context = context.to(torch.float32) if context.dtype != torch.float32 else context
    if context_mask is not None:
        mask = context_mask.to(context.dtype)
    else:
        mask = torch.isnan(context).logical_not().to(context.dtype)
    B, L = context.shape
    if L > cfg.context_length:  # model.py:487-489
        context = context[..., -cfg.context_length:]
        mask = mask[..., -cfg.context_length:]
    normed, loc, scale = instance_norm(context, use_arcsinh=cfg.use_arcsinh)
    normed = normed.to(dtype)
    mask = mask.to(dtype)
    ps = cfg.input_patch_size
    pc = patch(normed, ps)
    pm = torch.nan_to_num(patch(mask, ps), nan=0.0)
    pc = torch.where(pm > 0.0, pc, torch.zeros((), dtype=pc.dtype))
    attn = pm.sum(dim=-1) > 0
    P = attn.shape[-1]
    te = torch.arange(-P * ps, 0, dtype=torch.float32).view(1, P, ps).expand(B, -1, -1)
    te = te.div(cfg.time_encoding_scale).to(dtype)
    return torch.cat([te, pc, pm], dim=-1), attn, loc, scale


def prepare_patched_future(cfg: OracleConfig, N: int, B: int, dtype: torch.dtype):
    """_prepare_patched_future (cutechronos/model.py:521-549)."""
    ps = cfg.output_patch_size
    z = torch.zeros(B, N, ps, dtype=dtype)
    te = torch.arange(0, N * ps, dtype=torch.float32).view(1, N, ps).expand(B, -1, -1)
    te = te.div(cfg.time_encoding_scale).to(dtype)
    return torch.cat([te, z, z.clone()], dim=-1)


# ---------------------------------------------------------------------------
# Encoder pieces
# ---------------------------------------------------------------------------

def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """T5 RMSNorm, torch path (cutechronos/modules/_fallbacks.py:14-22): fp32
    variance, x*rsqrt in x's dtype promotion, cast to the weight dtype for
    half types, then weight * x."""
    var = x.float().pow(2).mean(-1, keepdim=True)
    y = x * torch.rsqrt(var + eps)
    if w.dtype in (torch.float16, torch.bfloat16):
        y = y.to(w.dtype)
    return w * y


def residual_block(x, W, prefix):
    """ResidualBlock.forward (cutechronos/model.py:176-181)."""
    hid = F.relu(F.linear(x, W[prefix + "hidden_layer.weight"], W[prefix + "hidden_layer.bias"]))
    out = F.linear(hid, W[prefix + "output_layer.weight"], W[prefix + "output_layer.bias"])
    res = F.linear(x, W[prefix + "residual_layer.weight"], W[prefix + "residual_layer.bias"])
    return out + res


def rope_cos_sin(cfg: OracleConfig, S: int, dtype: torch.dtype):
    """inv_freq (model.py:200-203) and compute_cos_sin_fallback (model.py:94-109)."""
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.d_kv, 2, dtype=torch.int64).float() / cfg.d_kv))
    pos = torch.arange(S, dtype=torch.long).unsqueeze(0)
    freqs = (inv_freq[None, :, None].float() @ pos[:, None, :].float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def unscaled_attention(q, k, v, mask):
    """unscaled_attention_fallback (cutechronos/model.py:131-142): scores in
    the input dtype (no 1/sqrt(d)), additive mask, fp32 softmax cast back."""
    s = torch.matmul(q, k.transpose(-2, -1))
    if mask is not None:
        s = s + mask
    w = torch.softmax(s.float(), dim=-1).to(q.dtype)
    return torch.matmul(w, v)


def time_self_attention(cfg, W, p, x, ext_mask, cos, sin, kv_hook=None):
    """TimeSelfAttentionFallback.forward, CPU branch (model.py:209-275).
    ``kv_hook(k, v) -> (k, v)`` stands for the key/value quantisers of
    model.py:243-248 (applied after RoPE)."""
    B, S, _ = x.shape
    H, Dh = cfg.num_heads, cfg.d_kv
    n = rms_norm(x, W[p + "layer_norm_weight"], cfg.layer_norm_epsilon)
    q = F.linear(n, W[p + "q.weight"]).view(B, S, H, Dh).transpose(1, 2)
    k = F.linear(n, W[p + "k.weight"]).view(B, S, H, Dh).transpose(1, 2)
    v = F.linear(n, W[p + "v.weight"]).view(B, S, H, Dh).transpose(1, 2)
    c, s_ = cos.unsqueeze(1), sin.unsqueeze(1)  # apply_rope_fallback (model.py:112-128)
    q, k = q * c + _rotate_half(q) * s_, k * c + _rotate_half(k) * s_
    if kv_hook is not None:
        k, v = kv_hook(k, v)
    a = unscaled_attention(q, k, v, ext_mask).transpose(1, 2).reshape(B, S, H * Dh)
    return x + F.linear(a, W[p + "o.weight"])


def group_self_attention(cfg, W, p, x, group_time_mask):
    """GroupSelfAttentionFallback.forward (model.py:295-312): attention across
    the series of a group at each time step, no RoPE."""
    xt = x.transpose(0, 1)
    n = rms_norm(xt, W[p + "layer_norm_weight"], cfg.layer_norm_epsilon)
    T, B = n.shape[0], n.shape[1]
    H, Dh = cfg.num_heads, cfg.d_kv
    q = F.linear(n, W[p + "q.weight"]).view(T, B, H, Dh).permute(0, 2, 1, 3)
    k = F.linear(n, W[p + "k.weight"]).view(T, B, H, Dh).permute(0, 2, 1, 3)
    v = F.linear(n, W[p + "v.weight"]).view(T, B, H, Dh).permute(0, 2, 1, 3)
    a = unscaled_attention(q, k, v, group_time_mask).permute(0, 2, 1, 3).reshape(T, B, H * Dh)
    return (xt + F.linear(a, W[p + "o.weight"])).transpose(0, 1)


def feed_forward(cfg, W, p, x):
    """FeedForwardFallback.forward (model.py:326-332)."""
    n = rms_norm(x, W[p + "layer_norm_weight"], cfg.layer_norm_epsilon)
    return x + F.linear(F.relu(F.linear(n, W[p + "wi.weight"])), W[p + "wo.weight"])


# ---------------------------------------------------------------------------
# Whole forward
# ---------------------------------------------------------------------------

@torch.no_grad()
def forward(cfg: OracleConfig, W: dict, context: torch.Tensor, context_mask=None,
            num_output_patches: int = 1, group_ids=None, dtype=torch.float32,
            return_intermediates: bool = False, kv_hooks=None):
    """CuteChronos2Model.forward (cutechronos/model.py:738-831) on the CPU.

    ``W`` maps reference parameter names to CPU tensors (any dtype; they are
    cast to ``dtype``).  Returns (B, Q, 16*N) in ``dtype``; with
    ``return_intermediates`` also a dict of stage outputs; ``kv_hooks`` (one
    callable per layer or None) quantise the time attention's K and V."""
    W = {k: v.detach().to("cpu", dtype) for k, v in W.items()}
    context = context.detach().cpu()
    B = context.shape[0]
    N = num_output_patches
    inter = {}

    patched, attn, loc, scale = prepare_patched_context(cfg, context, context_mask, dtype)
    inter.update(patched=patched, attn=attn, loc=loc, scale=scale)
    emb = residual_block(patched, W, "input_patch_embedding.")
    amask = attn.to(dtype)
    if cfg.use_reg_token:  # model.py:768-778
        reg = W["shared.weight"][cfg.reg_token_id].view(1, 1, -1).expand(B, 1, -1)
        emb = torch.cat([emb, reg], dim=-2)
        amask = torch.cat([amask, torch.ones(B, 1, dtype=dtype)], dim=-1)
    fut = residual_block(prepare_patched_future(cfg, N, B, dtype), W, "input_patch_embedding.")
    x = torch.cat([emb, fut], dim=-2)
    amask = torch.cat([amask, torch.ones(B, N, dtype=dtype)], dim=-1)
    inter["embeds"] = x
    inter["token_mask"] = amask
    if group_ids is None:
        group_ids = torch.arange(B)
    group_ids = torch.as_tensor(group_ids).cpu()
    S = x.shape[1]
    fmin = torch.finfo(dtype).min
    ext = (1.0 - amask[:, None, None, :]) * fmin  # model.py:552-558
    gm = (group_ids[:, None] == group_ids[None, :]).to(dtype)  # model.py:561-569
    gtm = torch.einsum("qb, bt -> qbt", gm, amask).permute(2, 0, 1).unsqueeze(1)
    gtm = (1.0 - gtm) * fmin
    cos, sin = rope_cos_sin(cfg, S, dtype)
    for i in range(cfg.num_layers):
        p = f"blocks.{i}."
        x = time_self_attention(cfg, W, p + "time_attn.", x, ext, cos, sin,
                                kv_hooks[i] if kv_hooks is not None else None)
        x = group_self_attention(cfg, W, p + "group_attn.", x, gtm)
        x = feed_forward(cfg, W, p + "feed_forward.", x)
        if return_intermediates:
            inter[f"layer{i}"] = x
    x = rms_norm(x, W["final_layer_norm_weight"], cfg.layer_norm_epsilon)
    fe = x[:, -N:]
    q = residual_block(fe, W, "output_patch_embedding.")
    Q, ps = cfg.num_quantiles, cfg.output_patch_size
    inter["quantile_raw"] = q
    q = q.view(B, N, Q, ps).permute(0, 2, 1, 3).reshape(B, Q * N * ps)
    q = instance_norm_inverse(q, loc, scale, cfg.use_arcsinh).view(B, Q, N * ps)
    if return_intermediates:
        return q, inter
    return q


def output_transform(x: torch.Tensor, loc, scale, num_quantiles: int, patch_size: int,
                     use_arcsinh: bool = True) -> torch.Tensor:
    """Rearrange ``b n (q p) -> b q (n p)`` then InstanceNorm.inverse
    (cutechronos/model.py:816-829; triton_kernels/fused_output.py:20-80)."""
    B, N, _ = x.shape
    y = x.view(B, N, num_quantiles, patch_size).permute(0, 2, 1, 3).reshape(B, num_quantiles * N * patch_size)
    return instance_norm_inverse(y, loc.view(B, 1), scale.view(B, 1), use_arcsinh).view(B, num_quantiles, N * patch_size)


def forecast_flops(S: int, P: int, N: int, d=768, dff=3072, layers=12, g=1, out_dim=336, in_dim=48) -> float:
    """Algorithmic FLOPs per forecast (one series), counting group Q/K
    projections even for group size 1."""
    per_tok = 2 * d * d * 8 + 2 * 2 * d * dff + 4 * S * d + 4 * g * d
    return (layers * S * per_tok
            + (P + N) * (2 * in_dim * dff + 2 * dff * d + 2 * in_dim * d)
            + N * (2 * d * dff + 2 * dff * out_dim + 2 * d * out_dim))


def num_patches(cfg: OracleConfig, L: int) -> int:
    L = min(L, cfg.context_length)
    return math.ceil(L / cfg.input_patch_size)


# ---- pipeline host steps around the forward ---------------------------------------------------
def left_pad_and_stack(values: torch.Tensor, lens, context_length: int) -> torch.Tensor:
    """Ragged series (concatenated in ``values``, lengths ``lens``) -> (B, L)
    float32, each row right-aligned and NaN-left-padded to the longest row,
    then cut to the last ``context_length`` steps
    (cutechronos/pipeline.py:221-231 _left_pad_and_stack_rows, 239-243
    _finalize_context_batch)."""
    lens = [int(n) for n in lens]
    n = max(lens)
    out = torch.full((len(lens), n), float("nan"), dtype=torch.float32)
    pos = 0
    for i, k in enumerate(lens):
        if k:
            out[i, n - k:] = values[pos:pos + k]
        pos += k
    return out[:, -context_length:] if n > context_length else out


def select_quantiles(preds: torch.Tensor, training_quantiles, requested_quantiles) -> torch.Tensor:
    """(B, Q, H) float32 -> (B, H, len(requested)): a trained level is
    gathered; another level is ``a * (1 - frac) + b * frac`` between the
    trained neighbours found by searchsorted, clamped to [1, Q-1]
    (cutechronos/pipeline.py:24-58)."""
    bhq = preds.float().permute(0, 2, 1)
    tq = torch.tensor(training_quantiles, dtype=torch.float32)
    cols = []
    for ql in requested_quantiles:
        ql = float(ql)
        if ql in training_quantiles:
            cols.append(bhq[..., list(training_quantiles).index(ql)])
            continue
        hi = int(torch.searchsorted(tq, torch.tensor(ql, dtype=torch.float32)).clamp(1, len(tq) - 1))
        lo = hi - 1
        frac = (ql - tq[lo].item()) / max(tq[hi].item() - tq[lo].item(), 1e-9)
        cols.append(bhq[..., lo] * (1 - frac) + bhq[..., hi] * frac)
    return torch.stack(cols, dim=-1)

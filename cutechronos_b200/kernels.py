"""Torch-tensor entry points to the component kernels of the C ABI.

Each function mirrors the signature and output layout of the reference op it
replaces (paths inside lee101/cutedsl) and calls exactly one native kernel
(``rms_layernorm`` / ``linear`` / ``unscaled_attention`` one each):

  fused_preprocess        cutechronos/kernels.py:106-155 (-> cc2_preprocess)
  fused_output_transform  cutechronos/triton_kernels/fused_output.py:83-140
  rms_layernorm           cutechronos/kernel_backends.py:85-110
  linear                  F.linear call sites with fused epilogues (cc2_gemm)
  unscaled_attention      cutechronos/kernel_backends.py:113-153 (+ RoPE when
                          ``rope=True``: triton_kernels/rope.py:126-180)
  group_attention         cutechronos/model.py:295-312 attention core

All inputs must be CUDA tensors; nothing here runs on the CPU.
"""

from __future__ import annotations

import ctypes as C
import math

import torch

from . import _native as nat

_CODES = {torch.bfloat16: nat.CC2_BF16, torch.float32: nat.CC2_F32}


def _code(dt: torch.dtype) -> int:
    if dt not in _CODES:
        raise TypeError(f"dtype {dt} not supported (bfloat16 / float32)")
    return _CODES[dt]


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("cutechronos_b200 kernels take CUDA tensors only (no CPU path)")


def fused_preprocess(context: torch.Tensor, patch_size: int = 16, context_length: int = 512,
                     use_arcsinh: bool = False, *, context_mask: torch.Tensor | None = None,
                     time_encoding_scale: float | None = None, dtype: torch.dtype = torch.float32):
    """-> (patched (B,P,3ps), attention_mask (B,P) f32, loc (B,1), scale (B,1))."""
    _cuda(context, context_mask)
    lib = nat.load()
    ctx = context.float().contiguous()
    mask = context_mask.float().contiguous() if context_mask is not None else None
    B, L = ctx.shape
    Leff = min(L, context_length)
    P = math.ceil(Leff / patch_size)
    dev = ctx.device
    patched = torch.empty(B, P, 3 * patch_size, dtype=dtype, device=dev)
    tok = torch.empty(B * P, dtype=torch.uint8, device=dev)
    attn = torch.empty(B, P, dtype=torch.float32, device=dev)
    loc = torch.empty(B, 1, dtype=torch.float32, device=dev)
    scale = torch.empty(B, 1, dtype=torch.float32, device=dev)
    tes = float(time_encoding_scale if time_encoding_scale is not None else context_length)
    nat.check(lib.cc2_preprocess(ctx.data_ptr(), mask.data_ptr() if mask is not None else None, B, L, patch_size,
                                 context_length, tes, int(use_arcsinh), 0, 0, _code(dtype), patched.data_ptr(),
                                 3 * patch_size, 3 * patch_size, tok.data_ptr(), attn.data_ptr(), loc.data_ptr(),
                                 scale.data_ptr(), _stream(ctx)), "cc2_preprocess")
    return patched, attn, loc, scale


def fused_output_transform(x: torch.Tensor, loc: torch.Tensor, scale: torch.Tensor, num_quantiles: int = 21,
                           patch_size: int = 16, use_arcsinh: bool = True) -> torch.Tensor:
    """(B, N, Q*P) -> (B, Q, N*P): rearrange, sinh, * scale + loc (in x's dtype)."""
    _cuda(x, loc, scale)
    B, N, QP = x.shape
    if QP != num_quantiles * patch_size:
        raise ValueError(f"Last dim of x ({QP}) must equal num_quantiles * patch_size")
    x = x.contiguous()
    out = torch.empty(B, num_quantiles, N * patch_size, dtype=x.dtype, device=x.device)
    lf, sf = loc.reshape(B).float().contiguous(), scale.reshape(B).float().contiguous()
    nat.check(nat.load().cc2_output_transform(_code(x.dtype), x.data_ptr(), QP, lf.data_ptr(), sf.data_ptr(),
                                              out.data_ptr(), B, N, num_quantiles, patch_size, int(use_arcsinh),
                                              _stream(x)), "cc2_output_transform")
    return out


def rms_layernorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """T5 RMSNorm over the last dim: weight * cast(x * rsqrt(mean(x^2) + eps))."""
    _cuda(x, weight)
    shape = x.shape
    D = shape[-1]
    x2 = x.reshape(-1, D).contiguous()
    w = weight.to(x.dtype).contiguous()
    y = torch.empty_like(x2)
    rows = x2.shape[0]
    nat.check(nat.load().cc2_rmsnorm_rows(_code(x.dtype), x2.data_ptr(), D, w.data_ptr(), y.data_ptr(), D, rows, D,
                                          rows, 0, 0, float(eps), _stream(x)), "cc2_rmsnorm_rows")
    return y.reshape(shape)


def row_sumsq_parts(x: torch.Tensor) -> torch.Tensor:
    """(G, M) fp32 partial sums of squares over 64-column groups of x (M, K):
    the layout the SSQ epilogue writes and the ROWSCALE epilogue reads."""
    M, Kd = x.shape
    G = (Kd + 63) // 64
    xp = torch.nn.functional.pad(x.float(), (0, G * 64 - Kd))
    return xp.reshape(M, G, 64).pow(2).sum(-1).T.contiguous()


def lo_numel(M: int, N: int) -> int:
    """Elements of a low-halves buffer (CC2_EPI_LO) for an (M, N) result."""
    return -(-M // 32) * 32 * N


def rows_to_lo(t: torch.Tensor) -> torch.Tensor:
    """(M, N) row-major -> the 32-row interleaved layout of CC2_EPI_LO buffers:
    element (row, col) at ((row/32 * N/8 + col/8) * 32 + row%32) * 8 + col%8."""
    M, N = t.shape
    Mp = -(-M // 32) * 32
    p = torch.zeros(Mp, N, dtype=t.dtype, device=t.device)
    p[:M] = t
    return p.view(Mp // 32, 32, N // 8, 8).permute(0, 2, 1, 3).contiguous().view(-1)


def lo_to_rows(lo: torch.Tensor, M: int, N: int) -> torch.Tensor:
    """Inverse of :func:`rows_to_lo`."""
    Mp = -(-M // 32) * 32
    return lo.view(Mp // 32, N // 8, 32, 8).permute(0, 2, 1, 3).reshape(Mp, N)[:M]


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *, relu: bool = False,
           residual: torch.Tensor | None = None, row_ssq: torch.Tensor | None = None, norm_dim: int = 0,
           eps: float = 1e-6, ssq_out: torch.Tensor | None = None, out: torch.Tensor | None = None,
           rope_period: int = 0, rope_cols: int = 0, residual_lo: torch.Tensor | None = None,
           lo_out: torch.Tensor | None = None) -> torch.Tensor:
    """out = epilogue(x @ weight^T): optional row scale
    rsqrt(row_ssq.sum(0) / norm_dim + eps) with ``row_ssq`` (G, M) partial sums
    per 64-column group, + bias (fp32), ReLU, + residual, and ``ssq_out``
    (G', M) <- partial sums of squares of the stored output.  ``rope_period``
    > 0 (bf16 only) rotates every 64-column head below ``rope_cols`` at
    position row % rope_period with bf16 cos/sin, as the engine does for Q, K.
    ``lo_out`` (bf16 only; ``lo_numel(M, N)`` elements in the interleaved layout
    of :func:`rows_to_lo`) receives the low halves bf16(v - out) of the result
    v, and ``residual_lo`` (same layout) the residual's low halves (residual +
    residual_lo is the residual): the engine's hi + lo residual stream."""
    _cuda(x, weight, bias, residual, row_ssq, ssq_out, residual_lo, lo_out)
    K = x.shape[-1]
    x2 = x.reshape(-1, K).contiguous()
    M, N = x2.shape[0], weight.shape[0]
    w = weight.contiguous()
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    e = nat.Epilogue()
    flags = 0
    keep = []
    if row_ssq is not None:
        flags |= nat.EPI_ROWSCALE
        r = row_ssq.float().contiguous()
        keep.append(r)
        e.ssq_in, e.norm_dim, e.eps = r.data_ptr(), norm_dim, eps
        e.ssq_ld = r.shape[-1]
    if bias is not None:
        flags |= nat.EPI_BIAS
        b = bias.float().contiguous()
        keep.append(b)
        e.bias = b.data_ptr()
    if relu:
        flags |= nat.EPI_RELU
    if residual is not None:
        flags |= nat.EPI_RESID
        rr = residual.reshape(M, N).contiguous()
        keep.append(rr)
        e.resid, e.ld_resid = rr.data_ptr(), N
    if ssq_out is not None:
        flags |= nat.EPI_SSQ
        e.ssq_out = ssq_out.data_ptr()
        e.ssq_ld = ssq_out.shape[-1]
    if rope_period > 0:
        flags |= nat.EPI_ROPE
        tab = rope_table_bf16(rope_period, 64, 10000.0, x.device)
        keep.append(tab)
        e.rope_cs, e.rope_period, e.rope_cols = tab.data_ptr(), rope_period, rope_cols
    if lo_out is not None:
        n_lo = lo_numel(M, N)
        if x.dtype != torch.bfloat16 or lo_out.dtype != torch.bfloat16 or lo_out.numel() != n_lo \
                or not lo_out.is_contiguous() or N % 8:
            raise ValueError("lo_out must be a contiguous bf16 buffer of lo_numel(M, N) elements "
                             "(interleaved layout, see rows_to_lo) of a bf16 GEMM with N % 8 == 0")
        flags |= nat.EPI_LO
        e.lo_out, e.ld_lo = lo_out.data_ptr(), N
        if residual_lo is not None:
            if residual is None:
                raise ValueError("residual_lo needs residual")
            if residual_lo.dtype != torch.bfloat16 or residual_lo.numel() != n_lo or not residual_lo.is_contiguous():
                raise ValueError("residual_lo must be a contiguous bf16 buffer of lo_numel(M, N) elements")
            e.resid_lo = residual_lo.data_ptr()
        elif residual is not None:
            z = torch.zeros(n_lo, dtype=torch.bfloat16, device=x.device)
            keep.append(z)
            e.resid_lo = z.data_ptr()
    elif residual_lo is not None:
        raise ValueError("residual_lo needs lo_out")
    e.flags = flags
    nat.check(nat.load().cc2_gemm(_code(x.dtype), x2.data_ptr(), K, w.data_ptr(), K, out.data_ptr(), N, M, N, K,
                                  C.byref(e), _stream(x)), "cc2_gemm")
    return out.reshape(*x.shape[:-1], N)


_ROPE_CACHE: dict = {}


def rope_table(S: int, d_kv: int = 64, theta: float = 10000.0, device=None) -> torch.Tensor:
    """(S, d_kv/2, 2) fp32 (cos, sin) of inv_freq * pos, computed like the
    engine's table (fp32 angle, accurate cos/sin)."""
    key = (S, d_kv, theta, str(device))
    if key not in _ROPE_CACHE:
        inv = 1.0 / (theta ** (torch.arange(0, d_kv, 2, dtype=torch.int64).float() / d_kv))
        ang = (torch.arange(S, dtype=torch.float32)[:, None] * inv[None, :]).double()
        tab = torch.stack([ang.cos(), ang.sin()], dim=-1).float()
        _ROPE_CACHE[key] = tab.to(device)
    return _ROPE_CACHE[key]


def rope_table_bf16(S: int, d_kv: int = 64, theta: float = 10000.0, device=None) -> torch.Tensor:
    """(S, d_kv/2) int32 of packed bf16 (cos | sin << 16), the QKV-epilogue table."""
    t = rope_table(S, d_kv, theta, "cpu").to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF
    return (t[..., 0] | (t[..., 1] << 16)).to(torch.int32).contiguous().to(device)


def unscaled_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None = None, *,
                       rope: bool = False, rope_theta: float = 10000.0) -> torch.Tensor:
    """softmax(q k^T + mask) v with no 1/sqrt(d) factor; q,k,v (B,H,S,64).
    ``mask``: additive (B,1,1,S) float mask (finfo.min = masked) or (B,S)
    bool key mask.  ``rope=True`` rotates q and k at positions 0..S-1 first."""
    _cuda(q, k, v, mask)
    B, H, S, D = q.shape
    dev = q.device
    packed = torch.cat([t.transpose(1, 2).reshape(B, S, H * D) for t in (q, k, v)], dim=-1).reshape(B * S, 3 * H * D)
    packed = packed.contiguous()
    if mask is None:
        tok = torch.ones(B * S, dtype=torch.uint8, device=dev)
    elif mask.dtype == torch.bool:
        tok = mask.reshape(B * S).to(torch.uint8).contiguous()
    else:
        m = mask.reshape(B, -1)[:, -S:] if mask.numel() == B * S else mask.reshape(B, S)
        tok = (m > torch.finfo(m.dtype).min / 2).reshape(B * S).to(torch.uint8).contiguous()
    out = torch.empty(B * S, H * D, dtype=q.dtype, device=dev)
    cs = rope_table(S, D, rope_theta, dev) if rope else None
    nat.check(nat.load().cc2_attention(_code(q.dtype), 0, packed.data_ptr(), 3 * H * D, 0, H * D, 2 * H * D,
                                       out.data_ptr(), H * D, tok.data_ptr(), B, S, H, D, None, None, 0, 0,
                                       cs.data_ptr() if cs is not None else None, _stream(q)), "cc2_attention")
    return out.reshape(B, S, H, D).transpose(1, 2)


def attention_rows(qkv: torch.Tensor, token_mask: torch.Tensor, num_sets: int, S: int, num_heads: int,
                   rope: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
    """Time attention on token rows already packed as the engine keeps them:
    qkv (num_sets*S, 3*H*64) [Q|K|V], token_mask (num_sets*S,) uint8 ->
    (num_sets*S, H*64).  One kernel launch, no repacking."""
    _cuda(qkv, token_mask)
    HD = qkv.shape[1] // 3
    if out is None:
        out = torch.empty(qkv.shape[0], HD, dtype=qkv.dtype, device=qkv.device)
    cs = rope_table(S, HD // num_heads, 10000.0, qkv.device) if rope else None
    nat.check(nat.load().cc2_attention(_code(qkv.dtype), 0, qkv.data_ptr(), qkv.shape[1], 0, HD, 2 * HD,
                                       out.data_ptr(), HD, token_mask.data_ptr(), num_sets, S, num_heads,
                                       HD // num_heads, None, None, 0, 0,
                                       cs.data_ptr() if cs is not None else None, _stream(qkv)), "cc2_attention")
    return out


def group_attention_contig(qkv: torch.Tensor, token_mask: torch.Tensor, group_size: int, num_heads: int,
                           ) -> torch.Tensor:
    """Group self-attention on the tensor cores for groups of ``group_size``
    consecutive series (2..32, a power of two): qkv (B, S, 3*H*64) bf16
    packed [Q|K|V], token_mask (B, S) -> (B, S, H*64)."""
    _cuda(qkv, token_mask)
    B, S, W = qkv.shape
    HD = W // 3
    q = qkv.contiguous()
    tok = token_mask.to(torch.uint8).contiguous()
    out = torch.empty(B, S, HD, dtype=qkv.dtype, device=qkv.device)
    nat.check(nat.load().cc2_group_attention_tc(q.data_ptr(), W, 0, HD, 2 * HD, out.data_ptr(), HD, tok.data_ptr(),
                                                B, S, num_heads, group_size, _stream(qkv)), "cc2_group_attention_tc")
    return out


def group_attention(qkv: torch.Tensor, token_mask: torch.Tensor, group_ids: torch.Tensor, num_heads: int,
                    ) -> torch.Tensor:
    """Group self-attention core over token rows: qkv (B, S, 3*H*64) packed
    [Q|K|V], token_mask (B, S) bool, group_ids (B,) -> (B, S, H*64)."""
    _cuda(qkv, token_mask)
    B, S, W = qkv.shape
    HD = W // 3
    lib = nat.load()
    g = torch.as_tensor(group_ids).to("cpu", torch.int64).contiguous()
    mem = (C.c_int32 * B)()
    off = (C.c_int32 * (B + 1))()
    ng, mg = C.c_int(), C.c_int()
    nat.check(lib.cc2_group_layout(g.data_ptr(), B, mem, off, C.byref(ng), C.byref(mg)), "cc2_group_layout")
    dev = qkv.device
    mem_t = torch.tensor(list(mem), dtype=torch.int32).to(dev)
    off_t = torch.tensor(list(off)[: ng.value + 1], dtype=torch.int32).to(dev)
    x = qkv.reshape(B * S, W).contiguous()
    tok = token_mask.reshape(B * S).to(torch.uint8).contiguous()
    out = torch.empty(B * S, HD, dtype=qkv.dtype, device=dev)
    nat.check(lib.cc2_attention(_code(qkv.dtype), 1, x.data_ptr(), W, 0, HD, 2 * HD, out.data_ptr(), HD,
                                tok.data_ptr(), S * ng.value, S, num_heads, HD // num_heads, mem_t.data_ptr(),
                                off_t.data_ptr(), ng.value, mg.value, None, _stream(qkv)), "cc2_attention")
    return out.reshape(B, S, HD)


def stack_series(values: torch.Tensor, offsets: torch.Tensor, L: int) -> torch.Tensor:
    """Ragged series -> (B, L) float32, right-aligned, NaN-left-padded, each
    row's last L values kept (pipeline.py:221-243).  values (T,) float32 and
    offsets (B+1,) int64 on the device."""
    _cuda(values, offsets)
    B = offsets.numel() - 1
    out = torch.empty(B, L, dtype=torch.float32, device=values.device)
    nat.check(nat.load().cc2_stack_series(values.data_ptr(), offsets.data_ptr(), B, L, out.data_ptr(),
                                          _stream(values)), "cc2_stack_series")
    return out


def quantile_table(training_quantiles: list[float], levels: list[float]):
    """Per requested level: (lo, hi, w_lo, w_hi) as the reference's
    _select_quantiles (pipeline.py:24-58) picks them: a trained level is
    gathered (lo == hi); another level interpolates between the trained
    neighbours found by searchsorted (clamped to [1, Q-1]) with weights
    1 - frac and frac rounded to fp32."""
    index = {q: i for i, q in enumerate(training_quantiles)}
    tq = torch.tensor(training_quantiles, dtype=torch.float32)
    lo, hi, wl, wh = [], [], [], []
    for ql in levels:
        di = index.get(ql)
        if di is not None:
            lo.append(di), hi.append(di), wl.append(1.0), wh.append(0.0)
            continue
        h = int(torch.searchsorted(tq, torch.tensor(ql, dtype=torch.float32)).clamp(1, len(tq) - 1))
        frac = (ql - tq[h - 1].item()) / max(tq[h].item() - tq[h - 1].item(), 1e-9)
        lo.append(h - 1), hi.append(h), wl.append(1 - frac), wh.append(frac)
    return lo, hi, wl, wh


def select_quantiles(preds: torch.Tensor, H: int, training_quantiles: list[float], levels: list[float], *,
                     layout: int = 1, median_level: int | None = None, out: torch.Tensor | None = None):
    """preds (B, Q, ld) -> float32 levels: layout 0 (B, nq, H), layout 1
    (B, H, nq); with ``median_level`` also the gathered (B, H) row of that
    trained level.  ``out`` (optional) is a flat float32 device buffer that
    receives the levels followed by the median."""
    _cuda(preds)
    B, Q, ld = preds.shape
    if preds.stride(2) != 1 or preds.stride(1) != ld or preds.stride(0) != Q * ld:
        preds = preds.contiguous()
    nq = len(levels)
    lo, hi, wl, wh = quantile_table(training_quantiles, levels)
    n_lv, n_med = B * H * nq, (B * H if median_level is not None else 0)
    if out is None:
        out = torch.empty(n_lv + n_med, dtype=torch.float32, device=preds.device)
    ai = C.c_int * max(nq, 1)
    af = C.c_float * max(nq, 1)
    med_ptr = out.data_ptr() + 4 * n_lv if median_level is not None else None
    nat.check(nat.load().cc2_select_quantiles(
        _code(preds.dtype), preds.data_ptr(), B, Q, ld, H, nq, ai(*lo), ai(*hi), af(*wl), af(*wh), layout,
        out.data_ptr(), median_level if median_level is not None else 0, med_ptr, _stream(preds)),
        "cc2_select_quantiles")
    shape = (B, nq, H) if layout == 0 else (B, H, nq)
    lv = out[:n_lv].view(shape)
    return (lv, out[n_lv:n_lv + n_med].view(B, H)) if median_level is not None else lv

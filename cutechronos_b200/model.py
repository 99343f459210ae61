"""CuteChronos2Model for B200: the reference's module, API and tensor layouts,
computed by the native sm_100a engine.

Drop-in for ``cutechronos.model`` (lee101/cutedsl, cutechronos/model.py):
  * ``CuteChronos2Config`` mirrors model.py:59-91;
  * ``CuteChronos2Model`` registers the same parameters in the same order
    (model.py:419-468), so ``state_dict`` keys, ``load_chronos2_weights``
    (model.py:833-900), ``load_lora_adapter`` (902-950), ``from_pretrained``
    (952-1021) and ``from_original`` (1023-1062) behave like the reference;
  * ``forward(context, context_mask=None, num_output_patches=1,
    group_ids=None) -> (B, Q, 16*N)`` (model.py:738-831) runs entirely in the
    native library (``cc2_forward``); the parameters are packed once into the
    engine's layout (RMSNorm weights folded into the projections, Q/K/V
    fused, ResidualBlock hidden+skip fused) and re-packed when a parameter
    changes.

There is no CPU path: forward raises unless the parameters live on a CUDA
device and the native library is built.
"""

from __future__ import annotations

import ctypes as C
import json
import logging
from contextlib import contextmanager
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
import torch.nn as nn

from . import _native as nat

logger = logging.getLogger(__name__)


@dataclass
class CuteChronos2Config:
    d_model: int = 768
    d_kv: int = 64
    d_ff: int = 3072
    num_layers: int = 12
    num_heads: int = 12
    dropout_rate: float = 0.1
    layer_norm_epsilon: float = 1e-6
    dense_act_fn: str = "relu"
    rope_theta: float = 10000.0
    vocab_size: int = 2
    reg_token_id: int = 1
    context_length: int = 8192
    input_patch_size: int = 16
    input_patch_stride: int = 16
    output_patch_size: int = 16
    num_quantiles: int = 21
    quantiles: list[float] | None = None
    use_reg_token: bool = True
    use_arcsinh: bool = True
    time_encoding_scale: int | None = None
    max_output_patches: int = 64

    def __post_init__(self):
        if self.quantiles is None:
            self.quantiles = [
                0.01, 0.05, 0.1, 0.15, 0.2, 0.25, 0.3, 0.35, 0.4, 0.45,
                0.5, 0.55, 0.6, 0.65, 0.7, 0.75, 0.8, 0.85, 0.9, 0.95, 0.99,
            ]
        self.num_quantiles = len(self.quantiles)
        if self.time_encoding_scale is None:
            self.time_encoding_scale = self.context_length

    def to_native(self) -> nat.Config:
        if self.dense_act_fn != "relu":
            raise ValueError(f"dense_act_fn {self.dense_act_fn!r} is not supported (relu only)")
        if self.input_patch_stride != self.input_patch_size:
            raise ValueError("input_patch_stride must equal input_patch_size")
        return nat.Config(
            d_model=self.d_model, d_kv=self.d_kv, d_ff=self.d_ff, num_layers=self.num_layers,
            num_heads=self.num_heads, layer_norm_epsilon=self.layer_norm_epsilon,
            rope_theta=self.rope_theta, reg_token_id=self.reg_token_id,
            context_length=self.context_length, input_patch_size=self.input_patch_size,
            output_patch_size=self.output_patch_size, num_quantiles=self.num_quantiles,
            use_reg_token=int(self.use_reg_token), use_arcsinh=int(self.use_arcsinh),
            time_encoding_scale=float(self.time_encoding_scale),
            max_output_patches=self.max_output_patches)


# ---------------------------------------------------------------------------
# Parameter containers (same names and registration order as the reference)
# ---------------------------------------------------------------------------

class ResidualBlock(nn.Module):
    def __init__(self, in_dim: int, h_dim: int, out_dim: int):
        super().__init__()
        self.hidden_layer = nn.Linear(in_dim, h_dim)
        self.output_layer = nn.Linear(h_dim, out_dim)
        self.residual_layer = nn.Linear(in_dim, out_dim)


class _Attention(nn.Module):
    def __init__(self, config: CuteChronos2Config):
        super().__init__()
        inner = config.num_heads * config.d_kv
        self.layer_norm_weight = nn.Parameter(torch.ones(config.d_model))
        self.q = nn.Linear(config.d_model, inner, bias=False)
        self.k = nn.Linear(config.d_model, inner, bias=False)
        self.v = nn.Linear(config.d_model, inner, bias=False)
        self.o = nn.Linear(inner, config.d_model, bias=False)


class TimeSelfAttention(_Attention):
    pass


class GroupSelfAttention(_Attention):
    pass


class FeedForward(nn.Module):
    def __init__(self, config: CuteChronos2Config):
        super().__init__()
        self.layer_norm_weight = nn.Parameter(torch.ones(config.d_model))
        self.wi = nn.Linear(config.d_model, config.d_ff, bias=False)
        self.wo = nn.Linear(config.d_ff, config.d_model, bias=False)


class EncoderBlock(nn.Module):
    def __init__(self, config: CuteChronos2Config):
        super().__init__()
        self.time_attn = TimeSelfAttention(config)
        self.group_attn = GroupSelfAttention(config)
        self.feed_forward = FeedForward(config)


_DTYPES = {torch.bfloat16: nat.CC2_BF16, torch.float32: nat.CC2_F32}


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


class _Engine:
    """Packed weights + native model handle for one (device, dtype, version)."""

    def __init__(self, model: "CuteChronos2Model"):
        lib = nat.load()
        cfg = model.config
        dev = model._param_device()
        dt = model._param_dtype()
        if dt not in _DTYPES:
            raise TypeError(f"parameter dtype {dt} is not supported (bfloat16 or float32)")
        self.dtype_code = _DTYPES[dt]
        self.ncfg = cfg.to_native()
        nbytes = C.c_size_t()
        nat.check(lib.cc2_model_pack_bytes(C.byref(self.ncfg), self.dtype_code, C.byref(nbytes)),
                  "cc2_model_pack_bytes")
        self.pack = torch.empty(nbytes.value, dtype=torch.uint8, device=dev)
        b = model.blocks
        L = cfg.num_layers
        self._arrays = []
        keep = []  # contiguous views/copies must outlive the packing launches

        def P(t):
            t = t.detach().contiguous()
            keep.append(t)
            return _ptr(t)

        def arrp(fn):
            ts = [fn(b[i]).detach().contiguous() for i in range(L)]
            keep.extend(ts)
            a = (C.c_void_p * L)(*[_ptr(t) for t in ts])
            self._arrays.append(a)
            return C.cast(a, nat._PP)

        ie, oe = model.input_patch_embedding, model.output_patch_embedding
        w = nat.Weights(
            shared=P(model.shared.weight),
            in_hidden_w=P(ie.hidden_layer.weight), in_hidden_b=P(ie.hidden_layer.bias),
            in_output_w=P(ie.output_layer.weight), in_output_b=P(ie.output_layer.bias),
            in_residual_w=P(ie.residual_layer.weight), in_residual_b=P(ie.residual_layer.bias),
            time_ln=arrp(lambda x: x.time_attn.layer_norm_weight), time_q=arrp(lambda x: x.time_attn.q.weight),
            time_k=arrp(lambda x: x.time_attn.k.weight), time_v=arrp(lambda x: x.time_attn.v.weight),
            time_o=arrp(lambda x: x.time_attn.o.weight),
            group_ln=arrp(lambda x: x.group_attn.layer_norm_weight), group_q=arrp(lambda x: x.group_attn.q.weight),
            group_k=arrp(lambda x: x.group_attn.k.weight), group_v=arrp(lambda x: x.group_attn.v.weight),
            group_o=arrp(lambda x: x.group_attn.o.weight),
            ff_ln=arrp(lambda x: x.feed_forward.layer_norm_weight), ff_wi=arrp(lambda x: x.feed_forward.wi.weight),
            ff_wo=arrp(lambda x: x.feed_forward.wo.weight),
            final_ln=P(model.final_layer_norm_weight),
            out_hidden_w=P(oe.hidden_layer.weight), out_hidden_b=P(oe.hidden_layer.bias),
            out_output_w=P(oe.output_layer.weight), out_output_b=P(oe.output_layer.bias),
            out_residual_w=P(oe.residual_layer.weight), out_residual_b=P(oe.residual_layer.bias),
        )
        handle = C.c_void_p()
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            nat.check(lib.cc2_model_create(C.byref(self.ncfg), self.dtype_code, C.byref(w), _ptr(self.pack),
                                           nbytes.value, stream, C.byref(handle)), "cc2_model_create")
            torch.cuda.current_stream(dev).synchronize()
        del keep
        self.handle = handle
        self.device = dev
        self.dtype = dt
        self._ws = None
        self._lib = lib

    def workspace(self, B: int, L: int, N: int, max_group: int) -> tuple[int, int]:
        nbytes = C.c_size_t()
        nat.check(self._lib.cc2_forward_workspace_bytes(self.handle, B, L, N, max_group, C.byref(nbytes)),
                  "cc2_forward_workspace_bytes")
        if self._ws is None or self._ws.numel() < nbytes.value:
            self._ws = None
            self._ws = torch.empty(nbytes.value, dtype=torch.uint8, device=self.device)
        return _ptr(self._ws), nbytes.value

    def __del__(self):
        try:
            if getattr(self, "handle", None) and self.handle.value:
                self._lib.cc2_model_destroy(self.handle)
        except Exception:
            pass


class CuteChronos2Model(nn.Module):
    """Chronos-2 encoder with the reference's parameters, computed on B200."""

    def __init__(self, config: CuteChronos2Config):
        super().__init__()
        self.config = config
        self._offloaded = False
        self.shared = nn.Embedding(config.vocab_size, config.d_model)
        in_dim = config.input_patch_size * 3
        self.input_patch_embedding = ResidualBlock(in_dim, config.d_ff, config.d_model)
        self.blocks = nn.ModuleList([EncoderBlock(config) for _ in range(config.num_layers)])
        self.final_layer_norm_weight = nn.Parameter(torch.ones(config.d_model))
        self.output_patch_embedding = ResidualBlock(
            config.d_model, config.d_ff, config.num_quantiles * config.output_patch_size)
        self.register_buffer("quantiles", torch.tensor(config.quantiles, dtype=torch.float32), persistent=False)
        self._engine: _Engine | None = None
        self._engine_key = None
        self._cuda_graphs = False
        self._graphs: dict = {}
        self._tubroquant_config: dict | None = None
        self._tq_state = None  # (engine, per-layer params, stats tensor) of the enabled hook
        self._tq_last_rows = 0

    # -- helpers mirroring the reference ---------------------------------------------
    def _param_dtype(self) -> torch.dtype:
        return self.shared.weight.dtype

    def _param_device(self) -> torch.device:
        return self.shared.weight.device

    def _weights_key(self):
        def version(p):
            try:
                return p._version
            except RuntimeError:  # inference tensors carry no version counter
                return -1
        return tuple((p.data_ptr(), version(p), p.dtype) for p in self.parameters())

    def engine(self) -> _Engine:
        """The packed native model for the current parameters (re-packed when
        any parameter's storage, version or dtype changed)."""
        key = self._weights_key()
        if self._engine is None or self._engine_key != key:
            self._engine = None
            self._engine = _Engine(self)
            self._engine_key = key
        return self._engine

    # -- forward ---------------------------------------------------------------------------
    def forward(
        self,
        context: torch.Tensor,
        context_mask: torch.Tensor | None = None,
        num_output_patches: int = 1,
        group_ids: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """(B, L) context (NaN = missing) -> (B, num_quantiles, 16*num_output_patches)
        quantile forecasts in the parameter dtype (model.py:738-831)."""
        dev = self._param_device()
        if dev.type != "cuda":
            raise RuntimeError("CuteChronos2Model (B200 engine) runs on CUDA devices only; "
                               "move the model with .to('cuda') (there is no CPU path)")
        if context.dim() != 2:
            raise ValueError(f"context must be (B, L), got {tuple(context.shape)}")
        eng = self.engine()
        B, L = context.shape
        N = int(num_output_patches)
        ctx = context.to(device=dev, dtype=torch.float32).contiguous()
        mask = None
        if context_mask is not None:
            mask = context_mask.to(device=dev, dtype=torch.float32).contiguous()
            if mask.shape != ctx.shape:
                raise ValueError("context_mask must have the shape of context")
        gid_host = None
        max_group = 1
        if group_ids is not None:
            g = torch.as_tensor(group_ids).detach().to("cpu", torch.int64).contiguous()
            if g.numel() != B:
                raise ValueError("group_ids must have one entry per series")
            counts = torch.unique(g, return_counts=True)[1]
            max_group = int(counts.max())
            if max_group > 1:
                gid_host = g
        cfg = self.config
        if (self._cuda_graphs and gid_host is None and not torch.cuda.is_current_stream_capturing()):
            out = self._forward_graph(eng, dev, ctx, mask, B, L, N)
            self._check_device(dev)
            return out
        out = torch.empty(B, cfg.num_quantiles, N * cfg.output_patch_size, dtype=eng.dtype, device=dev)
        self._last_loc = torch.empty(B, dtype=torch.float32, device=dev)
        self._last_scale = torch.empty(B, dtype=torch.float32, device=dev)
        self._native_forward(eng, dev, ctx, mask, gid_host, B, L, N, max_group, out, self._last_loc,
                             self._last_scale)
        self._check_device(dev)
        return out

    def set_device_checks(self, enabled: bool = True) -> "CuteChronos2Model":
        """After every forward, synchronise the device and raise if a kernel's
        bounded wait ran out (its outputs are then incomplete although the launch
        succeeded).  Off by default: the check costs one device synchronisation."""
        self._device_checks = bool(enabled)
        return self

    def _check_device(self, dev) -> None:
        if not getattr(self, "_device_checks", False) or torch.cuda.is_current_stream_capturing():
            return
        with torch.cuda.device(dev):
            st = nat.load().cc2_device_status(1)
        if st < 0:
            nat.check(st, "cc2_device_status")
        if st:
            raise nat.NativeError(f"a kernel of the forward gave up waiting (device status {st}); "
                                  "its outputs are incomplete")

    def _native_forward(self, eng, dev, ctx, mask, gid_host, B, L, N, max_group, out, loc, scale):
        cfg = self.config
        ws, ws_bytes = eng.workspace(B, L, N, max_group)
        tq = self._turboquant_for(eng, dev)
        if tq is not None:
            tq[2].zero_()
            P = -(-min(L, cfg.context_length) // cfg.input_patch_size)
            self._tq_last_rows = B * (P + int(cfg.use_reg_token) + N)
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            st = eng._lib.cc2_forward(
                eng.handle, _ptr(ctx), _ptr(mask) if mask is not None else None, B, L, N,
                gid_host.data_ptr() if gid_host is not None else None, _ptr(out), _ptr(loc), _ptr(scale), ws,
                ws_bytes, stream)
        nat.check(st, "cc2_forward")
        return ws

    # -- CUDA-graph replay (the reference's compile_mode, model.py:1065-1140) ---------------
    def enable_cuda_graphs(self, enabled: bool = True) -> "CuteChronos2Model":
        """Replay one captured CUDA graph per (B, L, N, mask) shape instead of
        launching the forward's kernels one by one (the role torch.compile's
        "reduce-overhead" mode plays in the reference).  Series groups (group
        ids with repeated values) run eagerly.  Each call copies its inputs
        into the graph's buffers and returns copies of its outputs."""
        self._cuda_graphs = bool(enabled)
        self._graphs = {}
        return self

    def _forward_graph(self, eng, dev, ctx, mask, B, L, N):
        cfg = self.config
        ws_now = eng._ws.data_ptr() if eng._ws is not None else None
        key = (B, L, N, mask is not None, str(dev))
        ent = self._graphs.get(key)
        tq_id = id(self._tq_state) if self._tubroquant_config is not None else None
        if ent is not None and (ent["eng"] is not eng or ent["tq"] != tq_id or ent["ws"] != ws_now):
            ent = None
        if ent is None:
            ent = {"ctx": torch.empty_like(ctx), "mask": torch.empty_like(mask) if mask is not None else None,
                   "out": torch.empty(B, cfg.num_quantiles, N * cfg.output_patch_size, dtype=eng.dtype, device=dev),
                   "loc": torch.empty(B, dtype=torch.float32, device=dev),
                   "scale": torch.empty(B, dtype=torch.float32, device=dev)}
            ent["ctx"].copy_(ctx)
            if mask is not None:
                ent["mask"].copy_(mask)
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                # an eager run first: sizes the workspace and sets kernel attributes
                self._native_forward(eng, dev, ent["ctx"], ent["mask"], None, B, L, N, 1, ent["out"], ent["loc"],
                                     ent["scale"])
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    ws = self._native_forward(eng, dev, ent["ctx"], ent["mask"], None, B, L, N, 1, ent["out"],
                                              ent["loc"], ent["scale"])
            torch.cuda.current_stream(dev).wait_stream(s)
            # graphs of other shapes hold the workspace address they were captured with
            ws_addr = eng._ws.data_ptr()
            self._graphs = {k: e for k, e in self._graphs.items() if e["ws"] == ws_addr}
            ent.update(graph=g, eng=eng, ws=ws_addr,
                       tq=id(self._tq_state) if self._tubroquant_config is not None else None)
            self._graphs[key] = ent
        else:
            ent["ctx"].copy_(ctx)
            if mask is not None:
                ent["mask"].copy_(mask)
            ent["graph"].replay()
        self._last_loc = ent["loc"].clone()
        self._last_scale = ent["scale"].clone()
        return ent["out"].clone()

    @classmethod
    def from_pretrained_compiled(cls, model_path: str | Path, compile_mode: str = "reduce-overhead",
                                 adapter_path: str | Path | None = None) -> "CuteChronos2Model":
        """from_pretrained with CUDA-graph replay on (model.py:1065-1084);
        ``compile_mode`` is accepted for the reference's signature."""
        return cls.from_pretrained(model_path, adapter_path=adapter_path).enable_cuda_graphs(True)

    # -- TurboQuant K/V hook (model.py:615-688) ------------------------------------------
    def enable_turboquant_kv(self, bits: int = 4, *, key_mode: str = "prod", value_mode: str = "mse",
                             rotation: str = "hadamard", seed: int = 0,
                             norm_dtype: str = "float16") -> "CuteChronos2Model":
        """Quantise the time-attention K and V vectors of every layer with
        TurboQuant-style quantisers (layer i: key seed ``seed + 2i``, value seed
        ``seed + 2i + 1``); the device kernel runs inside the forward."""
        from .turboquant import TurboQuantParams
        # validate now, as the reference's constructor does
        TurboQuantParams.build(self.config.d_kv, bits, mode=key_mode, rotation=rotation, seed=seed,
                               norm_dtype=norm_dtype, device="cpu")
        TurboQuantParams.build(self.config.d_kv, bits, mode=value_mode, rotation=rotation, seed=seed + 1,
                               norm_dtype=norm_dtype, device="cpu")
        self._tubroquant_config = {"bits": bits, "key_mode": key_mode, "value_mode": value_mode,
                                   "rotation": rotation, "seed": seed, "norm_dtype": norm_dtype}
        self._tq_state = None
        self._tq_last_rows = 0
        return self

    def disable_turboquant_kv(self) -> "CuteChronos2Model":
        """Turn the hook off for every layer."""
        if self._tq_state is not None and self._engine is self._tq_state[0]:
            eng = self._engine
            for l in range(self.config.num_layers):
                nat.check(eng._lib.cc2_model_set_kv_quant(eng.handle, l, None, None, None), "cc2_model_set_kv_quant")
        self._tubroquant_config = None
        self._tq_state = None
        self._tq_last_rows = 0
        return self

    def _turboquant_for(self, eng: "_Engine", dev: torch.device):
        """The hook's device state for this engine (built and registered with the
        native model on first use after enabling or re-packing)."""
        if self._tubroquant_config is None:
            return None
        if self._tq_state is not None and self._tq_state[0] is eng:
            return self._tq_state
        from .turboquant import TurboQuantParams
        c = self._tubroquant_config
        layers = []
        stats = torch.zeros(self.config.num_layers, 4, dtype=torch.float32, device=dev)
        for l in range(self.config.num_layers):
            kq = TurboQuantParams.build(self.config.d_kv, c["bits"], mode=c["key_mode"], rotation=c["rotation"],
                                        seed=c["seed"] + 2 * l, norm_dtype=c["norm_dtype"], device=dev)
            vq = TurboQuantParams.build(self.config.d_kv, c["bits"], mode=c["value_mode"], rotation=c["rotation"],
                                        seed=c["seed"] + 2 * l + 1, norm_dtype=c["norm_dtype"], device=dev)
            kn, vn = kq.native(), vq.native()
            nat.check(eng._lib.cc2_model_set_kv_quant(eng.handle, l, C.byref(kn), C.byref(vn), stats[l].data_ptr()),
                      "cc2_model_set_kv_quant")
            layers.append((kq, vq))
        self._tq_state = (eng, layers, stats)
        return self._tq_state

    def get_tubroquant_summary(self) -> dict[str, Any]:
        """Per-layer statistics of the last forward (model.py:669-688): raw and
        packed bytes of K and V, compression ratio, mean squared and max
        absolute error of the reconstructions."""
        layers: list[dict[str, float]] = []
        if self._tq_state is not None and self._tq_last_rows > 0:
            _, params, stats = self._tq_state
            st = stats.cpu()
            cfg = self.config
            vectors = self._tq_last_rows * cfg.num_heads
            esz = torch.finfo(self._param_dtype()).bits // 8
            for l, (kq, vq) in enumerate(params):
                raw = 2.0 * vectors * cfg.d_kv * esz
                packed = float(vectors * (kq.quantized_bytes_per_vector() + vq.quantized_bytes_per_vector()))
                n = float(vectors * cfg.d_kv)
                layers.append({"layer": float(l), "raw_bytes": raw, "quantized_bytes": packed,
                               "compression_ratio": raw / max(packed, 1.0),
                               "key_mse": float(st[l, 0]) / n, "value_mse": float(st[l, 2]) / n,
                               "key_max_abs_error": float(st[l, 1]), "value_max_abs_error": float(st[l, 3])})
        total_raw = sum(x["raw_bytes"] for x in layers)
        total_q = sum(x["quantized_bytes"] for x in layers)
        return {"enabled": self._tubroquant_config is not None, "config": self._tubroquant_config,
                "layers": layers, "total_raw_bytes": total_raw, "total_quantized_bytes": total_q,
                "compression_ratio": total_raw / max(total_q, 1.0)}

    @torch.inference_mode()
    def predict(self, context: torch.Tensor, context_mask: torch.Tensor | None = None,
                num_output_patches: int = 1) -> torch.Tensor:
        """forward under inference_mode (model.py:1086-1107)."""
        return self.forward(context, context_mask=context_mask, num_output_patches=num_output_patches)

    # -- offload / onload (model.py:597-613) ----------------------------------------------
    def offload_to_cpu(self):
        self.to("cpu")
        self._engine = None
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        self._offloaded = True

    def onload_to_gpu(self, device: str = "cuda"):
        self.to(device)
        self._offloaded = False

    @property
    def is_offloaded(self) -> bool:
        return getattr(self, "_offloaded", False)

    @contextmanager
    def profile_allocations(self):
        """Allocation count and peak memory around a block (model.py:690-736)."""
        stats: dict[str, float] = {}
        dev = self._param_device()
        if dev.type == "cuda":
            torch.cuda.reset_peak_memory_stats(dev)
            torch.cuda.synchronize(dev)
            before = torch.cuda.memory_allocated(dev)
            torch.cuda.reset_accumulated_memory_stats(dev)
            yield stats
            torch.cuda.synchronize(dev)
            after = torch.cuda.memory_allocated(dev)
            st = torch.cuda.memory_stats(dev)
            stats["allocation_count"] = st.get("allocation.all.allocated", 0)
            stats["peak_memory_mb"] = torch.cuda.max_memory_allocated(dev) / 2**20
            stats["allocated_memory_mb"] = after / 2**20
            stats["memory_delta_mb"] = (after - before) / 2**20
        else:
            yield stats
            stats.update(allocation_count=0, peak_memory_mb=0.0, allocated_memory_mb=0.0, memory_delta_mb=0.0)

    # -- weight loading (model.py:833-1062) -------------------------------------------------
    def load_chronos2_weights(self, state_dict: dict[str, torch.Tensor]) -> None:
        """Load a Chronos-2 HuggingFace state dict (key mapping of model.py:833-900)."""
        mapping = {"shared.weight": self.shared.weight,
                   "encoder.final_layer_norm.weight": self.final_layer_norm_weight}
        for name in ("input_patch_embedding", "output_patch_embedding"):
            blk = getattr(self, name)
            for layer in ("hidden_layer", "output_layer", "residual_layer"):
                for prm in ("weight", "bias"):
                    mapping[f"{name}.{layer}.{prm}"] = getattr(getattr(blk, layer), prm)
        for i, b in enumerate(self.blocks):
            pre = f"encoder.block.{i}.layer"
            for j, att in ((0, b.time_attn), (1, b.group_attn)):
                mapping[f"{pre}.{j}.layer_norm.weight"] = att.layer_norm_weight
                for prj in "qkvo":
                    mapping[f"{pre}.{j}.self_attention.{prj}.weight"] = getattr(att, prj).weight
            mapping[f"{pre}.2.layer_norm.weight"] = b.feed_forward.layer_norm_weight
            mapping[f"{pre}.2.mlp.wi.weight"] = b.feed_forward.wi.weight
            mapping[f"{pre}.2.mlp.wo.weight"] = b.feed_forward.wo.weight
        with torch.no_grad():
            for key, prm in mapping.items():
                prm.copy_(state_dict[key])

    def load_lora_adapter(self, adapter_path: str | Path) -> None:
        """Merge a peft LoRA adapter: W += (alpha / r) * B @ A (model.py:902-950)."""
        adapter_path = Path(adapter_path)
        cfg = json.loads((adapter_path / "adapter_config.json").read_text())
        r, alpha = cfg["r"], cfg["lora_alpha"]
        fan_in_fan_out = cfg.get("fan_in_fan_out", False)
        targets = cfg.get("target_modules", ["q", "k", "v", "o"])
        scaling = alpha / r
        st_path, bin_path = adapter_path / "adapter_model.safetensors", adapter_path / "adapter_model.bin"
        if st_path.exists():
            from safetensors.torch import load_file
            sd = load_file(str(st_path))
        elif bin_path.exists():
            sd = torch.load(str(bin_path), map_location="cpu", weights_only=True)
        else:
            raise FileNotFoundError(f"No adapter weights in {adapter_path}")
        merged = 0
        with torch.no_grad():
            for i, b in enumerate(self.blocks):
                for li, att in ((0, b.time_attn), (1, b.group_attn)):
                    for prj in targets:
                        ka = f"base_model.model.encoder.block.{i}.layer.{li}.self_attention.{prj}.lora_A.weight"
                        kb = f"base_model.model.encoder.block.{i}.layer.{li}.self_attention.{prj}.lora_B.weight"
                        if ka not in sd:
                            continue
                        delta = sd[kb] @ sd[ka]
                        if fan_in_fan_out:
                            delta = delta.T
                        prm = getattr(att, prj).weight
                        prm.add_(delta.to(prm.dtype, ).to(prm.device) * scaling)
                        merged += 1
        logger.info("merged %d LoRA adapters (r=%d, alpha=%d)", merged, r, alpha)

    @staticmethod
    def _config_from_json(raw: dict[str, Any]) -> CuteChronos2Config:
        ch = raw.get("chronos_config", {})
        return CuteChronos2Config(
            d_model=raw.get("d_model", 768), d_kv=raw.get("d_kv", 64), d_ff=raw.get("d_ff", 3072),
            num_layers=raw.get("num_layers", 12), num_heads=raw.get("num_heads", 12),
            dropout_rate=raw.get("dropout_rate", 0.1), layer_norm_epsilon=raw.get("layer_norm_epsilon", 1e-6),
            dense_act_fn=raw.get("dense_act_fn", "relu"), rope_theta=raw.get("rope_theta", 10000.0),
            vocab_size=raw.get("vocab_size", 2), reg_token_id=raw.get("reg_token_id", 1),
            context_length=ch.get("context_length", 8192), input_patch_size=ch.get("input_patch_size", 16),
            input_patch_stride=ch.get("input_patch_stride", 16), output_patch_size=ch.get("output_patch_size", 16),
            quantiles=ch.get("quantiles"), use_reg_token=ch.get("use_reg_token", True),
            use_arcsinh=ch.get("use_arcsinh", True), time_encoding_scale=ch.get("time_encoding_scale"),
            max_output_patches=ch.get("max_output_patches", 64))

    @classmethod
    def from_pretrained(cls, model_path: str | Path, adapter_path: str | Path | None = None) -> "CuteChronos2Model":
        """config.json + model.safetensors / pytorch_model.bin (+ optional LoRA) (model.py:952-1021)."""
        model_path = Path(model_path)
        model = cls(cls._config_from_json(json.loads((model_path / "config.json").read_text())))
        st, binp = model_path / "model.safetensors", model_path / "pytorch_model.bin"
        if st.exists():
            from safetensors.torch import load_file
            sd = load_file(str(st))
        elif binp.exists():
            sd = torch.load(str(binp), map_location="cpu", weights_only=True)
        else:
            raise FileNotFoundError(f"No model weights found in {model_path}. "
                                    "Expected model.safetensors or pytorch_model.bin")
        model.load_chronos2_weights(sd)
        if adapter_path is None and (model_path / "adapter_config.json").exists():
            adapter_path = model_path
        if adapter_path is not None:
            model.load_lora_adapter(adapter_path)
        return model.eval()

    @classmethod
    def from_original(cls, original_model) -> "CuteChronos2Model":
        """Copy an upstream Chronos2Model's config and weights (model.py:1023-1062)."""
        oc, cc = original_model.config, original_model.chronos_config
        config = CuteChronos2Config(
            d_model=oc.d_model, d_kv=oc.d_kv, d_ff=oc.d_ff, num_layers=oc.num_layers, num_heads=oc.num_heads,
            dropout_rate=oc.dropout_rate, layer_norm_epsilon=oc.layer_norm_epsilon,
            dense_act_fn=oc.dense_act_fn, rope_theta=oc.rope_theta, vocab_size=oc.vocab_size,
            reg_token_id=getattr(oc, "reg_token_id", 1), context_length=cc.context_length,
            input_patch_size=cc.input_patch_size, input_patch_stride=cc.input_patch_stride,
            output_patch_size=cc.output_patch_size, quantiles=cc.quantiles, use_reg_token=cc.use_reg_token,
            use_arcsinh=cc.use_arcsinh, time_encoding_scale=cc.time_encoding_scale,
            max_output_patches=getattr(cc, "max_output_patches", 64))
        model = cls(config)
        model.load_chronos2_weights(original_model.state_dict())
        return model.eval()

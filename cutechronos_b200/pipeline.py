"""CuteChronos2Pipeline: the reference's pipeline API over the B200 engine.

Mirrors ``cutechronos/pipeline.py`` of lee101/cutedsl:
  * ``_select_quantiles`` (pipeline.py:24-58): gather trained levels, linearly
    interpolate the others;
  * ``_prepare_context`` (pipeline.py:244-322): 1-D / 2-D / 3-D tensors or a
    list of 1-D/2-D items -> flat (sum_variates, L) float32 batch, NaN
    left-padding of ragged rows, group ids (2-D: one group per row; 3-D and
    list items: one group per item), truncation to ``model_context_length``;
  * ``predict`` (327-417), ``predict_quantiles`` (420-474), ``predict_df``
    (476-566) with the same arguments, defaults, chunking rules and return
    types.
The model call is ``CuteChronos2Model.forward`` of this package.
"""

from __future__ import annotations

import logging
import math
import warnings
from pathlib import Path
from typing import Any, List, Optional, Union

import torch

from .model import CuteChronos2Model

logger = logging.getLogger(__name__)


def _select_quantiles(preds: torch.Tensor, training_quantiles: list[float],
                      requested_quantiles: list[float]) -> torch.Tensor:
    """(B, Q_train, H) -> (B, H, len(requested)); exact levels are gathered,
    others interpolated between the neighbouring trained levels."""
    bhq = preds.permute(0, 2, 1)
    index = {q: i for i, q in enumerate(training_quantiles)}
    direct = [index.get(q) for q in requested_quantiles]
    if all(i is not None for i in direct):
        return bhq[..., [int(i) for i in direct]]
    tq = torch.tensor(training_quantiles, dtype=torch.float32)
    cols = []
    for ql, di in zip(requested_quantiles, direct):
        if di is not None:
            cols.append(bhq[..., di])
            continue
        hi = int(torch.searchsorted(tq, torch.tensor(ql, dtype=torch.float32)).clamp(1, len(tq) - 1))
        lo = hi - 1
        frac = (ql - tq[lo].item()) / max(tq[hi].item() - tq[lo].item(), 1e-9)
        cols.append(bhq[..., lo] * (1 - frac) + bhq[..., hi] * frac)
    return torch.stack(cols, dim=-1)


class CuteChronos2Pipeline:
    """Forecasting pipeline over :class:`CuteChronos2Model` (pipeline.py:107-566)."""

    def __init__(self, model: CuteChronos2Model, *, device: str = "cuda", _is_cute: bool = True):
        self.model = model
        self._device = device
        self._is_cute = True

    # -- properties (pipeline.py:128-162) ------------------------------------------
    def _get_config(self):
        return self.model.config

    @property
    def device(self) -> str:
        return self._device

    @property
    def model_context_length(self) -> int:
        return self._get_config().context_length

    @property
    def model_output_patch_size(self) -> int:
        return self._get_config().output_patch_size

    @property
    def max_output_patches(self) -> int:
        return getattr(self._get_config(), "max_output_patches", 64)

    @property
    def model_prediction_length(self) -> int:
        return self.max_output_patches * self._get_config().output_patch_size

    @property
    def quantiles(self) -> list[float]:
        return self._get_config().quantiles

    # -- offload / onload (pipeline.py:165-180) --------------------------------------
    def offload(self):
        self.model.offload_to_cpu()

    def onload(self, device: str | None = None):
        self.model.onload_to_gpu(device or self._device)

    # -- factory (pipeline.py:185-215) ------------------------------------------------
    @classmethod
    def from_pretrained(cls, model_path: str, *, device: str = "cuda", dtype: torch.dtype = torch.bfloat16,
                        use_cute: bool = True, compile_mode: str | None = None) -> "CuteChronos2Pipeline":
        """Load a local Chronos-2 checkpoint directory.  ``compile_mode`` is
        accepted for API compatibility and ignored (the engine has no tracing
        compiler; use CUDA graphs for launch-bound batch sizes)."""
        if not use_cute:
            raise NotImplementedError("use_cute=False (upstream Chronos2Pipeline) is not part of this engine")
        if not Path(model_path).is_dir():
            raise FileNotFoundError(f"{model_path} is not a local checkpoint directory")
        model = CuteChronos2Model.from_pretrained(model_path).to(device=device, dtype=dtype).eval()
        return cls(model, device=device)

    # -- helpers (pipeline.py:221-322) ---------------------------------------------------
    @staticmethod
    def _left_pad_and_stack_rows(rows: List[torch.Tensor]) -> torch.Tensor:
        n = max(r.shape[-1] for r in rows)
        out = torch.full((len(rows), n), float("nan"), dtype=rows[0].dtype, device=rows[0].device)
        for i, r in enumerate(rows):
            if r.shape[-1]:
                out[i, n - r.shape[-1]:] = r
        return out

    @staticmethod
    def _as_tensor(value: Any) -> torch.Tensor:
        return value if isinstance(value, torch.Tensor) else torch.as_tensor(value)

    def _finalize_context_batch(self, context: torch.Tensor) -> torch.Tensor:
        if context.shape[-1] > self.model_context_length:
            context = context[..., -self.model_context_length:]
        return context.to(device=self._device, dtype=torch.float32)

    def _prepare_context(self, context):
        """-> (flat (sum_variates, L) float32 on device, group ids (int64), target index ranges)."""
        if isinstance(context, list):
            rows, gids, ranges = [], [], []
            for gi, item in enumerate(context):
                if isinstance(item, dict):
                    raise NotImplementedError(
                        "Covariate dictionaries are not supported by CuteChronos2Pipeline yet. "
                        "Pass raw targets only or use the upstream Chronos2Pipeline.")
                t = self._as_tensor(item)
                if t.ndim == 1:
                    t = t.unsqueeze(0)
                elif t.ndim != 2:
                    raise ValueError(f"Each list item must be 1-D or 2-D, got shape {tuple(t.shape)}")
                start = len(rows)
                rows.extend(t[i] for i in range(t.shape[0]))
                ranges.append((start, len(rows)))
                gids.extend([gi] * t.shape[0])
            flat = self._finalize_context_batch(self._left_pad_and_stack_rows(rows))
            return flat, torch.tensor(gids, dtype=torch.long), ranges
        t = self._as_tensor(context)
        if t.ndim == 1:
            return self._finalize_context_batch(t.unsqueeze(0)), torch.tensor([0], dtype=torch.long), [(0, 1)]
        if t.ndim == 2:
            batch = self._finalize_context_batch(t)
            return batch, torch.arange(batch.shape[0], dtype=torch.long), [(i, i + 1) for i in range(batch.shape[0])]
        if t.ndim == 3:
            B, V = t.shape[0], t.shape[1]
            flat = self._finalize_context_batch(t.reshape(B * V, t.shape[2]))
            gids = torch.arange(B, dtype=torch.long).repeat_interleave(V)
            return flat, gids, [(b * V, (b + 1) * V) for b in range(B)]
        raise ValueError(f"context must be 1-D, 2-D, or 3-D, got shape {tuple(t.shape)}")

    # -- prediction ----------------------------------------------------------------------
    @torch.inference_mode()
    def predict(self, context: Union[torch.Tensor, List[torch.Tensor]], prediction_length: Optional[int] = None,
                limit_prediction_length: bool = True, cross_learning: bool = False,
                batch_size: Optional[int] = None) -> List[torch.Tensor]:
        """List of (n_variates, Q, prediction_length) float32 CPU tensors, one per task."""
        if self.model.is_offloaded:
            self.model.onload_to_gpu(self._device)
        if prediction_length is None:
            prediction_length = self.model_prediction_length
        if prediction_length > self.model_prediction_length:
            msg = (f"prediction_length ({prediction_length}) exceeds model_prediction_length "
                   f"({self.model_prediction_length}). Quality may degrade.")
            if limit_prediction_length:
                raise ValueError(msg + " Set limit_prediction_length=False to allow this.")
            warnings.warn(msg)
        ctx, gids, ranges = self._prepare_context(context)
        total = ctx.shape[0]
        multivariate = any(e - s > 1 for s, e in ranges)
        N = min(math.ceil(prediction_length / self.model_output_patch_size), self.max_output_patches)

        def run(chunk, chunk_gids):
            g = torch.zeros(chunk.shape[0], dtype=torch.long) if cross_learning else chunk_gids
            return self.model(chunk, num_output_patches=N, group_ids=g)

        if batch_size is not None and batch_size < total:
            if cross_learning or multivariate:
                logger.warning("batch_size chunking disabled for multivariate inputs or cross_learning=True "
                               "(would break group attention semantics)")
                preds = run(ctx, gids)
            else:
                preds = torch.cat([run(ctx[i:i + batch_size], gids[i:i + batch_size])
                                   for i in range(0, total, batch_size)], dim=0)
        else:
            preds = run(ctx, gids)
        preds = preds[..., :prediction_length].to(dtype=torch.float32, device="cpu")
        return [preds[s:e] for s, e in ranges]

    @torch.inference_mode()
    def predict_quantiles(self, context, prediction_length: Optional[int] = None,
                          quantile_levels: Optional[List[float]] = None, limit_prediction_length: bool = True,
                          cross_learning: bool = False, batch_size: Optional[int] = None):
        """(quantiles: list of (V, H, len(levels)), mean: list of (V, H)); mean is the median."""
        if quantile_levels is None:
            quantile_levels = [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9]
        preds = self.predict(context, prediction_length=prediction_length,
                             limit_prediction_length=limit_prediction_length, cross_learning=cross_learning,
                             batch_size=batch_size)
        tq = self.quantiles
        quantiles = [_select_quantiles(p, tq, quantile_levels) for p in preds]
        mi = tq.index(0.5)
        mean = [p.permute(0, 2, 1)[..., mi] for p in preds]
        return quantiles, mean

    def predict_df(self, df, future_df=None, id_column: str = "item_id", timestamp_column: str = "timestamp",
                   target: str = "target", prediction_length: Optional[int] = None,
                   quantile_levels: Optional[List[float]] = None, batch_size: int = 256,
                   cross_learning: bool = False, **kwargs):
        """Long-format DataFrame in, DataFrame (id, step, one column per level) out."""
        import pandas as pd

        if future_df is not None:
            raise NotImplementedError("future_df (future covariates) is not supported by CuteChronos2Pipeline. "
                                      "Pass future_df=None or use the upstream Chronos2Pipeline.")
        if prediction_length is None:
            prediction_length = self.model_prediction_length
        if quantile_levels is None:
            quantile_levels = list(self.quantiles)
        groups = df.sort_values(timestamp_column).groupby(id_column, sort=False)
        ids = list(groups.groups.keys())
        tensors = [torch.tensor(g[target].values, dtype=torch.float32) for _, g in groups]
        preds = self.predict(tensors, prediction_length=prediction_length, cross_learning=cross_learning,
                             batch_size=batch_size, limit_prediction_length=False, **kwargs)
        allp = torch.cat(preds, dim=0)
        H = allp.shape[-1]
        sel = _select_quantiles(allp, self.quantiles, quantile_levels)
        out = {id_column: [i for i in ids for _ in range(H)], "step": list(range(H)) * len(ids)}
        flat = sel.reshape(len(ids) * H, len(quantile_levels))
        for qi, ql in enumerate(quantile_levels):
            out[str(ql)] = flat[:, qi].tolist()
        return pd.DataFrame(out)

"""CuteChronos2Pipeline: the reference's pipeline API over the B200 engine.

Mirrors ``cutechronos/pipeline.py`` of lee101/cutedsl:
  * ``_select_quantiles`` (pipeline.py:24-58): gather trained levels, linearly
    interpolate the others -- here one kernel on the device
    (``kernels.select_quantiles``) that also gathers the median;
  * ``_prepare_context`` (pipeline.py:244-322): 1-D / 2-D / 3-D tensors or a
    list of 1-D/2-D items -> flat (sum_variates, L) float32 batch, NaN
    left-padding of ragged rows, group ids (2-D: one group per row; 3-D and
    list items: one group per item), truncation to ``model_context_length``
    -- here ragged rows travel as one pinned buffer plus offsets and are
    stacked by a kernel (``kernels.stack_series``);
  * ``predict`` (327-417), ``predict_quantiles`` (420-474), ``predict_df``
    (476-566) with the same arguments, defaults, chunking rules and return
    types.
The model call is ``CuteChronos2Model.forward`` of this package.  Each call
makes one host-to-device copy of its inputs and one device-to-host copy of its
results, both through pinned memory.
"""

from __future__ import annotations

import logging
import math
import warnings
from dataclasses import dataclass
from pathlib import Path
from typing import Any, List, Optional, Union

import numpy as np
import torch

from . import kernels
from .model import CuteChronos2Model

logger = logging.getLogger(__name__)


def _select_quantiles(preds: torch.Tensor, training_quantiles: list[float],
                      requested_quantiles: list[float]) -> torch.Tensor:
    """(B, Q_train, H) -> (B, H, len(requested)) on preds' device: trained
    levels gathered, others interpolated between the neighbouring trained
    levels (pipeline.py:24-58); CPU tensors make a round trip to the GPU."""
    dev = preds if preds.is_cuda else preds.to("cuda")
    out = kernels.select_quantiles(dev, dev.shape[-1], training_quantiles, requested_quantiles, layout=1)
    return out if preds.is_cuda else out.cpu()


@dataclass
class _Ragged:
    """Univariate series concatenated in one 1-D float32 CPU tensor, one
    length per series (the packed form predict_df builds from a DataFrame)."""
    values: torch.Tensor
    lens: List[int]


def _group_series(df, id_column: str, timestamp_column: str, target: str):
    """``df.sort_values(ts).groupby(id, sort=False)`` of predict_df
    (pipeline.py:535-537), vectorised: ids in order of first appearance in the
    time-sorted frame, each series' values in time order, rows with a missing
    id dropped.  -> (ids, _Ragged)."""
    import pandas as pd
    sdf = df.sort_values(timestamp_column)
    codes, uniques = pd.factorize(sdf[id_column], sort=False)
    keep = codes >= 0
    codes = codes[keep]
    order = np.argsort(codes, kind="stable")
    values = sdf[target].to_numpy(dtype=np.float32)[keep][order]
    lens = np.bincount(codes, minlength=len(uniques)).tolist()
    return list(uniques), _Ragged(torch.from_numpy(np.ascontiguousarray(values)), lens)


def _to_host(t: torch.Tensor) -> torch.Tensor:
    """One asynchronous copy into pinned memory, then a wait on the stream."""
    host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    host.copy_(t, non_blocking=True)
    torch.cuda.current_stream(t.device).synchronize()
    return host


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
        """Load a local Chronos-2 checkpoint directory.  A ``compile_mode``
        (the reference's torch.compile mode, e.g. "reduce-overhead") turns on
        CUDA-graph replay of the forward per input shape; there is no tracing
        compiler."""
        if not use_cute:
            raise NotImplementedError("use_cute=False (upstream Chronos2Pipeline) is not part of this engine")
        if not Path(model_path).is_dir():
            raise FileNotFoundError(f"{model_path} is not a local checkpoint directory")
        model = CuteChronos2Model.from_pretrained(model_path).to(device=device, dtype=dtype).eval()
        if compile_mode:
            model.enable_cuda_graphs(True)
        return cls(model, device=device)

    # -- helpers (pipeline.py:221-322) ---------------------------------------------------
    def _upload_rows(self, rows) -> torch.Tensor:
        """1-D series (a list, or a :class:`_Ragged`) -> (B, L) float32 on the
        device, NaN-left-padded, truncated to model_context_length
        (pipeline.py:221-243): the rows are packed on the host into one pinned
        buffer, copied once with their offsets, and stacked by a kernel."""
        if isinstance(rows, _Ragged):
            lens, pieces = rows.lens, [rows.values]
        else:
            lens, pieces = [int(r.shape[-1]) for r in rows], rows
        if not lens:
            raise ValueError("context holds no series")
        L = min(max(lens), self.model_context_length)
        if L == 0:
            raise ValueError("context holds no time steps")
        total = sum(lens)
        t8 = total + (total & 1)  # the int64 offsets start 8-byte aligned
        host = torch.empty(t8 + 2 * (len(lens) + 1), dtype=torch.float32, pin_memory=True)
        torch.cat([r.reshape(-1).to("cpu", torch.float32) for r in pieces], out=host[:total])
        offs = host[t8:].view(torch.int64)
        offs[0] = 0
        torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0, out=offs[1:])
        dev = host.to(self._device, non_blocking=True)
        return kernels.stack_series(dev[:total], dev[t8:].view(torch.int64), L)

    @staticmethod
    def _as_tensor(value: Any) -> torch.Tensor:
        return value if isinstance(value, torch.Tensor) else torch.as_tensor(value)

    def _finalize_context_batch(self, context: torch.Tensor) -> torch.Tensor:
        """Keep the last model_context_length steps (a view; no copy)."""
        if context.shape[-1] > self.model_context_length:
            context = context[..., -self.model_context_length:]
        return context

    def _upload_batch(self, context: torch.Tensor) -> torch.Tensor:
        """(B, L) batch -> float32 on the device, through one pinned buffer."""
        if context.is_cuda:
            return context.to(device=self._device, dtype=torch.float32)
        host = torch.empty(context.shape, dtype=torch.float32, pin_memory=True)
        host.copy_(context)
        return host.to(self._device, non_blocking=True)

    def _plan_context(self, context):
        """Host half of ``_prepare_context`` (pipeline.py:244-322): ->
        (rows, gids, ranges) where ``rows`` is a list of 1-D series (ragged
        input: list items) or a (B, L) tensor already cut to
        model_context_length (1-D / 2-D / 3-D input)."""
        if isinstance(context, _Ragged):
            n = len(context.lens)
            return context, torch.arange(n, dtype=torch.long), [(i, i + 1) for i in range(n)]
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
            return rows, torch.tensor(gids, dtype=torch.long), ranges
        t = self._as_tensor(context)
        if t.ndim == 1:
            return self._finalize_context_batch(t.unsqueeze(0)), torch.tensor([0], dtype=torch.long), [(0, 1)]
        if t.ndim == 2:
            return (self._finalize_context_batch(t), torch.arange(t.shape[0], dtype=torch.long),
                    [(i, i + 1) for i in range(t.shape[0])])
        if t.ndim == 3:
            B, V = t.shape[0], t.shape[1]
            gids = torch.arange(B, dtype=torch.long).repeat_interleave(V)
            return (self._finalize_context_batch(t.reshape(B * V, t.shape[2])), gids,
                    [(b * V, (b + 1) * V) for b in range(B)])
        raise ValueError(f"context must be 1-D, 2-D, or 3-D, got shape {tuple(t.shape)}")

    def _prepare_context(self, context):
        """-> (flat (sum_variates, L) float32 on device, group ids (int64), target index ranges)."""
        rows, gids, ranges = self._plan_context(context)
        batch = self._upload_rows(rows) if isinstance(rows, (list, _Ragged)) else self._upload_batch(rows)
        return batch, gids, ranges

    # -- prediction ----------------------------------------------------------------------
    @torch.inference_mode()
    def predict(self, context: Union[torch.Tensor, List[torch.Tensor]], prediction_length: Optional[int] = None,
                limit_prediction_length: bool = True, cross_learning: bool = False,
                batch_size: Optional[int] = None) -> List[torch.Tensor]:
        """List of (n_variates, Q, prediction_length) float32 CPU tensors, one per task."""
        if self.model.is_offloaded:
            self.model.onload_to_gpu(self._device)
        prediction_length = self._check_horizon(prediction_length, limit_prediction_length)
        preds, ranges = self._forecast(context, prediction_length, cross_learning, batch_size)
        H = min(prediction_length, preds.shape[-1])  # N is clamped to max_output_patches
        out = kernels.select_quantiles(preds, H, self.quantiles, self.quantiles, layout=0)
        host = _to_host(out)
        return [host[s:e] for s, e in ranges]

    def _forecast(self, context, prediction_length: int, cross_learning: bool, batch_size: Optional[int]):
        """(B, Q, 16N) forecasts on the device, in the model dtype, + task ranges."""
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
        return preds, ranges

    def _check_horizon(self, prediction_length: Optional[int], limit_prediction_length: bool) -> int:
        if prediction_length is None:
            prediction_length = self.model_prediction_length
        if prediction_length > self.model_prediction_length:
            msg = (f"prediction_length ({prediction_length}) exceeds model_prediction_length "
                   f"({self.model_prediction_length}). Quality may degrade.")
            if limit_prediction_length:
                raise ValueError(msg + " Set limit_prediction_length=False to allow this.")
            warnings.warn(msg)
        return prediction_length

    @torch.inference_mode()
    def predict_quantiles(self, context, prediction_length: Optional[int] = None,
                          quantile_levels: Optional[List[float]] = None, limit_prediction_length: bool = True,
                          cross_learning: bool = False, batch_size: Optional[int] = None):
        """(quantiles: list of (V, H, len(levels)), mean: list of (V, H)); mean is the median."""
        if quantile_levels is None:
            quantile_levels = [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9]
        if self.model.is_offloaded:
            self.model.onload_to_gpu(self._device)
        H = self._check_horizon(prediction_length, limit_prediction_length)
        preds, ranges = self._forecast(context, H, cross_learning, batch_size)
        H = min(H, preds.shape[-1])
        tq = self.quantiles
        B = preds.shape[0]
        buf = torch.empty(B * H * (len(quantile_levels) + 1), dtype=torch.float32, device=preds.device)
        kernels.select_quantiles(preds, H, tq, quantile_levels, layout=1, median_level=tq.index(0.5), out=buf)
        host = _to_host(buf)
        nq = len(quantile_levels)
        q_all = host[:B * H * nq].view(B, H, nq)
        m_all = host[B * H * nq:].view(B, H)
        return [q_all[s:e] for s, e in ranges], [m_all[s:e] for s, e in ranges]

    @torch.inference_mode()
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
        ids, tensors = _group_series(df, id_column, timestamp_column, target)
        if self.model.is_offloaded:
            self.model.onload_to_gpu(self._device)
        H = self._check_horizon(prediction_length, False)
        preds, _ = self._forecast(tensors, H, cross_learning, batch_size)
        H = min(H, preds.shape[-1])  # may be < prediction_length when N is clamped
        sel = _to_host(kernels.select_quantiles(preds, H, self.quantiles, quantile_levels, layout=1)).numpy()
        out = {id_column: pd.Index(ids).repeat(H), "step": np.tile(np.arange(H), len(ids))}
        flat = sel.reshape(len(ids) * H, len(quantile_levels)).astype(np.float64)
        for qi, ql in enumerate(quantile_levels):
            out[str(ql)] = flat[:, qi]
        return pd.DataFrame(out)

"""Handle-based forecasting API for non-Python hosts (mirror of
cutechronos/foreign.py:1-190 of lee101/cutedsl).

Two routes to the same engine:

- the functions of this module (``init_pipeline``, ``predict_median``,
  ``predict_quantile``, ``destroy_pipeline``) keep a registry of
  :class:`CuteChronos2Pipeline` objects, as the reference module does for the
  C bridge that embeds CPython;
- :class:`NativeBridge` calls the native C bridge (``include/cutechronos_bridge.h``,
  exported by the engine's shared library), which loads the checkpoint and runs
  the forward without Python.  It is what a C, Go or ctypes host binds.
"""

from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass
from typing import Any

import torch

from .pipeline import CuteChronos2Pipeline

_DTYPE_MAP = {"float32": torch.float32, "bfloat16": torch.bfloat16}


@dataclass
class _PipelineSession:
    backend: str
    device: str
    dtype_name: str
    pipeline: Any


_PIPELINES: dict[int, _PipelineSession] = {}
_NEXT_HANDLE = 1


def _resolve_dtype(dtype_name: str) -> torch.dtype:
    try:
        return _DTYPE_MAP[dtype_name]
    except KeyError as exc:
        raise ValueError(f"Unsupported dtype '{dtype_name}'. Expected one of {sorted(_DTYPE_MAP)}") from exc


def _resolve_device(device: str | None) -> str:
    return device if device else "cuda"


def init_pipeline(model_id: str, backend: str = "cute", device: str | None = None, dtype_name: str = "bfloat16",
                  compile_mode: str | None = None) -> int:
    """Load a pipeline and return a numeric handle (foreign.py:85-123)."""
    global _NEXT_HANDLE
    device = _resolve_device(device)
    dtype = _resolve_dtype(dtype_name)
    if backend != "cute":
        raise ValueError(f"Unsupported backend '{backend}'. Expected 'cute'.")
    pipeline = CuteChronos2Pipeline.from_pretrained(model_id, device=device, dtype=dtype, use_cute=True,
                                                    compile_mode=compile_mode)
    handle = _NEXT_HANDLE
    _NEXT_HANDLE += 1
    _PIPELINES[handle] = _PipelineSession(backend=backend, device=device, dtype_name=dtype_name, pipeline=pipeline)
    return handle


def destroy_pipeline(handle: int) -> bool:
    """Remove a handle; its weights leave the device (foreign.py:126-143)."""
    session = _PIPELINES.pop(handle, None)
    if session is None:
        return False
    try:
        session.pipeline.offload()
    except Exception:
        pass
    return True


def predict_median(handle: int, context_values: list[float], prediction_length: int) -> tuple[list[float], float]:
    """``(forecast, latency_ms)`` of the 0.5 quantile (foreign.py:146-152)."""
    return predict_quantile(handle, context_values, prediction_length, 0.5)


def predict_quantile(handle: int, context_values: list[float], prediction_length: int,
                     quantile_level: float) -> tuple[list[float], float]:
    """``(forecast, latency_ms)`` of one quantile level (foreign.py:155-186)."""
    session = _PIPELINES[handle]
    context = torch.tensor(context_values, dtype=torch.float32)
    torch.cuda.synchronize()
    start = time.perf_counter()
    quantiles, _ = session.pipeline.predict_quantiles(context, prediction_length=prediction_length,
                                                      quantile_levels=[quantile_level])
    forecast = quantiles[0][0, :, 0]
    torch.cuda.synchronize()
    return forecast.tolist(), (time.perf_counter() - start) * 1000.0


def available_backends() -> list[str]:
    return ["cute"]


class BridgeError(RuntimeError):
    pass


class NativeBridge:
    """ctypes binding of the native C bridge; the same calls a C or Go host
    makes (examples of the reference: python/ctypes_runner.py)."""

    def __init__(self, lib: C.CDLL | None = None):
        if lib is None:
            from . import _native
            lib = _native.load()
        self._lib = lib
        lib.cutechronos_init_pipeline.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, C.c_char_p, C.c_char_p,
                                                  C.POINTER(C.c_int), C.c_char_p, C.c_size_t]
        lib.cutechronos_predict_median.argtypes = [C.c_int, C.POINTER(C.c_float), C.c_int, C.c_int,
                                                   C.POINTER(C.c_float), C.c_int, C.POINTER(C.c_int),
                                                   C.POINTER(C.c_double), C.c_char_p, C.c_size_t]
        lib.cutechronos_destroy_pipeline.argtypes = [C.c_int, C.c_char_p, C.c_size_t]
        for f in (lib.cutechronos_init_pipeline, lib.cutechronos_predict_median, lib.cutechronos_destroy_pipeline):
            f.restype = C.c_int

    @staticmethod
    def _enc(s: str | None) -> bytes | None:
        return None if s is None else s.encode()

    def init_pipeline(self, model_id: str, backend: str | None = "cute", device: str | None = None,
                      dtype_name: str | None = "bfloat16", compile_mode: str | None = None) -> int:
        err = C.create_string_buffer(4096)
        h = C.c_int(-1)
        st = self._lib.cutechronos_init_pipeline(self._enc(model_id), self._enc(backend), self._enc(device),
                                                 self._enc(dtype_name), self._enc(compile_mode), C.byref(h), err,
                                                 len(err))
        if st != 0:
            raise BridgeError(err.value.decode(errors="replace"))
        return h.value

    def predict_median(self, handle: int, context_values, prediction_length: int,
                       capacity: int | None = None) -> tuple[list[float], float]:
        ctx = (C.c_float * len(context_values))(*[float(v) for v in context_values])
        cap = prediction_length if capacity is None else capacity
        out = (C.c_float * max(cap, 1))()
        n, ms = C.c_int(0), C.c_double(0.0)
        err = C.create_string_buffer(4096)
        st = self._lib.cutechronos_predict_median(handle, ctx, len(context_values), prediction_length, out, cap,
                                                  C.byref(n), C.byref(ms), err, len(err))
        if st != 0:
            raise BridgeError(err.value.decode(errors="replace"))
        return list(out[:n.value]), ms.value

    def destroy_pipeline(self, handle: int) -> None:
        err = C.create_string_buffer(4096)
        if self._lib.cutechronos_destroy_pipeline(handle, err, len(err)) != 0:
            raise BridgeError(err.value.decode(errors="replace"))

"""ctypes bindings of the C ABI in ``include/cc2.h`` (``_lib/libcc2_b200.so``).

The library is the only compute path of this package: if it is missing or
fails to load, every entry point raises.  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libcc2_b200.so"

CC2_F32, CC2_BF16 = 0, 1
EPI_ROWSCALE, EPI_BIAS, EPI_RELU, EPI_RESID, EPI_SSQ, EPI_SPECIAL, EPI_ROPE, EPI_LO = 1, 2, 4, 8, 16, 32, 64, 128

EXPORTED = (
    "cc2_last_error", "cc2_version", "cc2_device_status", "cc2_model_pack_bytes", "cc2_model_create",
    "cc2_model_destroy", "cc2_group_layout", "cc2_forward_workspace_bytes", "cc2_forward",
    "cc2_preprocess", "cc2_gemm", "cc2_rmsnorm_rows", "cc2_attention", "cc2_output_transform",
    "cc2_profile_begin", "cc2_profile_read", "cc2_set_gemm_variant", "cc2_forward_noalloc",
    "cc2_stack_series", "cc2_select_quantiles", "cc2_set_attention_variant",
    "cc2_set_attention_trace", "cc2_set_gemm_trace", "cc2_kv_quant", "cc2_model_set_kv_quant",
    "cc2_set_launch_overlap", "cc2_test_starve_gemm", "cc2_group_attention_tc", "cc2_set_layer_chain",
    "cc2_test_starve_layer_barrier", "cc2_set_layer_trace",
)
KIND_NAMES = {1: "preprocess", 2: "gemm_tc", 3: "attn_time", 4: "attn_group", 5: "rmsnorm", 6: "output_transform",
              7: "gemm_qkv", 8: "gemm_o", 9: "gemm_group", 10: "gemm_ffn_up", 11: "gemm_ffn_down", 12: "gemm_io",
              13: "layers"}
GEMM_KINDS = (2, 7, 8, 9, 10, 11, 12)


class Config(C.Structure):
    _fields_ = [
        ("d_model", C.c_int), ("d_kv", C.c_int), ("d_ff", C.c_int), ("num_layers", C.c_int),
        ("num_heads", C.c_int), ("layer_norm_epsilon", C.c_float), ("rope_theta", C.c_float),
        ("reg_token_id", C.c_int), ("context_length", C.c_int), ("input_patch_size", C.c_int),
        ("output_patch_size", C.c_int), ("num_quantiles", C.c_int), ("use_reg_token", C.c_int),
        ("use_arcsinh", C.c_int), ("time_encoding_scale", C.c_float), ("max_output_patches", C.c_int),
    ]


_VP = C.c_void_p
_PP = C.POINTER(C.c_void_p)


class Weights(C.Structure):
    _fields_ = [
        ("shared", _VP),
        ("in_hidden_w", _VP), ("in_hidden_b", _VP), ("in_output_w", _VP), ("in_output_b", _VP),
        ("in_residual_w", _VP), ("in_residual_b", _VP),
        ("time_ln", _PP), ("time_q", _PP), ("time_k", _PP), ("time_v", _PP), ("time_o", _PP),
        ("group_ln", _PP), ("group_q", _PP), ("group_k", _PP), ("group_v", _PP), ("group_o", _PP),
        ("ff_ln", _PP), ("ff_wi", _PP), ("ff_wo", _PP),
        ("final_ln", _VP),
        ("out_hidden_w", _VP), ("out_hidden_b", _VP), ("out_output_w", _VP), ("out_output_b", _VP),
        ("out_residual_w", _VP), ("out_residual_b", _VP),
    ]


class Epilogue(C.Structure):
    _fields_ = [
        ("flags", C.c_int), ("ssq_in", _VP), ("norm_dim", C.c_int), ("eps", C.c_float),
        ("bias", _VP), ("resid", _VP), ("ld_resid", C.c_int), ("ssq_out", _VP), ("ssq_ld", C.c_int),
        ("special", _VP), ("special_period", C.c_int), ("special_offset", C.c_int),
        ("rope_cs", _VP), ("rope_period", C.c_int), ("rope_cols", C.c_int),
        ("lo_out", _VP), ("resid_lo", _VP), ("ld_lo", C.c_int),
    ]


class NativeError(RuntimeError):
    pass


_lib = None


def load(path: Path | str | None = None) -> C.CDLL:
    """Load (once) and return the native library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise NativeError(
            f"native library {p} not found; build it with `python -m cutechronos_b200.build` "
            "(there is no CPU fallback)")
    lib = C.CDLL(str(p))
    i, f, v, sz = C.c_int, C.c_float, C.c_void_p, C.c_size_t
    lib.cc2_last_error.restype = C.c_char_p
    lib.cc2_version.restype = C.c_char_p
    lib.cc2_device_status.argtypes = [i]
    lib.cc2_model_pack_bytes.argtypes = [C.POINTER(Config), i, C.POINTER(sz)]
    lib.cc2_model_create.argtypes = [C.POINTER(Config), i, C.POINTER(Weights), v, sz, v, C.POINTER(v)]
    lib.cc2_model_destroy.argtypes = [v]
    lib.cc2_group_layout.argtypes = [v, i, v, v, C.POINTER(i), C.POINTER(i)]
    lib.cc2_forward_workspace_bytes.argtypes = [v, i, i, i, i, C.POINTER(sz)]
    lib.cc2_forward.argtypes = [v, v, v, i, i, i, v, v, v, v, v, sz, v]
    lib.cc2_preprocess.argtypes = [v, v, i, i, i, i, f, i, i, i, i, v, i, i, v, v, v, v, v]
    lib.cc2_gemm.argtypes = [i, v, i, v, i, v, i, i, i, i, C.POINTER(Epilogue), v]
    lib.cc2_rmsnorm_rows.argtypes = [i, v, i, v, v, i, i, i, i, i, i, f, v]
    lib.cc2_attention.argtypes = [i, i, v, i, i, i, i, v, i, v, i, i, i, i, v, v, i, i, v, v]
    lib.cc2_output_transform.argtypes = [i, v, i, v, v, v, i, i, i, i, i, v]
    lib.cc2_profile_begin.argtypes = [i]
    lib.cc2_set_gemm_variant.argtypes = [i]
    lib.cc2_set_attention_variant.argtypes = [i]
    lib.cc2_set_attention_trace.argtypes = [v]
    lib.cc2_set_gemm_trace.argtypes = [v]
    lib.cc2_kv_quant.argtypes = [i, v, i, i, i, i, i, i, v, v, v, i, v, v]
    lib.cc2_model_set_kv_quant.argtypes = [v, i, v, v, v]
    lib.cc2_set_launch_overlap.argtypes = [i]
    lib.cc2_test_starve_gemm.argtypes = [i]
    lib.cc2_set_layer_chain.argtypes = [i]
    lib.cc2_test_starve_layer_barrier.argtypes = [i]
    lib.cc2_set_layer_trace.argtypes = [v]
    lib.cc2_group_attention_tc.argtypes = [v, i, i, i, i, v, i, v, i, i, i, i, v]
    lib.cc2_forward_noalloc.argtypes = [v, v, v, i, i, i, v, v, v, v, v]
    lib.cc2_profile_read.argtypes = [v, v, v, v, i, C.POINTER(i)]
    lib.cc2_stack_series.argtypes = [v, v, i, i, v, v]
    lib.cc2_select_quantiles.argtypes = [i, v, i, i, i, i, i, v, v, v, v, i, v, i, v, v]
    for name in EXPORTED:
        getattr(lib, name)  # every declared symbol must resolve
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().cc2_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed with status {status}: {msg}")

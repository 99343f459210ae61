"""The C-ABI library without a GPU: it loads, exports every entry point that
include/cc2.h declares, and its host-side logic (config validation, weight
pack sizing, group layout, argument checks) behaves as documented.  Nothing
here launches a kernel."""

import ctypes as C
import re
from pathlib import Path

import pytest
import torch

from cutechronos_b200 import _native as nat
from cutechronos_b200.model import CuteChronos2Config

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    if not nat.LIB_PATH.exists():
        from cutechronos_b200 import build
        build.build()
    return nat.load()


def declared_symbols():
    text = (ROOT / "include" / "cc2.h").read_text()
    return sorted(set(re.findall(r"CC2_API\s+[\w\s\*]+?\b(cc2_\w+)\s*\(", text)))


def test_header_declares_and_library_exports_everything(lib):
    names = declared_symbols()
    assert len(names) >= 17
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(nat.EXPORTED)


def test_version_and_error_strings(lib):
    assert b"sm_100a" in lib.cc2_version()
    st = lib.cc2_forward(None, None, None, 1, 1, 1, None, None, None, None, None, 0, None)
    assert st == -1 and b"null" in lib.cc2_last_error()


def _cfg(**kw):
    c = CuteChronos2Config(**kw)
    return c.to_native()


def test_pack_bytes_base_model(lib):
    n = C.c_size_t()
    assert lib.cc2_model_pack_bytes(C.byref(_cfg()), nat.CC2_BF16, C.byref(n)) == 0
    # 119,477,664 bf16 parameters
    # + the fused Wo.Wv group matrices, fp32 biases, RoPE table and packing scratch
    assert 2 * 119_477_664 <= n.value <= 2 * 119_477_664 + 32 * 2**20
    n32 = C.c_size_t()
    assert lib.cc2_model_pack_bytes(C.byref(_cfg()), nat.CC2_F32, C.byref(n32)) == 0
    assert n32.value > 1.9 * n.value


@pytest.mark.parametrize("kw,msg", [(dict(d_kv=32, num_heads=24), b"d_kv"), (dict(d_model=100, num_heads=1, d_kv=64), b"num_heads"),
                                    (dict(output_patch_size=8), b"patch")])
def test_pack_bytes_rejects_unsupported_configs(lib, kw, msg):
    n = C.c_size_t()
    assert lib.cc2_model_pack_bytes(C.byref(_cfg(**kw)), nat.CC2_BF16, C.byref(n)) == -1
    assert msg in lib.cc2_last_error()


def test_group_layout(lib):
    gid = torch.tensor([7, 3, 7, 7, 1, 3], dtype=torch.int64)
    mem = (C.c_int32 * 6)()
    off = (C.c_int32 * 7)()
    ng, mg = C.c_int(), C.c_int()
    assert lib.cc2_group_layout(gid.data_ptr(), 6, mem, off, C.byref(ng), C.byref(mg)) == 0
    assert ng.value == 3 and mg.value == 3
    assert list(mem) == [0, 2, 3, 1, 5, 4]          # groups by first appearance, order kept
    assert list(off)[:4] == [0, 3, 5, 6]


@pytest.mark.parametrize("args", [
    (1, None, 768, None, 768, None, 768, 0, 768, 768),    # M = 0
    (1, None, 768, None, 768, None, 768, 10, 768, 768),   # null operands
    (7, None, 768, None, 768, None, 768, 10, 768, 768),   # bad dtype
])
def test_gemm_argument_checks(lib, args):
    dt, A, lda, W, ldw, out, ldo, M, N, K = args
    st = lib.cc2_gemm(dt, A, lda, W, ldw, out, ldo, M, N, K, None, None)
    assert st == -1 and lib.cc2_last_error()


def test_forward_noalloc_argument_checks(lib):
    assert lib.cc2_forward_noalloc(None, None, None, 1, 16, 1, None, None, None, None, None) == -1

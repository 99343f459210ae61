"""cc2_forward_noalloc: the forward for callers that cannot allocate device
memory themselves (foreign-language front ends without a device allocator,
serving loops that must not stall on a synchronising cudaMalloc).  It runs the
same forward as cc2_forward with its scratch in the library's static device
array, so its forecasts must match cc2_forward's on the same inputs, call
after call, and requests larger than the array must be refused.

This file is collected last on purpose: a run that stops at the first failure
has already run every other test.  It also passes alone in a fresh process.
"""

import ctypes as C

import pytest
import torch

from cutechronos_b200 import _native as nat
from cutechronos_b200.model import CuteChronos2Config, CuteChronos2Model
from cutechronos_b200.workloads import seeded_init_, series_cfg1

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def model():
    return seeded_init_(CuteChronos2Model(CuteChronos2Config()), seed=0).to(DEV, torch.bfloat16).eval()


@pytest.fixture(scope="module")
def model_f32():
    return seeded_init_(CuteChronos2Model(CuteChronos2Config()), seed=0).to(DEV, torch.float32).eval()


def _forward_with_workspace(eng, ctx, N):
    """Existing entry point cc2_forward through the C ABI, caller-owned workspace."""
    B, L = ctx.shape
    out = torch.empty(B, 21, 16 * N, dtype=eng.dtype, device=DEV)
    ws, ws_bytes = eng.workspace(B, L, N, 1)
    st = torch.cuda.current_stream().cuda_stream
    nat.check(eng._lib.cc2_forward(eng.handle, ctx.data_ptr(), None, B, L, N, None, out.data_ptr(), None, None,
                                   ws, ws_bytes, st), "cc2_forward")
    return out


def _forward_noalloc(eng, ctx, N):
    B, L = ctx.shape
    out = torch.empty(B, 21, 16 * N, dtype=eng.dtype, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    nat.check(eng._lib.cc2_forward_noalloc(eng.handle, ctx.data_ptr(), None, B, L, N, None, out.data_ptr(), None,
                                           None, st), "cc2_forward_noalloc")
    return out


@pytest.mark.parametrize("which", ["bf16", "f32"])
def test_noalloc_matches_forward_on_two_calls_in_a_row(model, model_f32, which):
    # the forward has no atomics and a fixed reduction order, so the two entry
    # points must agree bit for bit
    eng = (model if which == "bf16" else model_f32).engine()
    a = series_cfg1(4, 2048, 11).to(DEV)
    b = series_cfg1(3, 512, 12).to(DEV)
    ya = _forward_noalloc(eng, a, 4)   # first call on this device sets the scratch address up
    yb = _forward_noalloc(eng, b, 2)   # second call reuses the same scratch with another shape
    torch.cuda.synchronize()
    ra = _forward_with_workspace(eng, a, 4)
    rb = _forward_with_workspace(eng, b, 2)
    torch.cuda.synchronize()
    assert torch.isfinite(ya.float()).all() and torch.isfinite(yb.float()).all()
    assert torch.equal(ya, ra)
    assert torch.equal(yb, rb)


def test_noalloc_refuses_requests_beyond_the_static_scratch(model):
    eng = model.engine()
    B, L, N = 64, 2048, 4  # about 8,500 token rows: more than the array holds
    need = C.c_size_t()
    nat.check(eng._lib.cc2_forward_workspace_bytes(eng.handle, B, L, N, 1, C.byref(need)), "workspace_bytes")
    assert need.value > (32 << 20)
    ctx = torch.zeros(B, L, device=DEV)
    out = torch.empty(B, 21, 64, dtype=torch.bfloat16, device=DEV)
    st = eng._lib.cc2_forward_noalloc(eng.handle, ctx.data_ptr(), None, B, L, N, None, out.data_ptr(), None, None,
                                      torch.cuda.current_stream().cuda_stream)
    assert st == -4  # CC2_E_WORKSPACE
    assert b"scratch" in eng._lib.cc2_last_error()

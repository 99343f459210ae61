"""Failure path of the bounded waits, exercised without a GPU fault.

Every mbarrier wait in the tcgen05 kernels gives up after 2 s, raises the
device error word, leaves its loops, frees TMEM and returns.  The test hook
cc2_test_starve_gemm makes a single-SM GEMM withhold one stage's load, so the
MMA warp's wait on it runs out: no trap, no bad address, nothing left in
flight.  The test checks that the launch returns, that cc2_device_status
reports the timeout, that the model's opt-in device check raises, and that
the next GEMM and forward are correct again.
"""

import pytest
import torch

from cutechronos_b200 import _native as nat
from cutechronos_b200 import kernels as K
from cutechronos_b200.model import CuteChronos2Model
from conftest import small_config
from cutechronos_b200.workloads import seeded_init_

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ref(x, w):
    return (x.float() @ w.float().t())


def test_gemm_wait_timeout_sets_status_and_recovers():
    lib = nat.load()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(64, 768, generator=g).to(DEV, torch.bfloat16)
    w = (0.02 * torch.randn(512, 768, generator=g)).to(DEV, torch.bfloat16)
    torch.cuda.synchronize()
    assert lib.cc2_device_status(1) == 0
    nat.check(lib.cc2_test_starve_gemm(1), "cc2_test_starve_gemm")
    try:
        K.linear(x, w)  # the launch itself succeeds; the kernel gives up after 2 s
        status = lib.cc2_device_status(1)
    finally:
        nat.check(lib.cc2_test_starve_gemm(0), "cc2_test_starve_gemm")
    assert status == 1  # CC2_DEV_GEMM_TIMEOUT
    assert lib.cc2_device_status(0) == 0  # cleared
    y = K.linear(x, w)
    torch.cuda.synchronize()
    assert lib.cc2_device_status(0) == 0
    ref = _ref(x, w)
    assert (y.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


def test_model_device_check_raises_then_recovers():
    lib = nat.load()
    m = seeded_init_(CuteChronos2Model(small_config()), seed=0).to(DEV, torch.bfloat16).eval()
    m.set_device_checks(True)
    ctx = torch.randn(1, 64).to(DEV)  # one series: 6 token rows, single-SM GEMMs only
    good = m(ctx, num_output_patches=2).clone()
    nat.check(lib.cc2_test_starve_gemm(1), "cc2_test_starve_gemm")
    try:
        with pytest.raises(nat.NativeError, match="gave up waiting"):
            m(ctx, num_output_patches=2)
    finally:
        nat.check(lib.cc2_test_starve_gemm(0), "cc2_test_starve_gemm")
        lib.cc2_device_status(1)
    again = m(ctx, num_output_patches=2)
    assert torch.equal(again, good)


def test_layer_barrier_timeout_sets_status_and_recovers():
    """The layer-persistent forward's grid barrier: one CTA withholds its
    arrival (test hook), every other CTA's bounded wait runs out, the launch
    ends with CC2_DEV_LAYER_TIMEOUT, and the next forward is correct again."""
    lib = nat.load()
    m = seeded_init_(CuteChronos2Model(small_config()), seed=0).to(DEV, torch.bfloat16).eval()
    ctx = torch.randn(1, 300).to(DEV)  # one series: 23 token rows, the layers in one launch
    old_c = lib.cc2_set_layer_chain(1)
    try:
        good = m(ctx, num_output_patches=3).clone()
        torch.cuda.synchronize()
        assert lib.cc2_device_status(1) == 0
        nat.check(lib.cc2_test_starve_layer_barrier(1), "cc2_test_starve_layer_barrier")
        try:
            m(ctx, num_output_patches=3)
            status = lib.cc2_device_status(1)
        finally:
            nat.check(lib.cc2_test_starve_layer_barrier(0), "cc2_test_starve_layer_barrier")
        assert status == 4  # CC2_DEV_LAYER_TIMEOUT
        again = m(ctx, num_output_patches=3)
        torch.cuda.synchronize()
        assert lib.cc2_device_status(0) == 0
        assert torch.equal(again, good)
    finally:
        lib.cc2_set_layer_chain(old_c)

"""Bounded device waits give up: every wait in the kernels has a limit, after
which the kernel records a timeout code in the device error word and returns
(once the copies it has in flight have landed), leaving the context usable.
The waits are made to run out on purpose here, with no GPU fault: a counter
that nothing increments, and weight tiles given no time to land."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from moe_data import activations, zipf_logits

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cache(pkg, cuda):
    pkg.moe_cache.configure(enabled=True)
    yield
    pkg.moe_cache.set_wait_limits(0, 0)
    pkg.moe_cache.set_layer_fused(True)
    pkg.moe_cache.reset()


def test_exchange_wait_runs_out(pkg, cuda):
    """moe_b200_ep_wait on a counter no GPU ever increments: the wait gives up
    after its limit (1 ms here) with MOE_DERR_TIMEOUT_FULL."""
    mc = pkg.moe_cache
    from importlib import import_module
    L = import_module("a6000-custom-kernels_b200._lib")
    flag = torch.zeros(4, dtype=torch.int32, device=cuda)
    mc.set_wait_limits(0, 1_000_000)
    stream = torch.cuda.current_stream(cuda)
    L.check(L.lib().moe_b200_ep_wait(ctypes.c_void_p(flag.data_ptr()), 1, ctypes.c_void_p(stream.cuda_stream)))
    assert mc.device_error() == mc.DERR_TIMEOUT_FULL
    # the stream finished and the context still works
    torch.cuda.synchronize()
    assert int(flag.sum().item()) == 0
    flag += 1
    L.check(L.lib().moe_b200_ep_wait(ctypes.c_void_p(flag.data_ptr()), 1, ctypes.c_void_p(stream.cuda_stream)))
    assert mc.device_error() == 0


def test_tile_waits_run_out_and_the_context_survives(pkg, cuda):
    """The GEMV's mbarrier waits with a 1 ns limit: a consumer warp that finds
    its weight tile not yet landed (or the producer a ring stage not yet free)
    gives up. The kernel still drains its copies, and a later launch with the
    default limit gives the same result as before."""
    mc = pkg.moe_cache
    H, F, E, k = 3072, 768, 64, 8
    t = O.Q2_K
    layer = pkg.MoELayer(H, F, E, k, {"gate": t, "up": t, "down": t}, shared=True, seed=21)
    mc.set_layer_fused(False)           # the per-op GEMV launches
    x = torch.from_numpy(activations((1, H), seed=5)).to(cuda)
    lg = torch.from_numpy(zipf_logits(1, E, seed=6)).to(cuda)
    ref = layer.decode(x, lg).clone()
    assert mc.device_error() == 0
    mc.set_wait_limits(1, 0)
    codes = []
    for _ in range(5):
        layer.decode(x, lg)
        codes.append(mc.device_error())
        if codes[-1]:
            break
    assert codes[-1] in (mc.DERR_TIMEOUT_FULL, mc.DERR_TIMEOUT_EMPTY), codes
    mc.set_wait_limits(0, 0)
    again = layer.decode(x, lg)
    assert mc.device_error() == 0
    assert torch.equal(again, ref)

"""moe_b200_layer_decode_noalloc: the layer decode for callers that cannot
allocate device memory where they run it (engines that pre-reserve and own all
device memory, plugins whose host framework forbids allocations in its compute
callback). Its scratch is one fixed file-scope device array; this checks,
through the C ABI, that two calls in a row give the same outputs as the
allocating entry point moe_b200_layer_decode (within the layer tests' stage
tolerance, 1e-4 of max |ref|) and report no device error.

Named to be collected last: a failure here leaves every other test already run.
"""
import ctypes
import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-4

Q2_K = 10


def test_noalloc_layer_matches_allocating_entry_point(cuda):
    import sys
    import os
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if repo not in sys.path:
        sys.path.insert(0, repo)
    pkg = importlib.import_module("a6000-custom-kernels_b200")
    lib = pkg.lib()
    mc = pkg.moe_cache
    mc.configure(enabled=True)
    try:
        H, F, E, k = 3072, 768, 64, 8
        layer = pkg.MoELayer(H, F, E, k, {"gate": Q2_K, "up": Q2_K, "down": Q2_K}, shared=True, seed=21)
        rng = np.random.default_rng(5)
        stream = torch.cuda.current_stream().cuda_stream
        for call, n_tok in enumerate((1, 3)):                    # two calls in a row
            x = torch.from_numpy(rng.normal(0, 1, (n_tok, H)).astype(np.float32)).to(cuda)
            logits = torch.from_numpy(rng.normal(0, 1, (n_tok, E)).astype(np.float32)).to(cuda)
            ref = layer.decode(x, logits)                        # allocating entry point (workspace)
            out = torch.full((n_tok, H), float("nan"), device=cuda)
            rc = lib.moe_b200_layer_decode_noalloc(ctypes.byref(layer.desc), x.data_ptr(), logits.data_ptr(),
                                                   out.data_ptr(), n_tok, ctypes.c_void_p(stream))
            assert rc == 0, lib.moe_b200_last_error()
            code = ctypes.c_int32(-1)
            assert lib.moe_b200_noalloc_device_error(ctypes.c_void_p(stream), ctypes.byref(code)) == 0
            assert code.value == 0
            got, want = out.cpu().numpy(), ref.cpu().numpy()
            assert np.isfinite(got).all(), call
            err = float(np.abs(got - want).max() / np.abs(want).max())
            assert err < TOL, (call, err)
        too_big = torch.zeros((9, H), device=cuda)
        rc = lib.moe_b200_layer_decode_noalloc(ctypes.byref(layer.desc), too_big.data_ptr(),
                                               torch.zeros((9, E), device=cuda).data_ptr(),
                                               torch.zeros((9, H), device=cuda).data_ptr(), 9,
                                               ctypes.c_void_p(stream))
        assert rc == pkg._lib.MOE_ERR_UNSUPPORTED
    finally:
        mc.reset()

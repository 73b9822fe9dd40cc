"""qma_cuda_moe_layer_noalloc: the MoE block for callers that cannot allocate
device memory (a host that reserves the device memory for its own pools, or
a step loop that cannot afford cudaMalloc's synchronisation).  It must give
the same result as qma_cuda_moe_layer, which takes caller scratch, on two
calls in a row (the second call reuses whatever the first left in the
library's fixed scratch array), and refuse more tokens than that array holds.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process (the first call on the device does the array's set-up)."""
import ctypes as C

import numpy as np
import pytest

import qma_cuda as Q
from helpers import MoeLayer, assert_close, empty_dev, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def layer(cuda):
    L = MoeLayer(il=0, seed=5)
    yield L
    L.close()


def _noalloc(layer, dx, T):
    import torch
    out = empty_dev((T, 2048), torch.float32)
    sel = empty_dev((T, 8), torch.int32)
    w = empty_dev((T, 8), torch.float32)
    Q.call("qma_cuda_moe_layer_noalloc", C.byref(layer.w), Q.ptr(dx), T, Q.ptr(out), Q.ptr(sel),
           Q.ptr(w), None)
    torch.cuda.synchronize()
    return out.cpu().numpy(), sel.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize("T", [1, 4])
def test_noalloc_matches_scratch_entry_point_twice(layer, T):
    rng = np.random.default_rng(40 + T)
    x2 = rng.standard_normal((T, 2048)).astype(np.float32)
    want, wsel, ww, _ = layer.gpu(x2)          # qma_cuda_moe_layer, caller scratch
    dx = to_dev(x2)
    for _ in range(2):
        got, gsel, gw = _noalloc(layer, dx, T)
        assert np.array_equal(gsel, wsel)
        assert np.abs(gw - ww).max() < 1e-5
        assert_close(got, want, 1e-3, f"noalloc T={T}")


def test_noalloc_rejects_more_tokens_than_its_scratch_holds(layer):
    T = 5
    dx = to_dev(np.zeros((T, 2048), np.float32))
    out = to_dev(np.zeros((T, 2048), np.float32))
    rc = Q.lib().qma_cuda_moe_layer_noalloc(C.byref(layer.w), Q.ptr(dx), T, Q.ptr(out), None, None,
                                            None)
    assert rc == Q.ERR_INVALID
    assert "exceeds" in Q.last_error()

"""GPU parity of the fused MoE block (router + top-8 + SwiGLU experts +
shared expert + combine + residual) against the oracle on synthetic
qwen35moe layer weights (configs[0]: N(0,0.02) weights, Q4_K gate/up, Q6_K
down, fp32 router; x ~ N(0,1)).

Bars: selected expert ids identical in order for every token; outputs within
1e-3 scaled relative error; weights within 1e-5."""
import numpy as np
import pytest

from helpers import MoeLayer, assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def layer(cuda):
    L = MoeLayer(il=0, seed=0)
    yield L
    L.close()


@pytest.mark.parametrize("T", [1, 4, 16, 37, 300])
def test_moe_block_matches_oracle(layer, T):
    rng = np.random.default_rng(100 + T)
    x2 = rng.standard_normal((T, 2048)).astype(np.float32)
    want, wsel, ww = layer.oracle(x2)
    got, gsel, gw, _ = layer.gpu(x2)
    assert np.array_equal(gsel, wsel), (gsel, wsel)
    assert np.abs(gw - ww).max() < 1e-5
    assert_close(got, want, 1e-3, f"moe T={T}")


def test_moe_routing_many_tokens(layer):
    rng = np.random.default_rng(7)
    x2 = (rng.standard_normal((64, 2048)) * rng.uniform(0.2, 3.0, (64, 1))).astype(np.float32)
    want, wsel, _ = layer.oracle(x2)
    got, gsel, _, _ = layer.gpu(x2)
    assert np.array_equal(gsel, wsel)
    assert_close(got, want, 1e-3, "moe T=64")


def test_moe_repeat_calls_reuse_scratch(layer):
    import torch
    rng = np.random.default_rng(8)
    x2 = rng.standard_normal((2, 2048)).astype(np.float32)
    scratch = torch.empty(layer.Q.lib().qma_cuda_moe_scratch_bytes(2), dtype=torch.uint8, device="cuda")
    a = layer.gpu(x2, scratch)[0]
    b = layer.gpu(x2, scratch)[0]
    assert np.array_equal(a, b)


def _underflow_router(W):
    """Rows 1..4 copy row 0 and rows 5..8 hold row 0's values permuted, all
    scaled up: the aligned input gives experts 0..4 logits ~100 above every
    other expert, so the reference's expf(l - max) underflows to exactly 0
    for all the rest and they tie at probability 0 (ranked by expert id)."""
    rng = np.random.default_rng(3)
    W[0] *= 6.0
    for e in range(1, 5):
        W[e] = W[0]
    for e in range(5, 9):
        W[e] = W[0][rng.permutation(2048)]


def _near_tie_router(W):
    """Rows 1..4 copy row 0 (exact logit ties, ranked by id); rows 5..8 are
    row 0 with one weight nudged by a few ulps (logits distinct in fp32 but
    far inside the summation-error bound), so only the reference-order
    recompute can rank them."""
    for e in range(1, 9):
        W[e] = W[0]
    for e in range(5, 9):
        i = 100 + 13 * e
        v = W[e, i]
        for _ in range(e - 4):
            v = np.nextafter(v, np.float32(np.inf) if e % 2 else np.float32(-np.inf))
        W[e, i] = v


def _aligned_inputs(L, T, scale, seed):
    rng = np.random.default_rng(seed)
    tr = L.t["ffn_gate_inp.weight"]
    W0 = L.blob[tr.off:tr.off + tr.nbytes].view(np.float32).reshape(256, 2048)[0]
    return (rng.standard_normal((T, 2048)) + scale * np.sign(W0)[None, :]).astype(np.float32)


@pytest.mark.parametrize("edit,scale", [(_near_tie_router, 0.3), (_underflow_router, 3.0)],
                         ids=["near_ties", "underflow_ties"])
def test_moe_exact_fallback_on_ties(cuda, edit, scale):
    L = MoeLayer(il=0, seed=0, edit_router=edit)
    try:
        x2 = _aligned_inputs(L, 6, scale, seed=11)
        want, wsel, _ = L.oracle(x2)
        got, gsel, _, fallbacks = L.gpu(x2)
        assert fallbacks > 0, "crafted ties should need the exact recompute"
        assert np.array_equal(gsel, wsel), (gsel, wsel)
        assert_close(got, want, 1e-3, "moe ties")
    finally:
        L.close()


@pytest.mark.parametrize("T", [16, 37, 300])
def test_grouped_gateup_tcgen05_bit_identical_to_mma_sync(layer, T):
    """The grouped path's gate/up GEMM on the 5th-generation tensor cores
    (tcgen05 int8 MMAs, accumulators in tensor memory, the Q4_K sub-block
    scales folded into two int8 digits of the weights) against the
    warp-level mma.sync kernel (QMA_CUDA_MMA_SYNC=1): the integer
    super-block sums are exact in both and the fp32 fold is shared, so the
    block's output is the same bits; both within the oracle's tolerance."""
    import os
    rng = np.random.default_rng(900 + T)
    x2 = rng.standard_normal((T, 2048)).astype(np.float32)
    got, gsel, _, _ = layer.gpu(x2)
    os.environ["QMA_CUDA_MMA_SYNC"] = "1"
    try:
        ref, rsel, _, _ = layer.gpu(x2)
    finally:
        del os.environ["QMA_CUDA_MMA_SYNC"]
    assert np.array_equal(gsel, rsel)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), \
        f"max |diff| {np.abs(got - ref).max():.3e}"
    want, wsel, _ = layer.oracle(x2)
    assert np.array_equal(gsel, wsel)
    assert_close(got, want, 1e-3, f"moe tc T={T}")

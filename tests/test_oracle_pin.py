"""Pins the C restatement (oracle/liboracle.so) to the qma reference compiled
from its own sources (oracle/_ref/libqmaref.so): every kernel and layer the
CUDA engine is checked against must agree bit for bit."""
import numpy as np
import pytest

import oracle as O
from helpers import aligned_inputs, near_tie_router, underflow_router


def p(a):
    return O._ptr(a)


def test_fp16_conversions_match(ref_lib, rng):
    L = O.lib()
    vals = np.concatenate([rng.standard_normal(5000) * 1e-3, rng.standard_normal(5000) * 300,
                           rng.standard_normal(2000) * 1e-6, [0.0, -0.0, 65504.0, 65520.0, 1e-8]])
    for v in vals.astype(np.float32):
        h = L.qo_float_to_half(float(v))
        assert h == ref_lib.qr_float_to_half(float(v)), v
        assert np.float32(L.qo_half_to_float(h)) == np.float32(ref_lib.qr_half_to_float(h))


def test_q8k_quant_matches(ref_lib, rng):
    x = (rng.standard_normal((6, 4096)) * rng.uniform(0.01, 10, (6, 1))).astype(np.float32)
    x[5, :256] = 0.0                                            # all-zero block: xd = 1
    xq, xd, xs = O.q8k_quant(x)
    for t in range(6):
        rq, rd, rs = np.zeros(4096, np.int8), np.zeros(16, np.float32), np.zeros(256, np.int16)
        ref_lib.qma_q8k_quant(p(x[t]), 4096, p(rq), p(rd), p(rs))
        assert np.array_equal(xq[t], rq) and np.array_equal(xs[t], rs)
        assert np.array_equal(xd[t].view(np.uint32), rd.view(np.uint32))


@pytest.mark.parametrize("wtype", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("n_in", [512, 2048, 4096])
def test_row_dots_bit_exact(ref_lib, rng, wtype, n_in):
    W = O.synth_matrix(f"pin.{wtype}.{n_in}", wtype, 48, n_in, seed=3)
    xq, xd, xs = O.q8k_quant(rng.standard_normal(n_in).astype(np.float32))
    ours, _ = O.dot_partials(W, wtype, n_in, xq[0], xd[0], xs[0])
    theirs = np.array([ref_lib.qma_q8k_dot(p(W[r]), wtype, p(xq[0]), p(xd[0]), p(xs[0]), n_in)
                       for r in range(48)], np.float32)
    assert np.array_equal(ours.view(np.uint32), theirs.view(np.uint32))


def test_reference_matmul_matches(ref_lib, rng):
    W = O.synth_matrix("pin.mm", O.Q4_K, 64, 2048, seed=5)
    x = rng.standard_normal((3, 2048)).astype(np.float32)
    ours = O.matmul(x, W, O.Q4_K, 2048, 64)
    theirs = np.zeros((3, 64), np.float32)
    ref_lib.qr_matmul(p(x), p(W), 2048, 64, 3, O.Q4_K, p(theirs), 1)
    assert np.array_equal(ours, theirs)


def test_kvq_records_and_kernels_match(ref_lib, rng):
    L = O.lib()
    for _ in range(20):
        v = (rng.standard_normal(256) * rng.uniform(0.1, 5)).astype(np.float32)
        q = rng.standard_normal(256).astype(np.float32)
        a, b = np.zeros(240, np.uint8), np.zeros(240, np.uint8)
        L.qo_kvq4_quant(p(v), p(a)); L.qo_kvq2_quant(p(v), p(a))
        ref_lib.kvq4_quant(p(v), 256, p(b)); ref_lib.kvq2_quant(p(v), 256, p(b))
        assert np.array_equal(a, b)
        assert L.qo_kvq4_dot(p(a), p(q)) == ref_lib.kvq4_dot(p(b), p(q), 256)
        assert L.qo_kvq2_dot(p(a[160:]), p(q)) == ref_lib.kvq2_dot(p(b[160:]), p(q), 256)
        o1 = q.copy(); o2 = q.copy()
        L.qo_kvq4_vacc(p(a), 0.3, p(o1)); ref_lib.kvq4_vacc(p(b), 0.3, p(o2), 256)
        L.qo_kvq2_vacc(p(a[160:]), 0.7, p(o1)); ref_lib.kvq2_vacc(p(b[160:]), 0.7, p(o2), 256)
        assert np.array_equal(o1, o2)
        assert L.qo_kvq4_qf(p(a), p(v)) == ref_lib.kvq4_qf(p(b), p(v), 256)


@pytest.fixture(scope="module")
def layer0(ref_lib):
    arr, n, size = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K)
    names = {arr[i].name.decode() for i in range(n) if arr[i].name.decode().startswith("blk.0.")}
    blob = O.synth_blob(arr, n, size, seed=0, names=names)
    om = O.lib().qo_model_new(arr, n, p(blob), O.N_VOCAB)
    rm = ref_lib.qr_model_new(arr, n, p(blob), size)
    assert om and rm
    yield om, rm, blob
    O.lib().qo_model_free(om)
    ref_lib.qr_model_free(rm)


@pytest.mark.parametrize("T", [1, 3])
def test_moe_layer_bit_exact(layer0, ref_lib, rng, T):
    om, rm, _ = layer0
    x = rng.standard_normal((T, 2048)).astype(np.float32)
    o1, o2 = np.zeros((T, 2048), np.float32), np.zeros((T, 2048), np.float32)
    sel = np.zeros((T, 8), np.int32)
    w = np.zeros((T, 8), np.float32)
    rsel = np.zeros(8, np.int32)
    O.lib().qo_moe_ffn(om, 0, p(x), T, p(o1), p(sel), p(w))
    ref_lib.qr_moe_ffn(rm, 0, p(x), T, p(o2), p(rsel))
    assert np.array_equal(o1, o2)
    assert np.array_equal(sel[-1], rsel)
    assert abs(w.sum(axis=1) - 1).max() < 1e-6


def test_gdn_layer_and_state_bit_exact(layer0, ref_lib, rng):
    om, rm, _ = layer0
    L = O.lib()
    os_, rs = L.qo_state_new(256), ref_lib.qr_state_new(256)
    try:
        for T in (1, 5, 1):
            x = rng.standard_normal((T, 2048)).astype(np.float32)
            o1, o2 = np.zeros((T, 2048), np.float32), np.zeros((T, 2048), np.float32)
            L.qo_gdn_layer(om, os_, 0, p(x), T, p(o1))
            ref_lib.qr_gdn_layer(rm, rs, 0, p(x), T, p(o2))
            assert np.array_equal(o1, o2)
            s1 = np.ctypeslib.as_array(L.qo_state_ssm(os_, 0), (32 * 128 * 128,))
            s2 = np.ctypeslib.as_array(ref_lib.qr_state_ssm(rs, 0), (32 * 128 * 128,))
            c1 = np.ctypeslib.as_array(L.qo_state_conv(os_, 0), (8192 * 3,))
            c2 = np.ctypeslib.as_array(ref_lib.qr_state_conv(rs, 0), (8192 * 3,))
            assert np.array_equal(s1, s2) and np.array_equal(c1, c2)
    finally:
        L.qo_state_free(os_)
        ref_lib.qr_state_free(rs)


@pytest.mark.parametrize("edit,scale", [(near_tie_router, 0.3), (underflow_router, 3.0)],
                         ids=["near_ties", "underflow_ties"])
def test_moe_crafted_router_ties_bit_exact(ref_lib, edit, scale):
    """Layer 0 with its router rewritten so that logits tie exactly, differ
    by a few ulps, or leave probabilities that underflow to 0: the oracle's
    experts and output equal the reference's token by token (one token per
    call, as the reference reports the last token's experts) and for all
    tokens in one call.  These are the routers the engine's exact fallback
    is tested on against the oracle."""
    arr, n, size = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K)
    names = {arr[i].name.decode() for i in range(n) if arr[i].name.decode().startswith("blk.0.")}
    blob = O.synth_blob(arr, n, size, seed=0, names=names)
    t = next(arr[i] for i in range(n) if arr[i].name.decode() == "blk.0.ffn_gate_inp.weight")
    W = blob[t.off:t.off + t.nbytes].view(np.float32).reshape(256, 2048)
    edit(W)                             # in place, in the blob
    om = O.lib().qo_model_new(arr, n, p(blob), O.N_VOCAB)
    rm = ref_lib.qr_model_new(arr, n, p(blob), size)
    assert om and rm
    try:
        T = 6
        x = aligned_inputs(W[0].copy(), T, scale, seed=11)
        o1, o2 = np.zeros((T, 2048), np.float32), np.zeros((T, 2048), np.float32)
        sel, w, rsel = np.zeros((T, 8), np.int32), np.zeros((T, 8), np.float32), np.zeros(8, np.int32)
        for k in range(T):
            xt = np.ascontiguousarray(x[k:k + 1])
            O.lib().qo_moe_ffn(om, 0, p(xt), 1, p(o1[k:k + 1]), p(sel[k:k + 1]), p(w[k:k + 1]))
            ref_lib.qr_moe_ffn(rm, 0, p(xt), 1, p(o2[k:k + 1]), p(rsel))
            assert np.array_equal(sel[k], rsel), (k, sel[k], rsel)
        assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))
        assert set(range(5)) <= set(sel[:, :5].ravel())      # the crafted rows lead the selection
        a1, a2 = np.zeros((T, 2048), np.float32), np.zeros((T, 2048), np.float32)
        O.lib().qo_moe_ffn(om, 0, p(x), T, p(a1), p(sel), p(w))
        ref_lib.qr_moe_ffn(rm, 0, p(x), T, p(a2), p(rsel))
        assert np.array_equal(a1.view(np.uint32), a2.view(np.uint32))
        assert np.array_equal(sel[-1], rsel)
    finally:
        O.lib().qo_model_free(om)
        ref_lib.qr_model_free(rm)


def test_zero_router_bias_is_the_unbiased_block(layer0, rng):
    """The biased oracle block (configs[4]'s router prior: one fp32 addition
    per logit, then the reference's selection) with a zero bias is the
    unbiased block bit for bit: the block whose moe_ffn is pinned to the
    reference above."""
    om, _, _ = layer0
    T = 3
    x = rng.standard_normal((T, 2048)).astype(np.float32)
    o1, o2 = np.zeros((T, 2048), np.float32), np.zeros((T, 2048), np.float32)
    s1, s2 = np.zeros((T, 8), np.int32), np.zeros((T, 8), np.int32)
    zero = np.zeros(256, np.float32)
    O.lib().qo_moe_block_biased(om, 0, p(x), T, p(zero), p(o1), p(s1), None)
    O.lib().qo_moe_block(om, 0, p(x), T, p(o2), p(s2), None)
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))
    assert np.array_equal(s1, s2)


def test_zipf_router_prior():
    """log p(rank) of a Zipf(1.1) law over a seeded per-layer ranking: a
    permutation of the same 256 log-probabilities in every layer, summing
    (as probabilities) to one, reproducible from the seed."""
    a, b = O.zipf_router_bias(7, 0), O.zipf_router_bias(7, 1)
    assert a.dtype == np.float32 and a.shape == (256,)
    assert np.array_equal(a, O.zipf_router_bias(7, 0))
    assert not np.array_equal(a, b) and np.array_equal(np.sort(a), np.sort(b))
    assert abs(np.exp(a.astype(np.float64)).sum() - 1.0) < 1e-5
    r = np.arange(1, 257, dtype=np.float64) ** -1.1
    assert np.allclose(np.sort(a)[::-1], np.log(r / r.sum()), atol=1e-6)

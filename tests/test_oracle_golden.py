"""The C restatement (oracle/liboracle.so) against committed known answers
of the qma reference (tests/golden/layer0_ref.npz, written by
tests/golden/make_layer_golden.py from the reference compiled from its own
sources).  These tests need no reference sources: they keep the oracle
pinned bit for bit wherever it runs.  The reference itself ships no golden
vectors, so these are its outputs on seeded inputs, stored with them."""
import hashlib
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "layer0_ref.npz")


def p(a):
    return O._ptr(a)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def digest(a):
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), np.uint8)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="module")
def layer0(golden):
    arr, n, size = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K)
    names = {arr[i].name.decode() for i in range(n) if arr[i].name.decode().startswith("blk.0.")}
    blob = O.synth_blob(arr, n, size, seed=int(golden["blob_seed"]), names=names)
    om = O.lib().qo_model_new(arr, n, p(blob), O.N_VOCAB)
    assert om
    yield om
    O.lib().qo_model_free(om)


def test_q8k_quant_matches_the_reference_answers(golden):
    """quantize_row_q8k (q8k.c:34-85), an all-zero block included."""
    xq, xd, xs = O.q8k_quant(golden["q8k_x"])
    assert np.array_equal(xq, golden["q8k_xq"])
    assert np.array_equal(xs, golden["q8k_xs"])
    assert np.array_equal(bits(xd), bits(golden["q8k_xd"]))


def test_kv_records_and_dots_match_the_reference_answers(golden):
    """The 240-byte q4 + q2 KV record (kvq.c) and both dot products."""
    L = O.lib()
    for i in range(len(golden["kv_v"])):
        v = np.ascontiguousarray(golden["kv_v"][i])
        q = np.ascontiguousarray(golden["kv_q"][i])
        rec = np.zeros(240, np.uint8)
        L.qo_kvq4_quant(p(v), p(rec))
        L.qo_kvq2_quant(p(v), p(rec))
        assert np.array_equal(rec, golden["kv_rec"][i])
        assert bits(L.qo_kvq4_dot(p(rec), p(q))) == bits(golden["kv_dot4"][i])
        assert bits(L.qo_kvq2_dot(p(rec[160:]), p(q))) == bits(golden["kv_dot2"][i])


def test_moe_block_matches_the_reference_answers(golden, layer0):
    """moe_ffn of layer 0 (nn.c:509-649) on 3 tokens: the output bit for bit
    and the last token's 8 experts."""
    x = np.ascontiguousarray(golden["moe_x"])
    T = x.shape[0]
    out = np.zeros((T, 2048), np.float32)
    sel = np.zeros((T, 8), np.int32)
    w = np.zeros((T, 8), np.float32)
    O.lib().qo_moe_ffn(layer0, 0, p(x), T, p(out), p(sel), p(w))
    assert np.array_equal(bits(out), bits(golden["moe_out"]))
    assert np.array_equal(sel[-1], golden["moe_sel_last"])


def test_gdn_mixer_and_states_match_the_reference_answers(golden, layer0):
    """The gated delta net mixer of layer 0 over calls of 1, 5 and 1 tokens:
    outputs bit for bit and the recurrent and conv states (SHA-256) after
    every call."""
    L = O.lib()
    s = L.qo_state_new(256)
    try:
        t0 = 0
        for k, T in enumerate(golden["gdn_calls"]):
            T = int(T)
            x = np.ascontiguousarray(golden["gdn_x"][t0:t0 + T])
            out = np.zeros((T, 2048), np.float32)
            L.qo_gdn_layer(layer0, s, 0, p(x), T, p(out))
            assert np.array_equal(bits(out), bits(golden["gdn_out"][t0:t0 + T])), k
            ssm = np.ctypeslib.as_array(L.qo_state_ssm(s, 0), (32 * 128 * 128,))
            conv = np.ctypeslib.as_array(L.qo_state_conv(s, 0), (8192 * 3,))
            assert np.array_equal(digest(ssm), golden["gdn_ssm_sha256"][k]), k
            assert np.array_equal(digest(conv), golden["gdn_conv_sha256"][k]), k
            t0 += T
    finally:
        L.qo_state_free(s)


def test_fixture_is_the_references_own_output(golden, ref_lib):
    """Where the reference is built here, it reproduces the committed answers
    from the committed inputs (so the fixture is the reference's output, not
    the restatement's)."""
    R = ref_lib
    for t in range(len(golden["q8k_x"])):
        x = np.ascontiguousarray(golden["q8k_x"][t])
        xq, xd, xs = np.zeros(4096, np.int8), np.zeros(16, np.float32), np.zeros(256, np.int16)
        R.qma_q8k_quant(p(x), 4096, p(xq), p(xd), p(xs))
        assert np.array_equal(xq, golden["q8k_xq"][t]) and np.array_equal(bits(xd), bits(golden["q8k_xd"][t]))
    arr, n, size = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K)
    names = {arr[i].name.decode() for i in range(n) if arr[i].name.decode().startswith("blk.0.")}
    blob = O.synth_blob(arr, n, size, seed=int(golden["blob_seed"]), names=names)
    rm = R.qr_model_new(arr, n, p(blob), size)
    assert rm
    try:
        x = np.ascontiguousarray(golden["moe_x"])
        out, sel = np.zeros_like(x), np.zeros(8, np.int32)
        R.qr_moe_ffn(rm, 0, p(x), x.shape[0], p(out), p(sel))
        assert np.array_equal(bits(out), bits(golden["moe_out"])) and np.array_equal(sel, golden["moe_sel_last"])
        rs = R.qr_state_new(256)
        try:
            t0 = 0
            for k, T in enumerate(golden["gdn_calls"]):
                T = int(T)
                xg = np.ascontiguousarray(golden["gdn_x"][t0:t0 + T])
                og = np.zeros_like(xg)
                R.qr_gdn_layer(rm, rs, 0, p(xg), T, p(og))
                assert np.array_equal(bits(og), bits(golden["gdn_out"][t0:t0 + T])), k
                ssm = np.ctypeslib.as_array(R.qr_state_ssm(rs, 0), (32 * 128 * 128,))
                assert np.array_equal(digest(ssm), golden["gdn_ssm_sha256"][k]), k
                t0 += T
        finally:
            R.qr_state_free(rs)
    finally:
        R.qr_model_free(rm)

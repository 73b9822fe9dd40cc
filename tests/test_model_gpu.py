"""Full-model parity: the engine's qma_eval replacement against the oracle's
restatement of qma_eval and the golden fixture from the reference itself, on
the 40-layer synthetic qwen35moe (configs[3] shapes; Q6_K embeddings and LM
head, the types the reference supports).

Bars: greedy tokens identical; last-token logits within 1e-3 scaled relative
error.  The weights are generated on the device
(byte-identical to the oracle's generator, tests/test_synth_gpu.py) and
copied to the host for the oracle."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
import qma_cuda as Q
from helpers import assert_close

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "full_model.npz")
SEED = 7
N_CTX = 4096
RTOL = 1e-3


def device_blob(arr, n, size, seed):
    """The synthetic data section, generated tensor by tensor on the GPU."""
    import torch
    biggest = max(arr[i].nbytes for i in range(n))
    tmp = torch.empty(int(biggest), dtype=torch.uint8, device="cuda")
    blob = np.empty(size, np.uint8)
    for i in range(n):
        t = arr[i]
        nel = int(t.ne[0]) * int(t.ne[1]) * int(t.ne[2])
        Q.call("qma_cuda_synth_tensor", t.name, int(t.type), nel, seed, Q.ptr(tmp), None)
        torch.from_numpy(blob[t.off:t.off + t.nbytes]).copy_(tmp[:t.nbytes])
    torch.cuda.synchronize()
    return blob


@pytest.fixture(scope="module")
def full(cuda):
    arr, n, size = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K)
    blob = device_blob(arr, n, size, SEED)
    tp = C.cast(arr, C.POINTER(Q.Tensor))
    model = Q.Model(tp, n, host_blob=blob)
    om = O.lib().qo_model_new(arr, n, O._ptr(blob), O.N_VOCAB)
    assert om
    yield {"arr": arr, "n": n, "tp": tp, "blob": blob, "model": model, "om": om}
    O.lib().qo_model_free(om)
    model.close()


def oracle_run(om, prompt, decode_tokens):
    L = O.lib()
    s = L.qo_state_new(N_CTX)
    out = []
    try:
        lo = np.zeros(O.N_VOCAB, np.float32)
        p = np.ascontiguousarray(prompt, np.int32)
        L.qo_eval(om, s, O._ptr(p), len(p), O._ptr(lo), 0)
        out.append(lo.copy())
        for tok in decode_tokens:
            one = np.array([tok], np.int32)
            L.qo_eval(om, s, O._ptr(one), 1, O._ptr(lo), 0)
            out.append(lo.copy())
    finally:
        L.qo_state_free(s)
    return out


@pytest.mark.parametrize("n_layers", [1, 3, 4, 8, 40])
def test_hidden_state_after_n_layers(full, n_layers):
    """Residual stream after the first n layers (GDN layers 0-2, attention
    layer 3, ...) for a 5-token prompt then one decode token."""
    prompt = np.array([11, 22, 33, 44, 55], np.int32)
    st = Q.State(full["model"], N_CTX)
    L = O.lib()
    os_ = L.qo_state_new(N_CTX)
    try:
        for toks in (prompt, np.array([66], np.int32)):
            got = st.eval_hidden(toks, n_layers)
            want = np.zeros_like(got)
            L.qo_eval_hidden(full["om"], os_, O._ptr(toks), len(toks), n_layers, O._ptr(want))
            assert_close(got, want, RTOL, f"hidden after {n_layers} layers, T={len(toks)}")
    finally:
        st.close()
        L.qo_state_free(os_)


def test_prompt_and_greedy_decode_match_reference_and_oracle(full):
    g = np.load(GOLDEN) if os.path.exists(GOLDEN) else None
    rng = np.random.default_rng(SEED)
    prompt = g["prompt"] if g is not None else rng.integers(0, O.N_VOCAB, 24).astype(np.int32)
    st = Q.State(full["model"], N_CTX)
    try:
        got0 = st.eval(prompt)
        tok0 = int(np.argmax(got0))
        toks, last = st.decode_greedy(tok0, 4)
    finally:
        st.close()
    want = oracle_run(full["om"], prompt, list(toks))
    assert_close(got0, want[0], RTOL, "prompt logits")
    assert tok0 == int(np.argmax(want[0]))
    assert_close(last, want[-1], RTOL, "decode logits")
    oracle_toks = [int(np.argmax(w)) for w in want[:-1]]
    assert list(toks) == oracle_toks
    if g is not None:
        # the reference's own run (oracle/_ref) on the same weights
        assert list(toks) == list(g["greedy"])
        ids, vals = g["top_ids"][0], g["top_vals"][0]
        assert_close(got0[ids], vals, RTOL, "prompt logits vs reference top-64")


def test_model_synth_matches_model_load(full):
    m2 = Q.Model(full["tp"], full["n"], seed=SEED)
    try:
        prompt = np.arange(5, 17, dtype=np.int32)
        a = Q.State(full["model"], 512)
        b = Q.State(m2, 512)
        try:
            la, lb = a.eval(prompt), b.eval(prompt)
        finally:
            a.close()
            b.close()
        assert np.array_equal(la, lb)
    finally:
        m2.close()


def test_decode_after_live_index_rebuild(full):
    # a 130-token prompt, then decoding: the first decode step (position 130
    # >= 128) rebuilds the HCM live index, so decoding attends live index +
    # tail rather than the dense range
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, O.N_VOCAB, 130).astype(np.int32)
    st = Q.State(full["model"], N_CTX)
    try:
        got = st.eval(prompt)
        toks, last = st.decode_greedy(int(np.argmax(got)), 2)
    finally:
        st.close()
    want = oracle_run(full["om"], prompt, list(toks))
    assert_close(got, want[0], RTOL, "130-token prompt")
    assert list(toks) == [int(np.argmax(w)) for w in want[:-1]]
    assert_close(last, want[-1], RTOL, "decode after rebuild")


def test_ecache_get_addresses_expert_records(full):
    g, u, d = C.c_void_p(), C.c_void_p(), C.c_void_p()
    Q.call("qma_cuda_ecache_get", full["model"].h, 3, 17, C.byref(g), C.byref(u), C.byref(d))
    g0, u0, d0 = C.c_void_p(), C.c_void_p(), C.c_void_p()
    Q.call("qma_cuda_ecache_get", full["model"].h, 3, 0, C.byref(g0), C.byref(u0), C.byref(d0))
    assert g.value - g0.value == 17 * 512 * 8 * 144
    assert d.value - d0.value == 17 * Q.packed_bytes(Q.Q6_K, 2048, 512)
    assert Q.lib().qma_cuda_ecache_get(full["model"].h, 40, 0, None, None, None) == Q.ERR_INVALID

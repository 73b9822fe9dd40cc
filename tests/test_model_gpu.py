"""Full-model parity of the engine's qma_eval replacement on the 40-layer
synthetic qwen35moe (configs[3] shapes; Q6_K embeddings and LM head, the
types the reference supports), against the oracle's restatement of qma_eval
(pinned bit-exact to the reference by tests/test_oracle_pin.py and the
golden fixture).

Why layer by layer: this random-init model is chaotic.  A 1-ulp difference
anywhere (fp32 summation order, a libm expf) flips an int8 of a later Q8_K
activation once in a while, and the top-8-of-256 routing of near-tied
random logits turns such flips into O(1) differences within a few layers:
the reference built with its own production flags (-O3 -ffast-math,
oracle/Makefile ref-fast) differs from its strict build by 0.68 norm-rel at
the first logits of the golden prompt.  So the gate is teacher forcing:
each oracle layer gets the engine's own input for that layer, and each
layer's output must agree within the fp32 tolerance.  What is integer or
byte work is compared exactly: embedding rows, quantized KV records, the
greedy decode graph against eager evaluation.

The weights are generated on the device (byte-identical to the oracle's
generator, tests/test_synth_gpu.py) and copied to the host for the oracle."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
import qma_cuda as Q

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "full_model.npz")
SEED = 7
N_CTX = 4096
# per-layer bars of the teacher-forced comparison: norm-relative error of
# the layer output over all tokens, and of the worst single token (a rare
# Q8_K int8 flip moves one token's output by ~1e-3)
RTOL_LAYER = 1e-3
RTOL_TOKEN = 5e-3


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
    O.lib().qo_set_threads(32)
    yield {"arr": arr, "n": n, "tp": tp, "blob": blob, "model": model, "om": om}
    O.lib().qo_model_free(om)
    model.close()


def gpu_hidden(model, prompt, n_layers, decode_token=None):
    """Residual stream after n_layers layers for the prompt (or, with
    decode_token, for that token evaluated after the whole prompt)."""
    st = Q.State(model, N_CTX)
    try:
        if decode_token is None:
            return st.eval_hidden(prompt, n_layers)
        st.eval(prompt)
        return st.eval_hidden(np.array([decode_token], np.int32), n_layers)
    finally:
        st.close()


def norm_rel(got, want, axis=None):
    return np.linalg.norm(got - want, axis=axis) / np.linalg.norm(want, axis=axis)


def test_oracle_full_forward_matches_reference_golden(full):
    """The teacher itself: the oracle's qma_eval on the golden prompt and
    greedy continuation reproduces the reference's own run (oracle/_ref,
    tests/golden/make_golden.py) bit for bit at its top-64 logits."""
    g = np.load(GOLDEN)
    L = O.lib()
    s = L.qo_state_new(N_CTX)
    try:
        lo = np.zeros(O.N_VOCAB, np.float32)
        p = np.ascontiguousarray(g["prompt"], np.int32)
        L.qo_eval(full["om"], s, O._ptr(p), len(p), O._ptr(lo), 0)
        toks = []
        for k in range(len(g["greedy"]) + 1):
            ids = g["top_ids"][k]
            assert np.array_equal(lo[ids].view(np.uint32), g["top_vals"][k].astype(np.float32).view(np.uint32))
            if k == len(g["greedy"]):
                break
            toks.append(int(np.argmax(lo)))
            L.qo_eval(full["om"], s, O._ptr(np.array([toks[-1]], np.int32)), 1, O._ptr(lo), 0)
        assert toks == list(g["greedy"])
    finally:
        L.qo_state_free(s)


def test_embedding_rows_bit_exact(full):
    prompt = np.array([0, 1, 7, 151935, 62913], np.int32)
    got = gpu_hidden(full["model"], prompt, 0)
    want = np.zeros_like(got)
    s = O.lib().qo_state_new(N_CTX)
    O.lib().qo_eval_hidden(full["om"], s, O._ptr(prompt), len(prompt), 0, O._ptr(want))
    O.lib().qo_state_free(s)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_layers_teacher_forced_prefill_and_decode(full):
    """Every layer (30 gated-delta-net, 10 attention, each with its MoE
    block) on a 24-token prompt at positions 0..23 and then on one decode
    token at position 24, the oracle's layer fed the engine's input."""
    L = O.lib()
    prompt = np.random.default_rng(SEED).integers(0, O.N_VOCAB, 24).astype(np.int32)
    tok = 62913
    xs = [gpu_hidden(full["model"], prompt, nl) for nl in range(41)]
    xd = [gpu_hidden(full["model"], prompt, nl, tok) for nl in range(41)]
    os_ = L.qo_state_new(N_CTX)
    report = []
    try:
        for il in range(40):
            out = np.zeros_like(xs[il])
            L.qo_layer_forward(full["om"], os_, il, O._ptr(np.ascontiguousarray(xs[il])), len(prompt), 0,
                               O._ptr(out))
            report.append(("prefill", il, norm_rel(xs[il + 1], out), norm_rel(xs[il + 1], out, axis=1).max()))
        for il in range(40):
            out = np.zeros_like(xd[il])
            L.qo_layer_forward(full["om"], os_, il, O._ptr(np.ascontiguousarray(xd[il])), 1, len(prompt),
                               O._ptr(out))
            e = norm_rel(xd[il + 1], out)
            report.append(("decode", il, e, e))
    finally:
        L.qo_state_free(os_)
    bad = [r for r in report if r[2] > RTOL_LAYER and r[0] == "prefill" or r[3] > RTOL_TOKEN]
    assert not bad, "layers over tolerance (phase, layer, all-token, worst-token): %r" % bad
    # a single decode token has no averaging: its layers must still be at
    # the fp32 level typically, with rare int8 flips
    dec = sorted(r[2] for r in report if r[0] == "decode")
    assert dec[len(dec) // 2] <= RTOL_LAYER


def test_long_context_attention_arena_teacher_forced(full):
    """The first attention layer (layer 3) past the 4096-position hot
    window.  A 4700-token prompt: the rebuild at position 4608 pins the
    508 positions older than the hot window into the heavy-hitter arena,
    which the last prompt chunk (92 queries, the multi-query kernel) and
    then 40 single-token steps (the decode kernel) read; the rebuild at
    4736 re-ranks the pinned entries by their salience.  The oracle's layer
    gets the engine's own layer-3 inputs (qo_mixer_forward: qma_eval's
    chunks and rebuilds, this layer only), and the attention's
    contribution to the residual must agree within the fp32 tolerance."""
    L = O.lib()
    rng = np.random.default_rng(31)
    prompt = rng.integers(0, O.N_VOCAB, 4700).astype(np.int32)
    dec = rng.integers(0, O.N_VOCAB, 40).astype(np.int32)
    n_ctx = 8192
    a, b, c = (Q.State(full["model"], n_ctx) for _ in range(3))
    try:
        xin = [a.eval_hidden(prompt, 3)] + [a.eval_hidden(dec[i:i + 1], 3) for i in range(len(dec))]
        got = [b.eval_hidden(prompt, -4)] + [b.eval_hidden(dec[i:i + 1], -4) for i in range(len(dec))]
        # the same steps with single tokens through the multi-query kernel
        c.eval_hidden(prompt, -4)
        os.environ["QMA_CUDA_ATTN_GENERAL"] = "1"
        try:
            gen = [c.eval_hidden(dec[i:i + 1], -4) for i in range(len(dec))]
        finally:
            del os.environ["QMA_CUDA_ATTN_GENERAL"]
    finally:
        a.close()
        b.close()
        c.close()
    os_ = L.qo_state_new(n_ctx)
    want = []
    try:
        for x in xin:
            out = np.zeros_like(x)
            L.qo_mixer_forward(full["om"], os_, 3, O._ptr(np.ascontiguousarray(x)), len(x), O._ptr(out))
            want.append(out)
    finally:
        L.qo_state_free(os_)
    x_all, g_all, w_all = (np.concatenate(v) for v in (xin, got, want))
    dg, dw = g_all - x_all, w_all - x_all           # the attention output projection
    e_tok = norm_rel(dg, dw, axis=1)
    arena_q = np.arange(4608, 4740)                 # queries that read the arena
    print("attention delta norm-rel: all %.2e, worst %.2e, arena queries median %.2e"
          % (norm_rel(dg, dw), e_tok.max(), np.median(e_tok[arena_q])))
    assert norm_rel(dg, dw) <= RTOL_LAYER
    assert np.median(e_tok[arena_q]) <= RTOL_LAYER
    assert e_tok.max() <= 10 * RTOL_TOKEN
    # decode kernel vs multi-query kernel on the same state: fp32 rounding,
    # which now and then flips an int8 of the output projection's Q8_K input
    d1 = np.concatenate(got[1:]) - np.concatenate(xin[1:])
    d2 = np.concatenate(gen) - np.concatenate(xin[1:])
    e_k = norm_rel(d1, d2, axis=1)
    print("decode vs multi-query kernel: median %.2e, worst %.2e" % (np.median(e_k), e_k.max()))
    assert np.median(e_k) <= 1e-4 and e_k.max() <= RTOL_TOKEN


def test_kv_records_bit_exact(full):
    """The quantized K/V records (q4 + q2, 240 bytes per slot and head) the
    first attention layer appends for a single token, engine vs oracle."""
    L = O.lib()
    L.qo_state_kv_slot.restype = C.POINTER(C.c_uint8)
    toks = np.array([11], np.int32)
    st = Q.State(full["model"], N_CTX)
    os_ = L.qo_state_new(N_CTX)
    try:
        st.eval_hidden(toks, -4)          # through the mixer of layer 3
        want_h = np.zeros((1, 2048), np.float32)
        L.qo_eval_hidden(full["om"], os_, O._ptr(toks), 1, -4, O._ptr(want_h))
        for head in range(4):
            got = np.zeros(240, np.uint8)
            Q.call("qma_cuda_state_kv_slot", st.h, 0, head, 0, Q.ptr(got))
            want = np.ctypeslib.as_array(L.qo_state_kv_slot(os_, 0, head, 0), (240,))
            assert np.array_equal(got, want), f"KV head {head}: bytes {np.nonzero(got != want)[0][:16]}"
    finally:
        st.close()
        L.qo_state_free(os_)


def test_greedy_graph_matches_eager_eval_across_rebuild(full):
    """decode_greedy (one CUDA graph per step, argmax on the device, the
    graph re-captured when the HCM live index is rebuilt at position 128)
    reproduces token by token what eager qma_cuda_eval calls compute
    (QMA_CUDA_EAGER=1: single-token eval launches every kernel itself
    instead of replaying the decode graph)."""
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, O.N_VOCAB, 122).astype(np.int32)
    a = Q.State(full["model"], N_CTX)
    b = Q.State(full["model"], N_CTX)
    try:
        la = a.eval(prompt)
        lb = b.eval(prompt)
        assert np.array_equal(la, lb)
        tok = int(np.argmax(la))
        toks, last = a.decode_greedy(tok, 12)     # toks[i]: step i's input token
        fed = []
        os.environ["QMA_CUDA_EAGER"] = "1"
        try:
            for _ in range(12):
                fed.append(tok)
                lb = b.eval(np.array([tok], np.int32))
                tok = int(np.argmax(lb))
        finally:
            del os.environ["QMA_CUDA_EAGER"]
        assert list(toks) == fed
        assert np.array_equal(last, lb)
        assert a.n_pos == b.n_pos == 122 + 12
    finally:
        a.close()
        b.close()


def test_single_token_eval_replays_the_decode_graph(full):
    """qma_cuda_eval of one token (a replay of the captured decode step)
    returns the logits eager launches compute, across the HCM rebuild."""
    rng = np.random.default_rng(22)
    prompt = rng.integers(0, O.N_VOCAB, 124).astype(np.int32)
    a = Q.State(full["model"], N_CTX)
    b = Q.State(full["model"], N_CTX)
    try:
        la, lb = a.eval(prompt), b.eval(prompt)
        for i in range(8):
            tok = np.array([int(np.argmax(la))], np.int32)
            la = a.eval(tok)
            os.environ["QMA_CUDA_EAGER"] = "1"
            try:
                lb = b.eval(tok)
            finally:
                del os.environ["QMA_CUDA_EAGER"]
            assert np.array_equal(la, lb), f"step {i}"
        assert a.n_pos == b.n_pos == 124 + 8
    finally:
        a.close()
        b.close()


def test_single_token_eval_after_logits_all(full):
    """A logits-for-every-token evaluation enlarges the state's logits
    buffer; single-token evaluations after it (decode graph replays) must
    return the new step's logits, as eager launches compute them."""
    rng = np.random.default_rng(23)
    prompt = rng.integers(0, O.N_VOCAB, 40).astype(np.int32)
    a = Q.State(full["model"], N_CTX)
    b = Q.State(full["model"], N_CTX)
    try:
        la, lb = a.eval(prompt[:30]), b.eval(prompt[:30])
        la = a.eval(np.array([int(np.argmax(la))], np.int32))    # captures a decode graph
        lb = b.eval(np.array([int(np.argmax(lb))], np.int32))
        all_a = a.eval(prompt[30:], logits_all=True)
        all_b = b.eval(prompt[30:], logits_all=True)
        assert np.array_equal(all_a.view(np.uint32), all_b.view(np.uint32))
        tok = np.array([int(np.argmax(all_a[-1]))], np.int32)
        la = a.eval(tok)
        os.environ["QMA_CUDA_EAGER"] = "1"
        try:
            lb = b.eval(tok)
        finally:
            del os.environ["QMA_CUDA_EAGER"]
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    finally:
        a.close()
        b.close()


def test_model_load_gguf_reads_the_file(full, tmp_path):
    """qma_cuda_model_load_gguf on a GGUF file of the full layout (a sparse
    file: token_embd's bytes written, every other tensor zero) yields the
    embedding rows qma_cuda_model_load gives from the same bytes."""
    import gguf_file as G
    arr, n = full["arr"], full["n"]
    tensors = []
    for i in range(n):
        ne = [int(d) for d in arr[i].ne]
        tensors.append((arr[i].name.decode(), int(arr[i].type), tuple(ne if ne[2] > 1 else ne[:2]),
                        int(arr[i].off)))
    idx = O.tensor_index(arr, n)
    emb = arr[idx["token_embd.weight"]]
    p = tmp_path / "full.gguf"
    start = G.write(p, G.qwen35moe_kv(), tensors, data_size=full["blob"].nbytes)
    with open(p, "r+b") as f:
        f.seek(start + emb.off)
        f.write(full["blob"][emb.off:emb.off + emb.nbytes].tobytes())
    m = Q.Model(gguf=str(p))
    try:
        assert m.n_vocab == full["model"].n_vocab
        prompt = np.array([0, 5, 77, 151935], np.int32)
        st = Q.State(m, 256)
        try:
            got = st.eval_hidden(prompt, 0)
        finally:
            st.close()
        want = gpu_hidden(full["model"], prompt, 0)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        m.close()


def _device_floats(dptr, n):
    """n floats at a raw device address, copied to the host (cudaMemcpy of
    the CUDA runtime the engine library already loaded)."""
    rt = C.CDLL("libcudart.so.12")
    host = np.zeros(n, np.float32)
    assert rt.cudaMemcpy(C.c_void_p(host.ctypes.data), C.c_void_p(dptr), C.c_size_t(4 * n), 2) == 0
    return host


def test_state_logits_feed_the_gpu_sampler(full, ref_lib):
    """A single-token eval without host logits leaves them on the device
    (qma_cuda_state_logits): the same values the host copy returns, and the
    GPU sampler's candidates on them equal the reference's
    sampler_candidates on the host copy."""
    rng = np.random.default_rng(23)
    prompt = rng.integers(0, O.N_VOCAB, 16).astype(np.int32)
    a, b = Q.State(full["model"], N_CTX), Q.State(full["model"], N_CTX)
    try:
        la = a.eval(prompt)
        b.eval(prompt)
        tok = np.array([int(np.argmax(la))], np.int32)
        want_logits = a.eval(tok)
        Q.call("qma_cuda_eval", full["model"].h, b.h, Q.ptr(tok), 1, None, 0)
        dptr = Q.lib().qma_cuda_state_logits(b.h)
        n = full["model"].n_vocab
        host = _device_floats(dptr, n)
        assert np.array_equal(host.view(np.uint32), want_logits.view(np.uint32))
        last = np.array(list(prompt[-10:]) + [int(tok[0])], np.int32)
        ids = np.zeros(64, np.int32)
        lgs = np.zeros(64, np.float32)
        cnt = C.c_int()
        Q.call("qma_cuda_sample_candidates", dptr, n, Q.ptr(last), len(last), 1.1, 0.7, 40, 40, Q.ptr(ids),
               Q.ptr(lgs), C.byref(cnt), None)
        rids, rlgs = np.zeros(64, np.int32), np.zeros(64, np.float32)
        rn = ref_lib.qr_sampler_candidates(n, want_logits.ctypes.data, last.ctypes.data, len(last), 1.1, 0.7, 40,
                                           rids.ctypes.data, rlgs.ctypes.data, 40)
        assert cnt.value == rn == 40
        assert np.array_equal(ids[:40], rids[:40])
        assert np.array_equal(lgs[:40].view(np.uint32), rlgs[:40].view(np.uint32))
    finally:
        a.close()
        b.close()


def test_session_files_round_trip_and_resume(full, ref_lib, tmp_path):
    """qma_cuda_state_save writes the reference's session files (state as
    runstate_save, the KV slab file, salience as hcm_save): the reference's
    own runstate_load reads the state file back (position and recurrent
    state bytes), the KV file holds the engine's records at the reference's
    offsets, a state loaded from the files saves them again byte for byte,
    and the resumed state continues the sequence: its first token's logits
    match the original state's within the fp32 tolerance (a resumed process
    rebuilds the live index at once, so its attention sums the same
    positions in another order) and two resumed states agree exactly."""
    n_ctx = 512
    rng = np.random.default_rng(29)
    prompt = rng.integers(0, O.N_VOCAB, 300).astype(np.int32)
    a = Q.State(full["model"], n_ctx)
    b, c = Q.State(full["model"], n_ctx), Q.State(full["model"], n_ctx)
    f1 = [tmp_path / n for n in ("state.bin", "kv.bin", "salience.bin")]
    f2 = [tmp_path / n for n in ("state2.bin", "kv2.bin", "salience2.bin")]
    try:
        la = a.eval(prompt)
        tok = int(np.argmax(la))
        for _ in range(3):
            tok = int(np.argmax(a.eval(np.array([tok], np.int32))))
        a.save(*f1)
        gdn = 30
        assert f1[0].stat().st_size == 4 + gdn * 4 * (8192 * 3 + 32 * 128 * 128)
        assert f1[1].stat().st_size == 10 * 4 * n_ctx * 240
        assert f1[2].stat().st_size == 4 + 4 * (10 * n_ctx + 2048 + 10 * 2048) + 10 * 4 * 2048 * 240
        rs = ref_lib.qr_state_new(n_ctx)
        try:
            assert ref_lib.qr_runstate_load(rs, str(f1[0]).encode()) == 0
            assert ref_lib.qr_state_n_pos(rs) == a.n_pos == 303
            raw = np.fromfile(f1[0], np.uint8)
            conv0 = np.ctypeslib.as_array(ref_lib.qr_state_conv(rs, 0), (8192 * 3,))
            ssm0 = np.ctypeslib.as_array(ref_lib.qr_state_ssm(rs, 0), (32 * 128 * 128,))
            assert np.array_equal(conv0.view(np.uint8), raw[4:4 + 8192 * 3 * 4])
            assert np.array_equal(ssm0.view(np.uint8), raw[4 + 8192 * 3 * 4:4 + 4 * (8192 * 3 + 32 * 128 * 128)])
        finally:
            ref_lib.qr_state_free(rs)
        kvf = np.fromfile(f1[1], np.uint8).reshape(10, 4, n_ctx, 240)
        for lay, head, slot in [(0, 0, 0), (3, 2, 17), (9, 3, 302)]:
            rec = np.zeros(240, np.uint8)
            Q.call("qma_cuda_state_kv_slot", a.h, lay, head, slot, Q.ptr(rec))
            assert np.array_equal(kvf[lay, head, slot], rec)
        sal = np.fromfile(f1[2], np.uint8)
        assert int(sal[:4].view(np.uint32)[0]) == n_ctx
        b.load(*f1)
        c.load(*f1)
        assert b.n_pos == 303
        b.save(*f2)
        for x, y in zip(f1, f2):
            assert x.read_bytes() == y.read_bytes(), x.name
        t = np.array([tok], np.int32)
        la, lb, lc = a.eval(t), b.eval(t), c.eval(t)
        assert np.array_equal(lb, lc)
        assert norm_rel(lb, la) < RTOL_LAYER and int(np.argmax(lb)) == int(np.argmax(la))
    finally:
        a.close()
        b.close()
        c.close()


def test_resumed_session_reads_the_q2_gist_teacher_forced(full, tmp_path):
    """A session resumed past the hot window: the engine saves the state of
    a 4700-token prompt (layers 0-2 and layer 3's mixer), two fresh states
    load the files, and the first resumed token rebuilds the live index
    with the tiers cleared, as a fresh qma process does -- the positions
    older than the hot window are pinned into the arena and also listed in
    the q2 gist segment, so the decode kernel reads q2 records.  The
    oracle resumes from the same files (qo_state_resume: hcm_load into
    hcm_init's fresh bookkeeping) and runs layer 3's mixer on the engine's
    layer-3 inputs; the attention's residual contribution must agree
    within the fp32 tolerance."""
    L = O.lib()
    n_ctx = 8192
    rng = np.random.default_rng(37)
    prompt = rng.integers(0, O.N_VOCAB, 4700).astype(np.int32)
    dec = rng.integers(0, O.N_VOCAB, 6).astype(np.int32)
    files = [tmp_path / n for n in ("state.bin", "kv.bin", "salience.bin")]
    a = Q.State(full["model"], n_ctx)
    try:
        a.eval_hidden(prompt, -4)
        a.save(*files)
    finally:
        a.close()
    b, c = Q.State(full["model"], n_ctx), Q.State(full["model"], n_ctx)
    try:
        b.load(*files)
        c.load(*files)
        xin = [b.eval_hidden(dec[i:i + 1], 3) for i in range(len(dec))]
        got = [c.eval_hidden(dec[i:i + 1], -4) for i in range(len(dec))]
    finally:
        b.close()
        c.close()
    os_ = L.qo_state_new(n_ctx)
    want = []
    try:
        assert L.qo_state_resume(os_, str(files[1]).encode(), str(files[2]).encode(), len(prompt)) == 0
        for x in xin:
            out = np.zeros_like(x)
            L.qo_mixer_forward(full["om"], os_, 3, O._ptr(np.ascontiguousarray(x)), 1, O._ptr(out))
            want.append(out)
        seg = [C.c_int(), C.c_int(), C.c_int()]
        L.qo_state_live_segments(os_, *[C.byref(v) for v in seg])
        n_ring_q4, n4, live_n = (v.value for v in seg)
    finally:
        L.qo_state_free(os_)
    assert n4 > n_ring_q4 and live_n > n4, (n_ring_q4, n4, live_n)    # arena and q2 gist in use
    x_all, g_all, w_all = (np.concatenate(v) for v in (xin, got, want))
    dg, dw = g_all - x_all, w_all - x_all
    e_tok = norm_rel(dg, dw, axis=1)
    print("resumed attention delta norm-rel: all %.2e, worst %.2e; live segments %d / %d / %d"
          % (norm_rel(dg, dw), e_tok.max(), n_ring_q4, n4, live_n))
    assert norm_rel(dg, dw) <= RTOL_LAYER and e_tok.max() <= 10 * RTOL_TOKEN


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


def test_ecache_get_addresses_expert_records(full):
    g, u, d = C.c_void_p(), C.c_void_p(), C.c_void_p()
    Q.call("qma_cuda_ecache_get", full["model"].h, 3, 17, C.byref(g), C.byref(u), C.byref(d))
    g0, u0, d0 = C.c_void_p(), C.c_void_p(), C.c_void_p()
    Q.call("qma_cuda_ecache_get", full["model"].h, 3, 0, C.byref(g0), C.byref(u0), C.byref(d0))
    assert g.value - g0.value == 17 * 512 * 8 * 144
    assert d.value - d0.value == 17 * Q.packed_bytes(Q.Q6_K, 2048, 512)
    assert Q.lib().qma_cuda_ecache_get(full["model"].h, 40, 0, None, None, None) == Q.ERR_INVALID


def test_model_moe_weights_run_the_layer_moe_block(full):
    """qma_cuda_model_moe_weights hands out layer il's MoE weights in the
    engine's layout: qma_cuda_moe_layer on them equals the oracle's FFN half
    of that layer (routing bit-exact, output within 1e-3)."""
    import torch
    il, T = 7, 3
    w = Q.MoeWeights()
    Q.call("qma_cuda_model_moe_weights", full["model"].h, il, C.byref(w))
    g0 = C.c_void_p()
    Q.call("qma_cuda_ecache_get", full["model"].h, il, 0, C.byref(g0), None, None)
    assert w.gate_exps == g0.value and w.down_type == Q.Q6_K
    x2 = np.random.default_rng(il).standard_normal((T, 2048)).astype(np.float32)
    dx = torch.from_numpy(x2).cuda()
    out = torch.empty_like(dx)
    sel = torch.empty((T, 8), dtype=torch.int32, device="cuda")
    scratch = torch.empty(Q.lib().qma_cuda_moe_scratch_bytes(T), dtype=torch.uint8, device="cuda")
    Q.call("qma_cuda_moe_layer", C.byref(w), Q.ptr(dx), T, Q.ptr(out), Q.ptr(sel), None, Q.ptr(scratch),
           scratch.numel(), None)
    torch.cuda.synchronize()
    want = np.zeros_like(x2)
    wsel = np.zeros((T, 8), np.int32)
    O.lib().qo_moe_block(full["om"], il, O._ptr(x2), T, O._ptr(want), O._ptr(wsel), None)
    assert np.array_equal(sel.cpu().numpy(), wsel)
    assert norm_rel(out.cpu().numpy(), want) < 1e-3
    assert Q.lib().qma_cuda_model_moe_weights(full["model"].h, 40, C.byref(w)) == Q.ERR_INVALID


def test_ecache_hint_prefetch_hold_release(full):
    """The rest of the expert-cache contract (ecache.h:97-123): hint and
    prefetch accept up to 64 ids (more are clamped, as the reference
    does) and leave results unchanged; hold hands out get()'s pointers and
    counts, the 65th hold before a release is refused, and one release
    ends every hold."""
    import torch
    m = full["model"].h
    ids = np.array([3, 200, 17, 255, 0, 9, 77, 128], np.int32)
    Q.call("qma_cuda_ecache_hint", m, 5, Q.ptr(ids), len(ids), None)
    many = np.arange(100, dtype=np.int32) % 256
    Q.call("qma_cuda_ecache_prefetch", m, 6, Q.ptr(many), len(many), None)
    torch.cuda.synchronize()
    bad = np.array([256], np.int32)
    assert Q.lib().qma_cuda_ecache_hint(m, 5, Q.ptr(bad), 1, None) == Q.ERR_INVALID
    assert Q.lib().qma_cuda_ecache_prefetch(m, 40, Q.ptr(ids), 1, None) == Q.ERR_INVALID
    g, u, d = C.c_void_p(), C.c_void_p(), C.c_void_p()
    g1, u1, d1 = C.c_void_p(), C.c_void_p(), C.c_void_p()
    Q.call("qma_cuda_ecache_release", m)
    for k in range(64):
        Q.call("qma_cuda_ecache_hold", m, 2, k, C.byref(g), C.byref(u), C.byref(d))
        Q.call("qma_cuda_ecache_get", m, 2, k, C.byref(g1), C.byref(u1), C.byref(d1))
        assert (g.value, u.value, d.value) == (g1.value, u1.value, d1.value)
    assert Q.lib().qma_cuda_ecache_held(m) == 64
    assert Q.lib().qma_cuda_ecache_hold(m, 2, 64, C.byref(g), None, None) == Q.ERR_STATE
    Q.call("qma_cuda_ecache_release", m)
    assert Q.lib().qma_cuda_ecache_held(m) == 0
    Q.call("qma_cuda_ecache_hold", m, 2, 64, C.byref(g), None, None)
    Q.call("qma_cuda_ecache_release", m)


# ---- layer-level parity points (qma_cuda_gdn_step / qma_cuda_attn_decode) --
GDN_STATE_FLOATS = 8192 * 3 + 32 * 128 * 128


def gpu_mixer(st, fn, il, x, advance=1):
    """One call of a layer-level entry point on device copies of x."""
    import torch
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    out = torch.empty_like(dx)
    Q.call(fn, st.h, il, Q.ptr(dx), len(x), Q.ptr(out), advance)
    return out.cpu().numpy()


def engine_gdn_state(st, il, path):
    """conv [8192*3] and ssm [32*128*128] of gated-delta-net layer il, read
    from the state's runstate_save-format file (nn.c:2011-2025)."""
    st.save(state_path=path)
    raw = np.fromfile(path, np.float32, offset=4)
    k = sum(1 for l in range(il) if (l + 1) % 4)
    s = raw[k * GDN_STATE_FLOATS:(k + 1) * GDN_STATE_FLOATS]
    return s[:8192 * 3], s[8192 * 3:]


def oracle_gdn_state(os_, il):
    L = O.lib()
    conv = np.ctypeslib.as_array(L.qo_state_conv(os_, il), (8192 * 3,)).copy()
    ssm = np.ctypeslib.as_array(L.qo_state_ssm(os_, il), (32 * 128 * 128,)).copy()
    return conv, ssm


def oracle_mixer(full, il, chunks, n_ctx):
    """qo_mixer_forward over the given input chunks on a fresh oracle state;
    returns the outputs and the state (caller frees it)."""
    L = O.lib()
    os_ = L.qo_state_new(n_ctx)
    outs = []
    for x in chunks:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        L.qo_mixer_forward(full["om"], os_, il, O._ptr(x), len(x), O._ptr(out))
        outs.append(out)
    return outs, os_


def test_gdn_step_configs2_decode_1024_steps(full, tmp_path):
    """configs[2], decode: gated-delta-net layer 0 for 1024 single-token
    steps from a zero state (inputs ~N(0,1), seeded) through
    qma_cuda_gdn_step, against the oracle's sequential gdn_worker
    restatement (qo_mixer_forward, nn.c:784-833 with its conv and
    projections).  The layer's contribution to the residual must agree
    within 1e-3 norm-relative over all steps (5e-3 for the worst step: a
    rare Q8_K int8 flip), and after 1024 steps the recurrent and conv
    state within 1e-3: no drift of the recurrence over a long decode."""
    import torch
    il, n = 0, 1024
    x = np.random.default_rng(2024).standard_normal((n, 2048)).astype(np.float32)
    st = Q.State(full["model"], 4096)
    try:
        got = np.concatenate([gpu_mixer(st, "qma_cuda_gdn_step", il, x[i:i + 1]) for i in range(n)])
        assert st.n_pos == n
        conv_g, ssm_g = engine_gdn_state(st, il, tmp_path / "state.bin")
    finally:
        st.close()
    # the same steps queued back to back (qma_cuda_gdn_decode): identical
    st = Q.State(full["model"], 4096)
    try:
        dx = torch.from_numpy(x).cuda()
        dout = torch.empty_like(dx)
        Q.call("qma_cuda_gdn_decode", st.h, il, Q.ptr(dx), n, Q.ptr(dout))
        assert st.n_pos == n
        assert np.array_equal(dout.cpu().numpy(), got)
    finally:
        st.close()
    (want,), os_ = oracle_mixer(full, il, [x], 4096)
    try:
        conv_w, ssm_w = oracle_gdn_state(os_, il)
    finally:
        O.lib().qo_state_free(os_)
    dg, dw = got - x, want - x
    e_tok = norm_rel(dg, dw, axis=1)
    print("gdn decode 1024: all %.2e worst %.2e last-64 %.2e ssm %.2e conv %.2e"
          % (norm_rel(dg, dw), e_tok.max(), norm_rel(dg[-64:], dw[-64:]), norm_rel(ssm_g, ssm_w),
             norm_rel(conv_g, conv_w)))
    assert norm_rel(dg, dw) <= RTOL_LAYER
    assert e_tok.max() <= RTOL_TOKEN
    assert norm_rel(dg[-64:], dw[-64:]) <= RTOL_LAYER
    assert norm_rel(ssm_g, ssm_w) <= RTOL_LAYER
    assert norm_rel(conv_g, conv_w) <= RTOL_LAYER


@pytest.mark.parametrize("form", ["chunked", "sequential"])
def test_gdn_step_configs2_prefill_4096(full, tmp_path, form):
    """configs[2], prefill: layer 0 over a 4096-token prompt (8 calls of
    512 tokens through qma_cuda_gdn_step) against the oracle's
    token-sequential recurrence over the same 4096 inputs; outputs and the
    final recurrent and conv state within 1e-3 norm-relative.  Both forms
    of the engine's multi-token recurrence: the chunked gated-delta form
    (64-token chunks, the default) and the token-sequential kernel
    (QMA_CUDA_GDN_SEQ=1)."""
    il, n = 0, 4096
    x = np.random.default_rng(4096).standard_normal((n, 2048)).astype(np.float32)
    st = Q.State(full["model"], 8192)
    if form == "sequential":
        os.environ["QMA_CUDA_GDN_SEQ"] = "1"
    try:
        got = np.concatenate([gpu_mixer(st, "qma_cuda_gdn_step", il, x[i:i + 512]) for i in range(0, n, 512)])
        conv_g, ssm_g = engine_gdn_state(st, il, tmp_path / "state.bin")
    finally:
        os.environ.pop("QMA_CUDA_GDN_SEQ", None)
        st.close()
    (want,), os_ = oracle_mixer(full, il, [x], 8192)
    try:
        conv_w, ssm_w = oracle_gdn_state(os_, il)
    finally:
        O.lib().qo_state_free(os_)
    dg, dw = got - x, want - x
    e_tok = norm_rel(dg, dw, axis=1)
    print("gdn prefill 4096 (%s): all %.2e worst %.2e ssm %.2e conv %.2e"
          % (form, norm_rel(dg, dw), e_tok.max(), norm_rel(ssm_g, ssm_w), norm_rel(conv_g, conv_w)))
    assert norm_rel(dg, dw) <= RTOL_LAYER
    assert e_tok.max() <= RTOL_TOKEN
    assert norm_rel(ssm_g, ssm_w) <= RTOL_LAYER
    assert norm_rel(conv_g, conv_w) <= RTOL_LAYER


def test_attn_decode_matches_oracle_mixer(full):
    """qma_cuda_attn_decode on attention layer 3 from an empty ring: a
    300-token chunk (multi-query kernel), then 30 single tokens (decode
    kernel) past the live-index rebuild at position 300, against the
    oracle's layer (qo_mixer_forward: the same chunks and rebuilds).  Also:
    advance 0 leaves the position alone, and the entry points refuse the
    other kind of layer."""
    il = 3
    rng = np.random.default_rng(333)
    x = rng.standard_normal((330, 2048)).astype(np.float32)
    chunks = [x[:300]] + [x[i:i + 1] for i in range(300, 330)]
    st = Q.State(full["model"], 4096)
    try:
        got = [gpu_mixer(st, "qma_cuda_attn_decode", il, c) for c in chunks]
        assert st.n_pos == 330
        again = gpu_mixer(st, "qma_cuda_attn_decode", il, x[329:330], advance=0)
        assert st.n_pos == 330 and np.isfinite(again).all()
        assert Q.lib().qma_cuda_attn_decode(st.h, 0, 1, 1, 1, 1) == Q.ERR_INVALID
        assert Q.lib().qma_cuda_gdn_step(st.h, 3, 1, 1, 1, 1) == Q.ERR_INVALID
    finally:
        st.close()
    want, os_ = oracle_mixer(full, il, chunks, 4096)
    O.lib().qo_state_free(os_)
    g_all, w_all = np.concatenate(got), np.concatenate(want)
    dg, dw = g_all - x, w_all - x
    e_tok = norm_rel(dg, dw, axis=1)
    print("attn mixer: all %.2e worst %.2e decode steps %.2e"
          % (norm_rel(dg, dw), e_tok.max(), norm_rel(dg[300:], dw[300:])))
    assert norm_rel(dg, dw) <= RTOL_LAYER
    assert norm_rel(dg[300:], dw[300:]) <= RTOL_LAYER
    assert e_tok.max() <= RTOL_TOKEN


def test_gdn_step_ragged_chunks_match_sequential(full):
    """The chunked form on chunk lengths that are not multiples of 64 (2,
    63, 65, 130, 511 tokens), continuing one state, against the
    token-sequential kernel on the same calls: outputs within 1e-4
    norm-relative (two fp32 orders of the same recurrence)."""
    import torch
    il = 4
    sizes = [2, 63, 65, 130, 511]
    x = np.random.default_rng(77).standard_normal((sum(sizes), 2048)).astype(np.float32)
    outs = {}
    for form in ("chunked", "sequential"):
        st = Q.State(full["model"], 4096)
        if form == "sequential":
            os.environ["QMA_CUDA_GDN_SEQ"] = "1"
        try:
            o, k = [], 0
            for n in sizes:
                o.append(gpu_mixer(st, "qma_cuda_gdn_step", il, x[k:k + n]))
                k += n
            outs[form] = np.concatenate(o)
        finally:
            os.environ.pop("QMA_CUDA_GDN_SEQ", None)
            st.close()
    d1, d2 = outs["chunked"] - x, outs["sequential"] - x
    e = norm_rel(d1, d2)
    print("gdn ragged chunks: chunked vs sequential %.2e" % e)
    # two fp32 orders of one recurrence; a rare Q8_K int8 flip of the
    # ssm_out input moves single tokens by ~1e-3
    assert e <= 5e-4


# ------------------------------------------------------ multi-sequence batch --
def _batch_prefill(batch, prompts, **kw):
    sids = np.concatenate([np.full(len(p), i, np.int32) for i, p in enumerate(prompts)])
    return batch.eval(sids, np.concatenate(prompts), **kw)


def test_batch_decode_layers_teacher_forced(full):
    """Three sequences with prompts of different lengths decode one token
    each in one batched step (per-row conv / gated-delta state through the
    sequence table, attention per sequence, shared projections and MoE);
    every layer of every row, fed to the oracle's layer with that sequence's
    own prefix, agrees within the single-token tolerance."""
    L = O.lib()
    rng = np.random.default_rng(SEED + 1)
    prompts = [rng.integers(0, O.N_VOCAB, n).astype(np.int32) for n in (24, 17, 30)]
    toks = np.array([62913, 5, 151935], np.int32)
    sids = np.arange(len(prompts), dtype=np.int32)

    def batch_hidden(nl):
        b = Q.Batch(full["model"], len(prompts), N_CTX)
        try:
            _batch_prefill(b, prompts, logits=False, greedy=False)
            h = b.eval_hidden(sids, toks, nl)
            assert [b.n_pos(i) for i in range(len(prompts))] == [len(p) + 1 for p in prompts]
            return h
        finally:
            b.close()

    xd = [batch_hidden(nl) for nl in range(41)]
    report = []
    for i, p in enumerate(prompts):
        xs = [gpu_hidden(full["model"], p, nl) for nl in range(41)]
        os_ = L.qo_state_new(N_CTX)
        try:
            for il in range(40):
                out = np.zeros_like(xs[il])
                L.qo_layer_forward(full["om"], os_, il, O._ptr(np.ascontiguousarray(xs[il])), len(p), 0,
                                   O._ptr(out))
            for il in range(40):
                x = np.ascontiguousarray(xd[il][i:i + 1])
                out = np.zeros_like(x)
                L.qo_layer_forward(full["om"], os_, il, O._ptr(x), 1, len(p), O._ptr(out))
                report.append((i, il, norm_rel(xd[il + 1][i:i + 1], out)))
        finally:
            L.qo_state_free(os_)
    worst = max(report, key=lambda r: r[2])
    print("batched decode, worst layer (seq, layer, norm-rel): %r" % (worst,))
    bad = [r for r in report if r[2] > RTOL_TOKEN]
    assert not bad, "rows over tolerance (seq, layer, norm-rel): %r" % bad


def test_batch_steps_independent_of_the_other_sequences(full):
    """32 sequences: their prompts prefilled in one call (each through its
    own state: the logits equal a lone state's bit for bit), then three
    decode steps taken once as one 32-row step and once as two 16-row steps
    (the second half first, in reverse order).  Every sequence's logits and
    greedy token agree bit for bit: a row's results do not depend on the
    other rows of its step (same path: the GEMM projections, the grouped
    experts)."""
    B, P = 32, 8
    rng = np.random.default_rng(SEED + 2)
    prompts = rng.integers(0, O.N_VOCAB, (B, P)).astype(np.int32)
    a = Q.Batch(full["model"], B, N_CTX)
    b = Q.Batch(full["model"], B, N_CTX)
    try:
        la, ga = _batch_prefill(a, list(prompts))
        lb, gb = _batch_prefill(b, list(prompts))
        last = np.arange(B) * P + P - 1
        assert np.array_equal(la[last].view(np.uint32), lb[last].view(np.uint32))
        assert np.array_equal(ga[last], np.argmax(la[last], axis=1))
        assert (np.delete(ga, last) == -1).all()
        st = Q.State(full["model"], N_CTX)
        try:
            lone = st.eval(prompts[5])
        finally:
            st.close()
        assert np.array_equal(lone.view(np.uint32), la[last[5]].view(np.uint32))
        tok = ga[last].astype(np.int32)
        sids = np.arange(B, dtype=np.int32)
        for step in range(3):
            la, ga = a.eval(sids, tok)
            h2, h1 = sids[16:][::-1].copy(), sids[:16].copy()
            l2, g2 = b.eval(h2, tok[h2])
            l1, g1 = b.eval(h1, tok[h1])
            lb = np.empty_like(la)
            gb = np.empty_like(ga)
            lb[h2], gb[h2] = l2, g2
            lb[h1], gb[h1] = l1, g1
            diff = np.nonzero((la.view(np.uint32) != lb.view(np.uint32)).any(axis=1))[0]
            assert diff.size == 0, "step %d: rows differ for sequences %r" % (step, diff.tolist())
            assert np.array_equal(ga, gb) and np.array_equal(ga, np.argmax(la, axis=1))
            tok = ga.astype(np.int32)
        assert [a.n_pos(i) for i in range(B)] == [P + 3] * B
        # the attention of all rows in one launch per kernel (row tables)
        # equals one sequence at a time, bit for bit
        os.environ["QMA_CUDA_ATTN_PER_SEQ"] = "1"
        try:
            lb, gb = b.eval(sids, tok)
        finally:
            os.environ.pop("QMA_CUDA_ATTN_PER_SEQ", None)
        la, ga = a.eval(sids, tok)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)) and np.array_equal(ga, gb)
    finally:
        a.close()
        b.close()

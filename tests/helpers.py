"""Small helpers shared by the GPU parity tests."""
import numpy as np


def to_dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def empty_dev(shape, dtype):
    import torch
    return torch.empty(shape, dtype=dtype, device="cuda")


def assert_close(got, want, rtol, what=""):
    """|got - want| <= rtol * (|want| + mean|want|) element-wise: relative
    error with a floor at the output's mean magnitude, so outputs that cancel
    to ~0 are measured against the scale of their neighbours."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    scale = np.abs(want).mean() + 1e-30
    err = np.abs(got - want) / (np.abs(want) + scale)
    worst = float(err.max()) if err.size else 0.0
    assert worst <= rtol, f"{what}: max scaled error {worst:.3e} > {rtol:.1e}"
    return worst


def underflow_router(W):
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


def near_tie_router(W):
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


def aligned_inputs(W0, T, scale, seed):
    """T tokens of N(0, 1) noise plus scale * sign(router row 0): inputs whose
    top experts are the crafted rows."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((T, 2048)) + scale * np.sign(W0)[None, :]).astype(np.float32)


MOE_TENSORS = ("post_attention_norm.weight", "ffn_gate_inp.weight", "ffn_gate_exps.weight",
               "ffn_up_exps.weight", "ffn_down_exps.weight", "ffn_gate_inp_shexp.weight",
               "ffn_gate_shexp.weight", "ffn_up_shexp.weight", "ffn_down_shexp.weight")


class MoeLayer:
    """One synthetic MoE layer held twice: in a host blob for the oracle and
    on the GPU in the engine's layout (down projections repacked)."""

    def __init__(self, il=0, seed=0, down_type=14, edit_router=None):
        import oracle as O
        import qma_cuda as Q
        import torch
        self.O, self.Q, self.il = O, Q, il
        self.arr, self.n, self.size = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K,
                                                     down_type=down_type)
        names = {f"blk.{il}.{t}" for t in MOE_TENSORS}
        self.blob = O.synth_blob(self.arr, self.n, self.size, seed=seed, names=names)
        idx = O.tensor_index(self.arr, self.n)
        self.t = {k[len(f"blk.{il}."):]: self.arr[idx[k]] for k in names}
        if edit_router is not None:
            tr = self.t["ffn_gate_inp.weight"]
            W = self.blob[tr.off:tr.off + tr.nbytes].view(np.float32).reshape(256, 2048)
            edit_router(W)
        self.model = O.lib().qo_model_new(self.arr, self.n, O._ptr(self.blob), O.N_VOCAB)
        assert self.model
        self.dev = {}
        for name, tr in self.t.items():
            raw = torch.from_numpy(self.blob[tr.off:tr.off + tr.nbytes]).cuda()
            if name in ("ffn_down_exps.weight", "ffn_down_shexp.weight") and tr.type != O.Q4_K:
                rows, n_in, nexp = int(tr.ne[1]), int(tr.ne[0]), int(tr.ne[2])
                pb = Q.packed_bytes(tr.type, rows, n_in)
                gb = O.row_bytes(tr.type, n_in) * rows
                packed = torch.empty(pb * nexp, dtype=torch.uint8, device="cuda")
                for e in range(nexp):
                    Q.call("qma_cuda_repack", tr.type, raw.data_ptr() + e * gb, rows, n_in,
                           packed.data_ptr() + e * pb, None)
                self.dev[name] = packed
            else:
                self.dev[name] = raw
        d = self.dev
        self.w = Q.MoeWeights(d["post_attention_norm.weight"].data_ptr(), d["ffn_gate_inp.weight"].data_ptr(),
                              d["ffn_gate_exps.weight"].data_ptr(), d["ffn_up_exps.weight"].data_ptr(),
                              d["ffn_down_exps.weight"].data_ptr(), d["ffn_gate_inp_shexp.weight"].data_ptr(),
                              d["ffn_gate_shexp.weight"].data_ptr(), d["ffn_up_shexp.weight"].data_ptr(),
                              d["ffn_down_shexp.weight"].data_ptr(), down_type, down_type)
        torch.cuda.synchronize()

    def oracle(self, x2):
        T = x2.shape[0]
        out = np.zeros((T, 2048), np.float32)
        sel = np.zeros((T, 8), np.int32)
        w = np.zeros((T, 8), np.float32)
        self.O.lib().qo_moe_block(self.model, self.il, self.O._ptr(x2), T, self.O._ptr(out),
                                  self.O._ptr(sel), self.O._ptr(w))
        return out, sel, w

    def gpu(self, x2, scratch=None):
        import torch
        import ctypes as C
        Q = self.Q
        T = x2.shape[0]
        dx = to_dev(x2)
        out = empty_dev((T, 2048), torch.float32)
        sel = empty_dev((T, 8), torch.int32)
        w = empty_dev((T, 8), torch.float32)
        nb = Q.lib().qma_cuda_moe_scratch_bytes(T)
        if scratch is None:
            scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
        Q.call("qma_cuda_moe_layer", C.byref(self.w), Q.ptr(dx), T, Q.ptr(out), Q.ptr(sel),
               Q.ptr(w), Q.ptr(scratch), nb, None)
        torch.cuda.synchronize()
        fb = C.c_int(0)
        Q.call("qma_cuda_moe_exact_fallbacks", Q.ptr(scratch), T, C.byref(fb))
        return out.cpu().numpy(), sel.cpu().numpy(), w.cpu().numpy(), fb.value

    def close(self):
        self.O.lib().qo_model_free(self.model)

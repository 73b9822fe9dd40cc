"""ctypes bindings of the CPU oracle (TEST INFRASTRUCTURE).

Loads ``oracle/liboracle.so`` (the C restatement of the qma hot path) and,
when it was built, ``oracle/_ref/libqmaref.so`` (the qma reference compiled
from its own sources).  Only tests/, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` import this module; the CUDA engine never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libqmaref.so")

F32, Q8_0, Q4_K, Q6_K = 0, 8, 12, 14
EMBD, FF, EXPERT, LAYER = 2048, 512, 256, 40
N_VOCAB = 151936


class Tensor(C.Structure):
    """One entry of a GGUF-style tensor table (mirrors tensor_t, qma.h:155-161)."""

    _fields_ = [("name", C.c_char * 64), ("type", C.c_uint32), ("ne", C.c_int64 * 3),
                ("off", C.c_uint64), ("nbytes", C.c_uint64)]


class SynthCfg(C.Structure):
    _fields_ = [("n_vocab", C.c_int), ("embd_type", C.c_int), ("out_type", C.c_int),
                ("down_type", C.c_int), ("proj_type", C.c_int)]


def build() -> None:
    """Compile liboracle.so (and _ref/ when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _ptr(a: np.ndarray, ctype=C.c_void_p):
    return a.ctypes.data_as(ctype)


_lib = None
_ref = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        vp, i32, f32 = C.c_void_p, C.c_int, C.c_float
        L.qo_set_threads.argtypes = [i32]
        L.qo_half_to_float.argtypes = [C.c_uint16]
        L.qo_half_to_float.restype = f32
        L.qo_float_to_half.argtypes = [f32]
        L.qo_float_to_half.restype = C.c_uint16
        L.qo_q8k_quant.argtypes = [vp, i32, vp, vp, vp]
        for fn in ("qo_dot_q4k",):
            getattr(L, fn).argtypes = [vp, vp, vp, vp, i32, vp]
            getattr(L, fn).restype = f32
        for fn in ("qo_dot_q6k", "qo_dot_q80"):
            getattr(L, fn).argtypes = [vp, vp, vp, i32, vp]
            getattr(L, fn).restype = f32
        L.qo_gateup_q4k.argtypes = [vp, vp, vp, vp, vp, i32, vp, vp]
        L.qo_dot.argtypes = [vp, i32, vp, vp, vp, i32]
        L.qo_dot.restype = f32
        L.qo_dequant_row.argtypes = [vp, i32, vp, i32]
        L.qo_matmul.argtypes = [vp, vp, i32, i32, i32, i32, vp]
        for fn in ("qo_quantize_q4k", "qo_quantize_q6k", "qo_quantize_q80"):
            getattr(L, fn).argtypes = [vp, vp]
        L.qo_synth_layout.argtypes = [C.POINTER(SynthCfg), C.POINTER(Tensor), i32,
                                      C.POINTER(C.c_uint64)]
        L.qo_synth_layout.restype = i32
        L.qo_synth_tensor.argtypes = [C.POINTER(Tensor), vp, C.c_uint64, i32]
        L.qo_model_new.argtypes = [C.POINTER(Tensor), i32, vp, i32]
        L.qo_model_new.restype = vp
        L.qo_model_free.argtypes = [vp]
        L.qo_moe_ffn.argtypes = [vp, i32, vp, i32, vp, vp, vp]
        L.qo_moe_block.argtypes = [vp, i32, vp, i32, vp, vp, vp]
        L.qo_moe_block_biased.argtypes = [vp, i32, vp, i32, vp, vp, vp, vp]
        L.qo_router_logits.argtypes = [vp, vp, vp]
        L.qo_route.argtypes = [vp, vp, vp, i32, vp, vp]
        L.qo_moe_route.argtypes = [vp, vp, vp, vp, i32, vp, vp]
        L.qo_state_new.argtypes = [i32]
        L.qo_state_new.restype = vp
        L.qo_state_free.argtypes = [vp]
        L.qo_state_n_pos.argtypes = [vp]
        L.qo_state_n_pos.restype = i32
        L.qo_eval.argtypes = [vp, vp, vp, i32, vp, i32]
        L.qo_eval.restype = i32
        L.qo_eval_hidden.argtypes = [vp, vp, vp, i32, i32, vp]
        L.qo_eval_hidden.restype = i32
        L.qo_layer_forward.argtypes = [vp, vp, i32, vp, i32, i32, vp]
        L.qo_mixer_forward.argtypes = [vp, vp, i32, vp, i32, vp]
        L.qo_state_resume.argtypes = [vp, C.c_char_p, C.c_char_p, i32]
        L.qo_state_resume.restype = i32
        L.qo_state_live_segments.argtypes = [vp, vp, vp, vp]
        L.qo_state_kv_slot.argtypes = [vp, i32, i32, i32]
        L.qo_state_kv_slot.restype = C.POINTER(C.c_uint8)
        L.qo_gdn_layer.argtypes = [vp, vp, i32, vp, i32, vp]
        L.qo_state_conv.argtypes = [vp, i32]
        L.qo_state_conv.restype = C.POINTER(C.c_float)
        L.qo_state_ssm.argtypes = [vp, i32]
        L.qo_state_ssm.restype = C.POINTER(C.c_float)
        for fn in ("qo_kvq4_quant", "qo_kvq2_quant"):
            getattr(L, fn).argtypes = [vp, vp]
        for fn in ("qo_kvq4_dot", "qo_kvq2_dot", "qo_kvq4_qf"):
            getattr(L, fn).argtypes = [vp, vp]
            getattr(L, fn).restype = f32
        for fn in ("qo_kvq4_vacc", "qo_kvq2_vacc"):
            getattr(L, fn).argtypes = [vp, f32, vp]
        L.qo_set_threads(min(os.cpu_count() or 1, 64))
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref() -> C.CDLL:
    """The reference engine compiled from its own sources (one per process:
    its HCM and routing history are process-global statics, nn.c:40-57)."""
    global _ref
    if _ref is None:
        R = C.CDLL(REF_PATH)
        vp, i32, f32 = C.c_void_p, C.c_int, C.c_float
        R.qr_init.argtypes = [i32]
        R.qr_n_vocab.restype = i32
        R.qr_model_new.argtypes = [C.POINTER(Tensor), i32, vp, C.c_uint64]
        R.qr_model_new.restype = vp
        R.qr_model_free.argtypes = [vp]
        R.qr_state_new.argtypes = [i32]
        R.qr_state_new.restype = vp
        R.qr_state_free.argtypes = [vp]
        R.qr_eval.argtypes = [vp, vp, vp, i32, vp, i32, i32]
        R.qr_eval.restype = i32
        R.qr_moe_ffn.argtypes = [vp, i32, vp, i32, vp, vp]
        R.qr_gdn_layer.argtypes = [vp, vp, i32, vp, i32, vp]
        R.qr_matmul.argtypes = [vp, vp, i32, i32, i32, i32, vp, i32]
        R.qr_state_conv.argtypes = [vp, i32]
        R.qr_state_conv.restype = C.POINTER(C.c_float)
        R.qr_state_ssm.argtypes = [vp, i32]
        R.qr_state_ssm.restype = C.POINTER(C.c_float)
        R.qr_half_to_float.argtypes = [C.c_uint16]
        R.qr_half_to_float.restype = f32
        R.qr_float_to_half.argtypes = [f32]
        R.qr_float_to_half.restype = C.c_uint16
        R.qr_gguf_load.argtypes = [C.c_char_p, C.POINTER(Tensor), i32, C.POINTER(C.c_int),
                                   C.POINTER(C.c_uint64), C.POINTER(C.c_int), C.c_char_p, i32]
        R.qr_gguf_load.restype = i32
        R.qr_sampler_candidates.argtypes = [i32, vp, vp, i32, f32, f32, i32, vp, vp, i32]
        R.qr_sampler_candidates.restype = i32
        R.qr_runstate_load.argtypes = [vp, C.c_char_p]
        R.qr_runstate_load.restype = i32
        R.qr_state_n_pos.argtypes = [vp]
        R.qr_state_n_pos.restype = i32
        R.qma_q8k_quant.argtypes = [vp, i32, vp, vp, vp]
        R.qma_q8k_dot.argtypes = [vp, i32, vp, vp, vp, i32]
        R.qma_q8k_dot.restype = f32
        R.qma_q8k_gateup.argtypes = [vp, vp, vp, vp, vp, i32, vp, vp]
        for fn in ("kvq4_quant", "kvq2_quant"):
            getattr(R, fn).argtypes = [vp, i32, vp]
        for fn in ("kvq4_dot", "kvq2_dot", "kvq4_qf"):
            getattr(R, fn).argtypes = [vp, vp, i32]
            getattr(R, fn).restype = f32
        for fn in ("kvq4_vacc", "kvq2_vacc"):
            getattr(R, fn).argtypes = [vp, f32, vp, i32]
        R.dequantize_row_q4_K.argtypes = [vp, vp, C.c_int64]
        R.dequantize_row_q6_K.argtypes = [vp, vp, C.c_int64]
        _ref = R
    return _ref


# --------------------------------------------------------------- helpers --
def row_bytes(wtype: int, n_in: int) -> int:
    return {Q4_K: n_in // 256 * 144, Q6_K: n_in // 256 * 210, Q8_0: n_in // 32 * 34,
            F32: n_in * 4}[wtype]


def q8k_quant(x: np.ndarray):
    """Q8_K-quantize rows of x [T][n] -> (xq int8 [T][n], xd f32 [T][n/256], xsum i16 [T][n/16])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    x2 = x.reshape(-1, x.shape[-1])
    T, n = x2.shape
    xq = np.zeros((T, n), np.int8)
    xd = np.zeros((T, n // 256), np.float32)
    xs = np.zeros((T, n // 16), np.int16)
    L = lib()
    for t in range(T):
        L.qo_q8k_quant(_ptr(x2[t]), n, _ptr(xq[t]), _ptr(xd[t]), _ptr(xs[t]))
    return xq, xd, xs


def quantize_rows(w: np.ndarray, wtype: int) -> np.ndarray:
    """Quantize fp32 rows [R][n] into GGUF blocks with the engine's quantizer."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    R, n = w.shape
    per = 32 if wtype == Q8_0 else 256
    bb = {Q4_K: 144, Q6_K: 210, Q8_0: 34}[wtype]
    out = np.zeros((R, n // per * bb), np.uint8)
    fn = {Q4_K: lib().qo_quantize_q4k, Q6_K: lib().qo_quantize_q6k, Q8_0: lib().qo_quantize_q80}[wtype]
    for r in range(R):
        for b in range(n // per):
            fn(_ptr(w[r, b * per:]), _ptr(out[r, b * bb:]))
    return out


def matmul(x: np.ndarray, W: np.ndarray, wtype: int, n_in: int, n_out: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_in)
    out = np.zeros((x.shape[0], n_out), np.float32)
    lib().qo_matmul(_ptr(x), _ptr(W), n_in, n_out, x.shape[0], wtype, _ptr(out))
    return out


def zipf_router_bias(seed: int, layer: int, s: float = 1.1, n: int = 256) -> np.ndarray:
    """configs[4]'s router prior for one layer: expert e gets log p(rank),
    p(r) = r^-s / sum_k k^-s, over a seeded per-layer random ranking of the
    experts (a skewed expert load).  float32 [n]."""
    rank = np.random.default_rng([seed, layer]).permutation(n) + 1
    p = rank.astype(np.float64) ** -s
    return np.log(p / p.sum()).astype(np.float32)


def moe_route(post_norm: np.ndarray, gate_inp: np.ndarray, x2: np.ndarray, bias=None):
    """Routing of the FFN half of a layer (rms_norm_m * post_norm, then the
    router of moe_ffn, nn.c:513-551) for tokens x2 [T][2048]: (sel int32
    [T][8], w float32 [T][8]) in selection order.  bias (256 floats,
    optional) is added to each logit (the configs[4] router prior)."""
    x2 = np.ascontiguousarray(x2, dtype=np.float32).reshape(-1, 2048)
    pn = np.ascontiguousarray(post_norm, dtype=np.float32)
    gi = np.ascontiguousarray(gate_inp, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    T = x2.shape[0]
    sel = np.zeros((T, 8), np.int32)
    w = np.zeros((T, 8), np.float32)
    lib().qo_moe_route(_ptr(pn), _ptr(gi), None if b is None else _ptr(b), _ptr(x2), T, _ptr(sel), _ptr(w))
    return sel, w


def dot_partials(W: np.ndarray, wtype: int, n_in: int, xq, xd, xs):
    """Per-row fp32 dots and exact int32 partials (per 32-lane sub-block for
    Q4_K/Q8_0, per super-block for Q6_K) of one Q8_K-quantized token."""
    L = lib()
    rows = W.shape[0]
    per = n_in // 256 if wtype == Q6_K else n_in // 32
    isum = np.zeros((rows, per), np.int32)
    out = np.zeros(rows, np.float32)
    for r in range(rows):
        if wtype == Q4_K:
            out[r] = L.qo_dot_q4k(_ptr(W[r]), _ptr(xq), _ptr(xd), _ptr(xs), n_in, _ptr(isum[r]))
        elif wtype == Q6_K:
            out[r] = L.qo_dot_q6k(_ptr(W[r]), _ptr(xq), _ptr(xd), n_in, _ptr(isum[r]))
        else:
            out[r] = L.qo_dot_q80(_ptr(W[r]), _ptr(xq), _ptr(xd), n_in, _ptr(isum[r]))
    return out, isum


# --------------------------------------------------------- synthetic model --
def synth_layout(n_vocab=N_VOCAB, embd_type=Q8_0, out_type=Q8_0, down_type=Q6_K, proj_type=Q4_K):
    cfg = SynthCfg(n_vocab, embd_type, out_type, down_type, proj_type)
    cap = 1024
    arr = (Tensor * cap)()
    size = C.c_uint64(0)
    n = lib().qo_synth_layout(C.byref(cfg), arr, cap, C.byref(size))
    assert n > 0
    return arr, n, int(size.value)


def tensor_index(arr, n) -> dict:
    return {arr[i].name.decode(): i for i in range(n)}


def synth_matrix(name: str, wtype: int, rows: int, n: int, seed: int = 0,
                 threads=None) -> np.ndarray:
    """GGUF-layout bytes [rows][row_bytes] of one synthetic weight matrix,
    values a seeded function of (seed, name, index), N(0, 0.02) before
    quantization (F32 matrices are returned as raw float bytes)."""
    t = Tensor()
    t.name = name.encode()
    t.type = wtype
    t.ne[0], t.ne[1], t.ne[2] = n, rows, 1
    t.off = 0
    rb = row_bytes(wtype, n)
    t.nbytes = rb * rows
    out = np.zeros((rows, rb), np.uint8)
    lib().qo_synth_tensor(C.byref(t), _ptr(out), seed, threads or min(os.cpu_count() or 1, 32))
    return out


def synth_blob(arr, n, size, seed, names=None, threads=None) -> np.ndarray:
    """Generate the synthetic data section (all tensors, or only `names`)."""
    blob = np.zeros(size, np.uint8)
    th = threads or min(os.cpu_count() or 1, 32)
    for i in range(n):
        if names is not None and arr[i].name.decode() not in names:
            continue
        lib().qo_synth_tensor(C.byref(arr[i]), _ptr(blob), seed, th)
    return blob

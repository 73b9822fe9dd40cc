"""ctypes binding of libqma_cuda.so, the engine's C ABI (include/qma_cuda.h).

This is the host-side mirror a Python caller (tests, bench) uses; C callers
(qma's own nn.c) link the library directly.  Device memory is passed as raw
pointers: torch tensors are used only as allocators (``t.data_ptr()``).

The library must exist: there is no fallback of any kind.  Build it with
``make -C qwen-mobile-agent_b200`` (``__graft_entry__.build()`` does).
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqma_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "qma_cuda.h")

OK = 0
ERR_INVALID, ERR_NOMEM, ERR_CUDA, ERR_UNSUPPORTED, ERR_STATE, ERR_TIMEOUT = -1, -2, -3, -4, -5, -6
F32, Q8_0, Q4_K, Q6_K = 0, 8, 12, 14

_vp, _i32, _f32, _u64, _sz = C.c_void_p, C.c_int, C.c_float, C.c_uint64, C.c_size_t

# name -> (restype, argtypes); every function declared in the header
_SIGS = {
    "qma_cuda_abi_version": (_i32, []),
    "qma_cuda_last_error": (C.c_char_p, []),
    "qma_cuda_init": (_i32, [_i32]),
    "qma_cuda_q8k_quant": (_i32, [_vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    "qma_cuda_packed_bytes": (_sz, [_i32, _i32, _i32]),
    "qma_cuda_repack": (_i32, [_i32, _vp, _i32, _i32, _vp, _vp]),
    "qma_cuda_matvec": (_i32, [_i32, _vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "qma_cuda_dot_partials": (_i32, [_i32, _vp, _i32, _i32, _vp, _vp, _vp]),
    "qma_cuda_synth_tensor": (_i32, [C.c_char_p, _i32, _u64, _u64, _vp, _vp]),
    "qma_cuda_moe_scratch_bytes": (_sz, [_i32]),
    "qma_cuda_moe_layer": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "qma_cuda_moe_exact_fallbacks": (_i32, [_vp, _i32, C.POINTER(C.c_int)]),
    "qma_cuda_moe_layer_noalloc": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp]),
}


class Tensor(C.Structure):
    """qma_cuda_tensor: one GGUF-style tensor (the layout of tensor_t, qma.h:155-161)."""

    _fields_ = [("name", C.c_char * 64), ("type", C.c_uint32), ("ne", C.c_int64 * 3),
                ("off", C.c_uint64), ("nbytes", C.c_uint64)]


_TP = C.POINTER(Tensor)
_SIGS.update({
    "qma_cuda_model_load": (_i32, [_i32, _TP, C.c_uint32, _vp, _u64, C.POINTER(_vp)]),
    "qma_cuda_model_synth": (_i32, [_i32, _TP, C.c_uint32, _u64, C.POINTER(_vp)]),
    "qma_cuda_model_check": (_i32, [_TP, C.c_uint32, _u64]),
    "qma_cuda_gguf_scan": (_i32, [C.c_char_p, _TP, C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(_u64),
                                  C.POINTER(_u64)]),
    "qma_cuda_model_load_gguf": (_i32, [_i32, C.c_char_p, C.POINTER(_vp)]),
    "qma_cuda_model_free": (_i32, [_vp]),
    "qma_cuda_model_n_vocab": (_i32, [_vp]),
    "qma_cuda_ecache_get": (_i32, [_vp, _i32, _i32, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp)]),
    "qma_cuda_ecache_hint": (_i32, [_vp, _i32, _vp, _i32, _vp]),
    "qma_cuda_ecache_prefetch": (_i32, [_vp, _i32, _vp, _i32, _vp]),
    "qma_cuda_ecache_hold": (_i32, [_vp, _i32, _i32, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp)]),
    "qma_cuda_ecache_release": (_i32, [_vp]),
    "qma_cuda_ecache_held": (_i32, [_vp]),
    "qma_cuda_state_create": (_i32, [_vp, _i32, C.POINTER(_vp)]),
    "qma_cuda_state_free": (_i32, [_vp]),
    "qma_cuda_state_n_pos": (_i32, [_vp]),
    "qma_cuda_eval": (_i32, [_vp, _vp, _vp, _i32, _vp, _i32]),
    "qma_cuda_decode_greedy": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp]),
    "qma_cuda_eval_hidden": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "qma_cuda_gdn_step": (_i32, [_vp, _i32, _vp, _i32, _vp, _i32]),
    "qma_cuda_gdn_decode": (_i32, [_vp, _i32, _vp, _i32, _vp]),
    "qma_cuda_attn_decode": (_i32, [_vp, _i32, _vp, _i32, _vp, _i32]),
    "qma_cuda_state_stream": (_vp, [_vp]),
    "qma_cuda_state_kv_slot": (_i32, [_vp, _i32, _i32, _i32, _vp]),
    "qma_cuda_state_stats": (_i32, [_vp, C.POINTER(_i32), C.POINTER(_u64)]),
    "qma_cuda_state_logits": (_vp, [_vp]),
    "qma_cuda_state_save": (_i32, [_vp, C.c_char_p, C.c_char_p, C.c_char_p]),
    "qma_cuda_state_load": (_i32, [_vp, C.c_char_p, C.c_char_p, C.c_char_p]),
    "qma_cuda_sample_candidates": (_i32, [_vp, _i32, _vp, _i32, _f32, _f32, _i32, _i32, _vp, _vp,
                                          C.POINTER(_i32), _vp]),
})


# ----------------------------------------------------- synthetic model table --
# The qwen35moe tensor table (the reference's tensor names, gguf.c:302-345,
# with the shapes of the hyper-parameters in qma.h:28-64) over one data
# section, each tensor 256-byte aligned: what a random-init model is
# generated into (qma_cuda_model_synth) or loaded from.
_BLOCK = {F32: (4, 1), Q8_0: (34, 32), Q4_K: (144, 256), Q6_K: (210, 256)}


def row_bytes(wtype: int, n: int) -> int:
    """GGUF bytes of one row of n elements of type wtype."""
    bs, blk = _BLOCK[wtype]
    return n // blk * bs


def synth_layout(n_vocab=151936, embd_type=Q8_0, out_type=Q8_0, down_type=Q6_K, proj_type=Q4_K):
    """(Tensor array, count, data-section bytes) of the 40-layer qwen35moe."""
    E, FF, NE = 2048, 512, 256
    t = []

    def add(name, typ, ne0, ne1=1, ne2=1):
        t.append((name, typ, (ne0, ne1, ne2)))

    add("token_embd.weight", embd_type, E, n_vocab)
    add("output_norm.weight", F32, E)
    add("output.weight", out_type, E, n_vocab)
    for il in range(40):
        b = f"blk.{il}."
        add(b + "attn_norm.weight", F32, E)
        add(b + "post_attention_norm.weight", F32, E)
        if (il + 1) % 4 == 0:                       # gated full attention
            add(b + "attn_q.weight", proj_type, E, 8192)
            add(b + "attn_k.weight", proj_type, E, 512)
            add(b + "attn_v.weight", proj_type, E, 512)
            add(b + "attn_output.weight", proj_type, 4096, E)
            add(b + "attn_q_norm.weight", F32, 256)
            add(b + "attn_k_norm.weight", F32, 256)
        else:                                       # gated delta net
            add(b + "attn_qkv.weight", proj_type, E, 8192)
            add(b + "attn_gate.weight", proj_type, E, 4096)
            add(b + "ssm_conv1d.weight", F32, 4, 8192)
            add(b + "ssm_dt.bias", F32, 32)
            add(b + "ssm_a", F32, 32)
            add(b + "ssm_beta.weight", proj_type, E, 32)
            add(b + "ssm_alpha.weight", proj_type, E, 32)
            add(b + "ssm_norm.weight", F32, 128)
            add(b + "ssm_out.weight", proj_type, 4096, E)
        add(b + "ffn_gate_inp.weight", F32, E, NE)
        add(b + "ffn_gate_exps.weight", Q4_K, E, FF, NE)
        add(b + "ffn_up_exps.weight", Q4_K, E, FF, NE)
        add(b + "ffn_down_exps.weight", down_type, FF, E, NE)
        add(b + "ffn_gate_inp_shexp.weight", F32, E)
        add(b + "ffn_gate_shexp.weight", Q4_K, E, FF)
        add(b + "ffn_up_shexp.weight", Q4_K, E, FF)
        add(b + "ffn_down_shexp.weight", down_type, FF, E)
    arr = (Tensor * len(t))()
    off = 0
    for i, (name, typ, ne) in enumerate(t):
        arr[i].name = name.encode()
        arr[i].type = typ
        for d in range(3):
            arr[i].ne[d] = ne[d]
        arr[i].off = off
        arr[i].nbytes = row_bytes(typ, ne[0]) * ne[1] * ne[2]
        off += (arr[i].nbytes + 255) // 256 * 256
    return arr, len(t), off


def tensor_index(arr, n) -> dict:
    return {arr[i].name.decode(): i for i in range(n)}


def model_check(arr, n, data_size: int = 0) -> None:
    """qma_cuda_model_check: raise QmaError unless the table has every
    tensor with the shapes and types the kernels are written for."""
    call("qma_cuda_model_check", arr, n, data_size)


def gguf_scan(path: str):
    """qma_cuda_gguf_scan: (tensor table, count, data section offset in the
    file, tokenizer token count)."""
    n, off, ntok = C.c_uint32(), C.c_uint64(), C.c_uint64()
    call("qma_cuda_gguf_scan", path.encode(), None, 0, C.byref(n), C.byref(off), C.byref(ntok))
    arr = (Tensor * max(n.value, 1))()
    call("qma_cuda_gguf_scan", path.encode(), arr, n.value, C.byref(n), C.byref(off), C.byref(ntok))
    return arr, n.value, off.value, ntok.value


class Model:
    """Device-resident qwen35moe weights (qma_cuda_model): from a tensor
    table plus a host data section, from random-init weights generated on
    the device (seed), or from a GGUF file (gguf=path)."""

    def __init__(self, tensors=None, n=0, host_blob=None, seed=None, device=0, gguf=None):
        h = _vp()
        if gguf is not None:
            call("qma_cuda_model_load_gguf", device, gguf.encode(), C.byref(h))
        elif host_blob is not None:
            call("qma_cuda_model_load", device, tensors, n, ptr(host_blob), host_blob.nbytes, C.byref(h))
        else:
            call("qma_cuda_model_synth", device, tensors, n, seed, C.byref(h))
        self.h = h
        self.n_vocab = lib().qma_cuda_model_n_vocab(h)

    def close(self):
        if self.h:
            call("qma_cuda_model_free", self.h)
            self.h = None


class State:
    """One sequence (qma_cuda_state): KV ring, recurrent state, HCM tiers."""

    def __init__(self, model: Model, n_ctx: int):
        h = _vp()
        call("qma_cuda_state_create", model.h, n_ctx, C.byref(h))
        self.h, self.model = h, model

    @property
    def n_pos(self) -> int:
        return lib().qma_cuda_state_n_pos(self.h)

    def eval(self, tokens, logits_all=False):
        import numpy as np
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        rows = len(toks) if logits_all else 1
        out = np.zeros((rows, self.model.n_vocab), np.float32)
        call("qma_cuda_eval", self.model.h, self.h, ptr(toks), len(toks), ptr(out), int(logits_all))
        return out if logits_all else out[0]

    def eval_hidden(self, tokens, n_layers: int):
        import numpy as np
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros((len(toks), 2048), np.float32)
        call("qma_cuda_eval_hidden", self.model.h, self.h, ptr(toks), len(toks), n_layers, ptr(out))
        return out

    def save(self, state_path=None, kv_path=None, salience_path=None):
        enc = lambda p: None if p is None else str(p).encode()
        call("qma_cuda_state_save", self.h, enc(state_path), enc(kv_path), enc(salience_path))

    def load(self, state_path=None, kv_path=None, salience_path=None):
        enc = lambda p: None if p is None else str(p).encode()
        call("qma_cuda_state_load", self.h, enc(state_path), enc(kv_path), enc(salience_path))

    def decode_greedy(self, token: int, n_steps: int):
        import numpy as np
        toks = np.zeros(n_steps, np.int32)
        logits = np.zeros(self.model.n_vocab, np.float32)
        call("qma_cuda_decode_greedy", self.model.h, self.h, token, n_steps, ptr(toks), ptr(logits))
        return toks, logits

    def close(self):
        if self.h:
            call("qma_cuda_state_free", self.h)
            self.h = None


class MoeWeights(C.Structure):
    """qma_cuda_moe_weights: device pointers of one layer's MoE tensors."""

    _fields_ = [("post_norm", _vp), ("gate_inp", _vp), ("gate_exps", _vp), ("up_exps", _vp),
                ("down_exps", _vp), ("gate_inp_shexp", _vp), ("gate_shexp", _vp),
                ("up_shexp", _vp), ("down_shexp", _vp), ("down_type", _i32),
                ("down_shexp_type", _i32), ("router_bias", _vp)]


_SIGS["qma_cuda_model_moe_weights"] = (_i32, [_vp, _i32, C.POINTER(MoeWeights)])
_SIGS["qma_cuda_model_set_router_bias"] = (_i32, [_vp, _i32, _vp])
_SIGS.update({
    "qma_cuda_ep_unique_id": (_i32, [_vp]),
    "qma_cuda_ep_init": (_i32, [_i32, _vp, _i32, _i32, _i32, C.POINTER(_vp)]),
    "qma_cuda_ep_init_timeout": (_i32, [_i32, _vp, _i32, _i32, _i32, _i32, C.POINTER(_vp)]),
    "qma_cuda_ep_free": (_i32, [_vp]),
    "qma_cuda_ep_moe_layer": (_i32, [_vp, C.POINTER(MoeWeights), _vp, _i32, _vp, _vp, _vp, _vp]),
    "qma_cuda_ep_stats": (_i32, [_vp, C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_i32)]),
    "qma_cuda_ep_sync": (_i32, [_vp, _vp]),
    "qma_cuda_batch_create": (_i32, [_vp, _i32, _i32, C.POINTER(_vp)]),
    "qma_cuda_batch_free": (_i32, [_vp]),
    "qma_cuda_batch_n_seq": (_i32, [_vp]),
    "qma_cuda_batch_seq": (_vp, [_vp, _i32]),
    "qma_cuda_batch_eval": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "qma_cuda_batch_eval_hidden": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "qma_cuda_batch_logits": (_vp, [_vp]),
    "qma_cuda_batch_set_ep": (_i32, [_vp, _vp, C.POINTER(MoeWeights)]),
})

EP_UID_BYTES = 128
N_EXPERT = 256


def ep_shard(rank: int, n_ranks: int) -> tuple[int, int]:
    """(first expert, expert count) of a rank's shard: rank r owns experts
    r * 256/N .. (r + 1) * 256/N - 1."""
    if n_ranks < 1 or n_ranks > 8 or N_EXPERT % n_ranks or not 0 <= rank < n_ranks:
        raise ValueError(f"rank {rank} of {n_ranks}: 1..8 ranks dividing 256")
    n_local = N_EXPERT // n_ranks
    return rank * n_local, n_local


class ExpertParallel:
    """One rank's handle on the expert-parallel MoE block (qma_cuda_ep_*).

    share_uid(uid_or_None) -> bytes carries the communicator id from rank 0
    to the others (rank 0 passes its id and gets it back; the others pass
    None): a torch.distributed broadcast, a store, a file."""

    def __init__(self, device: int, rank: int, n_ranks: int, t_max: int, share_uid, timeout_ms=None):
        ep_shard(rank, n_ranks)
        uid = (C.c_uint8 * EP_UID_BYTES)()
        if rank == 0:
            call("qma_cuda_ep_unique_id", uid)
        raw = share_uid(bytes(uid) if rank == 0 else None)
        if len(raw) != EP_UID_BYTES:
            raise ValueError(f"communicator id of {len(raw)} bytes")
        uid = (C.c_uint8 * EP_UID_BYTES).from_buffer_copy(raw)
        h = _vp()
        if timeout_ms is None:
            call("qma_cuda_ep_init", device, uid, rank, n_ranks, t_max, C.byref(h))
        else:
            call("qma_cuda_ep_init_timeout", device, uid, rank, n_ranks, t_max, int(timeout_ms), C.byref(h))
        self.h, self.rank, self.n_ranks, self.t_max = h, rank, n_ranks, t_max

    def moe_layer(self, w: MoeWeights, x2, T: int, x_out, sel=None, wts=None, stream=None) -> None:
        call("qma_cuda_ep_moe_layer", self.h, C.byref(w), ptr(x2), T, ptr(x_out), ptr(sel), ptr(wts), stream)

    def sync(self, stream=None) -> None:
        """Bounded wait for the stream's work, exchanges included."""
        call("qma_cuda_ep_sync", self.h, stream)

    def stats(self) -> tuple[int, int, int]:
        s, r, n = C.c_uint64(), C.c_uint64(), C.c_int()
        call("qma_cuda_ep_stats", self.h, C.byref(s), C.byref(r), C.byref(n))
        return s.value, r.value, n.value

    def close(self) -> None:
        if self.h:
            call("qma_cuda_ep_free", self.h)
            self.h = None


class Batch:
    """n_seq sequences decoded together (qma_cuda_batch)."""

    def __init__(self, model: Model, n_seq: int, n_ctx: int):
        h = _vp()
        call("qma_cuda_batch_create", model.h, n_seq, n_ctx, C.byref(h))
        self.h, self.model, self.n_seq = h, model, n_seq
        self._ep_w = None

    def n_pos(self, seq: int) -> int:
        return lib().qma_cuda_state_n_pos(lib().qma_cuda_batch_seq(self.h, seq))

    def eval(self, seq_ids, tokens, logits=True, greedy=True):
        """(logits [n][n_vocab] or None, greedy [n] or None); rows of each
        sequence's last token in the call are filled (-1 / 0 elsewhere)."""
        import numpy as np
        sids = np.ascontiguousarray(seq_ids, dtype=np.int32)
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        if len(sids) != len(toks):
            raise ValueError("seq_ids and tokens differ in length")
        lo = np.zeros((len(toks), self.model.n_vocab), np.float32) if logits else None
        g = np.full(len(toks), -1, np.int32) if greedy else None
        call("qma_cuda_batch_eval", self.h, ptr(sids), ptr(toks), len(toks), ptr(lo), ptr(g))
        return lo, g

    def eval_hidden(self, seq_ids, tokens, n_layers: int):
        import numpy as np
        sids = np.ascontiguousarray(seq_ids, dtype=np.int32)
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros((len(toks), 2048), np.float32)
        call("qma_cuda_batch_eval_hidden", self.h, ptr(sids), ptr(toks), len(toks), n_layers, ptr(out))
        return out

    def set_ep(self, ep, shard_weights) -> None:
        """Route the MoE blocks through ep (an ExpertParallel) with this
        rank's 40 shard views; ep None restores the local block."""
        if ep is None:
            call("qma_cuda_batch_set_ep", self.h, None, None)
            self._ep_w = None
            return
        arr = (MoeWeights * len(shard_weights))(*shard_weights)
        call("qma_cuda_batch_set_ep", self.h, ep.h, arr)
        self._ep_w = arr

    def close(self):
        if self.h:
            call("qma_cuda_batch_free", self.h)
            self.h = None


class QmaError(RuntimeError):
    """A qma_cuda_* call returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} -> {status}: {msg}")
        self.status = status


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build the CUDA engine (make -C {HERE}); "
                "there is no CPU fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def declared_functions() -> list[str]:
    """Every qma_cuda_* function declared in include/qma_cuda.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(qma_cuda_[a-z0-9_]+)\s*\(", text)))


def last_error() -> str:
    return lib().qma_cuda_last_error().decode()


def call(name: str, *args) -> int:
    """Call a status-returning entry point; raise QmaError on failure."""
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        raise QmaError(name, rc, last_error())
    return rc


def ptr(t) -> int:
    """Raw device (or host) address of a torch tensor / numpy array / int."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    return t.ctypes.data


def init(device: int = 0) -> None:
    call("qma_cuda_init", device)


def packed_bytes(wtype: int, rows: int, n: int) -> int:
    return int(lib().qma_cuda_packed_bytes(wtype, rows, n))

"""The C-ABI library loads on a CPU-only machine, exports every function the
header declares, and rejects bad arguments with a status (no GPU needed)."""
import ctypes as C
import os

import pytest

import qma_cuda as Q


def test_library_exports_every_declared_symbol():
    lib = Q.lib()
    declared = Q.declared_functions()
    assert len(declared) >= 8
    missing = [f for f in declared if not hasattr(lib, f)]
    assert not missing, f"declared in qma_cuda.h but not exported: {missing}"
    unbound = [f for f in declared if f not in Q._SIGS]
    assert not unbound, f"no ctypes signature for {unbound}"


def test_abi_version():
    assert Q.lib().qma_cuda_abi_version() == 2


def test_bad_arguments_return_invalid_without_touching_the_device():
    lib = Q.lib()
    assert lib.qma_cuda_matvec(Q.Q4_K, None, 2048, 8, 1, None, None, None, None, None) == Q.ERR_INVALID
    assert "qma_cuda_matvec" in Q.last_error()
    assert lib.qma_cuda_matvec(Q.Q4_K, 1, 100, 8, 1, 1, 1, 1, 1, None) == Q.ERR_INVALID  # n_in % 256
    assert lib.qma_cuda_q8k_quant(None, 1, 256, None, None, None, None) == Q.ERR_INVALID
    assert lib.qma_cuda_repack(Q.Q6_K, None, 4, 512, None, None) == Q.ERR_INVALID


def test_misaligned_device_pointers_are_refused():
    lib = Q.lib()
    # 16-byte vector loads read the activation sums and rows: an unaligned
    # buffer is refused before anything is launched
    assert lib.qma_cuda_matvec(Q.Q4_K, 256, 2048, 16, 16, 256, 256, 258, 256, None) == Q.ERR_INVALID
    assert lib.qma_cuda_matvec(Q.Q4_K, 256, 2048, 16, 16, 264, 256, 256, 256, None) == Q.ERR_INVALID
    assert "aligned" in Q.last_error()
    w = Q.MoeWeights(*([256] * 9), Q.Q6_K, Q.Q6_K)
    assert lib.qma_cuda_moe_layer(C.byref(w), 260, 1, 256, None, None, 512, 1 << 20, None) == Q.ERR_INVALID
    assert lib.qma_cuda_moe_layer(C.byref(w), 256, 1, 256, None, None, 512 + 16, 1 << 20, None) == Q.ERR_INVALID
    assert lib.qma_cuda_moe_layer_noalloc(C.byref(w), 256, 1, 260, None, None, None) == Q.ERR_INVALID


def test_packed_sizes():
    # Q4_K stays in GGUF order; Q6_K / Q8_0 planes hold exactly the GGUF bytes
    assert Q.packed_bytes(Q.Q4_K, 512, 2048) == 512 * 8 * 144
    assert Q.packed_bytes(Q.Q6_K, 2048, 512) == 2048 * 2 * 210
    assert Q.packed_bytes(Q.Q8_0, 151936, 2048) == 151936 * 64 * 34


def test_expert_parallel_arguments_and_shards():
    import pytest
    lib = Q.lib()
    uid = (C.c_uint8 * Q.EP_UID_BYTES)()
    h = C.c_void_p()
    # rank counts that do not divide 256, ranks out of range, oversized chunks
    for args in [(0, uid, 0, 3, 8), (0, uid, 2, 2, 8), (0, uid, 0, 2, 300), (0, uid, 0, 8, 128),
                 (0, None, 0, 2, 8)]:
        assert lib.qma_cuda_ep_init(*args, C.byref(h)) == Q.ERR_INVALID, args
        assert "qma_cuda_ep_init" in Q.last_error()
    assert lib.qma_cuda_ep_moe_layer(None, None, None, 1, None, None, None, None) == Q.ERR_INVALID
    assert lib.qma_cuda_ep_sync(None, None) == Q.ERR_INVALID
    assert lib.qma_cuda_ep_free(None) == Q.OK
    assert [Q.ep_shard(r, 4) for r in range(4)] == [(0, 64), (64, 64), (128, 64), (192, 64)]
    assert Q.ep_shard(0, 1) == (0, 256)
    with pytest.raises(ValueError):
        Q.ep_shard(0, 3)


def test_sampler_arguments():
    lib = Q.lib()
    ids = (C.c_int32 * 64)()
    lgs = (C.c_float * 64)()
    n = C.c_int()
    last = (C.c_int32 * 65)()
    for args in [(None, 10, None, 0, 1.0, 1.0, 5, 5), (1, 10, None, 0, 1.0, 1.0, 5, 65),
                 (1, 10, last, 65, 1.0, 1.0, 5, 5), (1, 10, None, 3, 1.0, 1.0, 5, 5), (1, 0, None, 0, 1.0, 1.0, 5, 5)]:
        assert lib.qma_cuda_sample_candidates(*args, ids, lgs, C.byref(n), None) == Q.ERR_INVALID, args
    assert lib.qma_cuda_state_logits(None) is None


def test_model_table_check_refuses_shapes_the_kernels_do_not_handle():
    """The loader's up-front table check (host only): the qwen35moe table
    passes; a table with another expert count, a short norm vector, a
    missing tensor or a tensor past the data section is refused before
    anything is allocated."""
    import pytest
    arr, n, size = Q.synth_layout()
    Q.model_check(arr, n)
    Q.model_check(arr, n, size)
    idx = Q.tensor_index(arr, n)

    def refused(mutate, what):
        arr2, n2, _ = Q.synth_layout()
        mutate(arr2)
        with pytest.raises(Q.QmaError) as e:
            Q.model_check(arr2, n2)
        assert e.value.status == Q.ERR_INVALID, what
        assert what in str(e.value), (what, str(e.value))

    refused(lambda a: a[idx["blk.3.ffn_gate_exps.weight"]].ne.__setitem__(2, 128), "blk.3.ffn_gate_exps.weight")
    refused(lambda a: a[idx["blk.7.ffn_down_exps.weight"]].ne.__setitem__(1, 1024), "blk.7.ffn_down_exps.weight")
    refused(lambda a: a[idx["blk.0.ssm_norm.weight"]].ne.__setitem__(0, 64), "blk.0.ssm_norm.weight")
    refused(lambda a: a[idx["blk.3.attn_k_norm.weight"]].ne.__setitem__(0, 128), "blk.3.attn_k_norm.weight")
    refused(lambda a: a[idx["blk.12.ffn_gate_inp.weight"]].ne.__setitem__(1, 64), "blk.12.ffn_gate_inp.weight")
    refused(lambda a: a[idx["output.weight"]].ne.__setitem__(1, 1000), "output.weight")
    refused(lambda a: setattr(a[idx["blk.39.ffn_up_shexp.weight"]], "name", b"blk.39.renamed"),
            "blk.39.ffn_up_shexp.weight")
    # a data section too short for the last tensor
    with pytest.raises(Q.QmaError) as e:
        Q.model_check(arr, n, size - 4096)
    assert e.value.status == Q.ERR_INVALID
    # an unsupported expert type
    arr3, n3, _ = Q.synth_layout()
    arr3[idx["blk.5.ffn_up_exps.weight"]].type = Q.Q8_0
    with pytest.raises(Q.QmaError) as e:
        Q.model_check(arr3, n3)
    assert e.value.status in (Q.ERR_UNSUPPORTED, Q.ERR_INVALID)


def test_expert_parallel_init_timeout_argument():
    lib = Q.lib()
    uid = (C.c_uint8 * Q.EP_UID_BYTES)()
    h = C.c_void_p()
    assert lib.qma_cuda_ep_init_timeout(0, uid, 0, 2, 8, 0, C.byref(h)) == Q.ERR_INVALID
    assert "timeout" in Q.last_error()


def test_layer_entry_points_and_ecache_reject_bad_arguments():
    lib = Q.lib()
    assert lib.qma_cuda_gdn_step(None, 0, 1, 1, 1, 1) == Q.ERR_INVALID
    assert "qma_cuda_gdn_step" in Q.last_error()
    assert lib.qma_cuda_attn_decode(None, 3, 1, 1, 1, 1) == Q.ERR_INVALID
    assert lib.qma_cuda_ecache_hint(None, 0, None, 0, None) == Q.ERR_INVALID
    assert lib.qma_cuda_ecache_prefetch(None, 0, None, 0, None) == Q.ERR_INVALID
    assert lib.qma_cuda_ecache_hold(None, 0, 0, None, None, None) == Q.ERR_INVALID
    assert lib.qma_cuda_ecache_release(None) == Q.ERR_INVALID
    assert lib.qma_cuda_ecache_held(None) == -1


def test_batch_entry_points_reject_bad_arguments():
    lib = Q.lib()
    h = C.c_void_p()
    assert lib.qma_cuda_batch_create(None, 4, 4096, C.byref(h)) == Q.ERR_INVALID
    assert lib.qma_cuda_batch_create(1, 0, 4096, C.byref(h)) == Q.ERR_INVALID
    assert lib.qma_cuda_batch_create(1, 4, 4, C.byref(h)) == Q.ERR_INVALID      # n_ctx below the sink
    ids = (C.c_int * 1)(0)
    assert lib.qma_cuda_batch_eval(None, ids, ids, 1, None, None) == Q.ERR_INVALID
    assert lib.qma_cuda_batch_eval_hidden(None, ids, ids, 1, 40, None) == Q.ERR_INVALID
    assert lib.qma_cuda_batch_set_ep(None, None, None) == Q.ERR_INVALID
    assert lib.qma_cuda_batch_seq(None, 0) is None
    assert lib.qma_cuda_batch_n_seq(None) == 0
    assert lib.qma_cuda_batch_logits(None) is None
    assert lib.qma_cuda_batch_free(None) == Q.OK
    assert lib.qma_cuda_model_set_router_bias(None, 0, None) == Q.ERR_INVALID


C_CALLER = r"""
/* A C99 caller of the engine, as qma's nn.c would bind it: every entry
 * point is called once with arguments the library refuses before touching
 * a device (null handles, bad sizes), so the program runs without a GPU. */
#include <stdio.h>
#include <string.h>
#include "qma_cuda.h"

int main(void)
{
    int bad = 0;
    qma_cuda_model *m = NULL;
    qma_cuda_state *s = NULL;
    qma_cuda_batch *b = NULL;
    qma_cuda_ep *ep = NULL;
    qma_cuda_moe_weights w;
    int ids[1] = {0}, toks[1] = {0}, greedy[1];
    memset(&w, 0, sizeof w);
    if (qma_cuda_abi_version() != QMA_CUDA_ABI_VERSION) bad |= 1;
    if (qma_cuda_state_create(NULL, 4096, &s) != QMA_CUDA_ERR_INVALID) bad |= 2;
    if (qma_cuda_eval(NULL, NULL, toks, 1, NULL, 0) != QMA_CUDA_ERR_INVALID) bad |= 4;
    if (qma_cuda_batch_create(NULL, 4, 4096, &b) != QMA_CUDA_ERR_INVALID) bad |= 8;
    if (qma_cuda_batch_eval(NULL, ids, toks, 1, NULL, greedy) != QMA_CUDA_ERR_INVALID) bad |= 16;
    if (strlen(qma_cuda_last_error()) == 0) bad |= 1024;     /* the refusal says why */
    if (qma_cuda_moe_layer(&w, NULL, 1, NULL, NULL, NULL, NULL, 0, NULL) != QMA_CUDA_ERR_INVALID) bad |= 32;
    if (qma_cuda_ep_moe_layer(ep, &w, NULL, 1, NULL, NULL, NULL, NULL) != QMA_CUDA_ERR_INVALID) bad |= 64;
    if (qma_cuda_gdn_step(NULL, 0, NULL, 1, NULL, 1) != QMA_CUDA_ERR_INVALID) bad |= 128;
    if (qma_cuda_ecache_get(m, 0, 0, NULL, NULL, NULL) == QMA_CUDA_OK) bad |= 256;
    if (qma_cuda_model_free(NULL) != QMA_CUDA_OK) bad |= 512;
    printf("%d\n", bad);
    return bad != 0;
}
"""


def test_header_is_c99_and_links(tmp_path):
    """include/qma_cuda.h compiles as strict C99 (the reference's language)
    and a C program calling the entry points links against libqma_cuda.so
    and runs (argument checks only, no device needed)."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = tmp_path / "caller.c"
    src.write_text(C_CALLER)
    exe = tmp_path / "caller"
    libdir = os.path.dirname(Q.LIB_PATH)
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", str(src),
                        "-I", os.path.join(root, "include"), "-L", libdir, "-lqma_cuda",
                        "-Wl,-rpath," + libdir, "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "0", (r.stdout, r.stderr)

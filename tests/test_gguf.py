"""The engine's GGUF reader (qma_cuda_gguf_scan) against the reference's own
loader (qma_load, gguf.c:104-513, compiled from its sources in oracle/_ref)
on GGUF files written here: the same tensor table (names, types, shapes,
offsets, sizes) and data-section offset, and the same files rejected --
bad magic, corrupt metadata, mismatched hyper-parameters, unsupported
types, partial blocks, tensors past the end of the file.  One deliberate
difference: the engine also reads Q8_0 tensors (qma_load rejects type 8).
Host only: no GPU.  The files hold every tensor name of the qwen35moe
layout with one row each (qma_load checks presence, not shapes)."""
import ctypes as C

import numpy as np
import pytest

import gguf_file as G
import oracle as O
import qma_cuda as Q


@pytest.fixture(scope="module")
def layout():
    arr, n, _ = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K)
    return arr, n


def ours(path):
    try:
        t, n, off, ntok = Q.gguf_scan(str(path))
    except Q.QmaError as e:
        return e.status, str(e)
    return 0, ([(t[i].name.decode(), int(t[i].type), tuple(t[i].ne), int(t[i].off), int(t[i].nbytes))
                for i in range(n)], off, ntok)


def reference(ref_lib, path):
    cap = 4096
    t = (O.Tensor * cap)()
    n, off, nv = C.c_int(), C.c_uint64(), C.c_int()
    err = C.create_string_buffer(512)
    rc = ref_lib.qr_gguf_load(str(path).encode(), t, cap, C.byref(n), C.byref(off), C.byref(nv), err, 512)
    if rc:
        return rc, err.value.decode()
    return 0, ([(t[i].name.decode(), int(t[i].type), tuple(t[i].ne), int(t[i].off), int(t[i].nbytes))
                for i in range(n.value)], off.value, nv.value)


def test_tensor_table_matches_qma_load(tmp_path, layout, ref_lib):
    tensors, size = G.small_layout(*layout)
    p = tmp_path / "m.gguf"
    start = G.write(p, G.qwen35moe_kv(), tensors, data_size=size)
    rc, got = ours(p)
    rr, want = reference(ref_lib, p)
    assert rc == 0 and rr == 0, (got, want)
    assert got == want
    assert got[1] == start and got[2] == 64 and len(got[0]) == 733


def test_alignment_prefix_and_unread_metadata(tmp_path, layout, ref_lib):
    """general.alignment 64, the "qwen35." key prefix, a 4-dim tensor info,
    and metadata of every value type that both readers must step over."""
    extra = [("x.f64", "f64", 1.5), ("x.i64", "i64", -3), ("x.bool", "bool", True), ("x.i8", "i8", -1),
             ("x.u16", "u16", 7), ("x.nested", "arr", ("arr", [("u8", [1, 2]), ("u8", [3])])),
             ("x.strs", "arr", ("str", ["p", "qq"])), ("tokenizer.chat_template", "str", "{{x}}")]
    arr, n = layout
    tensors, size = G.small_layout(arr, n, alignment=64,
                                   override={"blk.0.ffn_gate_inp.weight": (0, (2048, 1, 1, 1))})
    p = tmp_path / "m.gguf"
    G.write(p, G.qwen35moe_kv(prefix="qwen35.", alignment=64, extra=extra), tensors, data_size=size,
            alignment=64)
    rc, got = ours(p)
    rr, want = reference(ref_lib, p)
    assert rc == 0 and rr == 0, (got, want)
    assert got == want and got[1] % 64 == 0


@pytest.mark.parametrize("case", ["magic", "layers", "type", "partial_block", "past_end", "truncated_meta"])
def test_both_readers_reject(tmp_path, layout, ref_lib, case):
    arr, n = layout
    kv, override, cut, magic = G.qwen35moe_kv(), None, 0, False
    if case == "layers":
        kv = G.qwen35moe_kv(block_count=39)
    elif case == "type":            # Q4_0: neither engine computes with it
        override = {"blk.3.attn_q.weight": (2, (2048, 1))}
    elif case == "partial_block":
        override = {"blk.5.ffn_gate_shexp.weight": (12, (2000, 1))}
    tensors, size = G.small_layout(arr, n, override=override)
    if case == "past_end":          # the last tensor's final byte missing
        name, typ, ne, off = tensors[-1]
        cut = size - (off + G.tensor_bytes(typ, ne)) + 1
    p = tmp_path / "m.gguf"
    G.write(p, kv, tensors, data_size=size, truncate_by=cut)
    if case == "magic":
        with open(p, "r+b") as f:
            f.write(b"GGUX")
    elif case == "truncated_meta":
        with open(p, "r+b") as f:
            f.truncate(200)
    rc, msg = ours(p)
    rr, rmsg = reference(ref_lib, p)
    assert rc != 0 and rr != 0, (case, msg, rmsg)


def test_q8_0_tensors_read_by_the_engine_only(tmp_path, layout, ref_lib):
    tensors, size = G.small_layout(*layout, override={"token_embd.weight": (8, (2048, 3))})
    p = tmp_path / "m.gguf"
    G.write(p, G.qwen35moe_kv(), tensors, data_size=size)
    rc, got = ours(p)
    rr, rmsg = reference(ref_lib, p)
    assert rr != 0 and "unsupported type 8" in rmsg
    assert rc == 0
    emb = [t for t in got[0] if t[0] == "token_embd.weight"][0]
    assert emb[1] == 8 and emb[4] == 3 * 2048 // 32 * 34


def test_scan_sizes_with_zero_capacity(tmp_path, layout):
    tensors, size = G.small_layout(*layout)
    p = tmp_path / "m.gguf"
    G.write(p, G.qwen35moe_kv(), tensors, data_size=size)
    n = C.c_uint32()
    assert Q.lib().qma_cuda_gguf_scan(str(p).encode(), None, 0, C.byref(n), None, None) == Q.OK
    assert n.value == 733
    assert Q.lib().qma_cuda_gguf_scan(str(tmp_path / "absent.gguf").encode(), None, 0, C.byref(n), None,
                                      None) == Q.ERR_INVALID

"""Generate tests/golden/layer0_ref.npz: layer-sized known answers from the
qma reference compiled from its own sources (oracle/_ref), so that the C
restatement stays pinned where the reference sources are absent.

The reference ships no golden vectors; these are the reference's own
outputs on seeded inputs (the inputs are stored beside them):
  * Q8_K quantisation of 6 rows of 4096 values (quantize_row_q8k,
    q8k.c:34-85), one block of them all zeros;
  * the 4-bit and 2-bit KV records of 8 vectors and their dot products
    (kvq4_quant / kvq2_quant / kvq4_dot / kvq2_dot, kvq.c);
  * the MoE block of layer 0 of the seeded synthetic model on 3 tokens
    (moe_ffn, nn.c:509-649) and the last token's 8 experts;
  * the gated delta net mixer of layer 0 over calls of 1, 5 and 1 tokens
    (nn.c:2164-2244), its outputs and SHA-256 digests of the recurrent and
    conv states after each call.

Needs the reference sources (it builds oracle/_ref) and a few seconds:

  python tests/golden/make_layer_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "layer0_ref.npz")
BLOB_SEED = 0
GDN_CALLS = (1, 5, 1)


def p(a):
    return O._ptr(a)


def digest(a):
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), np.uint8)


def layer0_blob():
    """Layer 0's tensors of the synthetic model (the rest left zero)."""
    arr, n, size = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K)
    names = {arr[i].name.decode() for i in range(n) if arr[i].name.decode().startswith("blk.0.")}
    return arr, n, size, O.synth_blob(arr, n, size, seed=BLOB_SEED, names=names)


def main():
    O.build()
    R = O.ref()
    R.qr_init(1)
    rng = np.random.default_rng(20261202)
    g = {}

    # Q8_K quantisation
    x = (rng.standard_normal((6, 4096)) * rng.uniform(0.01, 10, (6, 1))).astype(np.float32)
    x[5, :256] = 0.0
    xq, xd, xs = np.zeros((6, 4096), np.int8), np.zeros((6, 16), np.float32), np.zeros((6, 256), np.int16)
    for t in range(6):
        R.qma_q8k_quant(p(x[t]), 4096, p(xq[t]), p(xd[t]), p(xs[t]))
    g.update(q8k_x=x, q8k_xq=xq, q8k_xd=xd, q8k_xs=xs)

    # KV records
    v = (rng.standard_normal((8, 256)) * rng.uniform(0.1, 5, (8, 1))).astype(np.float32)
    q = rng.standard_normal((8, 256)).astype(np.float32)
    rec = np.zeros((8, 240), np.uint8)
    d4, d2 = np.zeros(8, np.float32), np.zeros(8, np.float32)
    for i in range(8):
        R.kvq4_quant(p(v[i]), 256, p(rec[i]))
        R.kvq2_quant(p(v[i]), 256, p(rec[i]))
        d4[i] = R.kvq4_dot(p(rec[i]), p(q[i]), 256)
        d2[i] = R.kvq2_dot(p(rec[i, 160:]), p(q[i]), 256)
    g.update(kv_v=v, kv_q=q, kv_rec=rec, kv_dot4=d4, kv_dot2=d2)

    # layer 0: MoE block and gated delta net
    arr, n, size, blob = layer0_blob()
    rm = R.qr_model_new(arr, n, p(blob), size)
    assert rm
    try:
        T = 3
        xm = rng.standard_normal((T, 2048)).astype(np.float32)
        om = np.zeros((T, 2048), np.float32)
        sel = np.zeros(8, np.int32)
        R.qr_moe_ffn(rm, 0, p(xm), T, p(om), p(sel))
        g.update(moe_x=xm, moe_out=om, moe_sel_last=sel)
        rs = R.qr_state_new(256)
        try:
            xs_, os_, ssm_d, conv_d = [], [], [], []
            for Tg in GDN_CALLS:
                xg = rng.standard_normal((Tg, 2048)).astype(np.float32)
                og = np.zeros((Tg, 2048), np.float32)
                R.qr_gdn_layer(rm, rs, 0, p(xg), Tg, p(og))
                xs_.append(xg)
                os_.append(og)
                ssm_d.append(digest(np.ctypeslib.as_array(R.qr_state_ssm(rs, 0), (32 * 128 * 128,))))
                conv_d.append(digest(np.ctypeslib.as_array(R.qr_state_conv(rs, 0), (8192 * 3,))))
            g.update(gdn_calls=np.array(GDN_CALLS, np.int32), gdn_x=np.concatenate(xs_),
                     gdn_out=np.concatenate(os_), gdn_ssm_sha256=np.stack(ssm_d), gdn_conv_sha256=np.stack(conv_d))
        finally:
            R.qr_state_free(rs)
    finally:
        R.qr_model_free(rm)
    g["blob_seed"] = np.array(BLOB_SEED, np.int64)
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT) / 1024:.0f} KB)")


if __name__ == "__main__":
    main()

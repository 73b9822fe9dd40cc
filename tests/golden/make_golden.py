"""Generate golden fixtures from the qma reference compiled from its own
sources (oracle/_ref) on the full 40-layer synthetic qwen35moe model.

Runs where the reference sources exist (this builds oracle/_ref); needs
~24 GB of host memory and a few minutes.  Writes tests/golden/full_model.npz:
the prompt, the reference's last-token logits after the prompt and after
each greedy decode step (top-64 ids and values plus summary statistics),
and the greedy tokens.  The C restatement is checked against the same run
bit for bit before anything is written.

  python tests/golden/make_golden.py [--prompt 24] [--decode 4]
"""
import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

SEED = 7
N_CTX = 4096


def summarize(logits):
    top = np.argsort(-logits, kind="stable")[:64]
    return top.astype(np.int32), logits[top].astype(np.float32), np.array(
        [logits.sum(dtype=np.float64), (logits.astype(np.float64) ** 2).sum(), logits.max(), logits.min()])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompt", type=int, default=24)
    ap.add_argument("--decode", type=int, default=4)
    ap.add_argument("--threads", type=int, default=min(os.cpu_count() or 1, 16))
    args = ap.parse_args()
    O.build()
    R = O.ref()
    L = O.lib()
    R.qr_init(args.threads)
    O.lib().qo_set_threads(args.threads)
    arr, n, size = O.synth_layout(embd_type=O.Q6_K, out_type=O.Q6_K)
    t0 = time.time()
    blob = O.synth_blob(arr, n, size, seed=SEED, threads=args.threads)
    print(f"generated {size/1e9:.1f} GB in {time.time()-t0:.0f} s", flush=True)
    p = O._ptr
    rm = R.qr_model_new(arr, n, p(blob), size)
    om = L.qo_model_new(arr, n, p(blob), O.N_VOCAB)
    rs = R.qr_state_new(N_CTX)
    os_ = L.qo_state_new(N_CTX)
    rng = np.random.default_rng(SEED)
    prompt = rng.integers(0, O.N_VOCAB, args.prompt).astype(np.int32)
    V = O.N_VOCAB
    lr = np.zeros(V, np.float32)
    lo = np.zeros(V, np.float32)
    t0 = time.time()
    R.qr_eval(rm, rs, p(prompt), len(prompt), p(lr), args.threads, 0)
    t1 = time.time()
    L.qo_eval(om, os_, p(prompt), len(prompt), p(lo), 0)
    t2 = time.time()
    print(f"prompt: ref {t1-t0:.1f} s, oracle {t2-t1:.1f} s, bit-exact {np.array_equal(lr, lo)}", flush=True)
    assert np.array_equal(lr, lo), np.abs(lr - lo).max()
    tops, vals, stats, toks = [], [], [], []
    a, b, c = summarize(lr)
    tops.append(a); vals.append(b); stats.append(c)
    tok = int(np.argmax(lr))
    for _ in range(args.decode):
        toks.append(tok)
        one = np.array([tok], np.int32)
        R.qr_eval(rm, rs, p(one), 1, p(lr), args.threads, 0)
        L.qo_eval(om, os_, p(one), 1, p(lo), 0)
        assert np.array_equal(lr, lo), np.abs(lr - lo).max()
        a, b, c = summarize(lr)
        tops.append(a); vals.append(b); stats.append(c)
        tok = int(np.argmax(lr))
    print("decode bit-exact, tokens", toks, flush=True)
    np.savez_compressed(os.path.join(HERE, "full_model.npz"), seed=SEED, n_ctx=N_CTX,
                        embd_type=O.Q6_K, out_type=O.Q6_K, prompt=prompt,
                        greedy=np.array(toks, np.int32), top_ids=np.stack(tops),
                        top_vals=np.stack(vals), stats=np.stack(stats))
    print("wrote", os.path.join(HERE, "full_model.npz"))


if __name__ == "__main__":
    main()

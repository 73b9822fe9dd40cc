"""The GPU sampler's first phase (qma_cuda_sample_candidates) against the
reference's own sampler_candidates (sampler.c:36-95, compiled from its
sources in oracle/_ref): repeat penalty over repeated last tokens of both
signs, temperature, top-k clamped by max_k and the vocabulary; the same
token ids in the same order and bit-identical scaled logits.  Equal values
inside the list: the reference's qsort leaves their order unspecified, so
that case compares the lists ordered by (value, id)."""
import ctypes as C

import numpy as np
import pytest

import qma_cuda as Q

pytestmark = pytest.mark.gpu

V = 151936


def ours(logits, last, pen, temp, k, max_k):
    import torch
    dev = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    last = np.ascontiguousarray(last, np.int32)
    ids = np.zeros(64, np.int32)
    lgs = np.zeros(64, np.float32)
    n = C.c_int()
    Q.call("qma_cuda_sample_candidates", dev.data_ptr(), len(logits), Q.ptr(last) if len(last) else None,
           len(last), pen, temp, k, max_k, Q.ptr(ids), Q.ptr(lgs), C.byref(n), None)
    return ids[:n.value], lgs[:n.value]


def reference(ref_lib, logits, last, pen, temp, k, max_k):
    last = np.ascontiguousarray(last, np.int32)
    ids = np.zeros(64, np.int32)
    lgs = np.zeros(64, np.float32)
    n = ref_lib.qr_sampler_candidates(len(logits), logits.ctypes.data, last.ctypes.data, len(last), pen, temp,
                                      k, ids.ctypes.data, lgs.ctypes.data, max_k)
    return ids[:n], lgs[:n]


@pytest.mark.parametrize("pen,temp,k,max_k,n_last,nv", [
    (1.1, 0.7, 40, 40, 64, V),      # the agent's defaults (agent.c:935: max_k 40)
    (1.0, 0.0, 20, 40, 0, V),       # no penalty, greedy temperature
    (1.3, 1.0, 64, 64, 17, V),
    (1.1, 0.5, 1, 40, 5, V),
    (1.1, 0.8, 200, 40, 30, V),     # top_k above max_k
    (1.2, 0.9, 40, 40, 8, 33),      # vocabulary below max_k
])
def test_candidates_match_reference(cuda, ref_lib, pen, temp, k, max_k, n_last, nv):
    rng = np.random.default_rng(nv + n_last + k)
    logits = (rng.standard_normal(nv) * 4).astype(np.float32)
    # the last tokens hit the current leaders (both signs) several times
    top = np.argsort(-logits)[:6]
    neg = np.argsort(logits)[:2]
    pool = np.concatenate([top, neg, rng.integers(0, nv, 64)])
    last = np.array([pool[i % len(pool)] for i in range(n_last)], np.int32)
    last[::3] = top[0]
    got = ours(logits, last, pen, temp, k, max_k)
    want = reference(ref_lib, logits, last, pen, temp, k, max_k)
    assert np.array_equal(got[0], want[0]), (got[0][:8], want[0][:8])
    assert np.array_equal(got[1].view(np.uint32), want[1].view(np.uint32))


def test_equal_values_inside_the_list(cuda, ref_lib):
    rng = np.random.default_rng(5)
    logits = rng.standard_normal(V).astype(np.float32)
    order = np.argsort(-logits)
    logits[order[3]] = logits[order[2]]        # a tie inside the top 40
    logits[order[10]] = logits[order[9]]
    got = ours(logits, [], 1.0, 0.8, 40, 40)
    want = reference(ref_lib, logits, [], 1.0, 0.8, 40, 40)
    key = lambda ids, v: sorted(zip((-v).tolist(), ids.tolist()))
    assert key(*got) == key(*want)
    assert [i for _, i in key(*got)] == got[0].tolist()

"""GPU parity of Q8_K quantization and the quantized GEMV against the oracle
(configs[1] shapes: 512x2048, 2048x512, 4096x2048, 2048x4096 and the
151936x2048 LM head; Q4_K / Q6_K / Q8_0 weights; batch 1, 8, 64).

Bars: Q8_K activations and integer super-block partials bit-exact; fp32
outputs within 1e-4 scaled relative error (the contract is 1e-3; the only
difference is fp32 summation order)."""
import numpy as np
import pytest

import oracle as O
import qma_cuda as Q
from helpers import assert_close, empty_dev, to_dev

pytestmark = pytest.mark.gpu

SHAPES = [(512, 2048), (2048, 512), (4096, 2048), (2048, 4096)]   # (n_out, n_in)
RTOL = 1e-4


def gpu_quant(x):
    import torch
    T, n = x.shape
    dx = to_dev(x)
    dq = empty_dev((T, n), torch.int8)
    dd = empty_dev((T, n // 256), torch.float32)
    ds = empty_dev((T, n // 16), torch.int16)
    Q.call("qma_cuda_q8k_quant", Q.ptr(dx), T, n, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds), None)
    return dq, dd, ds


def gpu_pack(W, wtype, rows, n):
    import torch
    dW = to_dev(W)
    dP = empty_dev((Q.packed_bytes(wtype, rows, n),), torch.uint8)
    Q.call("qma_cuda_repack", wtype, Q.ptr(dW), rows, n, Q.ptr(dP), None)
    return dP


def test_q8k_quant_bit_exact(cuda, rng):
    import torch
    x = (rng.standard_normal((33, 4096)) * rng.uniform(1e-3, 50, (33, 1))).astype(np.float32)
    x[0, :256] = 0.0
    x[1, 7] = 1e-30
    xq, xd, xs = O.q8k_quant(x)
    dq, dd, ds = gpu_quant(x)
    torch.cuda.synchronize()
    assert np.array_equal(dq.cpu().numpy(), xq)
    assert np.array_equal(dd.cpu().numpy().view(np.uint32), xd.view(np.uint32))
    assert np.array_equal(ds.cpu().numpy(), xs)


@pytest.mark.parametrize("wtype", [O.Q4_K, O.Q6_K, O.Q8_0])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("T", [1, 8, 64])
def test_matvec_matches_oracle(cuda, rng, wtype, shape, T):
    import torch
    n_out, n_in = shape
    W = O.synth_matrix(f"gemv.{wtype}.{n_out}x{n_in}", wtype, n_out, n_in, seed=11)
    x = rng.standard_normal((T, n_in)).astype(np.float32)
    want = O.matmul(x, W, wtype, n_in, n_out)
    dq, dd, ds = gpu_quant(x)
    dP = gpu_pack(W, wtype, n_out, n_in)
    out = empty_dev((T, n_out), torch.float32)
    Q.call("qma_cuda_matvec", wtype, Q.ptr(dP), n_in, n_out, T, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds),
           Q.ptr(out), None)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), want, RTOL, f"type {wtype} {shape} T={T}")


@pytest.mark.parametrize("wtype", [O.Q4_K, O.Q6_K, O.Q8_0])
@pytest.mark.parametrize("shape", SHAPES)
def test_integer_partials_bit_exact(cuda, rng, wtype, shape):
    import torch
    n_out, n_in = shape
    W = O.synth_matrix(f"part.{wtype}.{n_out}x{n_in}", wtype, n_out, n_in, seed=12)
    x = rng.standard_normal((1, n_in)).astype(np.float32)
    xq, xd, xs = O.q8k_quant(x)
    _, want = O.dot_partials(W, wtype, n_in, xq[0], xd[0], xs[0])
    dq, _, _ = gpu_quant(x)
    dP = gpu_pack(W, wtype, n_out, n_in)
    got = empty_dev(want.shape, torch.int32)
    Q.call("qma_cuda_dot_partials", wtype, Q.ptr(dP), n_in, n_out, Q.ptr(dq), Q.ptr(got), None)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("wtype,T", [(O.Q8_0, 1), (O.Q4_K, 1), (O.Q6_K, 1), (O.Q8_0, 37)])
def test_lm_head_shape(cuda, rng, wtype, T):
    """The 151936 x 2048 LM head; Q8_0 with 37 tokens takes the MMA GEMM of a
    batched step (two token tiles, the second partial)."""
    import torch
    n_out, n_in = 151936, 2048
    W = O.synth_matrix(f"lmhead.{wtype}", wtype, n_out, n_in, seed=13)
    x = rng.standard_normal((T, n_in)).astype(np.float32)
    want = O.matmul(x, W, wtype, n_in, n_out)
    dq, dd, ds = gpu_quant(x)
    dP = gpu_pack(W, wtype, n_out, n_in)
    out = empty_dev((T, n_out), torch.float32)
    Q.call("qma_cuda_matvec", wtype, Q.ptr(dP), n_in, n_out, T, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds),
           Q.ptr(out), None)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert_close(got, want, RTOL, f"lm head type {wtype} T={T}")
    assert np.array_equal(got.argmax(axis=1), want.argmax(axis=1))


def test_matvec_is_deterministic(cuda, rng):
    import torch
    W = O.synth_matrix("det", O.Q4_K, 4096, 2048, seed=14)
    x = rng.standard_normal((1, 2048)).astype(np.float32)
    dq, dd, ds = gpu_quant(x)
    dP = gpu_pack(W, O.Q4_K, 4096, 2048)
    outs = []
    for _ in range(3):
        out = empty_dev((1, 4096), torch.float32)
        Q.call("qma_cuda_matvec", O.Q4_K, Q.ptr(dP), 2048, 4096, 1, Q.ptr(dq), Q.ptr(dd),
               Q.ptr(ds), Q.ptr(out), None)
        outs.append(out.cpu().numpy())
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


@pytest.mark.parametrize("shape", [(4096, 2048), (2048, 4096), (12352, 2048), (208, 2048)])
@pytest.mark.parametrize("T", [64, 130, 512])
def test_q4k_gemm_tcgen05_bit_identical_to_mma_sync(cuda, rng, shape, T):
    """Prefill-sized Q4_K GEMMs (64+ tokens) on the 5th-generation tensor
    cores (tcgen05 int8 MMAs into tensor memory, the sub-block scales folded
    into two int8 digits of the weights, 128 x 128 tiles; partial row and
    token tiles included) against the warp-level mma.sync kernel
    (QMA_CUDA_MMA_SYNC=1): exact integer super-block sums and a shared fp32
    fold, so the same bits; and against the oracle within the GEMV bar."""
    import os
    import torch
    n_out, n_in = shape
    W = O.synth_matrix(f"gemm.tc.{n_out}x{n_in}", O.Q4_K, n_out, n_in, seed=13)
    x = rng.standard_normal((T, n_in)).astype(np.float32)
    dq, dd, ds = gpu_quant(x)
    dW = gpu_pack(W, O.Q4_K, n_out, n_in)
    outs = {}
    for form in ("tc", "sync"):
        out = empty_dev((T, n_out), torch.float32)
        if form == "sync":
            os.environ["QMA_CUDA_MMA_SYNC"] = "1"
        try:
            Q.call("qma_cuda_matvec", O.Q4_K, Q.ptr(dW), n_in, n_out, T, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds),
                   Q.ptr(out), None)
            torch.cuda.synchronize()
        finally:
            os.environ.pop("QMA_CUDA_MMA_SYNC", None)
        outs[form] = out.cpu().numpy()
    a, b = outs["tc"], outs["sync"]
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"max |diff| {np.abs(a - b).max():.3e}"
    want = O.matmul(x, W, O.Q4_K, n_in, n_out)
    assert_close(a, want, RTOL, f"tc gemm {shape} T={T}")

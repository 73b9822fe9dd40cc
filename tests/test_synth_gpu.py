"""The on-device synthetic weight generator reproduces the oracle's CPU
generator byte for byte (so a model generated on the GPU and one generated on
the host for the CPU oracle hold identical weights)."""
import numpy as np
import pytest

import oracle as O
import qma_cuda as Q

pytestmark = pytest.mark.gpu

CASES = [
    ("blk.3.ffn_gate_exps.weight", O.Q4_K, 2048, 512 * 3),
    ("blk.3.ffn_down_exps.weight", O.Q6_K, 512, 2048 * 2),
    ("token_embd.weight", O.Q8_0, 2048, 300),
    ("output.weight", O.Q6_K, 2048, 64),
    ("blk.0.ffn_gate_inp.weight", O.F32, 2048, 256),
    ("blk.0.attn_norm.weight", O.F32, 2048, 1),
    ("blk.0.ssm_conv1d.weight", O.F32, 4, 8192),
    ("blk.0.ssm_a", O.F32, 32, 1),
    ("blk.0.ssm_dt.bias", O.F32, 32, 1),
]


@pytest.mark.parametrize("name,wtype,n,rows", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("seed", [0, 12345])
def test_device_generator_matches_oracle(cuda, name, wtype, n, rows, seed):
    import torch
    want = O.synth_matrix(name, wtype, rows, n, seed=seed).reshape(-1)
    dst = torch.zeros(want.size, dtype=torch.uint8, device="cuda")
    Q.call("qma_cuda_synth_tensor", name.encode(), wtype, n * rows, seed, Q.ptr(dst), None)
    got = dst.cpu().numpy()
    assert np.array_equal(got, want), f"{name}: {np.count_nonzero(got != want)} bytes differ"

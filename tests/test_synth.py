"""CPU checks of the synthetic generator: deterministic, and the
distributions the configs name (projections ~N(0, 0.02) before quantization,
norms near 1, ssm_a negative)."""
import numpy as np

import oracle as O


def test_generator_is_deterministic_and_seeded():
    a = O.synth_matrix("blk.1.attn_q.weight", O.Q4_K, 8, 2048, seed=1)
    b = O.synth_matrix("blk.1.attn_q.weight", O.Q4_K, 8, 2048, seed=1)
    c = O.synth_matrix("blk.1.attn_q.weight", O.Q4_K, 8, 2048, seed=2)
    assert np.array_equal(a, b) and not np.array_equal(a, c)


def test_distributions():
    W = O.synth_matrix("blk.0.ffn_gate_inp.weight", O.F32, 256, 2048).view(np.float32)
    assert abs(W.std() - 0.02) < 0.001 and abs(W.mean()) < 0.001
    q = O.synth_matrix("blk.0.attn_q.weight", O.Q4_K, 64, 2048)
    deq = np.zeros(2048, np.float32)
    vals = []
    for r in range(64):
        O.lib().qo_dequant_row(O._ptr(q[r]), O.Q4_K, O._ptr(deq), 2048)
        vals.append(deq.copy())
    v = np.concatenate(vals)
    assert abs(v.std() - 0.02) < 0.002
    n = O.synth_matrix("blk.0.attn_norm.weight", O.F32, 1, 2048).view(np.float32)
    assert abs(n.mean() - 1.0) < 0.01
    a = O.synth_matrix("blk.0.ssm_a", O.F32, 1, 32).view(np.float32)
    assert (a < 0).all()


def test_engine_tensor_table_matches_the_oracles():
    """qma_cuda.synth_layout (the table bench.py and the engine's users
    build the random-init model from) equals the oracle's qo_synth_layout:
    names, types, shapes, offsets and sizes."""
    import qma_cuda as Q
    for cfg in [dict(embd_type=O.Q6_K, out_type=O.Q6_K), dict(), dict(down_type=O.Q4_K, proj_type=O.Q6_K),
                dict(n_vocab=1000)]:
        a, n, size = Q.synth_layout(**cfg)
        b, m, size2 = O.synth_layout(**cfg)
        assert (n, size) == (m, size2)
        for i in range(n):
            assert (a[i].name, a[i].type, tuple(a[i].ne), a[i].off, a[i].nbytes) == \
                (b[i].name, b[i].type, tuple(b[i].ne), b[i].off, b[i].nbytes), i

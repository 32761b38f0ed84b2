"""Host-side MoE routing (ops.moe_align on CPU tensors) against the oracle's
loop restatement; the CPU oracle's GEMM against a direct dense computation."""
import numpy as np
import torch

from cutile_b200 import ops
from oracle import oracle as O


def test_moe_align_cpu_matches_loops():
    for (M, E, topk, seed), block in zip([(1, 4, 1, 0), (100, 8, 2, 1), (333, 9, 3, 2), (7, 64, 4, 3)],
                                         [128, 256, 128, 256]):
        g = torch.Generator().manual_seed(seed)
        ids = torch.argsort(torch.rand(M, E, generator=g), dim=1)[:, :topk].to(torch.int32)
        s, e, n = ops.moe_align(ids, E, block)
        rs, re, rn = O.moe_align(ids.numpy(), E, block)
        np.testing.assert_array_equal(s.numpy(), rs)
        np.testing.assert_array_equal(e.numpy(), re)
        assert int(n.item()) == rn
        assert s.numel() % block == 0 and e.numel() * block == s.numel()


def test_moe_oracle_against_dense():
    rng = np.random.default_rng(0)
    M, N, K, E, topk = 50, 24, 16, 5, 2
    A = rng.standard_normal((M, K))
    B = rng.standard_normal((E, N, K))
    ids = np.stack([rng.choice(E, topk, replace=False) for _ in range(M)])
    w = rng.random((M, topk))
    s, e, n = O.moe_align(ids, E)
    C = O.moe(A, B, s, e, n, topk, w)
    for t in range(M):
        for j in range(topk):
            np.testing.assert_allclose(C[t * topk + j], (A[t] @ B[ids[t, j]].T) * w[t, j],
                                       rtol=1e-12, atol=1e-12)

"""The CPU oracle against independent numpy restatements and its own
invariants (test infrastructure)."""
import numpy as np
import pytest

from oracle import oracle as O


def test_generator_is_deterministic_and_offsettable():
    a = O.uniform(1000, 7)
    b = O.uniform(500, 7, offset=500)
    np.testing.assert_array_equal(a[500:], b)
    assert a.min() >= -1 and a.max() < 1
    # 24-bit grid: every value is k/2^23 - 1 exactly
    k = (a.astype(np.float64) + 1.0) * 2 ** 23
    np.testing.assert_array_equal(k, np.round(k))
    n = O.normal(200000, 3)
    assert abs(n.mean()) < 0.01 and abs(n.std() - 1) < 0.01


def test_splitmix_known_answer():
    # SplitMix64 with state 0: first output 0xE220A8397B1DCDAF (Steele et al. 2014,
    # the reference sequence of java.util.SplittableRandom / splitmix64.c).
    u = O.uniform(1, 0, lo=0.0, hi=1.0, dtype=np.float64)[0]
    assert u == (0xE220A8397B1DCDAF >> 40) / 2 ** 24


@pytest.mark.parametrize("dt", [np.float16, np.float32, np.float64])
@pytest.mark.parametrize("n", [1_024_000, 999_999])
def test_vadd_bit_exact(dt, n):
    a = O.uniform(n, 1, dtype=dt)
    b = O.uniform(n, 2, dtype=dt)
    ref = (a.astype(np.float64) + b.astype(np.float64)).astype(dt)  # exact sum rounded once
    np.testing.assert_array_equal(O.vadd(a, b).view(np.uint8), ref.view(np.uint8))


def test_rowsum_matches_numpy():
    m, n = 4096, 128  # test/runtests.jl:58
    a = O.uniform(m * n, 3).reshape(n, m)  # Julia m x n column-major storage
    ref = a.astype(np.float64).sum(axis=0)
    assert O.isapprox(O.rowsum(a), ref, 1e-6)
    r = O.uniform(64 * 33, 4).reshape(64, 33)
    assert O.isapprox(O.rowsum_rowmajor(r), r.astype(np.float64).sum(axis=1), 1e-6)


def test_softmax_matches_numpy():
    x = (4 * O.normal(37 * 1000, 5)).reshape(37, 1000)
    xd = x.astype(np.float64)
    e = np.exp(xd - xd.max(axis=1, keepdims=True))
    ref = e / e.sum(axis=1, keepdims=True)
    got = O.softmax(x)
    assert O.isapprox(got, ref, 1e-6)
    np.testing.assert_allclose(got.sum(axis=1), 1.0, rtol=1e-5)


def test_layernorm_matches_numpy():
    rows, n = 33, 4096
    x = O.normal(rows * n, 6).reshape(rows, n)
    w = 1 + 0.1 * O.normal(n, 7)
    b = 0.1 * O.normal(n, 8)
    y, mu, rs = O.layernorm_fwd(x, w, b, 1e-5)
    xd = x.astype(np.float64)
    m = xd.mean(axis=1)
    v = xd.var(axis=1)  # biased
    ref = (xd - m[:, None]) / np.sqrt(v[:, None] + 1e-5) * w + b
    assert O.isapprox(y, ref, 1e-6)
    assert O.isapprox(mu, m, 1e-6)
    assert O.isapprox(rs, 1 / np.sqrt(v + 1e-5), 1e-6)


def test_matmul_and_metrics():
    M, N, K = 30, 20, 10
    A = O.uniform(M * K, 1).reshape(K, M)  # Julia A (M x K) storage
    B = O.uniform(K * N, 2).reshape(N, K)
    C = O.matmul(A, B)  # (N, M)
    ref = A.T.astype(np.float64) @ B.T.astype(np.float64)  # Julia-order (M, N)
    np.testing.assert_allclose(C.T, ref, rtol=1e-12)
    assert O.max_rel(C, C) == 0 and O.rel_fro(C, C) == 0


def test_fmha_oracle_properties():
    S, D = 64, 16
    q, k, v = (O.normal(S * D, s).reshape(S, D) for s in (1, 2, 3))
    o = O.fmha(q, k, v, 0.25)
    o_c = O.fmha(q, k, v, 0.25, causal=True)
    np.testing.assert_allclose(o_c[0], v[0], rtol=1e-6)  # first query sees only key 0
    np.testing.assert_allclose(o_c[-1], o[-1], rtol=1e-10)  # last query sees all keys
    sub = O.fmha(q, k, v, 0.25, causal=True, rows=[5, 9])
    np.testing.assert_allclose(sub, o_c[[5, 9]], rtol=1e-12)


def test_isapprox_semantics():
    assert O.isapprox([1.0, 2.0], [1.0, 2.0 + 1e-7], 1e-6)
    assert not O.isapprox([1.0, 2.0], [1.0, 2.1], 1e-6)
    assert not O.isapprox([np.nan], [np.nan], 1e-6)


def test_layernorm_bwd_matches_autograd():
    import torch

    rows, n = 33, 256
    x = O.normal(rows * n, 1).reshape(rows, n)
    dy = O.normal(rows * n, 2).reshape(rows, n)
    w = 1 + 0.1 * O.normal(n, 3)
    b = 0.1 * O.normal(n, 4)
    _, mu, rs = O.layernorm_fwd(x, w, b, 1e-5)
    dx, dw, db = O.layernorm_bwd(x, dy, w, mu, rs)
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    wt = torch.tensor(w, dtype=torch.float64, requires_grad=True)
    bt = torch.tensor(b, dtype=torch.float64, requires_grad=True)
    torch.nn.functional.layer_norm(xt, (n,), wt, bt, eps=1e-5).backward(
        torch.tensor(dy, dtype=torch.float64))
    assert O.isapprox(dx, xt.grad.numpy(), 1e-6)
    assert O.isapprox(dw, wt.grad.numpy(), 1e-6)
    assert O.isapprox(db, bt.grad.numpy(), 1e-6)

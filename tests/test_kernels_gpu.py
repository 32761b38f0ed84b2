"""Parity of the sm_100a kernels against the CPU oracle on seeded inputs.

Tolerances (from the reference's checks and the BASELINE configs):
  vadd                     bit-exact
  rowsum/softmax/layernorm Julia isapprox, rtol 1e-5 (norm-wise)
  f16 GEMM / batched GEMM  relative Frobenius error <= 2e-3 vs float64
  f32 matmul               max|err| / max|ref| < 1e-3 (test/runtests.jl:95-98)
  fmha                     isapprox rtol 1e-2 vs float64
Inputs are generated on the device by ctb_fill_* and copied to the host, so
the oracle sees exactly the bits the kernel saw.
"""
import math

import numpy as np
import pytest
import torch

import cutile_b200 as cb
from cutile_b200 import ops
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def U(shape, seed, dev, dtype=torch.float32, lo=-1.0, hi=1.0):
    t = torch.empty(shape, dtype=dtype, device=dev)
    return ops.fill_uniform(t, seed, lo, hi)


def N(shape, seed, dev, dtype=torch.float32, mean=0.0, std=1.0):
    t = torch.empty(shape, dtype=dtype, device=dev)
    return ops.fill_normal(t, seed, mean, std)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ----------------------------------------------------------------------------- fills
def test_device_uniform_is_bit_identical_to_host_generator(dev):
    for dt, npdt in [(torch.float32, np.float32), (torch.float16, np.float16),
                     (torch.float64, np.float64)]:
        t = U(100_003, 11, dev, dt)
        np.testing.assert_array_equal(host(t), O.uniform(100_003, 11, dtype=npdt))


def test_device_normal_matches_host_generator(dev):
    t = N(100_000, 12, dev)
    np.testing.assert_allclose(host(t), O.normal(100_000, 12), rtol=1e-6, atol=1e-6)


# ----------------------------------------------------------------------------- vadd
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.float64])
@pytest.mark.parametrize("n", [1_024_000, 999_999, 1, 7, 0])
def test_vadd_bit_exact(dev, dt, n):
    a, b = U(n, 1, dev, dt), U(n, 2, dev, dt)
    c = ops.vadd(a, b)
    ref = O.vadd(host(a), host(b))
    assert host(c).tobytes() == ref.tobytes()


def test_vadd_subnormals_survive(dev):
    tiny = np.array([1e-45, -1e-45, 1.1754942e-38, 3e-39], np.float32)  # subnormals
    a = torch.from_numpy(tiny).to(dev)
    c = ops.vadd(a, a)
    assert host(c).tobytes() == (tiny + tiny).tobytes()


def test_vadd_strided_and_unaligned(dev):
    base = U(10_001, 3, dev)
    a = base[1:]        # 4-byte offset: not 16-byte aligned
    b = base[:-1]
    c = torch.empty(5000, device=dev)
    ops.vadd(a[::2], b[::2], c)
    hb = host(base)
    ref = O.vadd(np.ascontiguousarray(hb[1:][::2]), np.ascontiguousarray(hb[:-1][::2]))
    assert host(c).tobytes() == ref.tobytes()


@pytest.mark.slow
def test_vadd_full_size(dev):
    n = 1 << 28  # BASELINE config: Float32, N = 2^28, U(-1, 1)
    a, b = U(n, 20261201, dev), U(n, 20261202, dev)
    c = ops.vadd(a, b)
    ref = O.vadd(host(a), host(b))
    assert host(c).tobytes() == ref.tobytes()


# ----------------------------------------------------------------------------- rowsum
@pytest.mark.parametrize("m,n", [(4096, 128), (131072, 512), (1000, 33), (4100, 7), (3, 1),
                                 (65536, 512), (32768, 300), (16384, 512)])
def test_rowsum_julia_colmajor(dev, m, n):
    a = N((n, m), 4, dev)  # Julia m x n, stride (1, m)
    out = ops.rowsum(a)
    assert O.isapprox(host(out), O.rowsum(host(a)), 1e-5)


@pytest.mark.parametrize("m,n", [(131072, 512), (999, 1000), (5, 3)])
def test_rowsum_rowmajor(dev, m, n):
    a = N((m, n), 5, dev)
    out = ops.rowsum(a, julia_colmajor=False)
    assert O.isapprox(host(out), O.rowsum_rowmajor(host(a)), 1e-5)


def test_rowsum_generic_strides(dev):
    big = N((64, 300), 6, dev)
    a = big[:, ::3]  # both strides non-unit
    out = ops.rowsum(a, julia_colmajor=False)
    assert O.isapprox(host(out), O.rowsum_rowmajor(np.ascontiguousarray(host(big)[:, ::3])), 1e-5)


# ----------------------------------------------------------------------------- softmax
@pytest.mark.parametrize("count,length", [(2048, 1000), (4096, 16384), (17, 1), (9, 3),
                                          (33, 4097), (5, 32768), (3, 40000), (64, 513),
                                          (512, 16384), (300, 12000), (1, 16384), (149, 8196)])
def test_softmax(dev, count, length):
    x = N((count, length), 7, dev, std=4.0)
    y = ops.softmax(x)
    assert O.isapprox(host(y), O.softmax(host(x)), 1e-5)


def test_softmax_unaligned_rows(dev):
    big = N((10, 1003), 8, dev, std=4.0)
    x = big[:, 1:1002]  # row starts not 16-byte aligned, odd length
    y = torch.empty(10, 1001, device=dev)
    ops.softmax(x, y)
    assert O.isapprox(host(y), O.softmax(np.ascontiguousarray(host(big)[:, 1:1002])), 1e-5)


def test_softmax_large_magnitude(dev):
    x = N((8, 4096), 9, dev, std=200.0)  # exp would overflow without max subtraction
    y = ops.softmax(x)
    assert np.all(np.isfinite(host(y)))
    assert O.isapprox(host(y), O.softmax(host(x)), 1e-5)


# ----------------------------------------------------------------------------- layernorm
@pytest.mark.parametrize("rows,n", [(16384, 4096), (100, 1), (37, 7), (64, 4095), (8, 12288),
                                    (4, 20000), (300, 512), (33, 3000), (5, 2052), (1, 4096)])
def test_layernorm_fwd(dev, rows, n):
    x = N((rows, n), 10, dev)
    w = N(n, 11, dev, mean=1.0, std=0.1)
    b = N(n, 12, dev, std=0.1)
    y, mu, rs = ops.layernorm_fwd(x, w, b, 1e-5)
    ry, rmu, rrs = O.layernorm_fwd(host(x), host(w), host(b), 1e-5)
    assert O.isapprox(host(y), ry, 1e-5)
    assert O.isapprox(host(mu), rmu, 1e-5)
    assert O.isapprox(host(rs), rrs, 1e-5)


@pytest.mark.parametrize("rows,n,groups", [(16384, 4096, None), (100, 4, None), (37, 1000, 5),
                                           (64, 8192, None), (8, 12288, 3), (5, 16384, None),
                                           (1000, 512, 1)])
def test_layernorm_bwd(dev, rows, n, groups):
    x = N((rows, n), 20, dev)
    dy = N((rows, n), 21, dev)
    w = N(n, 22, dev, mean=1.0, std=0.1)
    b = N(n, 23, dev, std=0.1)
    _, mu, rs = ops.layernorm_fwd(x, w, b, 1e-5)
    dx, dw, db = ops.layernorm_bwd(x, dy, w, mu, rs, groups=groups)
    rdx, rdw, rdb = O.layernorm_bwd(host(x), host(dy), host(w), host(mu), host(rs))
    assert O.isapprox(host(dx), rdx, 1e-5)
    assert O.isapprox(host(dw), rdw, 1e-5)
    assert O.isapprox(host(db), rdb, 1e-5)


def test_layernorm_bwd_registry(dev):
    from cutile_b200 import TileArray

    rows, n = 48, 1024
    k = cb.triton_kernel("layernorm_bwd", [TileArray(torch.float32, 2)] * 2 +
                         [TileArray(torch.float32, 1)] * 2 + [TileArray(torch.float32, 2)] +
                         [TileArray(torch.float32, 1)] * 3 + [TileArray(torch.float32, 2)])
    x, dy = N((rows, n), 24, dev), N((rows, n), 25, dev)
    w = N(n, 26, dev, mean=1.0, std=0.1)
    _, mu, rs = ops.layernorm_fwd(x, w, torch.zeros(n, device=dev))
    dx = torch.empty_like(x)
    dw, db = torch.empty(n, device=dev), torch.empty(n, device=dev)
    partial = torch.empty(2 * 7, n, device=dev)  # Julia (N, 2G), G = 7
    cb.launch(k, 1, dx, dy, dw, db, x, w, mu, rs, partial)
    rdx, rdw, rdb = O.layernorm_bwd(host(x), host(dy), host(w), host(mu), host(rs))
    assert O.isapprox(host(dx), rdx, 1e-5) and O.isapprox(host(dw), rdw, 1e-5)
    assert O.isapprox(host(db), rdb, 1e-5)


@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.float64])
@pytest.mark.parametrize("M,N_", [(8192, 8192), (1000, 37), (1, 5), (65, 129)])
def test_transpose_bit_exact(dev, dt, M, N_):
    x = U((N_, M), 90, dev, dt)  # Julia M x N
    y = ops.transpose(x)         # Julia N x M
    assert host(y).tobytes() == np.ascontiguousarray(host(x).T).tobytes()


def test_transpose_registry_padded_columns(dev):
    from cutile_b200 import TileArray

    k = cb.triton_kernel("transpose", [TileArray(torch.float32, 2)] * 2)
    store = U((50, 80), 91, dev)
    x = cb.JlArray(store[:, :70], (70, 50), (1, 80))  # Julia 70 x 50, column stride 80
    y = torch.zeros(70, 50, device=dev)               # Julia 50 x 70
    cb.launch(k, 1, x, y)
    assert host(y).tobytes() == np.ascontiguousarray(host(store)[:, :70].T).tobytes()


# ----------------------------------------------------------------------------- GEMM
def gemm_case(dev, M, N_, K, seed, lda=None, ldb=None):
    lda = lda or M
    ldb = ldb or K
    A_store = U((K, lda), seed, dev, torch.float16)
    B_store = U((N_, ldb), seed + 1, dev, torch.float16)
    A_t = A_store[:, :M]
    B_t = B_store[:, :K]
    C_t = ops.matmul(A_t, B_t)
    ref = O.matmul(host(A_t).astype(np.float64), host(B_t).astype(np.float64))
    return host(C_t), ref


@pytest.mark.parametrize("M,N_,K", [(128, 256, 64), (256, 512, 128), (512, 512, 512),
                                    (200, 300, 100), (136, 264, 72), (8, 8, 8), (1024, 768, 4096),
                                    (2048, 2048, 2048)])
def test_gemm_f16_tensor_core(dev, M, N_, K):
    got, ref = gemm_case(dev, M, N_, K, 30)
    err = O.rel_fro(got, ref)
    assert err <= 2e-3, err
    ops.check_device()


@pytest.mark.parametrize("M,N_,K", [(300, 260, 200), (33, 17, 5)])
def test_gemm_f16_general_path(dev, M, N_, K):
    got, ref = gemm_case(dev, M, N_, K, 31)  # lda = M * 2 bytes not 16B-aligned
    assert O.rel_fro(got, ref) <= 2e-3


def test_gemm_f16_padded_leading_dims(dev):
    got, ref = gemm_case(dev, 200, 136, 96, 32, lda=256, ldb=128)
    assert O.rel_fro(got, ref) <= 2e-3


def test_gemm_k_zero(dev):
    A_t = torch.empty(0, 64, dtype=torch.float16, device=dev)
    B_t = torch.empty(32, 0, dtype=torch.float16, device=dev)
    C = ops.matmul(A_t, B_t)
    assert torch.count_nonzero(C).item() == 0


@pytest.mark.slow
def test_gemm_f16_full_size_sampled(dev):
    M = N_ = K = 8192  # BASELINE config
    A_t = U((K, M), 20261204, dev, torch.float16)
    B_t = U((N_, K), 20261205, dev, torch.float16)
    C_t = ops.matmul(A_t, B_t)
    ops.check_device()
    rng = np.random.default_rng(0)
    cols = rng.choice(N_, 256, replace=False)  # 256 full columns of C, f64 reference
    A = host(A_t).astype(np.float64)
    Bs = host(B_t)[cols].astype(np.float64)
    ref = Bs @ A
    got = host(C_t)[cols]
    assert O.rel_fro(got, ref) <= 2e-3


@pytest.mark.parametrize("batch,M,N_,K", [(4, 256, 256, 128), (3, 200, 136, 72), (32, 128, 256, 64)])
def test_bgemm_f16(dev, batch, M, N_, K):
    A_t = U((batch, K, M), 40, dev, torch.float16)
    B_t = U((batch, N_, K), 41, dev, torch.float16)
    C_t = ops.bmm(A_t, B_t)
    ha, hb, hc = host(A_t), host(B_t), host(C_t)
    for i in range(batch):
        ref = O.matmul(ha[i].astype(np.float64), hb[i].astype(np.float64))
        assert O.rel_fro(hc[i], ref) <= 2e-3


@pytest.mark.slow
def test_bgemm_f16_full_size_sampled(dev):
    batch, S = 32, 2048  # BASELINE config
    A_t = U((batch, S, S), 20261206, dev, torch.float16)
    B_t = U((batch, S, S), 20261207, dev, torch.float16)
    C_t = ops.bmm(A_t, B_t)
    ops.check_device()
    for i in (0, 17, 31):
        ref = O.matmul(host(A_t[i]).astype(np.float64), host(B_t[i]).astype(np.float64))
        assert O.rel_fro(host(C_t[i]), ref) <= 2e-3


# ----------------------------------------------------------------------------- fmha
def fmha_case(dev, B, H, S, D, causal, seed, rows=None, pairs=None):
    q = N((B, H, S, D), seed, dev, torch.float16)
    k = N((B, H, S, D), seed + 1, dev, torch.float16)
    v = N((B, H, S, D), seed + 2, dev, torch.float16)
    scale = 1.0 / math.sqrt(D)
    o = ops.fmha(q, k, v, scale, causal)
    ops.check_device()
    hq, hk, hv, ho = host(q), host(k), host(v), host(o)
    pairs = pairs or [(b, h) for b in range(B) for h in range(H)]
    for b, h in pairs:
        ref = O.fmha(hq[b, h], hk[b, h], hv[b, h], scale, causal, rows)
        got = ho[b, h] if rows is None else ho[b, h][rows]
        assert O.isapprox(got, ref, 1e-2), (b, h)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,H,S,D", [(1, 2, 128, 128), (2, 2, 256, 64), (1, 1, 1000, 128),
                                     (1, 2, 1024, 128), (1, 1, 77, 64), (2, 1, 600, 128),
                                     (1, 1, 1536, 128), (1, 1, 200, 128), (1, 2, 1024, 64),
                                     (2, 1, 1000, 64), (1, 1, 1536, 64)])
def test_fmha(dev, B, H, S, D, causal):
    fmha_case(dev, B, H, S, D, causal, 50)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Sq,Sk", [(300, 1000), (1000, 300), (129, 77), (512, 2048), (2048, 129)])
def test_fmha_cross_lengths(dev, Sq, Sk, D, causal):
    """seq_q != seq_k (the ABI's separate lengths): ragged key blocks, query
    blocks past the last key, and causal masks that end inside a key block."""
    q = N((1, 2, Sq, D), 80, dev, torch.float16)
    k = N((1, 2, Sk, D), 81, dev, torch.float16)
    v = N((1, 2, Sk, D), 82, dev, torch.float16)
    scale = 1.0 / math.sqrt(D)
    o = ops.fmha(q, k, v, scale, causal)
    ops.check_device()
    hq, hk, hv, ho = host(q), host(k), host(v), host(o)
    for h in range(2):
        ref = O.fmha(hq[0, h], hk[0, h], hv[0, h], scale, causal)
        assert np.all(np.isfinite(ho[0, h]))
        assert O.isapprox(ho[0, h], ref, 1e-2), h


@pytest.mark.parametrize("causal", [False, True])
def test_fmha_running_max_grows(dev, causal):
    """Scores that grow along the key axis force the running max up by more
    than the rescale threshold many times (the O rescale and exponential-redo
    paths), and large negative early scores exercise exp2 underflow."""
    B, H, S, D = 1, 2, 1024, 128
    q = N((B, H, S, D), 70, dev, torch.float16)
    k = N((B, H, S, D), 71, dev, torch.float16)
    v = N((B, H, S, D), 72, dev, torch.float16)
    ramp = torch.linspace(0.2, 6.0, S, device=dev, dtype=torch.float16).view(1, 1, S, 1)
    k = (k * ramp).contiguous()
    q = (q.abs() * 0 + 1.0).to(torch.float16) * torch.sign(k.sum(dim=2, keepdim=True))  # aligned with keys
    q = q.contiguous()
    scale = 1.0 / math.sqrt(D)
    o = ops.fmha(q, k, v, scale, causal)
    ops.check_device()
    hq, hk, hv, ho = host(q), host(k), host(v), host(o)
    for h in range(H):
        ref = O.fmha(hq[0, h], hk[0, h], hv[0, h], scale, causal)
        assert np.all(np.isfinite(ho[0, h]))
        assert O.isapprox(ho[0, h], ref, 1e-2), h


@pytest.mark.slow
@pytest.mark.parametrize("causal", [False, True])
def test_fmha_full_size_sampled(dev, causal):
    # BASELINE: batch 8, 32 heads, seqlen 8192, head_dim 128; every (b, h) pair
    # would take minutes in float64 on the host, so sample rows and pairs.
    rows = np.arange(0, 8192, 61)
    fmha_case(dev, 8, 32, 8192, 128, causal, 60, rows=rows,
              pairs=[(0, 0), (3, 17), (7, 31)])


# ----------------------------------------------------------------------------- registry
def test_registry_launch_like_runtests(dev):
    """The reference test's flow: triton_kernel + launch! + compare
    (test/runtests.jl:39-47, 58-66, 120-132)."""
    from cutile_b200 import TileArray, Constant

    def vadd(a, b, c, tile):
        pass

    def rowsum(a, out, tm, tn):
        pass

    def softmax(output, input, TILE_SIZE):
        pass

    for n in (1_024_000, 999_999):
        k = cb.triton_kernel(vadd, [TileArray(torch.float32, 1)] * 3 + [Constant(1024)])
        a, b = U(n, 1, dev), U(n, 2, dev)
        c = torch.zeros(n, device=dev)
        cb.launch(k, (n + 1023) // 1024, a, b, c)
        assert host(c).tobytes() == O.vadd(host(a), host(b)).tobytes()

    m, n = 4096, 128
    k = cb.triton_kernel(rowsum, [TileArray(torch.float32, 2)] * 2 + [Constant(64), Constant(128)])
    a = U((n, m), 3, dev)  # Julia m x n
    out = torch.zeros(1, m, device=dev)  # Julia m x 1
    cb.launch(k, m // 64, a, out)
    assert O.isapprox(host(out).ravel(), O.rowsum(host(a)), 1e-5)

    nrow, mcol = 1000, 2048
    k = cb.triton_kernel(softmax, [TileArray(torch.float32, 2)] * 2 + [Constant(1024)])
    x = U((mcol, nrow), 4, dev)  # Julia n x m: 2048 columns of 1000
    y = torch.zeros_like(x)
    cb.launch(k, 512, y, x)
    assert O.isapprox(host(y), O.softmax(host(x)), 1e-5)


def test_registry_matmul_f32_like_runtests(dev):
    from cutile_b200 import TileArray, Constant

    def matmul(A, B, C, tm, tn, tk):
        pass

    for (M, N_, K) in ((512, 512, 512), (300, 260, 200)):
        k = cb.triton_kernel(matmul, [TileArray(torch.float32, 2)] * 3 +
                             [Constant(128), Constant(128), Constant(32)])
        A, B = U((K, M), 5, dev, lo=0.0), U((N_, K), 6, dev, lo=0.0)  # CUDA.rand: U(0,1)
        C = torch.zeros(N_, M, device=dev)
        cb.launch(k, ((M + 127) // 128, (N_ + 127) // 128), A, B, C)
        ref = O.matmul(host(A), host(B))
        assert O.max_rel(host(C), ref) < 1e-3


def test_registry_layernorm_bmm_fmha(dev):
    from cutile_b200 import TileArray, Constant

    k = cb.triton_kernel("layer_norm_fwd", [TileArray(torch.float32, 2)] + [TileArray(torch.float32, 1)] * 2 +
                         [TileArray(torch.float32, 2)] + [TileArray(torch.float32, 1)] * 2 + [float, Constant(1024)])
    rows, n = 64, 1024
    X = N((rows, n), 1, dev)
    W, Bv = N(n, 2, dev, mean=1.0, std=0.1), N(n, 3, dev, std=0.1)
    Y, Mu, Rs = torch.empty_like(X), torch.empty(rows, device=dev), torch.empty(rows, device=dev)
    cb.launch(k, rows, X, W, Bv, Y, Mu, Rs, 1e-5)
    ry, rmu, rrs = O.layernorm_fwd(host(X), host(W), host(Bv))
    assert O.isapprox(host(Y), ry, 1e-5) and O.isapprox(host(Rs), rrs, 1e-5)

    k = cb.triton_kernel("batchmatmul", [TileArray(torch.float16, 3)] * 3)
    A, B = U((2, 64, 128), 4, dev, torch.float16), U((2, 256, 64), 5, dev, torch.float16)
    C = torch.empty(2, 256, 128, dtype=torch.float16, device=dev)
    cb.launch(k, 1, A, B, C)
    for i in range(2):
        assert O.rel_fro(host(C[i]), O.matmul(host(A[i]).astype(np.float64),
                                               host(B[i]).astype(np.float64))) <= 2e-3

    k = cb.triton_kernel("fmha", [TileArray(torch.float16, 4)] * 4 + [float, int])
    q, kk, v = (N((1, 2, 128, 64), s, dev, torch.float16) for s in (7, 8, 9))
    o = torch.empty_like(q)
    cb.launch(k, 1, q, kk, v, o, 0.125, 1)
    for h in range(2):
        ref = O.fmha(host(q)[0, h], host(kk)[0, h], host(v)[0, h], 0.125, True)
        assert O.isapprox(host(o)[0, h], ref, 1e-2)


def test_layout_errors_are_reported(dev):
    from cutile_b200 import TileArray

    k = cb.triton_kernel("softmax", [TileArray(torch.float32, 2)] * 2)
    x = torch.zeros(8, 16, device=dev).t()  # Julia dim 1 not contiguous
    with pytest.raises(cb.B200Error) as e:
        cb.launch(k, 1, torch.zeros(8, 16, device=dev).t(), x)
    assert e.value.status == "CTB_ERR_LAYOUT"

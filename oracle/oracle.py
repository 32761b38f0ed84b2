"""CPU oracle for the cuTile kernels of the B200 backend — TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs as the checker and the timed CPU stand-in. Nothing in
the product package imports it.

The C restatement (oracle/ctb_oracle.c) covers vadd, rowsum, softmax and
layernorm with OpenMP; GEMM and attention are restated here in numpy float64
(OpenBLAS dgemm). Reference expressions followed:

* vadd:     ``Array(a) .+ Array(b)``                  test/runtests.jl:46
* rowsum:   ``sum(Array(a); dims=2)``                 test/runtests.jl:66
* softmax:  ``exp.(xh .- maximum(xh; dims=1)) ./ sum(...)``  test/runtests.jl:129-131
* matmul:   ``Float32.(A) * Float32.(B)``; error = max|got-ref| / max|ref|
            bench/bench_f16.jl:27, 49-50; test/runtests.jl:95-98
* isapprox: Julia ``≈`` = norm(x-y) <= rtol*max(norm(x), norm(y))
* layernorm fwd/bwd / batchmatmul / fmha / moe: the cuTile examples are not vendored in the
  reference (parity unpinned); restated from their standard definitions.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ctb_oracle.c")
LIBDIR = os.path.join(HERE, "_build")
LIB = os.path.join(LIBDIR, "libctb_oracle.so")

# x86-64-v3 (AVX2/FMA) so the library built here also runs on the GPU hosts.
CFLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c11"]


def build(force=False):
    os.makedirs(LIBDIR, exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(SRC) > os.path.getmtime(LIB):
        subprocess.run(["gcc"] + CFLAGS + [SRC, "-o", LIB, "-lm"], check=True)
    return LIB


_lib = None
_P = ctypes.c_void_p
_I = ctypes.c_int64
_D = ctypes.c_double
_U = ctypes.c_uint64


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        sig = {
            "oracle_uniform_f64": [_P, _I, _U, _U, _D, _D],
            "oracle_uniform_f32": [_P, _I, _U, _U, _D, _D],
            "oracle_normal_f32": [_P, _I, _U, _U, _D, _D],
            "oracle_vadd_f32": [_P, _P, _P, _I],
            "oracle_vadd_f64": [_P, _P, _P, _I],
            "oracle_rowsum": [_P, _P, _I, _I, _I, _I],
            "oracle_rowsum_f32": [_P, _P, _I, _I, _I, _I],
            "oracle_softmax": [_P, _P, _I, _I, _I, _I],
            "oracle_softmax_f32": [_P, _P, _I, _I, _I, _I],
            "oracle_layernorm_fwd": [_P] * 6 + [_I, _I, _I, _I, _D],
            "oracle_layernorm_fwd_f32": [_P] * 6 + [_I, _I, _I, _I, _D],
            "oracle_layernorm_bwd": [_P] * 8 + [_I, _I],
            "oracle_set_threads": [ctypes.c_int],
        }
        for name, args in sig.items():
            getattr(L, name).argtypes = args
            getattr(L, name).restype = None
        L.oracle_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def threads():
    return lib().oracle_threads()


def set_threads(n):
    lib().oracle_set_threads(int(n))


# ---- seeded inputs (same stream as ctb_fill_uniform / ctb_fill_normal) --------
def uniform(n, seed, lo=-1.0, hi=1.0, offset=0, dtype=np.float32):
    """Element i = lo + (hi-lo) * (top 24 bits of splitmix64(seed, offset+i)) / 2^24,
    rounded to `dtype` (round to nearest). Bit-identical to ctb_fill_uniform."""
    d = np.empty(n, np.float64)
    lib().oracle_uniform_f64(_p(d), n, seed, offset, lo, hi)
    return d.astype(dtype)


def normal(n, seed, mean=0.0, std=1.0, offset=0):
    """Box-Muller normals in double rounded to float32 (matches ctb_fill_normal
    up to the last bit of the host/device log and cos)."""
    out = np.empty(n, np.float32)
    lib().oracle_normal_f32(_p(out), n, seed, offset, mean, std)
    return out


# ---- the kernels (checker: double accumulation) --------------------------------
def vadd(a, b):
    """``a .+ b`` elementwise in the arrays' own type (bit-exact reference)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.dtype == np.float32:
        c = np.empty_like(a)
        lib().oracle_vadd_f32(_p(a), _p(b), _p(c), a.size)
        return c
    if a.dtype == np.float64:
        c = np.empty_like(a)
        lib().oracle_vadd_f64(_p(a), _p(b), _p(c), a.size)
        return c
    if a.dtype == np.float16:
        # Julia's Float16 + rounds the exact float32 sum to Float16; with 24 >=
        # 2*11+2 significand bits this equals the correctly rounded f16 add.
        return (a.astype(np.float32) + b.astype(np.float32)).astype(np.float16)
    raise TypeError(a.dtype)


def rowsum(a_jl):
    """``sum(a; dims=2)`` of a Julia-layout (m x n) array given as the numpy
    array of its column-major storage, i.e. shape (n, m) row-major."""
    a = np.ascontiguousarray(a_jl, dtype=np.float32)
    n, m = a.shape
    out = np.empty(m, np.float32)
    lib().oracle_rowsum(_p(a), _p(out), m, n, 1, m)
    return out


def rowsum_rowmajor(a):
    """Sum of each row of a row-major (rows x n) float32 matrix."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    m, n = a.shape
    out = np.empty(m, np.float32)
    lib().oracle_rowsum(_p(a), _p(out), m, n, n, 1)
    return out


def softmax(x):
    """Row-wise softmax of a (count x len) row-major float32 matrix."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    count, length = x.shape
    y = np.empty_like(x)
    lib().oracle_softmax(_p(x), _p(y), length, count, length, length)
    return y


def layernorm_fwd(x, w, b, eps=1e-5):
    """LayerNorm over each row of a (rows x n) float32 matrix -> (y, mean, rstd)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    rows, n = x.shape
    y = np.empty_like(x)
    mu = np.empty(rows, np.float32)
    rs = np.empty(rows, np.float32)
    lib().oracle_layernorm_fwd(_p(x), _p(w), _p(b), _p(y), _p(mu), _p(rs), n, rows, n, n, eps)
    return y, mu, rs


def layernorm_bwd(x, dy, w, mean, rstd):
    """LayerNorm backward on (rows x n) float32 matrices -> (dx f32, dw f64, db f64)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    dy = np.ascontiguousarray(dy, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    mean = np.ascontiguousarray(mean, dtype=np.float32)
    rstd = np.ascontiguousarray(rstd, dtype=np.float32)
    rows, n = x.shape
    dx = np.empty_like(x)
    dw = np.empty(n, np.float64)
    db = np.empty(n, np.float64)
    lib().oracle_layernorm_bwd(_p(x), _p(dy), _p(w), _p(mean), _p(rstd), _p(dx), _p(dw), _p(db),
                               n, rows)
    return dx, dw, db


def matmul(A, B):
    """Float64 product of column-major Julia operands given in numpy as their
    transposes' storage: A_jl (M x K) is passed as a (K, M) array etc.
    Returns C_jl as a (N, M) float64 array (C^T row-major = C column-major)."""
    At = np.asarray(A, dtype=np.float64)  # (K, M) = A^T
    Bt = np.asarray(B, dtype=np.float64)  # (N, K) = B^T
    return Bt @ At  # (N, M) = (A B)^T


def fmha(q, k, v, scale, causal=False, rows=None):
    """Attention for one (batch, head): q (Sq, D), k/v (Sk, D) in float64.
    `rows` optionally restricts to a subset of query rows. Causal masks key
    j > query i (top-left aligned)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    idx = np.arange(q.shape[0]) if rows is None else np.asarray(rows)
    s = (q[idx] @ k.T) * scale
    if causal:
        mask = np.arange(k.shape[0])[None, :] > idx[:, None]
        s = np.where(mask, -np.inf, s)
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return p @ v


def moe_align(topk_ids, num_experts, block=128):
    """Fused-MoE routing restated with plain loops: slots (token*topk + j) of
    each expert in slot order, each expert padded to a multiple of `block`
    with the id M*topk; returns (sorted_ids, expert_ids, num_post_padded)."""
    flat = np.asarray(topk_ids, np.int64).ravel()
    n = flat.size
    sorted_ids, expert_ids = [], []
    for e in range(num_experts):
        slots = [s for s in range(n) if flat[s] == e]
        pad = (-len(slots)) % block
        sorted_ids += slots + [n] * pad
        expert_ids += [e] * ((len(slots) + pad) // block)
    em = len(sorted_ids)
    if em == 0:
        sorted_ids, expert_ids = [n] * block, [-1]
    return (np.asarray(sorted_ids, np.int32), np.asarray(expert_ids, np.int32), em)


def moe(A, B, sorted_ids, expert_ids, num_post_padded, topk, weights=None, block=128):
    """Float64 fused-MoE GEMM: rows C[s] = A[s // topk] @ B[e].T (* weights[s])
    for each listed slot s < M*topk of a block (below num_post_padded) of a
    valid expert e; rows never listed stay zero. A (M, K); B (E, N, K)."""
    A = np.asarray(A, np.float64)
    B = np.asarray(B, np.float64)
    M = A.shape[0]
    E, N, _ = B.shape
    w = None if weights is None else np.asarray(weights, np.float64).ravel()
    C = np.zeros((M * topk, N))
    nblk = min(len(expert_ids), (int(num_post_padded) + block - 1) // block)
    for b in range(nblk):
        e = int(expert_ids[b])
        if not 0 <= e < E:
            continue
        ids = np.asarray(sorted_ids[b * block:(b + 1) * block], np.int64)
        ids = ids[(ids >= 0) & (ids < M * topk)]
        if ids.size == 0:
            continue
        rows = A[ids // topk] @ B[e].T
        if w is not None:
            rows *= w[ids][:, None]
        C[ids] = rows
    return C


# ---- float-accumulating variants: the timed CPU baseline ------------------------
def vadd_f32_into(a, b, c):
    lib().oracle_vadd_f32(_p(a), _p(b), _p(c), a.size)


def rowsum_f32_into(a, out, m, n, si, sj):
    lib().oracle_rowsum_f32(_p(a), _p(out), m, n, si, sj)


def softmax_f32_into(x, y, length, count):
    lib().oracle_softmax_f32(_p(x), _p(y), length, count, length, length)


def layernorm_f32_into(x, w, b, y, mu, rs, n, rows, eps):
    lib().oracle_layernorm_fwd_f32(_p(x), _p(w), _p(b), _p(y), _p(mu), _p(rs), n, rows, n, n, eps)


# ---- comparison helpers ------------------------------------------------------------
def isapprox(got, ref, rtol):
    """Julia ``isapprox`` on arrays: norm(got-ref) <= rtol*max(norm(got), norm(ref))."""
    g = np.asarray(got, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    if not (np.all(np.isfinite(g)) and np.all(np.isfinite(r))):
        return False
    return np.linalg.norm(g - r) <= rtol * max(np.linalg.norm(g), np.linalg.norm(r))


def rel_fro(got, ref):
    """Relative Frobenius error ||got-ref|| / ||ref||."""
    g = np.asarray(got, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    return float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-300))


def max_rel(got, ref):
    """The reference matmul metric: max|got-ref| / max(max|ref|, 1)
    (test/runtests.jl:95-98)."""
    g = np.asarray(got, np.float64)
    r = np.asarray(ref, np.float64)
    return float(np.max(np.abs(g - r)) / max(np.max(np.abs(r)), 1.0))

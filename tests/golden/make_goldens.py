"""Generates the golden vectors in tests/golden/ by running the REFERENCE's own
kernels on a GPU — test infrastructure.

The kernels are the reference's TileTriton-emitted TTIR (vadd, rowsum) and
its Python-Triton twin of the persistent column softmax, compiled for sm_100
by oracle/build_ref.py into oracle/_ref/ (run that first, in a tree that has
the reference). This script loads those cubins with the CUDA driver API,
feeds them seeded inputs from the oracle's SplitMix64 generator (the same
bits tests regenerate on the host), and writes:

  ref_goldens.json  sha256 of every full output + metadata
  ref_goldens.npz   rowsum outputs and sampled softmax columns

With `matmul` as the first argument it instead runs the reference's tf32
matmul TTIR (test/runtests.jl:70-98 shapes, grid (cld(M,128), cld(N,128)))
and writes ref_goldens_matmul.json / .npz (full outputs).

With `softmax_baseline` it runs the reference's softmax twin compiled with
TILE = 16384 on the BASELINE config (4096 vectors of 16384 Float32, entries
4*N(0,1) from oracle.normal, seed 20261201) and writes
ref_goldens_softmax_baseline.json / .npz: the sha256 of the full output,
per-vector checksums (max, sum and index-weighted sum, in float64) of all
4096 vectors, and 4 sampled vectors in full.

Usage (on a machine with a B200):
    python tests/golden/make_goldens.py [matmul | softmax_baseline] [OUT_DIR]
(OUT_DIR defaults to tests/golden/).
"""
import ctypes
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
REF = os.path.join(ROOT, "oracle", "_ref")

# Shapes: the reference's own test cases (test/runtests.jl:39, 58, 120) and
# the BASELINE vadd size.
VADD_CASES = [(1_024_000, 1, 2), (999_999, 1, 2), (1 << 28, 20261201, 20261202)]
ROWSUM_CASES = [(4096, 128, 3), (131072, 128, 5)]
SOFTMAX_CASE = (1000, 2048, 4, 512)  # n_rows, n_cols, seed, grid
SOFTMAX_COLS = list(range(8)) + list(range(8, 2048, 256))
SOFTMAX_BASELINE = (16384, 4096, 20261201, 1184)  # length, count, seed, grid (8 x 148)
SOFTMAX_BASELINE_VECS = [0, 1, 2047, 4095]


def softmax_vector_stats(y):
    """Per-vector (max, sum, index-weighted sum) of a (count, length) softmax
    output in float64: a checksum of every vector, compared with the rtol."""
    y64 = y.astype(np.float64)
    idx = np.arange(1, y.shape[1] + 1, dtype=np.float64) / y.shape[1]
    return np.stack([y64.max(axis=1), y64.sum(axis=1), y64 @ idx], axis=1)


MATMUL_CASES = [(512, 512, 512, 31, 32), (300, 260, 200, 33, 34)]  # test/runtests.jl:86


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    import torch
    from cuda.bindings import driver as cu

    from oracle import oracle as O

    torch.cuda.init()
    dev = torch.device("cuda:0")
    torch.zeros(1, device=dev)  # creates the primary context
    (err,) = cu.cuInit(0)
    assert err == cu.CUresult.CUDA_SUCCESS, err

    def load(name):
        md = json.load(open(os.path.join(REF, name + ".json")))
        data = open(os.path.join(REF, name + ".cubin"), "rb").read()
        err, mod = cu.cuModuleLoadData(data)
        assert err == cu.CUresult.CUDA_SUCCESS, (name, err)
        err, fn = cu.cuModuleGetFunction(mod, md["name"].encode())
        assert err == cu.CUresult.CUDA_SUCCESS, (name, err)
        return mod, fn, md

    def launch(k, grid, args):
        _, fn, md = k
        ptrs = (ctypes.c_void_p * len(args))(*[ctypes.addressof(a) for a in args])
        st = torch.cuda.current_stream().cuda_stream
        gx, gy = grid if isinstance(grid, tuple) else (grid, 1)
        if md["shared"] > 48 * 1024:
            (err,) = cu.cuFuncSetAttribute(
                fn, cu.CUfunction_attribute.CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                md["shared"])
            assert err == cu.CUresult.CUDA_SUCCESS, err
        (err,) = cu.cuLaunchKernel(fn, gx, gy, 1, md["num_warps"] * 32, 1, 1, md["shared"], st,
                                   ctypes.addressof(ptrs), 0)
        assert err == cu.CUresult.CUDA_SUCCESS, err
        torch.cuda.synchronize()

    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    I = ctypes.c_int32  # noqa: E741
    NULL = ctypes.c_void_p(0)
    if len(sys.argv) > 1 and sys.argv[1] == "softmax_baseline":
        k = load("softmax_py_16384")
        length, count, seed, grid = SOFTMAX_BASELINE
        xh = O.normal(length * count, seed, 0.0, 4.0).reshape(count, length)
        x = torch.from_numpy(xh).to(dev)
        y = torch.zeros_like(x)
        launch(k, grid, [P(y), P(x), I(length), I(count), I(length), I(length), NULL, NULL])
        hy = y.cpu().numpy()
        st = softmax_vector_stats(hy)
        res = {"kernel": "bench/bench_compile.py:45-57 softmax, TILE 16384, 16 warps",
               "length": length, "count": count, "seed": seed, "mean": 0.0, "std": 4.0,
               "generator": "oracle.normal (SplitMix64 + Box-Muller)", "grid": grid,
               "sha256_input": sha(xh), "sha256": sha(hy), "sampled_vectors": SOFTMAX_BASELINE_VECS}
        dst = sys.argv[2] if len(sys.argv) > 2 else HERE
        os.makedirs(dst, exist_ok=True)
        with open(os.path.join(dst, "ref_goldens_softmax_baseline.json"), "w") as f:
            json.dump(res, f, indent=1)
        np.savez_compressed(os.path.join(dst, "ref_goldens_softmax_baseline.npz"), stats=st,
                            vectors=hy[SOFTMAX_BASELINE_VECS])
        print("softmax baseline", sha(hy)[:16])
        return 0
    if len(sys.argv) > 1 and sys.argv[1] == "matmul":
        k = load("matmul_ttir")
        gss, gsa = k[2]["global_scratch_size"], k[2]["global_scratch_align"]
        mout = {"generator": "SplitMix64 counter stream, oracle.uniform(lo=0, hi=1)",
                "kernel": "research/matmul_emitted.ttir (tf32, 128x128x32, 8 warps)",
                "cases": []}
        marrays = {}
        for M, N, K, sa, sb in MATMUL_CASES:
            A_jl = O.uniform(M * K, sa, lo=0.0, hi=1.0).reshape(K, M)  # Julia M x K, stride (1, M)
            B_jl = O.uniform(K * N, sb, lo=0.0, hi=1.0).reshape(N, K)  # Julia K x N, stride (1, K)
            A, B = torch.from_numpy(A_jl).to(dev), torch.from_numpy(B_jl).to(dev)
            C = torch.zeros(N, M, device=dev)  # Julia M x N
            grid = ((M + 127) // 128, (N + 127) // 128)
            scratch = torch.zeros(grid[0] * grid[1] * gss + gsa, dtype=torch.uint8, device=dev)
            sp = ctypes.c_void_p((scratch.data_ptr() + gsa - 1) // gsa * gsa)
            launch(k, grid, [P(A), I(M), I(K), I(1), I(M), P(B), I(K), I(N), I(1), I(K),
                             P(C), I(M), I(N), I(1), I(M), sp, NULL])
            hc = C.cpu().numpy()
            mout["cases"].append({"M": M, "N": N, "K": K, "seed_a": sa, "seed_b": sb,
                                  "sha256": sha(hc)})
            marrays[f"matmul_{M}x{N}x{K}"] = hc
            print("matmul", M, N, K, sha(hc)[:16])
        dst = sys.argv[2] if len(sys.argv) > 2 else HERE
        os.makedirs(dst, exist_ok=True)
        with open(os.path.join(dst, "ref_goldens_matmul.json"), "w") as f:
            json.dump(mout, f, indent=1)
        np.savez_compressed(os.path.join(dst, "ref_goldens_matmul.npz"), **marrays)
        print("written", os.path.join(dst, "ref_goldens_matmul.json"))
        return 0

    out = {"generator": "SplitMix64 counter stream, oracle.uniform (see oracle/ctb_oracle.c)",
           "kernels": "reference TTIR / Python-Triton twins compiled by oracle/build_ref.py",
           "vadd": [], "rowsum": [], "softmax": {}}
    arrays = {}

    k = load("vadd_ttir")
    for n, sa, sb in VADD_CASES:
        a = torch.from_numpy(O.uniform(n, sa)).to(dev)
        b = torch.from_numpy(O.uniform(n, sb)).to(dev)
        c = torch.zeros(n, device=dev)
        launch(k, (n + 1023) // 1024, [P(a), I(n), I(1), P(b), I(n), I(1), P(c), I(n), I(1), NULL, NULL])
        hc = c.cpu().numpy()
        out["vadd"].append({"n": n, "seed_a": sa, "seed_b": sb, "sha256": sha(hc),
                            "head": hc[:8].tolist()})
        print("vadd", n, sha(hc)[:16])

    k = load("rowsum_ttir")
    gss, gsa = k[2]["global_scratch_size"], k[2]["global_scratch_align"]
    for m, n, seed in ROWSUM_CASES:
        a_jl = O.uniform(m * n, seed, lo=0.0, hi=1.0).reshape(n, m)  # Julia m x n, stride (1, m)
        a = torch.from_numpy(a_jl).to(dev)
        o = torch.zeros(m, device=dev)
        grid = (m + 63) // 64
        scratch = torch.zeros(grid * gss + gsa, dtype=torch.uint8, device=dev)
        sp = ctypes.c_void_p((scratch.data_ptr() + gsa - 1) // gsa * gsa)
        launch(k, grid, [P(a), I(m), I(n), I(1), I(m), P(o), I(m), I(1), I(1), I(m), sp, NULL])
        ho = o.cpu().numpy()
        out["rowsum"].append({"m": m, "n": n, "seed": seed, "lo": 0.0, "hi": 1.0, "sha256": sha(ho)})
        arrays[f"rowsum_{m}x{n}"] = ho
        print("rowsum", m, n, sha(ho)[:16])

    k = load("softmax_py")
    n_rows, n_cols, seed, grid = SOFTMAX_CASE
    x_jl = O.uniform(n_rows * n_cols, seed, lo=0.0, hi=1.0).reshape(n_cols, n_rows)
    x = torch.from_numpy(x_jl).to(dev)
    y = torch.zeros_like(x)
    launch(k, grid, [P(y), P(x), I(n_rows), I(n_cols), I(n_rows), I(n_rows), NULL, NULL])
    hy = y.cpu().numpy()
    out["softmax"] = {"n_rows": n_rows, "n_cols": n_cols, "seed": seed, "lo": 0.0, "hi": 1.0,
                      "grid": grid, "sha256": sha(hy), "sampled_columns": SOFTMAX_COLS}
    arrays["softmax_sampled"] = hy[SOFTMAX_COLS]
    print("softmax", sha(hy)[:16])

    dst = sys.argv[1] if len(sys.argv) > 1 else HERE
    os.makedirs(dst, exist_ok=True)
    with open(os.path.join(dst, "ref_goldens.json"), "w") as f:
        json.dump(out, f, indent=1)
    np.savez_compressed(os.path.join(dst, "ref_goldens.npz"), **arrays)
    print("written", os.path.join(dst, "ref_goldens.json"))
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""The sm_100a kernels against golden vectors produced by the reference's own
kernels (tests/golden/make_goldens.py): bit-exact vadd, rowsum and softmax
within the reference's ≈ tolerance."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from cutile_b200 import ops
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
G = json.load(open(os.path.join(HERE, "ref_goldens.json")))
A = np.load(os.path.join(HERE, "ref_goldens.npz"))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", G["vadd"], ids=lambda c: f"n={c['n']}")
def test_vadd_matches_reference_kernel_bits(dev, case):
    n = case["n"]
    a = ops.fill_uniform(torch.empty(n, device=dev), case["seed_a"])
    b = ops.fill_uniform(torch.empty(n, device=dev), case["seed_b"])
    c = ops.vadd(a, b)
    torch.cuda.synchronize()
    assert sha(c.cpu().numpy()) == case["sha256"]


@pytest.mark.parametrize("case", G["rowsum"], ids=lambda c: f"{c['m']}x{c['n']}")
def test_rowsum_matches_reference_kernel(dev, case):
    m, n = case["m"], case["n"]
    a = ops.fill_uniform(torch.empty(n, m, device=dev), case["seed"], case["lo"], case["hi"])
    out = ops.rowsum(a)
    torch.cuda.synchronize()
    assert O.isapprox(out.cpu().numpy(), A[f"rowsum_{m}x{n}"], 1e-5)


def test_softmax_matches_reference_kernel(dev):
    c = G["softmax"]
    x = ops.fill_uniform(torch.empty(c["n_cols"], c["n_rows"], device=dev), c["seed"], c["lo"],
                         c["hi"])
    y = ops.softmax(x)
    torch.cuda.synchronize()
    got = y.cpu().numpy()[c["sampled_columns"]]
    assert O.isapprox(got, A["softmax_sampled"], 1e-5)


GM = json.load(open(os.path.join(HERE, "ref_goldens_matmul.json")))
AM = np.load(os.path.join(HERE, "ref_goldens_matmul.npz"))


@pytest.mark.parametrize("case", GM["cases"], ids=lambda c: f"{c['M']}x{c['N']}x{c['K']}")
def test_float32_matmul_matches_reference_tf32_kernel(dev, case):
    """Our Float32 matmul (registry `matmul`, the reference test's launch) on the
    inputs the reference's tf32 kernel saw, against that kernel's output with
    test/runtests.jl:95-98's metric and tolerance."""
    import cutile_b200 as cb
    from cutile_b200 import Constant, TileArray

    def matmul(A, B, C, tm, tn, tk):
        pass

    M, N, K = case["M"], case["N"], case["K"]
    A = torch.empty(K, M, device=dev)
    B = torch.empty(N, K, device=dev)
    ops.fill_uniform(A, case["seed_a"], 0.0, 1.0)
    ops.fill_uniform(B, case["seed_b"], 0.0, 1.0)
    C = torch.zeros(N, M, device=dev)
    k = cb.triton_kernel(matmul, [TileArray(torch.float32, 2)] * 3 +
                         [Constant(128), Constant(128), Constant(32)])
    cb.launch(k, ((M + 127) // 128, (N + 127) // 128), A, B, C)
    torch.cuda.synchronize()
    got = C.cpu().numpy()
    if M == 512:
        cols = GM["sampled"]["512x512x512"]["julia_columns_n"]
        got, ref = got[cols], AM["matmul_512x512x512_cols"]
    else:
        ref = AM[f"matmul_{M}x{N}x{K}"]
    assert O.max_rel(got, ref) < 1e-3


_SB = os.path.join(HERE, "ref_goldens_softmax_baseline.json")


@pytest.mark.slow
@pytest.mark.skipif(not os.path.exists(_SB), reason="BASELINE-size softmax golden not generated")
def test_softmax_baseline_config_matches_reference_kernel(dev):
    """The headline config (4096 vectors of 16384 Float32, 4*N(0,1)) against
    the reference's own softmax kernel compiled with TILE = 16384: every
    vector's checksums and four whole vectors within rtol 1e-5."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_goldens",
                                                  os.path.join(HERE, "make_goldens.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    softmax_vector_stats = mg.softmax_vector_stats
    c = json.load(open(_SB))
    g = np.load(_SB.replace(".json", ".npz"))
    xh = O.normal(c["length"] * c["count"], c["seed"], c["mean"], c["std"]).reshape(
        c["count"], c["length"])
    assert sha(xh) == c["sha256_input"]
    y = ops.softmax(torch.from_numpy(xh).to(dev))
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    st = softmax_vector_stats(got)
    ref = g["stats"]
    for j in range(3):
        assert O.isapprox(st[:, j], ref[:, j], 1e-5), j
    rel = np.abs(st - ref) / np.abs(ref)
    assert rel.max() < 1e-4, rel.max()
    for i, v in zip(c["sampled_vectors"], g["vectors"]):
        assert O.isapprox(got[i], v, 1e-5), i

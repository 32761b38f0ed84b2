"""Parity of the gather-routed MoE GEMM (ctb_moe_gemm_f16) against the float64
oracle. Tolerance: relative Frobenius error <= 2e-3 (the f16 GEMM bound), and
rows that no block lists must be left untouched (exactly as preset)."""
import numpy as np
import pytest
import torch

from cutile_b200 import _lib, ops
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def routing(M, E, topk, seed, skew=False):
    g = torch.Generator().manual_seed(seed)
    r = torch.rand(M, E, generator=g)
    if skew:  # expert 0 never chosen, expert 1 almost always
        r[:, 0] = -1.0
        r[:, 1] += 1.0
    return torch.argsort(r, dim=1, descending=True)[:, :topk].to(torch.int32)


def make(dev, M, N, K, E, seed):
    A = torch.empty(M, K, dtype=torch.float16, device=dev)
    B = torch.empty(E, N, K, dtype=torch.float16, device=dev)
    ops.fill_uniform(A, seed, -1.0, 1.0)
    ops.fill_uniform(B, seed + 1, -1.0, 1.0)
    return A, B


@pytest.mark.parametrize("block", [128, 256])
@pytest.mark.parametrize("M,N,K,E,topk,weighted,skew", [
    (64, 256, 128, 4, 2, False, False),
    (300, 200, 136, 7, 3, True, False),
    (1000, 512, 64, 8, 2, True, True),
    (5, 64, 8, 3, 1, False, False),
    (2048, 768, 512, 16, 4, True, False),
])
def test_moe_gemm(dev, M, N, K, E, topk, weighted, skew, block):
    A, B = make(dev, M, N, K, E, 21 + M)
    ids = routing(M, E, topk, M, skew)
    sid, eid, ntp = ops.moe_align(ids.to(dev), E, block)
    w = torch.rand(M, topk, generator=torch.Generator().manual_seed(3)).to(dev) if weighted else None
    C = ops.moe_gemm(A, B, sid, eid, ntp, topk, w)
    torch.cuda.synchronize()
    ref = O.moe(A.cpu().numpy(), B.cpu().numpy(), sid.cpu().numpy(), eid.cpu().numpy(),
                int(ntp.item()), topk, None if w is None else w.cpu().numpy(), block=block)
    got = C.cpu().numpy().astype(np.float64)
    assert O.rel_fro(got, ref) <= 2e-3
    assert np.all(np.isfinite(got))


@pytest.mark.parametrize("block", [128, 256])
def test_moe_align_matches_oracle_loops(dev, block):
    """The device routing kernel against the oracle's loops: the oracle's
    exact-size lists are a prefix of the worst-case-size device outputs, the
    rest holds the padding id (sorted ids) and -1 (expert ids)."""
    cases = [(333, 9, 3, 5, True), (1, 4, 1, 0, False), (7, 64, 4, 3, False),
             (5000, 256, 2, 9, True), (2048, 8, 2, 11, False)]
    for M, E, topk, seed, skew in cases:
        ids = routing(M, E, topk, seed, skew=skew)
        s, e, n = ops.moe_align(ids.to(dev), E, block)
        rs, re, rn = O.moe_align(ids.numpy(), E, block)
        s, e = s.cpu().numpy(), e.cpu().numpy()
        cap = int(_lib.load().ctb_moe_align_capacity(M * topk, E, block))
        assert s.size == cap and e.size == cap // block
        np.testing.assert_array_equal(s[:rs.size], rs)
        assert np.all(s[rs.size:] == M * topk)
        np.testing.assert_array_equal(e[:re.size], re)
        assert np.all(e[re.size:] == -1)
        assert int(n.item()) == rn


def test_moe_align_empty_and_errors(dev):
    ids = torch.empty(0, 2, dtype=torch.int32, device=dev)
    s, e, n = ops.moe_align(ids, 4, 128)
    assert int(n.item()) == 0 and bool((e.cpu() == -1).all()) and bool((s.cpu() == 0).all())
    with pytest.raises(_lib.B200Error):
        ops.moe_align(torch.zeros(4, 2, dtype=torch.int32, device=dev), 300, 128)


@pytest.mark.parametrize("block", [128, 256])
def test_moe_unlisted_rows_and_invalid_blocks_untouched(dev, block):
    """Blocks past num_tokens_post_padded and blocks with expert id -1 are
    skipped; the rows they list keep their preset value."""
    M, N, K, E, topk = 2 * block, 256, 128, 2, 1
    A, B = make(dev, M, N, K, E, 7)
    sid = torch.arange(M, dtype=torch.int32, device=dev)            # 2 blocks
    eid = torch.tensor([-1, 1], dtype=torch.int32, device=dev)
    ntp = torch.tensor([M], dtype=torch.int32, device=dev)
    out = torch.full((M, N), 3.0, dtype=torch.float16, device=dev)
    ops.moe_gemm(A, B, sid, eid, ntp, topk, out=out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(got[:block] == 3.0)
    ref = A.cpu().double()[block:] @ B.cpu().double()[1].T
    assert O.rel_fro(got[block:], ref.numpy()) <= 2e-3
    # num_tokens_post_padded below EM: the second block is no longer in use
    out.fill_(3.0)
    ntp.fill_(block)
    eid[0] = 0
    ops.moe_gemm(A, B, sid, eid, ntp, topk, out=out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(got[block:] == 3.0)
    assert O.rel_fro(got[:block], (A.cpu().double()[:block] @ B.cpu().double()[0].T).numpy()) <= 2e-3


def test_moe_bad_layout_reported(dev):
    A = torch.zeros(16, 12, dtype=torch.float16, device=dev)  # K % 8 != 0
    B = torch.zeros(2, 64, 12, dtype=torch.float16, device=dev)
    sid = torch.zeros(128, dtype=torch.int32, device=dev)
    eid = torch.zeros(1, dtype=torch.int32, device=dev)
    ntp = torch.tensor([128], dtype=torch.int32, device=dev)
    with pytest.raises(Exception):
        ops.moe_gemm(A, B, sid, eid, ntp, 1)


def test_moe_through_the_registry(dev):
    """triton_kernel("moe", ...) / launch with TileArrays in cuTile order, as
    the TileTriton shim calls it."""
    import cutile_b200 as cb
    from cutile_b200 import TileArray

    M, N, K, E, topk = 200, 256, 192, 5, 2
    A, B = make(dev, M, N, K, E, 99)
    ids = routing(M, E, topk, 9)
    sid, eid, ntp = ops.moe_align(ids.to(dev), E)
    w = torch.rand(M, topk, generator=torch.Generator().manual_seed(4)).to(dev)
    C = torch.zeros(M * topk, N, dtype=torch.float16, device=dev)
    ws = torch.empty(sid.numel() * K, dtype=torch.float16, device=dev)
    k = cb.triton_kernel("moe", [TileArray(torch.float16, 2), TileArray(torch.float16, 3),
                                 TileArray(torch.float16, 2)] + [TileArray(torch.int32, 1)] * 3 +
                         [TileArray(torch.float32, 2), TileArray(torch.float16, 1), int, int])
    cb.launch(k, 1, A, B, C, sid, eid, ntp, w, ws, topk, 1)
    torch.cuda.synchronize()
    ref = O.moe(A.cpu().numpy(), B.cpu().numpy(), sid.cpu().numpy(), eid.cpu().numpy(),
                int(ntp.item()), topk, w.cpu().numpy(), block=sid.numel() // eid.numel())
    assert O.rel_fro(C.cpu().numpy().astype(np.float64), ref) <= 2e-3


def test_transpose_int32_bitwise(dev):
    x = torch.randint(-2**31, 2**31 - 1, (300, 517), dtype=torch.int32, device=dev)
    y = torch.empty(517, 300, dtype=torch.int32, device=dev)
    ops.transpose(x, y)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), x.cpu().T)


def test_moe_256_row_blocks_on_the_single_sm_kernel():
    """256-row routing blocks also run on the single-SM kernel (the fallback
    when no CTA pair can be resident), forced with CTB_MOE_PAIR=0 in a child."""
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = r"""
import json, sys
sys.path.insert(0, "cutile-triton_b200"); sys.path.insert(0, ".")
import numpy as np, torch
from cutile_b200 import _lib, ops
from oracle import oracle as O
dev = torch.device("cuda", 0)
A = ops.fill_uniform(torch.empty(700, 136, dtype=torch.float16, device=dev), 1)
B = ops.fill_uniform(torch.empty(5, 296, 136, dtype=torch.float16, device=dev), 2)
g = torch.Generator().manual_seed(3)
ids = torch.argsort(torch.rand(700, 5, generator=g), dim=1)[:, :2].to(torch.int32).to(dev)
w = torch.rand(700, 2, generator=g).to(dev)
sid, eid, ntp = ops.moe_align(ids, 5, 256)
C = ops.moe_gemm(A, B, sid, eid, ntp, 2, w)
torch.cuda.synchronize(); ops.check_device()
ref = O.moe(A.cpu().numpy(), B.cpu().numpy(), sid.cpu().numpy(), eid.cpu().numpy(),
            int(ntp.item()), 2, w.cpu().numpy(), block=256)
print(json.dumps(O.rel_fro(C.cpu().numpy().astype(np.float64), ref)))
"""
    env = dict(os.environ, CTB_MOE_PAIR="0")
    r = subprocess.run([sys.executable, "-c", script], cwd=root, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert json.loads(r.stdout.strip().splitlines()[-1]) <= 2e-3

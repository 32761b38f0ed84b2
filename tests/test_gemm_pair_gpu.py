"""The CTA-pair GEMM kernel (tcgen05 cta_group::2, 256 x 256 tiles over two
SMs) on ragged shapes. The library picks it for large problems; here it is
forced with CTB_GEMM_PAIR=1 (read once per process, hence the subprocess) so
that small and ragged shapes take it too. Tolerance: relative Frobenius error
<= 2e-3 against the float64 oracle, as for the other f16 GEMM tests."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import json, sys
sys.path.insert(0, "cutile-triton_b200"); sys.path.insert(0, ".")
import numpy as np, torch
from cutile_b200 import ops
from oracle import oracle as O
dev = torch.device("cuda", 0)
out = []
for (batch, M, N, K) in [(1, 256, 256, 64), (1, 300, 260, 200), (1, 1000, 700, 136),
                         (3, 200, 520, 72), (2, 513, 257, 1000)]:
    A = ops.fill_uniform(torch.empty(batch, K, M, dtype=torch.float16, device=dev), 1)
    B = ops.fill_uniform(torch.empty(batch, N, K, dtype=torch.float16, device=dev), 2)
    C = torch.full((batch, N, M), 7.0, dtype=torch.float16, device=dev)
    if batch == 1:
        ops.matmul(A[0], B[0], C[0])
    else:
        ops.bmm(A, B, C)
    torch.cuda.synchronize()
    ops.check_device()
    errs = [O.rel_fro(C[i].cpu().numpy(), O.matmul(A[i].cpu().numpy(), B[i].cpu().numpy()))
            for i in range(batch)]
    out.append([batch, M, N, K, max(errs)])
print(json.dumps(out))
"""


def test_pair_kernel_ragged_shapes():
    env = dict(os.environ, CTB_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-c", SCRIPT], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    for batch, M, N, K, err in json.loads(r.stdout.strip().splitlines()[-1]):
        assert err <= 2e-3, (batch, M, N, K, err)

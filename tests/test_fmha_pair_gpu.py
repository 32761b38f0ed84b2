"""The CTA-pair attention kernel (tcgen05 cta_group::2: 256-row query tiles
over two SMs, each SM loading half of every K and V block). It is opt-in,
selected with CTB_FMHA_PAIR=1 (read once per process, hence the subprocess).
Shapes cover one and several 512-row query blocks, ragged lengths, causal
masks whose diagonal falls inside a block, and a running max that grows past
the rescale threshold. Tolerance: isapprox rtol 1e-2 against the float64
oracle, as for the other attention tests."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import json, math, sys
sys.path.insert(0, "cutile-triton_b200"); sys.path.insert(0, ".")
import numpy as np, torch
from cutile_b200 import ops
from oracle import oracle as O
dev = torch.device("cuda", 0)
out = []
def randn(shape, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(shape, generator=g).to(torch.float16).to(dev)
for (B, H, S, Sk, causal, ramp) in [(1, 1, 512, 512, False, False), (1, 1, 512, 512, True, False),
                                    (1, 2, 1024, 1024, True, False), (2, 1, 600, 600, False, False),
                                    (1, 1, 1000, 1000, True, False), (1, 1, 77, 77, True, False),
                                    (1, 2, 1536, 1536, False, False), (1, 1, 1024, 1024, True, True),
                                    (1, 1, 300, 1000, True, False), (1, 1, 1000, 300, True, False),
                                    (1, 1, 700, 129, False, False)]:
    q, k, v = randn((B, H, S, 128), 1), randn((B, H, Sk, 128), 2), randn((B, H, Sk, 128), 3)
    if ramp:  # scores grow along the keys: the running max moves many times
        k = (k * torch.linspace(0.2, 6.0, Sk, device=dev, dtype=torch.float16).view(1, 1, S, 1)).contiguous()
        q = (torch.ones_like(q) * torch.sign(k.sum(dim=2, keepdim=True))).contiguous()
    o = ops.fmha(q, k, v, 1.0 / math.sqrt(128), causal)
    torch.cuda.synchronize()
    ops.check_device()
    ok = True
    hq, hk, hv, ho = (t.float().cpu().numpy() for t in (q, k, v, o))
    for b in range(B):
        for h in range(H):
            ref = O.fmha(hq[b, h], hk[b, h], hv[b, h], 1.0 / math.sqrt(128), causal)
            ok = ok and bool(np.all(np.isfinite(ho[b, h]))) and bool(O.isapprox(ho[b, h], ref, 1e-2))
    out.append([B, H, S, Sk, causal, ramp, ok])
print(json.dumps(out))
"""


def test_pair_kernel_parity():
    env = dict(os.environ, CTB_FMHA_PAIR="1")
    r = subprocess.run([sys.executable, "-c", SCRIPT], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    rows = json.loads(r.stdout.strip().splitlines()[-1])
    assert len(rows) == 11
    for B, H, S, Sk, causal, ramp, ok in rows:
        assert ok, (B, H, S, Sk, causal, ramp)

"""Launch-path overhead: the C ABI launches on the caller's stream and
allocates nothing, so a sequence of launches can be captured once into a
CUDA graph and replayed without per-launch host work (what the reference's
`run(; nruns)` loops pay per call: argument flattening, a scratch CuArray per
TMA launch, src/runtime.jl:206-222). Replays must reproduce the eager results
bit for bit (same kernels, same inputs)."""
import math

import pytest
import torch

from cutile_b200 import ops

pytestmark = pytest.mark.gpu


def test_captured_launches_replay_bit_exact(dev):
    x = ops.fill_normal(torch.empty(512, 4096, device=dev), 1, 0.0, 4.0)
    A = ops.fill_uniform(torch.empty(1024, 512, dtype=torch.float16, device=dev), 2)
    B = ops.fill_uniform(torch.empty(768, 1024, dtype=torch.float16, device=dev), 3)
    q, k, v = (ops.fill_normal(torch.empty(1, 2, 512, 128, dtype=torch.float16, device=dev), s)
               for s in (4, 5, 6))
    w = ops.fill_normal(torch.empty(4096, device=dev), 7, 1.0, 0.1)
    b = torch.zeros(4096, device=dev)
    y, C, o = torch.empty_like(x), torch.empty(768, 512, dtype=torch.float16, device=dev), torch.empty_like(q)
    ln_y, mu, rs = torch.empty_like(x), torch.empty(512, device=dev), torch.empty(512, device=dev)
    groups = ops.layernorm_bwd_groups(4096, 512)
    dx, dw, db = torch.empty_like(x), torch.empty(4096, device=dev), torch.empty(4096, device=dev)
    part = torch.empty(2 * groups * 4096, device=dev)

    def work():
        ops.softmax(x, y)
        ops.matmul(A, B, C)
        ops.fmha(q, k, v, 1 / math.sqrt(128), True, o)
        ops.layernorm_fwd(x, w, b, 1e-5, ln_y, mu, rs)
        ops.layernorm_bwd(x, y, w, mu, rs, dx, dw, db, part, groups)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        work()  # eager run: per-device set-up happens here, outside capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager = [t.clone() for t in (y, C, o, ln_y, dx, dw, db)]
    for t in (y, C, o, ln_y, dx, dw, db):
        t.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        work()
    for _ in range(2):
        g.replay()
        torch.cuda.synchronize()
        for got, ref in zip((y, C, o, ln_y, dx, dw, db), eager):
            assert torch.equal(got, ref)
    ops.check_device()

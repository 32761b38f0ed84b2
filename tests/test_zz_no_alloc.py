"""The allocation-free LayerNorm backward entry point, called through the C ABI.

ctb_layernorm_bwd_f32_noalloc serves callers that cannot allocate device
memory when they run the backward pass (a process whose whole memory budget
is already reserved for its own pool, or Julia code where CUDA.jl's
allocator must not be entered). Its dW/dB workspace is a fixed array inside
the library, shared by every call, so this test makes two calls in a row with
different shapes and checks each against the regular entry point
(ctb_layernorm_bwd_f32, caller-provided workspace) and against the CPU oracle,
at the tolerance the other layernorm tests use (Julia isapprox, rtol 1e-5).
This file is collected last.
"""
import ctypes

import pytest
import torch

from cutile_b200 import _lib, ops
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _case(dev, rows, n, seed):
    x = ops.fill_normal(torch.empty(rows, n, device=dev), seed)
    dy = ops.fill_normal(torch.empty(rows, n, device=dev), seed + 1)
    w = ops.fill_normal(torch.empty(n, device=dev), seed + 2, 1.0, 0.1)
    b = ops.fill_normal(torch.empty(n, device=dev), seed + 3, 0.0, 0.1)
    _, mu, rs = ops.layernorm_fwd(x, w, b, 1e-5)
    return x, dy, w, mu, rs


def _noalloc(x, dy, w, mu, rs, groups=0):
    rows, n = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(n, device=x.device)
    db = torch.empty(n, device=x.device)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _lib.load().ctb_layernorm_bwd_f32_noalloc(
        x.data_ptr(), dy.data_ptr(), w.data_ptr(), mu.data_ptr(), rs.data_ptr(), dx.data_ptr(),
        dw.data_ptr(), db.data_ptr(), n, rows, x.stride(0), dy.stride(0), dx.stride(0), groups, st)
    return rc, dx, dw, db


def test_noalloc_matches_regular_entry_point_twice(dev):
    for rows, n, seed in ((4096, 4096, 70), (1000, 2048, 80)):
        x, dy, w, mu, rs = _case(dev, rows, n, seed)
        rc, dx, dw, db = _noalloc(x, dy, w, mu, rs)
        assert rc == 0, _lib.load().ctb_last_error()
        rdx, rdw, rdb = ops.layernorm_bwd(x, dy, w, mu, rs)
        torch.cuda.synchronize()
        for got, ref in ((dx, rdx), (dw, rdw), (db, rdb)):
            assert O.isapprox(got.cpu().numpy(), ref.cpu().numpy(), 1e-5)
        # and directly against the CPU oracle (float64 accumulation)
        odx, odw, odb = O.layernorm_bwd(*(t.cpu().numpy() for t in (x, dy, w, mu, rs)))
        for got, ref in ((dx, odx), (dw, odw), (db, odb)):
            assert O.isapprox(got.cpu().numpy(), ref, 1e-5)


def test_noalloc_rejects_workspace_beyond_the_built_in_array(dev):
    x, dy, w, mu, rs = _case(dev, 2048, 4096, 90)
    rc, *_ = _noalloc(x, dy, w, mu, rs, groups=1000)  # 2 x 1000 x 4096 floats > 2,097,152
    assert rc == -3
    assert b"built-in scratch" in _lib.load().ctb_last_error()

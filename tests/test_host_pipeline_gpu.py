"""Host-buffer entry points (ctb_*_host): data in host memory, chunks pipelined
through a device workspace on three streams. Same tolerances as the device
calls: vadd bit-exact, softmax / layernorm Julia isapprox rtol 1e-5."""
import numpy as np
import pytest
import torch

from cutile_b200 import ops
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def pinned(a):
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


@pytest.mark.parametrize("count,length", [(4096, 16384), (1000, 2048), (1, 1024), (37, 4000)])
def test_softmax_host(dev, count, length):
    x = pinned(4 * O.normal(count * length, 5).reshape(count, length))
    y = torch.empty_like(x).pin_memory()
    ops.softmax_host(x, y)
    torch.cuda.synchronize()
    assert O.isapprox(y.numpy(), O.softmax(x.numpy()), 1e-5)


def test_softmax_host_pageable_and_stream_order(dev):
    # Pageable host memory still gives correct results (copies just do not overlap);
    # work already on the caller's stream is ordered before the pipeline.
    x = torch.from_numpy(O.normal(300 * 512, 6).reshape(300, 512))
    y = torch.full_like(x, 3.0)
    d = torch.empty(1 << 24, device=dev)
    d.fill_(1.0)  # pending work on the current stream
    ops.softmax_host(x, y)
    torch.cuda.synchronize()
    assert O.isapprox(y.numpy(), O.softmax(x.numpy()), 1e-5)


@pytest.mark.parametrize("rows,n", [(16384, 4096), (333, 1000)])
def test_layernorm_host(dev, rows, n):
    x = pinned(O.normal(rows * n, 7).reshape(rows, n))
    w = pinned(O.normal(n, 8, 1.0, 0.1))
    b = pinned(O.normal(n, 9, 0.0, 0.1))
    y, mu, rs = ops.layernorm_fwd_host(x, w, b, 1e-5)
    torch.cuda.synchronize()
    ry, rmu, rrs = O.layernorm_fwd(x.numpy(), w.numpy(), b.numpy())
    assert O.isapprox(y.numpy(), ry, 1e-5)
    assert O.isapprox(mu.numpy(), rmu, 1e-5) and O.isapprox(rs.numpy(), rrs, 1e-5)


@pytest.mark.parametrize("dt", [np.float32, np.float16, np.float64])
@pytest.mark.parametrize("n", [1 << 26, 999_999, 7])
def test_vadd_host_bit_exact(dev, dt, n):
    a = pinned(O.uniform(n, 1, dtype=dt))
    b = pinned(O.uniform(n, 2, dtype=dt))
    c = ops.vadd_host(a, b)
    torch.cuda.synchronize()
    assert c.numpy().tobytes() == O.vadd(a.numpy(), b.numpy()).tobytes()

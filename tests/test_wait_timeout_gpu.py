"""A bounded device-side wait really runs out: a self-test kernel waits
~1 ms on an mbarrier that nothing arrives on. ctb_check_device must report
CTB_ERR_TIMEOUT once (and clear the error word), the other warp must leave
through the CTA abort flag rather than its own 4 s limit, the TMEM the CTA
held must be released (a tensor-core launch afterwards allocates it again),
and ordinary launches on the same device must still pass parity."""
import numpy as np
import pytest
import torch

from cutile_b200 import _lib, ops
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _check():
    L = _lib.load()
    rc = L.ctb_check_device(torch.cuda.current_stream().cuda_stream)
    return rc, L.ctb_last_error().decode()


def test_bounded_wait_gives_up_and_context_survives(dev):
    assert _check()[0] == 0
    status = torch.full((3,), -1, dtype=torch.int32, device=dev)
    for _ in range(2):  # twice: the error word is cleared between the two
        status.fill_(-1)
        _lib.call("ctb_selftest_wait_timeout", 1_000_000, status.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        rc, msg = _check()
        assert rc == -7, (rc, msg)  # CTB_ERR_TIMEOUT
        assert "gave up" in msg and "32" in msg, msg
        st = status.cpu().tolist()
        assert st[0] == 1 and st[1] == 1, st
        assert 0 < st[2] < 500_000_000, st  # left through the abort flag, not its 4 s limit
        assert _check()[0] == 0  # cleared
    # The same context still runs ordinary kernels correctly, tensor-core ones included.
    x = ops.fill_normal(torch.empty(64, 4096, device=dev), 3, 0.0, 4.0)
    y = ops.softmax(x)
    torch.cuda.synchronize()
    assert O.isapprox(y.cpu().numpy(), O.softmax(x.cpu().numpy()), 1e-5)
    A = ops.fill_uniform(torch.empty(256, 512, dtype=torch.float16, device=dev), 7)
    B = ops.fill_uniform(torch.empty(384, 256, dtype=torch.float16, device=dev), 8)
    C = ops.matmul(A, B)
    ref = O.matmul(A.cpu().numpy().astype(np.float64), B.cpu().numpy().astype(np.float64))
    assert O.rel_fro(C.cpu().numpy(), ref) <= 2e-3
    ops.check_device()


def test_selftest_rejects_bad_limits(dev):
    status = torch.zeros(3, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    for bad in (0, -5, 2_000_000_000):
        with pytest.raises(_lib.B200Error):
            _lib.call("ctb_selftest_wait_timeout", bad, status.data_ptr(), st)

"""Typed torch-facing calls of the kernels (the C ABI's typed entry
points). Every call runs on the current torch CUDA stream and raises
:class:`B200Error` on failure; there is no CPU or eager fallback.

Layout notes: ``softmax``/``layernorm_fwd`` take row-major torch matrices
(rows of contiguous elements = Julia columns). ``matmul``/``bmm`` take the
Julia column-major storage as torch tensors: the Julia M x K matrix A is the
torch tensor ``A_t`` of shape (K, M) (row stride = Julia column stride).
``fmha`` takes row-major [B, H, S, D] tensors (= Julia (D, S, H, B)).
"""
import ctypes

import torch

from . import _lib
from .runtime import current_stream_handle

_DT = {torch.float16: _lib.CTB_F16, torch.bfloat16: _lib.CTB_BF16, torch.float32: _lib.CTB_F32,
       torch.float64: _lib.CTB_F64, torch.int32: _lib.CTB_I32}


def _st():
    return current_stream_handle()


def _need_cuda(*ts):
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise _lib.B200Error(-1, "expected CUDA tensors")


def init(device=0):
    _lib.call("ctb_init", int(device))


def check_device():
    """Synchronises and raises CTB_ERR_TIMEOUT if a bounded device wait gave up."""
    _lib.call("ctb_check_device", _st())


def fill_uniform(t, seed, lo=-1.0, hi=1.0, offset=0):
    _need_cuda(t)
    assert t.is_contiguous()
    _lib.call("ctb_fill_uniform", t.data_ptr(), _DT[t.dtype], t.numel(), seed, offset, lo, hi,
              _st())
    return t


def fill_normal(t, seed, mean=0.0, std=1.0, offset=0):
    _need_cuda(t)
    assert t.is_contiguous()
    _lib.call("ctb_fill_normal", t.data_ptr(), _DT[t.dtype], t.numel(), seed, offset, mean, std,
              _st())
    return t


def vadd(a, b, out=None):
    _need_cuda(a, b)
    if out is None:
        out = torch.empty_like(a)
    n = out.numel()
    _lib.call("ctb_vadd", _DT[a.dtype], a.data_ptr(), b.data_ptr(), out.data_ptr(), n,
              a.stride(0) if a.dim() else 1, b.stride(0) if b.dim() else 1,
              out.stride(0) if out.dim() else 1, _st())
    return out


def rowsum(a, out=None, julia_colmajor=True):
    """``sum(a; dims=2)``. With ``julia_colmajor`` the torch tensor (n, m) is the
    Julia m x n array (stride (1, m)); otherwise a is a row-major (m, n)
    matrix whose rows are summed."""
    _need_cuda(a)
    if julia_colmajor:
        n, m = a.shape
        si, sj = a.stride(1), a.stride(0)
    else:
        m, n = a.shape
        si, sj = a.stride(0), a.stride(1)
    if out is None:
        out = torch.empty(m, dtype=torch.float32, device=a.device)
    _lib.call("ctb_rowsum_f32", a.data_ptr(), out.data_ptr(), m, n, si, sj, out.stride(0), _st())
    return out


def softmax(x, out=None):
    """Row-wise softmax of a (count, len) float32 tensor with unit inner stride."""
    _need_cuda(x)
    if out is None:
        out = torch.empty_like(x)
    count, length = x.shape
    if x.stride(1) != 1 or out.stride(1) != 1:
        raise _lib.B200Error(-4, "softmax: rows must be contiguous")
    _lib.call("ctb_softmax_f32", x.data_ptr(), out.data_ptr(), length, count, x.stride(0),
              out.stride(0), _st())
    return out


def layernorm_fwd(x, w, b, eps=1e-5, out=None, mean=None, rstd=None):
    _need_cuda(x, w, b)
    rows, n = x.shape
    if x.stride(1) != 1:
        raise _lib.B200Error(-4, "layernorm_fwd: rows must be contiguous")
    out = torch.empty_like(x) if out is None else out
    mean = torch.empty(rows, dtype=torch.float32, device=x.device) if mean is None else mean
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device) if rstd is None else rstd
    _lib.call("ctb_layernorm_fwd_f32", x.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(),
              mean.data_ptr(), rstd.data_ptr(), n, rows, x.stride(0), out.stride(0),
              ctypes.c_float(eps), _st())
    return out, mean, rstd


def layernorm_bwd_groups(n, rows):
    g = _lib.load().ctb_layernorm_bwd_groups(n, rows)
    if g < 1:
        _lib.check(-8)
    return g


def layernorm_bwd(x, dy, w, mean, rstd, dx=None, dw=None, db=None, partial=None, groups=None):
    """LayerNorm backward on row-major (rows, n) float32 tensors -> (dx, dw, db).
    `partial` (2 * groups * n floats) is the workspace; allocated here when None."""
    _need_cuda(x, dy, w, mean, rstd)
    rows, n = x.shape
    groups = layernorm_bwd_groups(n, rows) if groups is None else groups
    dx = torch.empty_like(x) if dx is None else dx
    dw = torch.empty(n, dtype=torch.float32, device=x.device) if dw is None else dw
    db = torch.empty(n, dtype=torch.float32, device=x.device) if db is None else db
    if partial is None:
        partial = torch.empty(2 * groups * n, dtype=torch.float32, device=x.device)
    _lib.call("ctb_layernorm_bwd_f32", x.data_ptr(), dy.data_ptr(), w.data_ptr(), mean.data_ptr(),
              rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(), n, rows, x.stride(0),
              dy.stride(0), dx.stride(0), partial.data_ptr(), groups, _st())
    return dx, dw, db


def layernorm_bwd_noalloc(x, dy, w, mean, rstd, dx, dw, db, groups=0):
    """LayerNorm backward through the allocation-free entry point: the dW/dB
    workspace is the library's built-in array, so nothing is allocated on
    the device here (every output must be passed in)."""
    _need_cuda(x, dy, w, mean, rstd, dx, dw, db)
    rows, n = x.shape
    _lib.call("ctb_layernorm_bwd_f32_noalloc", x.data_ptr(), dy.data_ptr(), w.data_ptr(),
              mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(), n,
              rows, x.stride(0), dy.stride(0), dx.stride(0), int(groups), _st())
    return dx, dw, db


def transpose(x, out=None):
    """Julia y = x' on column-major storage: x_t (N, M) holds the Julia M x N
    matrix; returns y_t (M, N) holding the Julia N x M transpose."""
    _need_cuda(x)
    N, M = x.shape
    if x.stride(1) != 1:
        raise _lib.B200Error(-4, "transpose: columns must be contiguous")
    out = torch.empty(M, N, dtype=x.dtype, device=x.device) if out is None else out
    _lib.call("ctb_transpose", _DT[x.dtype], x.data_ptr(), out.data_ptr(), M, N, x.stride(0),
              out.stride(0), _st())
    return out


def matmul(A_t, B_t, C_t=None):
    """Julia C = A*B on column-major storage: A_t (K, M), B_t (N, K), C_t (N, M)."""
    _need_cuda(A_t, B_t)
    K, M = A_t.shape
    N = B_t.shape[0]
    if C_t is None:
        C_t = torch.empty(N, M, dtype=A_t.dtype, device=A_t.device)
    if A_t.dtype != torch.float16:
        raise _lib.B200Error(-2, "matmul: typed entry is Float16")
    _lib.call("ctb_gemm_f16", A_t.data_ptr(), B_t.data_ptr(), C_t.data_ptr(), M, N, K,
              A_t.stride(0), B_t.stride(0), C_t.stride(0), _st())
    return C_t


def bmm(A_t, B_t, C_t=None):
    """Batched Julia C_b = A_b*B_b: A_t (batch, K, M), B_t (batch, N, K), C_t (batch, N, M)."""
    _need_cuda(A_t, B_t)
    batch, K, M = A_t.shape
    N = B_t.shape[1]
    if C_t is None:
        C_t = torch.empty(batch, N, M, dtype=A_t.dtype, device=A_t.device)
    _lib.call("ctb_bgemm_f16", A_t.data_ptr(), B_t.data_ptr(), C_t.data_ptr(), M, N, K, batch,
              A_t.stride(1), B_t.stride(1), C_t.stride(1), A_t.stride(0), B_t.stride(0),
              C_t.stride(0), _st())
    return C_t


def fmha(q, k, v, scale, causal=False, out=None):
    """Attention forward on contiguous [B, H, S, D] float16 tensors."""
    _need_cuda(q, k, v)
    for t in (q, k, v):
        if not t.is_contiguous():
            raise _lib.B200Error(-4, "fmha: tensors must be contiguous [B, H, S, D]")
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    out = torch.empty_like(q) if out is None else out
    _lib.call("ctb_fmha_fwd_f16", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H,
              Sq, Sk, D, ctypes.c_float(scale), 1 if causal else 0, _st())
    return out


MOE_BLOCK = 256  # rows per routing block: 256 runs the CTA-pair kernel, 128 the single-SM one


def moe_align(topk_ids, num_experts, block=MOE_BLOCK):
    """Routing in the fused-MoE layout: returns (sorted_token_ids int32 [EM],
    expert_ids int32 [EM/block], num_tokens_post_padded int32 [1]) on the
    device of `topk_ids` ((M, topk) int tensor). Slots of each expert are
    listed in token order and padded to a multiple of `block` with M*topk.

    On a CUDA tensor this is one device kernel (ctb_moe_align_i32) and never
    waits for the GPU: EM is the worst case for the routing
    (ctb_moe_align_capacity), entries past num_tokens_post_padded hold the
    padding id and blocks past it expert -1, which the MoE GEMM skips. On a
    host tensor the exact-size layout is computed on the host."""
    if topk_ids.is_cuda:
        n = topk_ids.numel()
        ids = topk_ids.reshape(-1)
        if ids.dtype != torch.int32:
            ids = ids.to(torch.int32)
        ids = ids.contiguous()
        cap = int(_lib.load().ctb_moe_align_capacity(n, num_experts, block))
        if cap < 0:
            _lib.check(-3)
        sorted_ids = torch.empty(cap, dtype=torch.int32, device=ids.device)
        expert_ids = torch.empty(cap // block, dtype=torch.int32, device=ids.device)
        ntp = torch.empty(1, dtype=torch.int32, device=ids.device)
        _lib.call("ctb_moe_align_i32", ids.data_ptr(), n, num_experts, block,
                  sorted_ids.data_ptr(), expert_ids.data_ptr(), ntp.data_ptr(), cap, _st())
        return sorted_ids, expert_ids, ntp
    flat = topk_ids.reshape(-1).to(torch.int64)
    n = flat.numel()
    counts = torch.bincount(flat, minlength=num_experts)
    padded = (counts + block - 1) // block * block
    em = int(padded.sum().item())
    order = torch.argsort(flat * n + torch.arange(n, device=flat.device))  # stable by expert
    sorted_ids = torch.full((max(em, block),), n, dtype=torch.int32, device=flat.device)
    starts = torch.cumsum(padded, 0) - padded
    cstarts = torch.cumsum(counts, 0) - counts
    pos = starts[flat[order]] + (torch.arange(n, device=flat.device) - cstarts[flat[order]])
    sorted_ids[pos] = order.to(torch.int32)
    expert_ids = torch.repeat_interleave(torch.arange(num_experts, device=flat.device),
                                         padded // block).to(torch.int32)
    if expert_ids.numel() * block < sorted_ids.numel():
        expert_ids = torch.cat([expert_ids, torch.full((1,), -1, dtype=torch.int32,
                                                       device=flat.device)])
    ntp = torch.tensor([em], dtype=torch.int32, device=flat.device)
    return sorted_ids, expert_ids, ntp


_moe_ws = {}


def moe_workspace(EM, K, device):
    """The routed-rows workspace for ctb_moe_gemm_f16, cached per device and
    grown on demand (EM x K Float16)."""
    need = int(_lib.load().ctb_moe_workspace_bytes(EM, K))
    key = torch.device(device)
    ws = _moe_ws.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device=key)
        _moe_ws[key] = ws
    return ws


def moe_gemm(A, B, sorted_ids, expert_ids, ntp, topk, weights=None, out=None, workspace=None):
    """Fused-MoE GEMM: A (M, K) f16, B (E, N, K) f16 -> C (M*topk, N) f16 with
    C[s] = A[s // topk] @ B[e].T (* weights[s]) for the slots s routed to e.
    Rows of C that no block in use lists are left as they were."""
    _need_cuda(A, B, sorted_ids, expert_ids, ntp)
    M, K = A.shape
    E, N, _ = B.shape
    EM = sorted_ids.numel()
    out = torch.zeros(M * topk, N, dtype=A.dtype, device=A.device) if out is None else out
    w = weights.reshape(-1).contiguous() if weights is not None else None
    ws = moe_workspace(EM, K, A.device) if workspace is None else workspace
    block_m = EM // max(expert_ids.numel(), 1)
    _lib.call("ctb_moe_gemm_f16", A.data_ptr(), B.data_ptr(), out.data_ptr(),
              sorted_ids.data_ptr(), expert_ids.data_ptr(), ntp.data_ptr(),
              w.data_ptr() if w is not None else None, 1 if w is not None else 0,
              M, N, K, E, EM, topk, block_m, A.stride(0), B.stride(1), out.stride(0),
              ws.data_ptr(), ws.numel() * ws.element_size(), _st())
    return out


# ---- host-buffer calls (three-stream chunk pipeline inside the library) -------
_host_ws = {}


def _host_workspace(nbytes, device):
    """One workspace per device for the host-buffer calls; they run on the
    current stream, which orders successive calls that share it."""
    key = torch.device(device)
    ws = _host_ws.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=key)
        _host_ws[key] = ws
    return ws


def _need_host(*ts):
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.device.type == "cpu" and t.is_contiguous()):
            raise _lib.B200Error(-1, "expected contiguous host (CPU) tensors")


def softmax_host(x, y=None, device=0):
    """Row softmax of a host (count, len) float32 tensor through the GPU;
    x and y should be pinned (``pin_memory()``) for the copies to overlap."""
    _need_host(x)
    count, length = x.shape
    y = torch.empty_like(x) if y is None else y
    L = _lib.load()
    ws = _host_workspace(L.ctb_host_workspace_bytes(4 * length, 4 * length, count), device)
    with torch.cuda.device(device):
        _lib.call("ctb_softmax_f32_host", x.data_ptr(), y.data_ptr(), length, count,
                  ws.data_ptr(), ws.numel(), _st())
    return y


def layernorm_fwd_host(x, w, b, eps=1e-5, y=None, mean=None, rstd=None, device=0):
    """LayerNorm over rows of a host (rows, n) float32 tensor through the GPU."""
    _need_host(x, w, b)
    rows, n = x.shape
    y = torch.empty_like(x) if y is None else y
    mean = torch.empty(rows, dtype=torch.float32) if mean is None else mean
    rstd = torch.empty(rows, dtype=torch.float32) if rstd is None else rstd
    L = _lib.load()
    wb = 2 * ((4 * n + 255) // 256 * 256)
    ws = _host_workspace(L.ctb_host_workspace_bytes(4 * n, 4 * n + 8, rows) + wb, device)
    with torch.cuda.device(device):
        _lib.call("ctb_layernorm_fwd_f32_host", x.data_ptr(), w.data_ptr(), b.data_ptr(),
                  y.data_ptr(), mean.data_ptr(), rstd.data_ptr(), n, rows, eps, ws.data_ptr(),
                  ws.numel(), _st())
    return y, mean, rstd


def vadd_host(a, b, c=None, device=0):
    """c = a + b for host vectors through the GPU."""
    _need_host(a, b)
    c = torch.empty_like(a) if c is None else c
    L = _lib.load()
    es = a.element_size()
    ws = _host_workspace(L.ctb_host_workspace_bytes(2 * es, es, a.numel()) + 16 * 256, device)
    with torch.cuda.device(device):
        _lib.call("ctb_vadd_host", _DT[a.dtype], a.data_ptr(), b.data_ptr(), c.data_ptr(),
                  a.numel(), ws.data_ptr(), ws.numel(), _st())
    return c

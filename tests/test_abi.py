"""The C-ABI library loads without a GPU and exports every symbol the public
header declares; host-side argument validation answers before any CUDA call."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
import cutile_b200
from cutile_b200 import _lib

HEADER = os.path.join(ROOT, "include", "cutile_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(ctb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ["ctb_version", "ctb_find_kernel", "ctb_launch", "ctb_vadd", "ctb_rowsum_f32",
              "ctb_softmax_f32", "ctb_layernorm_fwd_f32", "ctb_gemm_f16", "ctb_bgemm_f16",
              "ctb_fmha_fwd_f16"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    for s in declared_symbols():
        assert hasattr(L, s), f"{s} declared in include/cutile_b200.h but not exported"
    # every declared function has a Python signature
    for s in declared_symbols():
        assert s in _lib.SIGNATURES or s == "ctb_last_error", s


def test_version_matches_header():
    m = re.search(r"#define CTB_ABI_VERSION (\d+)", open(HEADER).read())
    assert _lib.load().ctb_version() == int(m.group(1))


@pytest.mark.parametrize("name,n", [("vadd", 3), ("rowsum", 2), ("softmax", 2),
                                    ("layernorm_fwd", 6), ("layer_norm_fwd", 6), ("layernorm_bwd", 9), ("matmul", 3),
                                    ("matmul16", 3), ("batchmatmul", 3), ("fmha", 4), ("transpose", 2), ("moe", 8)])
def test_registry_knows_the_seven_kernels(name, n):
    L = _lib.load()
    dt = (ctypes.c_int32 * n)(*([_lib.CTB_F32] * n))
    h = ctypes.c_int32(-1)
    assert L.ctb_find_kernel(name.encode(), dt, n, None, 0, ctypes.byref(h)) == 0
    info = _lib.CtbKernelInfo()
    assert L.ctb_kernel_info_get(h.value, ctypes.byref(info)) == 0
    assert info.narrays == n


def test_unknown_kernel_is_an_error_not_a_fallback():
    L = _lib.load()
    h = ctypes.c_int32(-1)
    rc = L.ctb_find_kernel(b"fft", None, 0, None, 0, ctypes.byref(h))
    assert rc == -5
    assert b"no prebuilt sm_100a kernel" in L.ctb_last_error()


def test_wrong_dtype_count():
    L = _lib.load()
    dt = (ctypes.c_int32 * 2)(_lib.CTB_F32, _lib.CTB_F32)
    h = ctypes.c_int32(-1)
    assert L.ctb_find_kernel(b"vadd", dt, 2, None, 0, ctypes.byref(h)) == -1


def test_launch_validates_argument_counts_before_touching_the_device():
    L = _lib.load()
    dt = (ctypes.c_int32 * 3)(*([_lib.CTB_F32] * 3))
    h = ctypes.c_int32(-1)
    assert L.ctb_find_kernel(b"vadd", dt, 3, None, 0, ctypes.byref(h)) == 0
    arrs = (_lib.CtbArray * 2)()
    rc = L.ctb_launch(h.value, arrs, 2, None, 0, None, None)
    assert rc == -1
    assert b"expected 3" in L.ctb_last_error()
    assert L.ctb_launch(999, arrs, 2, None, 0, None, None) == -1


def test_typed_entry_points_reject_bad_sizes_without_gpu():
    L = _lib.load()
    assert L.ctb_vadd(_lib.CTB_F32, None, None, None, -1, 1, 1, 1, None) == -3
    assert L.ctb_vadd(_lib.CTB_F32, None, None, None, 10, 1, 1, 1, None) == -1
    assert L.ctb_softmax_f32(None, None, -1, 4, 4, 4, None) == -3
    assert L.ctb_layernorm_fwd_f32(None, None, None, None, None, None, 0, 4, 4, 4,
                                   ctypes.c_float(1e-5), None) == -3
    assert L.ctb_fmha_fwd_f16(None, None, None, None, 1, 1, 1, 0, 64, ctypes.c_float(1.0), 0,
                              None) == -3


def test_python_error_carries_status():
    with pytest.raises(cutile_b200.B200Error) as e:
        cutile_b200.triton_kernel("fft", [cutile_b200.TileArray(__import__("torch").float32, 1)])
    assert e.value.status == "CTB_ERR_UNKNOWN_KERNEL"


def test_new_entry_points_validate_without_gpu():
    L = _lib.load()
    # MoE: routing block must be 128 or 256, EM a multiple of it; checked before any device call.
    args = [None] * 7 + [0, 16, 64, 64, 2, 256, 1]
    assert L.ctb_moe_gemm_f16(*args, 64, 64, 64, 64, None, 0, None) == -3
    assert L.ctb_moe_gemm_f16(*args[:12], 384, 1, 256, 64, 64, 64, None, 0, None) == -3
    assert b"multiple of block_m" in L.ctb_last_error()
    assert L.ctb_moe_workspace_bytes(256, 64) == 256 * 64 * 2
    # Host-buffer calls: NULL pointers and bad sizes are reported, empty work is a no-op.
    assert L.ctb_softmax_f32_host(None, None, 16, 4, None, 0, None) == -1
    assert L.ctb_softmax_f32_host(None, None, -1, 4, None, 0, None) == -3
    assert L.ctb_softmax_f32_host(None, None, 16, 0, None, 0, None) == 0
    assert L.ctb_vadd_host(99, None, None, None, 8, None, 0, None) == -2
    assert L.ctb_layernorm_fwd_f32_host(None, None, None, None, None, None, 0, 4,
                                        ctypes.c_float(1e-5), None, 0, None) == -3
    ws = L.ctb_host_workspace_bytes(4 * 16384, 4 * 16384, 4096)
    assert ws >= 3 * (4096 // 8) * 8 * 16384  # three slots of 1/8 of the rows
    assert L.ctb_host_workspace_bytes(4, 4, 0) == 0

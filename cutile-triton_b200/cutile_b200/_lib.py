"""ctypes binding of libcutile_b200.so (declared in include/cutile_b200.h).

This is the Python twin of the Julia ``ccall`` layer: plain pointers, sizes,
strides and a stream handle cross the boundary, nothing else. The library is
loaded from ``$CUTILE_B200_LIB`` or from this package directory; a missing
library is an error (there is no fallback path).
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_LIB = os.path.join(HERE, "libcutile_b200.so")

CTB_MAX_DIMS = 5
CTB_F16, CTB_BF16, CTB_F32, CTB_F64, CTB_I32 = 1, 2, 3, 4, 5

STATUS = {
    0: "CTB_OK",
    -1: "CTB_ERR_ARG",
    -2: "CTB_ERR_DTYPE",
    -3: "CTB_ERR_SHAPE",
    -4: "CTB_ERR_LAYOUT",
    -5: "CTB_ERR_UNKNOWN_KERNEL",
    -6: "CTB_ERR_CUDA",
    -7: "CTB_ERR_TIMEOUT",
    -8: "CTB_ERR_NO_DEVICE",
}


class CtbArray(ctypes.Structure):
    """``ctb_array``: one flattened TileArray (Julia dim order, element units)."""

    _fields_ = [
        ("ptr", ctypes.c_void_p),
        ("ndim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("sizes", ctypes.c_int32 * CTB_MAX_DIMS),
        ("strides", ctypes.c_int32 * CTB_MAX_DIMS),
    ]


class CtbKernelInfo(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 32),
        ("narrays", ctypes.c_int32),
        ("nscalars", ctypes.c_int32),
        ("num_warps", ctypes.c_int32),
        ("shared_bytes", ctypes.c_int32),
    ]


class B200Error(RuntimeError):
    """A non-zero ctb_status, carrying the library's message (the analogue of
    the reference's ``error("...")`` on compile/ABI failures)."""

    def __init__(self, code, msg):
        self.code = code
        self.status = STATUS.get(code, str(code))
        super().__init__(f"b200: {self.status}: {msg}")


_P, _I32, _I64, _U64, _D, _F = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                ctypes.c_uint64, ctypes.c_double, ctypes.c_float)

# name -> argtypes; every function returns int except ctb_last_error.
SIGNATURES = {
    "ctb_version": [],
    "ctb_init": [ctypes.c_int],
    "ctb_check_device": [_P],
    "ctb_find_kernel": [ctypes.c_char_p, ctypes.POINTER(_I32), _I32, ctypes.POINTER(_I64), _I32,
                        ctypes.POINTER(_I32)],
    "ctb_kernel_info_get": [_I32, ctypes.POINTER(CtbKernelInfo)],
    "ctb_launch": [_I32, ctypes.POINTER(CtbArray), _I32, ctypes.POINTER(_D), _I32,
                   ctypes.POINTER(_I32), _P],
    "ctb_vadd": [_I32, _P, _P, _P, _I64, _I64, _I64, _I64, _P],
    "ctb_rowsum_f32": [_P, _P, _I32, _I32, _I64, _I64, _I64, _P],
    "ctb_softmax_f32": [_P, _P, _I32, _I32, _I64, _I64, _P],
    "ctb_layernorm_fwd_f32": [_P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _F, _P],
    "ctb_layernorm_bwd_f32": [_P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _I64, _P,
                              _I32, _P],
    "ctb_layernorm_bwd_groups": [_I32, _I32],
    "ctb_layernorm_bwd_f32_noalloc": [_P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _I64,
                                      _I64, _I32, _P],
    "ctb_transpose": [_I32, _P, _P, _I32, _I32, _I64, _I64, _P],
    "ctb_gemm_f16": [_P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _P],
    "ctb_bgemm_f16": [_P, _P, _P, _I32, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _I64, _I64,
                      _P],
    "ctb_fmha_fwd_f16": [_P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P],
    "ctb_moe_workspace_bytes": [_I32, _I32],
    "ctb_moe_align_capacity": [_I32, _I32, _I32],
    "ctb_moe_align_i32": [_P, _I32, _I32, _I32, _P, _P, _P, _I32, _P],
    "ctb_host_workspace_bytes": [_I64, _I64, _I64],
    "ctb_softmax_f32_host": [_P, _P, _I32, _I32, _P, _I64, _P],
    "ctb_layernorm_fwd_f32_host": [_P, _P, _P, _P, _P, _P, _I32, _I32, _F, _P, _I64, _P],
    "ctb_vadd_host": [_I32, _P, _P, _P, _I64, _P, _I64, _P],
    "ctb_moe_gemm_f16": [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _I32,
                         _I32, _I64, _I64, _I64, _P, _I64, _P],
    "ctb_fill_uniform": [_P, _I32, _I64, _U64, _U64, _D, _D, _P],
    "ctb_fill_normal": [_P, _I32, _I64, _U64, _U64, _D, _D, _P],
    "ctb_selftest_wait_timeout": [_I64, _P, _P],
}

_lib = None


def lib_path():
    return os.environ.get("CUTILE_B200_LIB", DEFAULT_LIB)


def load():
    """Loads the library once and declares every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise B200Error(-8, f"libcutile_b200.so not found at {path}; build it with "
                            "`python cutile-triton_b200/build.py`")
    L = ctypes.CDLL(path)
    for name, args in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    L.ctb_moe_workspace_bytes.restype = ctypes.c_int64
    L.ctb_host_workspace_bytes.restype = ctypes.c_int64
    L.ctb_last_error.argtypes = []
    L.ctb_last_error.restype = ctypes.c_char_p
    _lib = L
    return L


def check(rc):
    """Raises B200Error for a non-zero status."""
    if rc != 0:
        msg = load().ctb_last_error().decode(errors="replace")
        raise B200Error(rc, msg)
    return rc


def call(name, *args):
    return check(getattr(load(), name)(*args))

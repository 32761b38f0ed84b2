"""B200 twin of TileTriton's ``TritonRun`` module (reference: src/runtime.jl).

Same entry points, names and argument meaning, with the Triton compile
replaced by a lookup of the prebuilt sm_100a kernel in libcutile_b200.so:

* ``triton_kernel(f, argtypes; name, num_warps, num_stages, use_tma)``
  (runtime.jl:128-137) -> ``B200Kernel``; unknown kernels raise, there is no
  Triton fallback.
* ``triton_kernel_candidates`` (runtime.jl:109-126) -> a single candidate:
  one hand-tuned kernel per op, nothing to race.
* ``flatten_args(spec, args)`` (runtime.jl:163-198) -> ctb_array per
  TileArray (pointer, Julia-order sizes and strides) and doubles for
  scalars; the same checks and error messages (eltype / ndims mismatch).
* ``launch(k, grid, *args)`` (``launch!``, runtime.jl:206-222) -> one
  ``ctb_launch`` on the current torch stream.
* ``set_target(backend, arch, warp_size)`` (runtime.jl:14-31) accepts only
  the sm_100 CUDA target this backend is built for.

Arrays: a :class:`JlArray` is a device tensor seen with Julia (column-major)
sizes and strides. ``jl(t)`` views a torch tensor that way (dims reversed),
so a row-major torch (R, C) tensor is the Julia C x R array with strides
(1, C), as TileTriton would receive a CuArray.
"""
import ctypes
from dataclasses import dataclass

import torch

from . import _lib

_DTYPES = {
    torch.float16: _lib.CTB_F16,
    torch.bfloat16: _lib.CTB_BF16,
    torch.float32: _lib.CTB_F32,
    torch.float64: _lib.CTB_F64,
    torch.int32: _lib.CTB_I32,
}


@dataclass(frozen=True)
class TargetInfo:
    backend: str
    arch: int
    warp_size: int
    binkey: str


ACTIVE_TARGET = [TargetInfo("cuda", 100, 32, "sm_100a")]


def set_target(backend, arch, warp_size):
    """Only the CUDA sm_100 target exists: the kernels are prebuilt for sm_100a."""
    if backend != "cuda" or int(arch) != 100 or int(warp_size) != 32:
        raise ValueError("b200 backend: only set_target('cuda', 100, 32) is supported")
    ACTIVE_TARGET[0] = TargetInfo("cuda", 100, 32, "sm_100a")


class JlArray:
    """A device tensor with Julia-order sizes and strides (element units)."""

    __slots__ = ("tensor", "sizes", "strides")

    def __init__(self, tensor, sizes=None, strides=None):
        self.tensor = tensor
        self.sizes = tuple(reversed(tensor.shape)) if sizes is None else tuple(sizes)
        self.strides = tuple(reversed(tensor.stride())) if strides is None else tuple(strides)

    @property
    def dtype(self):
        return self.tensor.dtype

    @property
    def ndims(self):
        return len(self.sizes)

    def pointer(self):
        return self.tensor.data_ptr()


def jl(t):
    """Julia view of a torch tensor: dims reversed (row-major -> column-major)."""
    return t if isinstance(t, JlArray) else JlArray(t)


@dataclass(frozen=True)
class TileArray:
    """Argument type of a TileArray parameter (``ct.TileArray{T, N, Spec}``)."""

    elty: torch.dtype
    ndims: int


@dataclass(frozen=True)
class Constant:
    """A ghost ``ct.Constant{Int, V}`` parameter (tile sizes): identifies the
    specialisation only and contributes no bytes to the launch."""

    value: int


@dataclass(frozen=True)
class ArgSpec:
    """Per-parameter ABI record (reference ArgSpec, src/emitter.jl:163-167)."""

    kind: str  # "tilearray" | "scalar"
    elty: object
    ndims: int


@dataclass
class B200Kernel:
    """A prebuilt kernel handle (the TritonKernel analogue, runtime.jl:85-95)."""

    handle: int
    name: str
    num_warps: int
    warp_size: int
    shared: int
    global_scratch_size: int
    argspec: list
    nscalars: int


def _name_of(f):
    if isinstance(f, str):
        return f
    return getattr(f, "__name__", str(f))


def _argspec(argtypes):
    spec, consts = [], []
    for t in argtypes:
        if isinstance(t, TileArray):
            spec.append(ArgSpec("tilearray", t.elty, t.ndims))
        elif isinstance(t, Constant):
            consts.append(int(t.value))
        elif t in (float, int, bool) or isinstance(t, type):
            spec.append(ArgSpec("scalar", t, 0))
        else:
            raise TypeError(f"unsupported kernel argument type {t!r}")
    return spec, consts


def triton_kernel(f, argtypes, *, name=None, num_warps=None, num_stages=None, use_tma=True):
    """Returns the prebuilt sm_100a kernel for cuTile function ``f`` specialised
    on ``argtypes``. ``num_warps``/``num_stages``/``use_tma`` are accepted for
    signature compatibility; the kernel's schedule is fixed per op."""
    L = _lib.load()
    kname = _name_of(f)  # the cuTile function identifies the kernel; `name` labels it
    spec, consts = _argspec(argtypes)
    arrays = [s for s in spec if s.kind == "tilearray"]
    dt = (ctypes.c_int32 * max(1, len(arrays)))(*[_DTYPES[s.elty] for s in arrays])
    cs = (ctypes.c_int64 * max(1, len(consts)))(*consts)
    h = ctypes.c_int32(-1)
    _lib.check(L.ctb_find_kernel(kname.encode(), dt, len(arrays), cs, len(consts),
                                 ctypes.byref(h)))
    info = _lib.CtbKernelInfo()
    _lib.check(L.ctb_kernel_info_get(h.value, ctypes.byref(info)))
    nscal = sum(1 for s in spec if s.kind == "scalar")
    if nscal != info.nscalars:
        raise _lib.B200Error(-1, f"{kname}: expected {info.nscalars} scalar parameters, got {nscal}")
    return B200Kernel(h.value, info.name.decode(), info.num_warps, 32, info.shared_bytes, 0,
                      spec, info.nscalars)


def triton_kernel_candidates(f, argtypes, *, name=None, use_tma=True):
    """One candidate per op: the hand-written kernel has no variants to race."""
    return [triton_kernel(f, argtypes, name=name, use_tma=use_tma)]


def flatten_args(spec, args):
    """TileArray -> ctb_array (ptr, Julia sizes, strides); scalars -> doubles.
    Mirrors runtime.jl:163-198, including its argument checks."""
    if len(spec) != len(args):
        raise _lib.B200Error(-1, f"expected {len(spec)} kernel arguments")
    arrays, scalars = [], []
    for s, a in zip(spec, args):
        if s.kind == "tilearray":
            if isinstance(a, torch.Tensor):
                a = jl(a)
            if not isinstance(a, JlArray):
                raise _lib.B200Error(-1, "expected a GPU array for tilearray argument")
            if a.dtype != s.elty:
                raise _lib.B200Error(-2, f"eltype mismatch: {a.dtype} vs {s.elty}")
            if a.ndims != s.ndims:
                raise _lib.B200Error(-3, "ndims mismatch")
            if not a.tensor.is_cuda:
                raise _lib.B200Error(-1, "expected a GPU array for tilearray argument")
            c = _lib.CtbArray()
            c.ptr = a.pointer()
            c.ndim = a.ndims
            c.dtype = _DTYPES[a.dtype]
            for d in range(a.ndims):
                c.sizes[d] = int(a.sizes[d])
                c.strides[d] = int(a.strides[d])
            arrays.append(c)
        else:
            scalars.append(float(a))
    return arrays, scalars


def current_stream_handle(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def launch(k, grid, *args, stream=None):
    """``launch!(k, grid, args...)``: flatten and make one ctb_launch on the
    current torch stream. ``grid`` (Int or tuple) is advisory."""
    arrays, scalars = flatten_args(k.argspec, list(args))
    g = (int(grid), 1, 1) if isinstance(grid, int) else tuple(grid) + (1,) * (3 - len(grid))
    arr = (_lib.CtbArray * max(1, len(arrays)))(*arrays)
    sc = (ctypes.c_double * max(1, len(scalars)))(*scalars)
    gr = (ctypes.c_int32 * 3)(*g)
    st = stream if stream is not None else current_stream_handle()
    _lib.check(_lib.load().ctb_launch(k.handle, arr, len(arrays), sc, len(scalars), gr, st))


def code_triton(*_args, **_kwargs):
    """Reflection of the Triton pipeline has no counterpart: there is no TTIR
    or compiled stage on this path."""
    raise NotImplementedError("b200 backend: kernels are prebuilt; there is no TTIR to show")

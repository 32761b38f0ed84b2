"""B200 twin of TileTriton's ``TritonShim`` (reference: src/shim.jl).

``install_shim(ct)`` overrides ``ct.cufunction`` so that every cuTile launch
of one of the registered kernels goes to the prebuilt sm_100a library, exactly as
the reference's ``install_shim!`` (shim.jl:126-131) routes them to Triton.
``get_kernel`` keeps the reference cache key ``(f, tt, world)`` (shim.jl:20-36)
and raises for a kernel the library does not have. The call operator takes
cuTile's ``blocks``/``threads`` keywords and launches once: there is a single
candidate, so the first-launch race of shim.jl:97-111 has nothing to do.
"""
from . import runtime

KERNEL_CACHE = {}
_WORLD = [0]


def bump_world():
    """Method redefinition analogue: invalidates cached kernels."""
    _WORLD[0] += 1


class ShimKernel:
    def __init__(self, f, tt, kernel):
        self.f = f
        self.tt = tt
        self.candidates = [kernel]
        self.chosen = 1

    def __call__(self, *args, blocks=1, threads=1, stream=None, **_kw):
        runtime.launch(self.candidates[self.chosen - 1], blocks, *args, stream=stream)


def get_kernel(f, tt):
    key = (f, tuple(tt), _WORLD[0])
    k = KERNEL_CACHE.get(key)
    if k is None:
        k = ShimKernel(f, tuple(tt), runtime.triton_kernel(f, list(tt)))
        KERNEL_CACHE[key] = k
    return k


def install_shim(ct):
    """Route ``ct.cufunction`` (and so ``ct.launch``) to this backend."""

    def cufunction(f, tt=(), **_kwargs):
        return get_kernel(f, tt)

    ct.cufunction = cufunction
    return None

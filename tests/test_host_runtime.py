"""Host-side logic of the TritonRun / TritonShim twins, on CPU: argument
specs, flattening checks and the shim cache (reference: src/runtime.jl:109-198,
src/shim.jl:16-36, 126-131)."""
import pytest
import torch

import cutile_b200 as cb
from cutile_b200 import Constant, TileArray, runtime, shim


def vadd(a, b, c, tile):  # stands for the cuTile kernel function
    pass


def softmax(output, input, TILE_SIZE):
    pass


def test_triton_kernel_specialisation():
    k = cb.triton_kernel(vadd, [TileArray(torch.float32, 1)] * 3 + [Constant(1024)], name="vadd",
                         num_warps=4)
    assert k.name == "vadd"
    assert [s.kind for s in k.argspec] == ["tilearray"] * 3
    assert k.nscalars == 0
    assert k.global_scratch_size == 0  # no per-launch scratch allocation (runtime.jl:211-215)


def test_candidates_is_one_kernel():
    ks = cb.triton_kernel_candidates(softmax, [TileArray(torch.float32, 2)] * 2 + [Constant(1024)])
    assert len(ks) == 1


def test_scalar_count_checked():
    with pytest.raises(cb.B200Error):
        cb.triton_kernel("layernorm_fwd", [TileArray(torch.float32, 2)] + [TileArray(torch.float32, 1)] * 2 +
                         [TileArray(torch.float32, 2)] + [TileArray(torch.float32, 1)] * 2)


def test_jl_view_reverses_dims():
    t = torch.empty(4096, 16384)
    a = cb.jl(t)
    assert a.sizes == (16384, 4096) and a.strides == (1, 16384)


def test_flatten_args_checks_like_the_reference():
    k = cb.triton_kernel(vadd, [TileArray(torch.float32, 1)] * 3 + [Constant(1024)])
    cpu = torch.zeros(8)
    with pytest.raises(cb.B200Error, match="expected 3 kernel arguments"):
        runtime.flatten_args(k.argspec, [cpu, cpu])
    with pytest.raises(cb.B200Error, match="eltype mismatch"):
        runtime.flatten_args(k.argspec, [cpu.double(), cpu, cpu])
    with pytest.raises(cb.B200Error, match="ndims mismatch"):
        runtime.flatten_args(k.argspec, [torch.zeros(2, 2), cpu, cpu])
    with pytest.raises(cb.B200Error, match="GPU array"):
        runtime.flatten_args(k.argspec, [cpu, cpu, cpu])


def test_set_target_only_sm100():
    cb.set_target("cuda", 100, 32)
    with pytest.raises(ValueError):
        cb.set_target("hip", "gfx942", 64)


def test_code_triton_has_no_stages():
    with pytest.raises(NotImplementedError):
        cb.code_triton(vadd, [])


def test_install_shim_routes_cufunction_and_caches():
    class FakeCuTile:  # the cuTile module surface install_shim! overwrites
        def cufunction(self, f, tt=()):
            raise AssertionError("original cufunction must be replaced")

    ct = FakeCuTile()
    cb.install_shim(ct)
    tt = (TileArray(torch.float32, 1),) * 3 + (Constant(1024),)
    k1 = ct.cufunction(vadd, tt)
    k2 = ct.cufunction(vadd, tt)
    assert k1 is k2 and isinstance(k1, shim.ShimKernel)
    shim.bump_world()
    assert ct.cufunction(vadd, tt) is not k1
    with pytest.raises(cb.B200Error):
        ct.cufunction(lambda x: x, (TileArray(torch.float32, 1),))

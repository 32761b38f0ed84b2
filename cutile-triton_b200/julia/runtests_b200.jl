# The reference's correctness tests (test/runtests.jl) on the B200 path:
# same cuTile kernels, same shapes, same CPU checks; kernels come from
# libcutile_b200.so through TileTritonB200 instead of the Triton compiler.
#   julia --project=<TileTriton env> cutile-triton_b200/julia/runtests_b200.jl
include(joinpath(@__DIR__, "TileTritonB200.jl"))
using .TileTritonB200
const TR = TileTritonB200
using CUDA
import cuTile as ct

TR.use_b200!()

const Spec1 = typeof(ct.ArraySpec{1}(128, true, (1,), (0,)))
const Spec2 = typeof(ct.ArraySpec{2}(128, true, (1, 0), (0, 0)))
TA1(T) = ct.TileArray{T, 1, Spec1}
TA2(T) = ct.TileArray{T, 2, Spec2}

npass = 0
function check(name, ok)
    global npass
    ok || error("FAIL: $name")
    npass += 1
    println("  pass: $name")
end

# kernel bodies are never traced on this path; the names select the kernels
function vadd(a, b, c, tile::Int) end
function rowsum(a, out, tm::Int, tn::Int) end
function matmul(A, B, C, tm::Int, tn::Int, tk::Int) end
function softmax(output, input, TILE_SIZE::Int) end

for T in (Float32, Float16, Float64), n in (1_024_000, 999_999)
    k = TR.triton_kernel(vadd, Tuple{TA1(T), TA1(T), TA1(T), ct.Constant{Int, 1024}}; name="vadd")
    a = CUDA.rand(T, n); b = CUDA.rand(T, n); c = CUDA.zeros(T, n)
    TR.launch!(k, cld(n, 1024), a, b, c)
    CUDA.synchronize()
    check("vadd $T n=$n (bit-exact)", Array(c) == Array(a) .+ Array(b))
end

let m = 4096, n = 128
    k = TR.triton_kernel(rowsum, Tuple{TA2(Float32), TA2(Float32), ct.Constant{Int, 64}, ct.Constant{Int, 128}})
    a = CUDA.rand(Float32, m, n); out = CUDA.zeros(Float32, m, 1)
    TR.launch!(k, cld(m, 64), a, out)
    CUDA.synchronize()
    check("rowsum $m x $n", Array(out) ≈ sum(Array(a); dims=2))
end

for (M, N, K) in ((512, 512, 512), (300, 260, 200))
    k = TR.triton_kernel(matmul, Tuple{TA2(Float32), TA2(Float32), TA2(Float32),
                                       ct.Constant{Int, 128}, ct.Constant{Int, 128}, ct.Constant{Int, 32}})
    A = CUDA.rand(Float32, M, K); B = CUDA.rand(Float32, K, N); C = CUDA.zeros(Float32, M, N)
    TR.launch!(k, (cld(M, 128), cld(N, 128)), A, B, C)
    CUDA.synchronize()
    ref = Array(A) * Array(B)
    err = maximum(abs.(Array(C) .- ref)) / max(maximum(abs.(ref)), 1)
    check("matmul $M x $N x $K (rel err $(round(err; sigdigits=2)))", err < 1e-3)
end

let n = 1000, m = 2048
    k = TR.triton_kernel(softmax, Tuple{TA2(Float32), TA2(Float32), ct.Constant{Int, 1024}})
    x = CUDA.rand(Float32, n, m); y = CUDA.zeros(Float32, n, m)
    TR.launch!(k, 512, y, x)
    CUDA.synchronize()
    xh = Array(x); eh = exp.(xh .- maximum(xh; dims=1))
    check("softmax $n x $m", Array(y) ≈ eh ./ sum(eh; dims=1))
end

println("ALL $npass TESTS PASSED")

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

# ---- the next kernels: transpose, moe (registry) and the host-buffer calls ----
function transpose_k(x, y) end  # registry name "transpose" (Base.transpose is not touched)
function moe(A, B, C, sorted, expert_ids, ntp, W, WS, topk, mul) end

let m = 300, n = 517
    k = TR.triton_kernel(transpose_k, Tuple{TA2(Float32), TA2(Float32)}; name="transpose")
    x = CUDA.rand(Float32, m, n); y = CUDA.zeros(Float32, n, m)
    TR.launch!(k, 1, x, y)
    CUDA.synchronize()
    check("transpose $m x $n (bit-exact)", Array(y) == permutedims(Array(x)))
end

let M = 300, N = 256, K = 128, E = 4, topk = 2
    ids = [rand(0:E-1) for _ in 1:topk, _ in 1:M]                      # (topk, M) expert of each slot
    for t in 1:M  # distinct experts per token
        while ids[1, t] == ids[2, t]; ids[2, t] = rand(0:E-1); end
    end
    sorted, experts, ntp = TR.moe_align(ids, E; block=256)
    A = CuArray(rand(Float16, K, M) .- Float16(0.5)); B = CuArray(rand(Float16, K, N, E) .- Float16(0.5))
    W = CuArray(rand(Float32, topk, M)); C = CUDA.zeros(Float16, N, M * topk)
    WS = CUDA.zeros(Float16, K * length(sorted))
    k = TR.triton_kernel(moe, Tuple{TA2(Float16), ct.TileArray{Float16, 3, typeof(ct.ArraySpec{3}(128, true, (1, 0, 0), (0, 0, 0)))},
                                    TA2(Float16), TA1(Int32), TA1(Int32), TA1(Int32), TA2(Float32), TA1(Float16), Int, Int})
    TR.launch!(k, 1, A, B, C, CuArray(sorted), CuArray(experts), CuArray(ntp), W, WS, topk, 1)
    CUDA.synchronize()
    Ah, Bh, Wh, Ch = Float64.(Array(A)), Float64.(Array(B)), Float64.(Array(W)), Float64.(Array(C))
    ref = zeros(N, M * topk)
    for s in 0:M*topk-1  # slot s = token * topk + choice
        t, j = divrem(s, topk)
        ref[:, s+1] = (transpose(Bh[:, :, ids[j+1, t+1]+1]) * Ah[:, t+1]) .* Wh[j+1, t+1]
    end
    err = sqrt(sum(abs2, Ch .- ref) / sum(abs2, ref))
    check("moe $M tokens top-$topk of $E (rel err $(round(err; sigdigits=2)))", err <= 2e-3)
end

let n = 1000, m = 2048
    x = CUDA.pin(rand(Float32, n, m)); y = CUDA.pin(zeros(Float32, n, m))
    TR.softmax_host!(y, x)
    eh = exp.(x .- maximum(x; dims=1))
    check("softmax_host! $n x $m", y ≈ eh ./ sum(eh; dims=1))
    a = CUDA.pin(rand(Float32, 999_999)); b = CUDA.pin(rand(Float32, 999_999)); c = similar(a)
    TR.vadd_host!(c, a, b)
    check("vadd_host! (bit-exact)", c == a .+ b)
end

println("ALL $npass TESTS PASSED")

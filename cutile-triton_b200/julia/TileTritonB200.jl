"""
    TileTritonB200

B200 (sm_100a) backend for TileTriton: the same user-facing API as
`TritonRun` / `TritonShim` (reference: src/runtime.jl, src/shim.jl), with the
TTIR -> Triton -> cubin pipeline replaced by prebuilt kernels in
`libcutile_b200.so`, reached through `ccall` on the C ABI declared in
include/cutile_b200.h.

- `triton_kernel(f, argtypes; name, num_warps, num_stages, use_tma)` returns a
  `B200Kernel` handle (no compilation; unknown kernels raise).
- `launch!(k, grid, args...)` flattens exactly like `TritonRun.flatten_args`
  (runtime.jl:163-198) into `ctb_array`s and launches on CUDA.jl's stream.
- `install_shim!()` overwrites `cuTile.cufunction` so `ct.launch` /
  `@cuda backend=cuTile` of the registered kernels run here (shim.jl:126-131).
- `use_b200!()` selects this backend for `TileTriton.triton_kernel` /
  `launch!` callers (TileTriton's own `triton_kernel`/`launch!` forward here
  when the active target's backend is "b200").

The library path is `ENV["CUTILE_B200_LIB"]`, else the in-tree build.
"""
module TileTritonB200

using CUDA
using Libdl
import cuTile as ct

export triton_kernel, triton_kernel_candidates, launch!, install_shim!, use_b200!, B200Kernel,
       softmax_host!, layernorm_fwd_host!, vadd_host!, moe_align

# ---------------------------------------------------------------------------- library
const LIBPATH = Ref{String}("")
const LIB = Ref{Ptr{Cvoid}}(C_NULL)
const SYMS = Dict{Symbol,Ptr{Cvoid}}()

default_libpath() = get(ENV, "CUTILE_B200_LIB",
                        normpath(joinpath(@__DIR__, "..", "cutile_b200", "libcutile_b200.so")))

function sym(name::Symbol)
    if LIB[] == C_NULL
        LIBPATH[] = default_libpath()
        isfile(LIBPATH[]) || error("b200: libcutile_b200.so not found at $(LIBPATH[])")
        LIB[] = Libdl.dlopen(LIBPATH[])
    end
    get!(() -> Libdl.dlsym(LIB[], name), SYMS, name)
end

lasterror() = unsafe_string(ccall(sym(:ctb_last_error), Cstring, ()))
check(rc::Integer) = rc == 0 ? nothing : error("b200: " * lasterror())

# ---------------------------------------------------------------------------- ABI types
const CTB_MAX_DIMS = 5

"`ctb_array`: one flattened TileArray (pointer, Julia-order sizes and strides)."
struct CtbArray
    ptr::Ptr{Cvoid}
    ndim::Int32
    dtype::Int32
    sizes::NTuple{CTB_MAX_DIMS,Int32}
    strides::NTuple{CTB_MAX_DIMS,Int32}
end

struct CtbKernelInfo
    name::NTuple{32,UInt8}
    narrays::Int32
    nscalars::Int32
    num_warps::Int32
    shared_bytes::Int32
end

dtype_code(::Type{Float16}) = Int32(1)
dtype_code(::Type{Float32}) = Int32(3)
dtype_code(::Type{Float64}) = Int32(4)
dtype_code(::Type{Int32}) = Int32(5)
dtype_code(T::Type) = T === ct.TFloat32 ? error("b200: tf32 inputs are stored as Float32 arrays") :
                      (nameof(T) === :BFloat16 ? Int32(2) : error("b200: unsupported element type $T"))

pad5(t) = ntuple(i -> i <= length(t) ? Int32(t[i]) : Int32(0), CTB_MAX_DIMS)

ctb_array(a::CuArray{T,N}) where {T,N} =
    CtbArray(reinterpret(Ptr{Cvoid}, UInt(pointer(a))), Int32(N), dtype_code(T),
             pad5(size(a)), pad5(strides(a)))

# A converted cuTile argument (what ShimKernel receives; shim.jl:42-63).
ctb_array(x::ct.TileArray) =
    CtbArray(reinterpret(Ptr{Cvoid}, UInt(x.ptr)), Int32(length(x.sizes)),
             dtype_code(eltype(x)), pad5(x.sizes), pad5(x.strides))

# ---------------------------------------------------------------------------- kernels
"Per-parameter ABI record (the reference ArgSpec, src/emitter.jl:163-167)."
struct B200ArgSpec
    kind::Symbol      # :tilearray | :scalar
    elty::Type
    ndims::Int
end

"A prebuilt-kernel handle (the TritonKernel analogue, runtime.jl:85-95)."
struct B200Kernel
    handle::Int32
    name::String
    num_warps::Int
    warp_size::Int
    shared::Int
    global_scratch_size::Int
    argspec::Vector{B200ArgSpec}
end

function argspec_of(argtypes::Type{<:Tuple})
    specs = B200ArgSpec[]
    consts = Int64[]
    for T in argtypes.parameters
        if T <: ct.TileArray
            push!(specs, B200ArgSpec(:tilearray, eltype(T), ndims(T)))
        elseif T <: ct.Constant
            push!(consts, Int64(T.parameters[2]))   # Constant{Int, V}: ghost
        else
            push!(specs, B200ArgSpec(:scalar, T, 0))
        end
    end
    return specs, consts
end

"""
    triton_kernel(f, argtypes; name, num_warps, num_stages, use_tma) -> B200Kernel

Looks up the prebuilt sm_100a kernel for cuTile function `f`. The keyword
arguments are accepted for signature compatibility with
`TritonRun.triton_kernel`; the schedule of each kernel is fixed.
"""
function triton_kernel(@nospecialize(f), @nospecialize(argtypes); name::String=string(nameof(f)),
                       num_warps=nothing, num_stages=nothing, use_tma::Bool=true)
    specs, consts = argspec_of(argtypes)
    dts = Int32[dtype_code(s.elty) for s in specs if s.kind === :tilearray]
    h = Ref{Int32}(-1)
    kname = string(nameof(f))
    check(ccall(sym(:ctb_find_kernel), Cint,
                (Cstring, Ptr{Int32}, Int32, Ptr{Int64}, Int32, Ref{Int32}),
                kname, dts, length(dts), consts, length(consts), h))
    info = Ref{CtbKernelInfo}()
    check(ccall(sym(:ctb_kernel_info_get), Cint, (Int32, Ref{CtbKernelInfo}), h[], info))
    nscal = count(s -> s.kind === :scalar, specs)
    nscal == info[].nscalars ||
        error("b200: $kname expects $(info[].nscalars) scalar parameters, got $nscal")
    return B200Kernel(h[], kname, info[].num_warps, 32, info[].shared_bytes, 0, specs)
end

"One candidate: the hand-written kernel has no variants to race."
triton_kernel_candidates(@nospecialize(f), @nospecialize(argtypes); name::String=string(nameof(f)),
                         use_tma::Bool=true) = [triton_kernel(f, argtypes; name, use_tma)]

function flatten_args(spec::Vector{B200ArgSpec}, args)
    length(spec) == length(args) || error("expected $(length(spec)) kernel arguments")
    arrays = CtbArray[]
    scalars = Float64[]
    for (s, a) in zip(spec, args)
        if s.kind === :tilearray
            a isa AbstractArray || a isa ct.TileArray || error("expected a GPU array for tilearray argument")
            eltype(a) === s.elty || error("eltype mismatch: $(eltype(a)) vs $(s.elty)")
            (a isa ct.TileArray ? length(a.sizes) : ndims(a)) == s.ndims || error("ndims mismatch")
            push!(arrays, ctb_array(a))
        else
            push!(scalars, Float64(a))
        end
    end
    return arrays, scalars
end

function raw_launch(handle::Int32, arrays::Vector{CtbArray}, scalars::Vector{Float64}, g)
    grid = Int32[g[1], g[2], g[3]]
    rc = ccall(sym(:ctb_launch), Cint,
               (Int32, Ptr{CtbArray}, Int32, Ptr{Float64}, Int32, Ptr{Int32}, Ptr{Cvoid}),
               handle, arrays, length(arrays), scalars, length(scalars), grid,
               CUDA.stream().handle)
    check(rc)
end

normgrid(grid) = grid isa Integer ? (Int(grid), 1, 1) :
                 length(grid) == 2 ? (grid[1], grid[2], 1) : Tuple(grid)

"""
    launch!(k::B200Kernel, grid, args...)

`grid` is advisory (outputs never depend on it); `args` are the kernel's
Julia-level arguments in order, skipping `ct.Constant` slots.
"""
function launch!(k::B200Kernel, grid, args...)
    arrays, scalars = flatten_args(k.argspec, args)
    GC.@preserve args raw_launch(k.handle, arrays, scalars, normgrid(grid))
    return nothing
end

# ---------------------------------------------------------------------------- shim
mutable struct B200ShimKernel{F,TT} <: ct.AbstractKernel{F,TT}
    kernel::B200Kernel
    f::F
end

const KERNEL_CACHE = Dict{Any,Any}()

function get_kernel(@nospecialize(f), @nospecialize(tt))
    key = (f, tt, Base.get_world_counter())
    haskey(KERNEL_CACHE, key) && return KERNEL_CACHE[key]
    k = B200ShimKernel{typeof(f),tt}(triton_kernel(f, tt), f)
    KERNEL_CACHE[key] = k
    return k
end

# Ghost arguments (Constant and other singletons) carry no bytes; dropping them
# with a recursive tuple filter is specialised per signature, with no Any[].
drop_ghosts() = ()
drop_ghosts(a, rest...) = Base.issingletontype(typeof(a)) ? drop_ghosts(rest...) :
                          (a, drop_ghosts(rest...)...)

# cuTile calls the kernel with converted arguments (TileArrays, ghosts, primitives).
function (k::B200ShimKernel)(args...; blocks=1, threads=1, convert=Val(false), kwargs...)
    arrays, scalars = flatten_args(k.kernel.argspec, drop_ghosts(args...))
    GC.@preserve args raw_launch(k.kernel.handle, arrays, scalars, normgrid(blocks))
    return nothing
end

"""
    install_shim!()

Route cuTile compilation of the registered kernels to libcutile_b200.so by
overwriting `cuTile.cufunction` (opt-in, like the reference's shim).
"""
function install_shim!()
    @eval ct function cufunction(@nospecialize(f), tt::Type{<:Tuple}=Tuple{}; kwargs...)
        return $(TileTritonB200).get_kernel(f, tt)
    end
    return nothing
end

# ---- host-buffer calls: arrays in (pinned) host memory, chunks pipelined through
# a device workspace on the library's streams; synchronise the stream to read results.
const HOST_WS = Ref{Any}(nothing)
function host_workspace(nbytes::Integer)
    ws = HOST_WS[]
    if ws === nothing || sizeof(ws) < nbytes
        ws = CuArray{UInt8}(undef, max(Int(nbytes), 256))
        HOST_WS[] = ws
    end
    return ws
end
wsbytes(inb, outb, units) = ccall(sym(:ctb_host_workspace_bytes), Int64, (Int64, Int64, Int64),
                                  inb, outb, units)

"y = softmax over each column of the host matrix x (len x count), through the GPU."
function softmax_host!(y::Matrix{Float32}, x::Matrix{Float32})
    len, count = size(x)
    ws = host_workspace(wsbytes(4len, 4len, count))
    check(ccall(sym(:ctb_softmax_f32_host), Cint,
                (Ptr{Float32}, Ptr{Float32}, Int32, Int32, CuPtr{UInt8}, Int64, Ptr{Cvoid}),
                x, y, len, count, ws, sizeof(ws), CUDA.stream().handle))
    CUDA.synchronize()
    return y
end

"LayerNorm over each column of the host matrix x (n x rows): y, mean, rstd on the host."
function layernorm_fwd_host!(y::Matrix{Float32}, mean::Vector{Float32}, rstd::Vector{Float32},
                             x::Matrix{Float32}, w::Vector{Float32}, b::Vector{Float32}, eps=1f-5)
    n, rows = size(x)
    ws = host_workspace(wsbytes(4n, 4n + 8, rows) + 2 * cld(4n, 256) * 256)
    check(ccall(sym(:ctb_layernorm_fwd_f32_host), Cint,
                (Ptr{Float32}, Ptr{Float32}, Ptr{Float32}, Ptr{Float32}, Ptr{Float32}, Ptr{Float32},
                 Int32, Int32, Float32, CuPtr{UInt8}, Int64, Ptr{Cvoid}),
                x, w, b, y, mean, rstd, n, rows, eps, ws, sizeof(ws), CUDA.stream().handle))
    CUDA.synchronize()
    return y, mean, rstd
end

"c = a + b for host vectors, through the GPU."
function vadd_host!(c::Vector{T}, a::Vector{T}, b::Vector{T}) where {T<:Union{Float16,Float32,Float64}}
    ws = host_workspace(wsbytes(2sizeof(T), sizeof(T), length(a)) + 16 * 256)
    check(ccall(sym(:ctb_vadd_host), Cint,
                (Int32, Ptr{T}, Ptr{T}, Ptr{T}, Int64, CuPtr{UInt8}, Int64, Ptr{Cvoid}),
                dtype_code(T), a, b, c, length(a), ws, sizeof(ws), CUDA.stream().handle))
    CUDA.synchronize()
    return c
end

"""
    moe_align(topk_ids::Matrix{<:Integer}, num_experts; block=256)

Fused-MoE routing for the `moe` kernel from a (topk, tokens) matrix of
0-based expert ids: (sorted_token_ids, expert_ids, num_tokens_post_padded) as
Int32 vectors, slots grouped by expert in slot order, each expert padded to a
multiple of `block` (256: CTA-pair kernel, 128: single-SM kernel) with the id
tokens*topk. Move them to the device with `CuArray`.
"""
function moe_align(topk_ids::AbstractMatrix{<:Integer}, num_experts::Integer; block::Integer=256)
    flat = vec(topk_ids)  # slot s = token * topk + choice (column-major (topk, tokens))
    n = length(flat)
    sorted = Int32[]
    experts = Int32[]
    for e in 0:num_experts-1
        slots = [Int32(s - 1) for s in 1:n if flat[s] == e]
        pad = mod(-length(slots), block)
        append!(sorted, slots, fill(Int32(n), pad))
        append!(experts, fill(Int32(e), (length(slots) + pad) ÷ block))
    end
    em = length(sorted)
    if em == 0  # nothing routed: one padding block with no expert, none in use
        sorted = fill(Int32(n), block)
        experts = Int32[-1]
    end
    return sorted, experts, Int32[em]
end

"""
    moe_align(topk_ids::CuMatrix{Int32}, num_experts; block=256)

The same routing on the device (`ctb_moe_align_i32`), with no host round trip:
the outputs are CuArrays sized for the worst case (`ctb_moe_align_capacity`);
entries past num_tokens_post_padded hold the padding id and blocks past it the
expert -1, which the `moe` kernel skips. At most 256 experts.
"""
function moe_align(topk_ids::CuMatrix{Int32}, num_experts::Integer; block::Integer=256)
    n = length(topk_ids)
    cap = ccall(sym(:ctb_moe_align_capacity), Int32, (Int32, Int32, Int32), n, num_experts, block)
    cap < 0 && error("b200: moe_align: bad sizes")
    sorted = CuArray{Int32}(undef, cap)
    experts = CuArray{Int32}(undef, cap ÷ block)
    ntp = CuArray{Int32}(undef, 1)
    check(ccall(sym(:ctb_moe_align_i32), Cint,
                (CuPtr{Int32}, Int32, Int32, Int32, CuPtr{Int32}, CuPtr{Int32}, CuPtr{Int32},
                 Int32, Ptr{Cvoid}),
                topk_ids, n, num_experts, block, sorted, experts, ntp, cap,
                CUDA.stream().handle))
    return sorted, experts, ntp
end

"Initialises the library on the active CUDA device (kernel attributes, checks sm_100)."
function use_b200!()
    check(ccall(sym(:ctb_init), Cint, (Cint,), CUDA.deviceid(CUDA.device())))
    @info "TileTriton: using the B200 sm_100a kernel library $(LIBPATH[])"
    return nothing
end

end # module

"""
    KernelIntrinsicsB200

Julia host binding of `libki_b200.so` (the C ABI in `include/ki_b200.h`) for CUDA.jl arrays on
NVIDIA B200 GPUs.  Names mirror KernelIntrinsics.jl (src/KernelIntrinsics.jl:5-10, src/warp.jl:188-315,
src/vectorization.jl:1-129, src/device.jl:1-19): the warp-level intrinsics run over whole warps of an
array, and the device-wide operations those intrinsics build (`sum`, `cumsum`, `filter`/`findall`,
`copyto!`) run as hand-written sm_100a kernels.  Every call is stream-ordered on `CUDA.stream()`;
`Idx` lanes and device numbers are 1-based here, as in the reference, and 0-based at the C ABI.

Errors follow the reference: misuse raises `ArgumentError` (the reference raises it at macro
expansion), a device-side bounded wait that ran out raises `KITimeoutError`, anything else `KIError`.
"""
module KernelIntrinsicsB200

using CUDA

export get_warpsize, devices, deviceid, context, check_device,
       Workgroup, Device, System, Weak, Volatile, Relaxed, Acquire, Release, AcqRel, SeqCst,
       Up, Down, Xor, Idx, All, AnyLane, Uni, Ballot,
       shfl!, warpreduce!, warpfold!, vote!, vload, vstore!, access_roundtrip!,
       warpfold_reduce, reduce_ki, mapreduce_ki, reduce_rows_ki,
       warpreduce_scan!, warpreduce_scan_host!, warpreduce_scan_noalloc!, accumulate_ki!, accumulate_rows_ki!,
       vote_compact, filter_ki, count_ki,
       vcopy!, vcopy2d!, vcopy_strided!, fp8_gemm!,
       Comm, comm_id, comms, sum_sharded, cumsum_sharded!, cumsum_sharded_host!, findall_sharded, shard_range,
       abort!

const libki = normpath(joinpath(@__DIR__, "..", "lib", "libki_b200.so"))

# ---- status codes (ki_status) ----------------------------------------------------------------
const KI_OK = Cint(0)
const KI_ERR_ARG = Cint(1)
const KI_ERR_TIMEOUT = Cint(3)

struct KIError <: Exception
    status::Cint
    msg::String
end
Base.showerror(io::IO, e::KIError) = print(io, "KIError(", e.status, "): ", e.msg)
struct KITimeoutError <: Exception
    msg::String
end
Base.showerror(io::IO, e::KITimeoutError) = print(io, "KITimeoutError: ", e.msg)

_errstr(ctx::Ptr{Cvoid}) = unsafe_string(ccall((:ki_last_error_string, libki), Cstring, (Ptr{Cvoid},), ctx))
_statusstr(st) = unsafe_string(ccall((:ki_status_string, libki), Cstring, (Cint,), st))

function _check(st::Cint, ctx::Ptr{Cvoid} = C_NULL)
    st == KI_OK && return nothing
    msg = _errstr(ctx)
    st == KI_ERR_ARG && throw(ArgumentError(msg))
    st == KI_ERR_TIMEOUT && throw(KITimeoutError(msg))
    throw(KIError(st, isempty(msg) ? _statusstr(st) : msg))
end

# ---- type lattices (src/scopes_orderings.jl:13-120, src/warp.jl:16-106) -----------------------
abstract type Scope end
struct Workgroup <: Scope end
struct Device <: Scope end
struct System <: Scope end
abstract type Ordering end
struct Weak <: Ordering end
struct Volatile <: Ordering end
struct Relaxed <: Ordering end
struct Acquire <: Ordering end
struct Release <: Ordering end
struct AcqRel <: Ordering end
struct SeqCst <: Ordering end
abstract type Direction end
struct Up <: Direction end
struct Down <: Direction end
struct Xor <: Direction end
struct Idx <: Direction end
abstract type Mode end
struct All <: Mode end
struct AnyLane <: Mode end
struct Uni <: Mode end
struct Ballot <: Mode end

_code(::Type{Nothing}) = Cint(0)
_code(::Type{Workgroup}) = Cint(1); _code(::Type{Device}) = Cint(2); _code(::Type{System}) = Cint(3)
_code(::Type{Weak}) = Cint(1); _code(::Type{Volatile}) = Cint(2); _code(::Type{Relaxed}) = Cint(3)
_code(::Type{Acquire}) = Cint(4); _code(::Type{Release}) = Cint(5); _code(::Type{AcqRel}) = Cint(6)
_code(::Type{SeqCst}) = Cint(7)
_code(::Type{Up}) = Cint(0); _code(::Type{Down}) = Cint(1); _code(::Type{Xor}) = Cint(2); _code(::Type{Idx}) = Cint(3)
_code(::Type{All}) = Cint(0); _code(::Type{AnyLane}) = Cint(1); _code(::Type{Uni}) = Cint(2)
_code(::Type{Ballot}) = Cint(3)

const _dtype = Dict{DataType,Cint}(Int8 => 0, UInt8 => 1, Int16 => 2, UInt16 => 3, Int32 => 4, UInt32 => 5,
                                   Int64 => 6, UInt64 => 7, Float32 => 8, Float64 => 9)
const _op = Dict{Any,Cint}(+ => 0, max => 1, min => 2, (|) => 3, (&) => 4, xor => 5, (*) => 6)
const _map = Dict{Any,Cint}(identity => 0, abs => 1, abs2 => 2)
const _pred = Dict{Any,Cint}(> => 0, >= => 1, < => 2, <= => 3, == => 4, != => 5)
_dt(::Type{T}) where {T} = haskey(_dtype, T) ? _dtype[T] : throw(ArgumentError("unsupported element type $T"))
_opc(op) = haskey(_op, op) ? _op[op] : throw(ArgumentError("unsupported operator $op"))
# Base's result type of sum / prod (Base.add_sum, Base.mul_prod); every other operator keeps T
_rt(::Type{T}, op) where {T} = (op in (+, *) && T <: Union{Int8,Int16,Int32}) ? Int64 :
                               (op in (+, *) && T <: Union{UInt8,UInt16,UInt32}) ? UInt64 : T

# ---- devices and contexts (src/device.jl:1-19, ext/CUDA/device.jl:4-13) ------------------------
function devices()
    n = Ref{Cint}(0)
    ccall((:ki_device_count, libki), Cint, (Ref{Cint},), n)
    return collect(1:Int(n[]))
end
deviceid(x::CuArray) = CUDA.deviceid(CUDA.device(x)) + 1
function get_warpsize(dev::Integer = 1)
    ws = Ref{Cint}(0)
    _check(ccall((:ki_device_info, libki), Cint, (Cint, Ptr{Cint}, Ref{Cint}, Ptr{Cint}, Ptr{Cint}),
                 dev - 1, C_NULL, ws, C_NULL, C_NULL))
    return Int(ws[])
end

const _ctx_lock = ReentrantLock()
const _ctxs = Dict{Tuple{Int,Int},Ptr{Cvoid}}()

"The calling thread's libki_b200 context on the current CUDA device (created on first use)."
function context()
    dev = CUDA.deviceid(CUDA.device())
    key = (Threads.threadid(), dev)
    lock(_ctx_lock) do
        get!(_ctxs, key) do
            r = Ref{Ptr{Cvoid}}(C_NULL)
            _check(ccall((:ki_ctx_create, libki), Cint, (Cint, Ref{Ptr{Cvoid}}), dev, r))
            r[]
        end
    end
end
_stream() = CUDA.stream().handle
_call(f) = (c = context(); _check(f(c), c))

"Synchronise the stream and raise if a device-side bounded wait of this context ran out."
check_device() = _call(c -> ccall((:ki_ctx_check, libki), Cint, (Ptr{Cvoid}, Ptr{Cvoid}), c, _stream()))

# ---- warp intrinsics over whole warps (element i is lane i % 32 of warp i / 32) -------------------
"@shfl(Dir, val, src) on every warp of `x`: src is the offset (Up/Down), the lane mask (Xor) or the 1-based lane (Idx)."
function shfl!(y::CuVector{T}, ::Type{D}, x::CuVector{T}, src::Integer) where {T,D<:Direction}
    s = D === Idx ? (1 <= src <= 32 ? src - 1 : throw(ArgumentError("Idx lane must be in 1..32"))) : src
    _call(c -> ccall((:ki_warp_shfl, libki), Cint, (Ptr{Cvoid}, Cint, CuPtr{T}, CuPtr{T}, Csize_t, Csize_t, Cint, Ptr{Cvoid}),
                     c, _code(D), x, y, sizeof(T), length(x), s, _stream()))
    return y
end
"@warpreduce(val, op): inclusive scan of every warp with Up shuffles."
warpreduce!(y::CuVector{T}, op, x::CuVector{T}) where {T} =
    (_call(c -> ccall((:ki_warp_reduce, libki), Cint, (Ptr{Cvoid}, Cint, Cint, CuPtr{T}, CuPtr{T}, Csize_t, Ptr{Cvoid}),
                      c, _opc(op), _dt(T), x, y, length(x), _stream())); y)
"@warpfold(val, op): form :xor (every lane holds the total) or :down (the reference's Down fold, lane 1)."
warpfold!(y::CuVector{T}, op, x::CuVector{T}; form::Symbol = :xor) where {T} =
    (_call(c -> ccall((:ki_warp_fold, libki), Cint, (Ptr{Cvoid}, Cint, Cint, Cint, CuPtr{T}, CuPtr{T}, Csize_t, Ptr{Cvoid}),
                      c, _opc(op), _dt(T), form === :down ? 1 : 0, x, y, length(x), _stream())); y)
"@vote(Mode, pred): one UInt32 per lane (0/1, or the ballot mask)."
vote!(y::CuVector{UInt32}, ::Type{M}, pred::CuVector{UInt8}) where {M<:Mode} =
    (_call(c -> ccall((:ki_warp_vote, libki), Cint, (Ptr{Cvoid}, Cint, CuPtr{UInt8}, CuPtr{UInt32}, Csize_t, Ptr{Cvoid}),
                      c, _code(M), pred, y, length(pred), _stream())); y)

"vload(A, idx, Val(N)) run by one device thread: 1-based block index (rebase) or element index."
function vload(a::CuVector{T}, idx::Integer, ::Val{N}, ::Val{Rebase} = Val(true)) where {T,N,Rebase}
    out = CuVector{T}(undef, N)
    _call(c -> ccall((:ki_vload, libki), Cint, (Ptr{Cvoid}, CuPtr{T}, Csize_t, Int64, Cint, Cint, CuPtr{T}, Ptr{Cvoid}),
                     c, a, sizeof(T), idx - 1, N, Rebase ? 1 : 0, out, _stream()))
    return NTuple{N,T}(Array(out))
end
function vstore!(a::CuVector{T}, idx::Integer, values::NTuple{N,T}, ::Val{Rebase} = Val(true)) where {T,N,Rebase}
    v = CuVector{T}(collect(values))
    _call(c -> ccall((:ki_vstore, libki), Cint, (Ptr{Cvoid}, CuPtr{T}, Csize_t, Int64, Cint, Cint, CuPtr{T}, Ptr{Cvoid}),
                     c, a, sizeof(T), idx - 1, N, Rebase ? 1 : 0, v, _stream()))
    return a
end

"@access store with (S, store order), @fence(FS, FO), @access load with (S, load order) on one slot."
function access_roundtrip!(slot::CuVector{T}, value::CuVector{T}, readback::CuVector{T};
                           scope = Nothing, store = Nothing, load = Nothing,
                           fence_scope = Nothing, fence_order = Nothing) where {T}
    _call(c -> ccall((:ki_access_roundtrip, libki), Cint,
                     (Ptr{Cvoid}, Cint, Cint, Cint, Cint, Cint, Cint, CuPtr{T}, CuPtr{T}, CuPtr{T}, Ptr{Cvoid}),
                     c, _dt(T), _code(scope), _code(store), _code(load), _code(fence_scope), _code(fence_order),
                     slot, value, readback, _stream()))
    return readback
end

# ---- device-wide reduce (the @warpfold-built sum) ---------------------------------------------
"sum(x) of Float32 `x` with Float64 accumulation (returns the Float64 value)."
function warpfold_reduce(x::CuVector{Float32})
    out = CuVector{Float64}(undef, 1)
    _call(c -> ccall((:ki_reduce_sum_f32, libki), Cint,
                     (Ptr{Cvoid}, CuPtr{Float32}, Csize_t, CuPtr{Float32}, CuPtr{Float64}, Ptr{Cvoid}),
                     c, x, length(x), CuPtr{Float32}(0), out, _stream()))
    return Array(out)[1]
end
"reduce(op, x) with Base's result types (sum/prod/maximum/minimum/reduce(|, &, xor))."
function reduce_ki(op, x::CuVector{T}) where {T}
    out = CuVector{_rt(T, op)}(undef, 1)
    _call(c -> ccall((:ki_reduce, libki), Cint, (Ptr{Cvoid}, Cint, Cint, CuPtr{T}, Csize_t, CuPtr{_rt(T, op)}, Ptr{Cvoid}),
                     c, _opc(op), _dt(T), x, length(x), out, _stream()))
    return Array(out)[1]
end
"mapreduce(f, op, x) for f in identity, abs, abs2 and op in +, max, min."
function mapreduce_ki(f, op, x::CuVector{T}) where {T}
    R = _rt(T, op)
    out = CuVector{R}(undef, 1)
    _call(c -> ccall((:ki_mapreduce, libki), Cint, (Ptr{Cvoid}, Cint, Cint, Cint, CuPtr{T}, Csize_t, CuPtr{R}, Ptr{Cvoid}),
                     c, _map[f], _opc(op), _dt(T), x, length(x), out, _stream()))
    return Array(out)[1]
end
"reduce(op, A; dims=1) of a column-major matrix (one result per column)."
function reduce_rows_ki(op, A::CuMatrix{T}) where {T}
    R = _rt(T, op)
    out = CuVector{R}(undef, size(A, 2))
    _call(c -> ccall((:ki_reduce_rows, libki), Cint,
                     (Ptr{Cvoid}, Cint, Cint, CuPtr{T}, Csize_t, Csize_t, Csize_t, CuPtr{R}, Ptr{Cvoid}),
                     c, _opc(op), _dt(T), A, size(A, 2), size(A, 1), stride(A, 2), out, _stream()))
    return out
end

# ---- device-wide scan (the @warpreduce-built single-pass scan) --------------------------------
"cumsum of Int64 `x` into `y` (plus `seed`)."
warpreduce_scan!(y::CuVector{Int64}, x::CuVector{Int64}; seed::Integer = 0) =
    (_call(c -> ccall((:ki_scan_inclusive_i64, libki), Cint, (Ptr{Cvoid}, CuPtr{Int64}, CuPtr{Int64}, Csize_t, Int64, Ptr{Cvoid}),
                      c, x, y, length(x), seed, _stream())); y)
"""cumsum of a HOST Int64 array through the GPU (16 MiB chunks cross PCIe, are scanned on the device,
each seeded there with the previous chunk's last value, and come back; both directions overlap).
Pin the arrays (CUDA.Mem.pin) for the copies to be asynchronous; returns after synchronising."""
function warpreduce_scan_host!(y::Vector{Int64}, x::Vector{Int64}; seed::Integer = 0)
    length(y) == length(x) || throw(DimensionMismatch("warpreduce_scan_host!"))
    GC.@preserve x y _call(c -> ccall((:ki_scan_inclusive_i64_host, libki), Cint,
                                      (Ptr{Cvoid}, Ptr{Int64}, Ptr{Int64}, Csize_t, Int64, Ptr{Cvoid}),
                                      c, pointer(x), pointer(y), length(x), seed, _stream()))
    CUDA.synchronize()
    return y
end
"""The same scan without a context and without allocating (callers that may not allocate device
memory); n <= 2^28, calls must not overlap on the GPU, first call per device before any capture."""
function warpreduce_scan_noalloc!(y::CuVector{Int64}, x::CuVector{Int64}; seed::Integer = 0)
    st = ccall((:ki_scan_inclusive_i64_noalloc, libki), Cint, (CuPtr{Int64}, CuPtr{Int64}, Csize_t, Int64, Ptr{Cvoid}),
               x, y, length(x), seed, _stream())
    st == KI_ERR_ARG && throw(ArgumentError("noalloc scan: n above 2^28 or bad pointers"))
    st == KI_OK || throw(KIError(st, _statusstr(st)))
    return y
end
"accumulate(op, x; init) / cumsum / cumprod, inclusive or exclusive, into `y` of Base's result type."
function accumulate_ki!(y::CuVector{R}, op, x::CuVector{T}; init = nothing, exclusive::Bool = false) where {R,T}
    r = Ref{R}(init === nothing ? zero(R) : convert(R, init))
    GC.@preserve r _call(c -> ccall((:ki_scan, libki), Cint,
                                    (Ptr{Cvoid}, Cint, Cint, Cint, CuPtr{T}, CuPtr{R}, Csize_t, Ptr{Cvoid}, Ptr{Cvoid}),
                                    c, _opc(op), _dt(T), exclusive, x, y, length(x),
                                    init === nothing ? C_NULL : Base.unsafe_convert(Ptr{Cvoid}, r), _stream()))
    return y
end
"accumulate(op, A; dims=1) of a column-major matrix into `B`."
function accumulate_rows_ki!(B::CuMatrix{R}, op, A::CuMatrix{T}; init = nothing, exclusive::Bool = false) where {R,T}
    r = Ref{R}(init === nothing ? zero(R) : convert(R, init))
    GC.@preserve r _call(c -> ccall((:ki_scan_rows, libki), Cint,
                                    (Ptr{Cvoid}, Cint, Cint, Cint, CuPtr{T}, Csize_t, CuPtr{R}, Csize_t, Csize_t, Csize_t,
                                     Ptr{Cvoid}, Ptr{Cvoid}),
                                    c, _opc(op), _dt(T), exclusive, A, stride(A, 2), B, stride(B, 2), size(A, 2),
                                    size(A, 1), init === nothing ? C_NULL : Base.unsafe_convert(Ptr{Cvoid}, r), _stream()))
    return B
end

# ---- compaction (the @vote Ballot compaction) ---------------------------------------------------
"filter(>(t), x) and findall(>(t), x) for Float32 (1-based Int32 indices)."
function vote_compact(x::CuVector{Float32}, t::Real)
    n = length(x)
    vals = CuVector{Float32}(undef, n); idx = CuVector{Int32}(undef, n); cnt = CUDA.zeros(UInt64, 1)
    _call(c -> ccall((:ki_compact_gt_f32, libki), Cint,
                     (Ptr{Cvoid}, CuPtr{Float32}, Csize_t, Float32, CuPtr{Float32}, CuPtr{Int32}, Int64, CuPtr{UInt64}, Ptr{Cvoid}),
                     c, x, n, Float32(t), vals, idx, 1, cnt, _stream()))
    k = Int(Array(cnt)[1])
    return vals[1:k], idx[1:k]
end
"filter(v -> f(v) pred t, x) and its findall; pred in >, >=, <, <=, ==, !=; f in identity, abs, abs2."
function filter_ki(x::CuVector{T}, pred, t; f = identity) where {T}
    n = length(x)
    vals = CuVector{T}(undef, n); idx = CuVector{Int32}(undef, n); cnt = CUDA.zeros(UInt64, 1)
    r = Ref{T}(convert(T, t))
    GC.@preserve r _call(c -> ccall((:ki_compact_map, libki), Cint,
                                    (Ptr{Cvoid}, Cint, Cint, Cint, CuPtr{T}, Csize_t, Ptr{Cvoid}, CuPtr{T}, CuPtr{Int32}, Int64,
                                     CuPtr{UInt64}, Ptr{Cvoid}),
                                    c, _map[f], _pred[pred], _dt(T), x, n, Base.unsafe_convert(Ptr{Cvoid}, r), vals, idx, 1,
                                    cnt, _stream()))
    k = Int(Array(cnt)[1])
    return vals[1:k], idx[1:k]
end
"count(v -> f(v) pred t, x)."
function count_ki(x::CuVector{T}, pred, t; f = identity) where {T}
    cnt = CUDA.zeros(UInt64, 1)
    r = Ref{T}(convert(T, t))
    GC.@preserve r _call(c -> ccall((:ki_compact_map, libki), Cint,
                                    (Ptr{Cvoid}, Cint, Cint, Cint, CuPtr{T}, Csize_t, Ptr{Cvoid}, CuPtr{T}, CuPtr{Int32}, Int64,
                                     CuPtr{UInt64}, Ptr{Cvoid}),
                                    c, _map[f], _pred[pred], _dt(T), x, length(x), Base.unsafe_convert(Ptr{Cvoid}, r),
                                    CuPtr{T}(0), CuPtr{Int32}(0), 1, cnt, _stream()))
    return Int(Array(cnt)[1])
end

# ---- copies (vload_multi / vstore_multi! over whole ranges) ------------------------------------
"copyto!(dst, src) of the bytes of two device arrays at any byte alignment."
function vcopy!(dst::CuArray, src::CuArray)
    nb = min(sizeof(dst), sizeof(src))
    _call(c -> ccall((:ki_vcopy, libki), Cint, (Ptr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Csize_t, Ptr{Cvoid}),
                     c, dst, src, nb, _stream()))
    return dst
end
"copyto!(dst, src) of two host arrays through the GPU (pin them with CUDA.Mem.pin to overlap)."
function vcopy!(dst::Array{T}, src::Array{T}) where {T}
    nb = min(sizeof(dst), sizeof(src))
    GC.@preserve dst src _call(c -> ccall((:ki_vcopy_host, libki), Cint, (Ptr{Cvoid}, Ptr{T}, Ptr{T}, Csize_t, Ptr{Cvoid}),
                                          c, pointer(dst), pointer(src), nb, _stream()))
    CUDA.synchronize()
    return dst
end
"copyto!(B, A) of two 2-D strided views of device matrices (a block of a column-major matrix)."
function vcopy2d!(B::SubArray{T,2}, A::SubArray{T,2}) where {T}
    size(B) == size(A) || throw(DimensionMismatch("copyto!"))
    _call(c -> ccall((:ki_vcopy_2d, libki), Cint, (Ptr{Cvoid}, CuPtr{T}, Csize_t, CuPtr{T}, Csize_t, Csize_t, Csize_t, Ptr{Cvoid}),
                     c, pointer(B), stride(B, 2) * sizeof(T), pointer(A), stride(A, 2) * sizeof(T),
                     size(A, 1) * sizeof(T), size(A, 2), _stream()))
    return B
end
"copyto!(y, x) of two 1-D strided views (strides in elements, either sign), elements of any size."
function vcopy_strided!(y::SubArray{T,1}, x::SubArray{T,1}) where {T}
    length(y) == length(x) || throw(DimensionMismatch("copyto!"))
    _call(c -> ccall((:ki_vcopy_strided, libki), Cint, (Ptr{Cvoid}, CuPtr{T}, Int64, CuPtr{T}, Int64, Csize_t, Csize_t, Ptr{Cvoid}),
                     c, pointer(y), stride(y, 1), pointer(x), stride(x, 1), sizeof(T), length(x), _stream()))
    return y
end

# ---- fp8 e4m3 GEMM on tcgen05 ------------------------------------------------------------------
"""C = sa*sb * A*B for e4m3 codes (UInt8).  The ABI is row-major; a column-major Julia matrix is the
row-major transpose, so C' = B' * A' is computed: pass A (K x M), B (N x K) and get C (N x M)."""
function fp8_gemm!(C::CuMatrix{Float32}, A::CuMatrix{UInt8}, B::CuMatrix{UInt8}; sa = 1f0, sb = 1f0)
    # row-major views: Ct (M x N) = At (M x K) * Bt (K x N) with At = A' etc.
    M, K = size(A, 2), size(A, 1)
    N = size(B, 1)
    size(B, 2) == K || throw(DimensionMismatch("fp8_gemm!"))
    _call(c -> ccall((:ki_gemm_e4m3_f32, libki), Cint,
                     (Ptr{Cvoid}, CuPtr{UInt8}, CuPtr{UInt8}, CuPtr{Float32}, Cint, Cint, Cint, Float32, Float32, Ptr{Cvoid}),
                     c, A, B, C, M, N, K, sa, sb, _stream()))
    return C
end

# ---- several GPUs: communicators and sharded operations ---------------------------------------
"""One rank of a libki_b200 communicator.  Every rank calls the same sharded operations in the same
order, each on its own contiguous shard; only one 8-byte value per rank and operation crosses NVLink."""
mutable struct Comm
    handle::Ptr{Cvoid}
    ctx::Ptr{Cvoid}
    nranks::Int
    rank::Int        # 0-based, as the shard order
    device::Int      # 0-based CUDA ordinal
end

function _wrap_comm(h::Ptr{Cvoid})
    nr, rk, dv, ex = Ref{Cint}(0), Ref{Cint}(0), Ref{Cint}(0), Ref{Cint}(0)
    ccall((:ki_comm_info, libki), Cint, (Ptr{Cvoid}, Ref{Cint}, Ref{Cint}, Ref{Cint}, Ref{Cint}), h, nr, rk, dv, ex)
    c = Ref{Ptr{Cvoid}}(C_NULL)
    ccall((:ki_comm_get_ctx, libki), Cint, (Ptr{Cvoid}, Ref{Ptr{Cvoid}}), h, c)
    return Comm(h, c[], Int(nr[]), Int(rk[]), Int(dv[]))
end

"A 128-byte id made by one rank and handed to the others (e.g. with MPI.Bcast!)."
function comm_id()
    id = zeros(UInt8, 128)
    st = ccall((:ki_comm_get_id, libki), Cint, (Ptr{UInt8},), id)
    st == KI_OK || throw(KIError(st, _statusstr(st)))
    return id
end
"One process per GPU: join communicator `id` as `rank` of `nranks` on the current CUDA device."
function Comm(id::Vector{UInt8}, nranks::Integer, rank::Integer; exchange::Symbol = :auto)
    length(id) == 128 || throw(ArgumentError("communicator id must be 128 bytes"))
    h = Ref{Ptr{Cvoid}}(C_NULL)
    x = exchange === :peer ? 1 : exchange === :nccl ? 2 : 0
    st = ccall((:ki_comm_init_rank, libki), Cint, (Cint, Cint, Cint, Ptr{UInt8}, Cint, Ref{Ptr{Cvoid}}),
               CUDA.deviceid(CUDA.device()), nranks, rank, id, x, h)
    _check(st)
    return _wrap_comm(h[])
end
"One process driving several GPUs (1-based device numbers): one Comm per device."
function comms(devs::AbstractVector{<:Integer})
    n = length(devs)
    hs = Vector{Ptr{Cvoid}}(undef, n)
    st = ccall((:ki_comm_create, libki), Cint, (Cint, Ptr{Cint}, Ptr{Ptr{Cvoid}}), n, Cint.(devs .- 1), hs)
    _check(st)
    return [_wrap_comm(h) for h in hs]
end
Base.close(c::Comm) = (c.handle == C_NULL || _check(ccall((:ki_comm_destroy, libki), Cint, (Ptr{Cvoid},), c.handle));
                       c.handle = C_NULL; nothing)
abort!(c::Comm) = (c.handle == C_NULL || ccall((:ki_comm_abort, libki), Cint, (Ptr{Cvoid},), c.handle);
                   c.handle = C_NULL; nothing)
"1-based global index range of `rank`'s shard of n elements (the first n % nranks shards hold one more)."
function shard_range(n::Integer, nranks::Integer, rank::Integer)
    lo, cnt = Ref{Csize_t}(0), Ref{Csize_t}(0)
    _check(ccall((:ki_comm_shard_range, libki), Cint, (Csize_t, Cint, Cint, Ref{Csize_t}, Ref{Csize_t}),
                 n, nranks, rank, lo, cnt))
    return Int(lo[]) + 1:Int(lo[] + cnt[])
end
_ccheck(c::Comm, st::Cint) = _check(st, c.ctx)

"sum over all ranks' Float32 shards; every rank gets the same Float64 bits."
function sum_sharded(c::Comm, x::CuVector{Float32})
    out = CuVector{Float64}(undef, 1)
    _ccheck(c, ccall((:ki_reduce_sum_f32_sharded, libki), Cint,
                     (Ptr{Cvoid}, CuPtr{Float32}, Csize_t, CuPtr{Float32}, CuPtr{Float64}, Ptr{Cvoid}),
                     c.handle, x, length(x), CuPtr{Float32}(0), out, _stream()))
    return Array(out)[1]
end
"This rank's slice of cumsum over the concatenated Int64 shards."
cumsum_sharded!(c::Comm, y::CuVector{Int64}, x::CuVector{Int64}) =
    (_ccheck(c, ccall((:ki_scan_inclusive_i64_sharded, libki), Cint,
                      (Ptr{Cvoid}, CuPtr{Int64}, CuPtr{Int64}, Csize_t, Ptr{Cvoid}),
                      c.handle, x, y, length(x), _stream())); y)
"""cumsum_sharded! with this rank's shard in HOST memory (pinned for asynchrony)."""
function cumsum_sharded_host!(c::Comm, y::Vector{Int64}, x::Vector{Int64})
    length(y) == length(x) || throw(DimensionMismatch("cumsum_sharded_host!"))
    GC.@preserve x y _ccheck(c, ccall((:ki_scan_inclusive_i64_sharded_host, libki), Cint,
                                      (Ptr{Cvoid}, Ptr{Int64}, Ptr{Int64}, Csize_t, Ptr{Cvoid}),
                                      c.handle, pointer(x), pointer(y), length(x), _stream()))
    CUDA.synchronize()
    return y
end
"""filter(>(t)) / findall(>(t)) over the concatenated Float32 shards; `first` is the 1-based global
index of this shard's first element.  Returns (vals, idx, offset, total): this rank's part belongs
at offset+1:offset+length(vals) of the global result."""
function findall_sharded(c::Comm, x::CuVector{Float32}, t::Real, first::Integer)
    n = length(x)
    vals = CuVector{Float32}(undef, n); idx = CuVector{Int32}(undef, n)
    w = CUDA.zeros(UInt64, 3)  # count, offset, total
    _ccheck(c, ccall((:ki_compact_gt_f32_sharded, libki), Cint,
                     (Ptr{Cvoid}, CuPtr{Float32}, Csize_t, Float32, CuPtr{Float32}, CuPtr{Int32}, Int64, CuPtr{UInt64},
                      CuPtr{UInt64}, CuPtr{UInt64}, Ptr{Cvoid}),
                     c.handle, x, n, Float32(t), vals, idx, first, pointer(w, 1), pointer(w, 2), pointer(w, 3), _stream()))
    k, off, tot = Int.(Array(w))
    return vals[1:k], idx[1:k], off, tot
end

end # module

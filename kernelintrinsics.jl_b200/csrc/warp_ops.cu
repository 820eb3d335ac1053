// warp_ops.cu -- the reference's per-thread intrinsics run over whole warps of an array, so that a
// host can check them against the reference's known answers: @shfl, @warpreduce, @warpfold, @vote,
// vload / vstore! and @access / @fence.  Element i of an array is lane i % 32 of warp i / 32.
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"

namespace {

constexpr int kThreads = 256;

template <int NW>
struct Words {
    uint32_t w[NW];
};

// ---- @shfl --------------------------------------------------------------------------------------
template <int NW>
__global__ void warp_shfl_kernel(int dir, const uint8_t* src, uint8_t* dst, size_t esz, size_t n, int arg) {
    const size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
    if (i >= n) return;  // n % 32 == 0: whole warps leave together
    Words<NW> v;
#pragma unroll
    for (int k = 0; k < NW; ++k) v.w[k] = 0;
    memcpy(&v, src + i * esz, esz);
    Words<NW> r;
    switch (dir) {
        case KI_SHFL_UP: r = ki::shfl<ki::Dir::Up>(v, arg); break;
        case KI_SHFL_DOWN: r = ki::shfl<ki::Dir::Down>(v, arg); break;
        case KI_SHFL_XOR: r = ki::shfl<ki::Dir::Xor>(v, arg); break;
        default: r = ki::shfl<ki::Dir::Idx>(v, arg); break;
    }
    memcpy(dst + i * esz, &r, esz);
}

template <int NW>
void launch_shfl(int dir, const void* s, void* d, size_t esz, size_t n, int arg, cudaStream_t st) {
    warp_shfl_kernel<NW><<<(unsigned)((n + kThreads - 1) / kThreads), kThreads, 0, st>>>(
        dir, (const uint8_t*)s, (uint8_t*)d, esz, n, arg);
}

// ---- @warpreduce / @warpfold ---------------------------------------------------------------------
template <class T, class Op>
__global__ void warp_scan_kernel(const T* src, T* dst, size_t n) {
    const size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
    if (i >= n) return;
    dst[i] = ki::warpreduce(src[i], Op{});
}

template <class T, class Op>
__global__ void warp_fold_kernel(const T* src, T* dst, size_t n, int form) {
    const size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
    if (i >= n) return;
    dst[i] = form ? ki::warpfold_down(src[i], Op{}) : ki::warpfold(src[i], Op{});
}

template <class T, class Op>
void launch_scan_fold(bool fold, int form, const void* s, void* d, size_t n, cudaStream_t st) {
    const unsigned g = (unsigned)((n + kThreads - 1) / kThreads);
    if (fold) warp_fold_kernel<T, Op><<<g, kThreads, 0, st>>>((const T*)s, (T*)d, n, form);
    else warp_scan_kernel<T, Op><<<g, kThreads, 0, st>>>((const T*)s, (T*)d, n);
}

template <class T>
int dispatch_op(int op, bool fold, int form, const void* s, void* d, size_t n, cudaStream_t st) {
    switch (op) {
        case KI_OP_ADD: launch_scan_fold<T, ki::Add>(fold, form, s, d, n, st); return KI_OK;
        case KI_OP_MAX: launch_scan_fold<T, ki::Max>(fold, form, s, d, n, st); return KI_OK;
        case KI_OP_MIN: launch_scan_fold<T, ki::Min>(fold, form, s, d, n, st); return KI_OK;
        default: break;
    }
    if constexpr (std::is_integral<T>::value) {
        switch (op) {
            case KI_OP_OR: launch_scan_fold<T, ki::BitOr>(fold, form, s, d, n, st); return KI_OK;
            case KI_OP_AND: launch_scan_fold<T, ki::BitAnd>(fold, form, s, d, n, st); return KI_OK;
            case KI_OP_XOR: launch_scan_fold<T, ki::BitXor>(fold, form, s, d, n, st); return KI_OK;
            default: break;
        }
    }
    return KI_ERR_ARG;
}

int dispatch_dtype(int dtype, int op, bool fold, int form, const void* s, void* d, size_t n, cudaStream_t st) {
    switch (dtype) {
        case KI_I8: return dispatch_op<int8_t>(op, fold, form, s, d, n, st);
        case KI_U8: return dispatch_op<uint8_t>(op, fold, form, s, d, n, st);
        case KI_I16: return dispatch_op<int16_t>(op, fold, form, s, d, n, st);
        case KI_U16: return dispatch_op<uint16_t>(op, fold, form, s, d, n, st);
        case KI_I32: return dispatch_op<int32_t>(op, fold, form, s, d, n, st);
        case KI_U32: return dispatch_op<uint32_t>(op, fold, form, s, d, n, st);
        case KI_I64: return dispatch_op<int64_t>(op, fold, form, s, d, n, st);
        case KI_U64: return dispatch_op<uint64_t>(op, fold, form, s, d, n, st);
        case KI_F32: return dispatch_op<float>(op, fold, form, s, d, n, st);
        case KI_F64: return dispatch_op<double>(op, fold, form, s, d, n, st);
        default: return KI_ERR_ARG;
    }
}

size_t dtype_size(int dtype) {
    switch (dtype) {
        case KI_I8: case KI_U8: return 1;
        case KI_I16: case KI_U16: return 2;
        case KI_I32: case KI_U32: case KI_F32: return 4;
        case KI_I64: case KI_U64: case KI_F64: return 8;
        default: return 0;
    }
}

// ---- @vote ----------------------------------------------------------------------------------------
__global__ void warp_vote_kernel(int mode, const uint8_t* pred, uint32_t* out, size_t n) {
    const size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
    if (i >= n) return;
    const bool p = pred[i] != 0;
    uint32_t r;
    switch (mode) {
        case KI_VOTE_ALL: r = ki::vote_all(p); break;
        case KI_VOTE_ANY: r = ki::vote_any(p); break;
        case KI_VOTE_UNI: r = ki::vote_uni(p); break;
        default: r = ki::ballot(p); break;
    }
    out[i] = r;
}

// ---- vload / vstore! -------------------------------------------------------------------------------
template <int B>
struct Elem {
    uint8_t b[B];
};
template <>
struct Elem<1> {
    uint8_t v;
};
template <>
struct Elem<2> {
    uint16_t v;
};
template <>
struct Elem<4> {
    uint32_t v;
};
template <>
struct Elem<8> {
    uint64_t v;
};
template <>
struct __align__(16) Elem<16> {
    uint4 v;
};

// Rebase: idx is a block index; the aligned batch access is taken when the pointer is a multiple of
// N elements (src/vectorization.jl:168-181), else vload_multi from element idx*N.
template <class T, int N>
__global__ void vload_kernel(const T* a, int64_t idx, int rebase, T* out) {
    T r[N];
    if (rebase) {
        const int64_t start = idx * N;
        if (((uintptr_t)a / sizeof(T)) % N == 0) ki::detail::ld_aligned<(int)(N * sizeof(T))>(a + start, r);
        else ki::vload_multi<T, N>(a, start, r);
    } else {
        ki::vload_multi<T, N>(a, idx, r);
    }
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = r[k];
}

template <class T, int N>
__global__ void vstore_kernel(T* a, int64_t idx, int rebase, const T* vals) {
    T r[N];
#pragma unroll
    for (int k = 0; k < N; ++k) r[k] = vals[k];
    if (rebase) {
        const int64_t start = idx * N;
        if (((uintptr_t)a / sizeof(T)) % N == 0) ki::detail::st_aligned<(int)(N * sizeof(T))>(a + start, r);
        else ki::vstore_multi<T, N>(a, start, r);
    } else {
        ki::vstore_multi<T, N>(a, idx, r);
    }
}

// Non power-of-two element sizes: the scalar tuple path (src/vectorization.jl:136-145,218-233).
__global__ void vscalar_kernel(const uint8_t* src, uint8_t* dst, size_t bytes) {
    for (size_t k = 0; k < bytes; ++k) dst[k] = src[k];
}

template <int B, int N>
void launch_vload(bool store, void* a, int64_t idx, int rebase, void* v, cudaStream_t s) {
    using T = Elem<B>;
    if (store) vstore_kernel<T, N><<<1, 1, 0, s>>>((T*)a, idx, rebase, (const T*)v);
    else vload_kernel<T, N><<<1, 1, 0, s>>>((const T*)a, idx, rebase, (T*)v);
}

template <int B>
int dispatch_vload_n(bool store, int nitem, void* a, int64_t idx, int rebase, void* v, cudaStream_t s) {
    switch (nitem) {
        case 1: launch_vload<B, 1>(store, a, idx, rebase, v, s); return KI_OK;
        case 2: launch_vload<B, 2>(store, a, idx, rebase, v, s); return KI_OK;
        case 4: launch_vload<B, 4>(store, a, idx, rebase, v, s); return KI_OK;
        case 8: launch_vload<B, 8>(store, a, idx, rebase, v, s); return KI_OK;
        case 16: launch_vload<B, 16>(store, a, idx, rebase, v, s); return KI_OK;
        default: return KI_ERR_ARG;
    }
}

int vload_vstore(ki_ctx* ctx, bool store, void* a, size_t esz, int64_t idx, int nitem, int rebase, void* v,
                 void* stream) {
    KI_CHECK_CTX(ctx);
    if (!a || !v || esz == 0 || idx < 0) return ki::set_error(ctx, KI_ERR_ARG, "vload/vstore: bad argument");
    if (nitem != 1 && nitem != 2 && nitem != 4 && nitem != 8 && nitem != 16)
        return ki::set_error(ctx, KI_ERR_ARG, "vload/vstore: nitem must be 1, 2, 4, 8 or 16");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    const bool pow2 = (esz & (esz - 1)) == 0 && esz <= 16;
    if (!pow2) {
        const int64_t start = rebase ? idx * nitem : idx;
        uint8_t* base = (uint8_t*)a + (size_t)start * esz;
        if (store) vscalar_kernel<<<1, 1, 0, s>>>((const uint8_t*)v, base, esz * nitem);
        else vscalar_kernel<<<1, 1, 0, s>>>(base, (uint8_t*)v, esz * nitem);
        return ki::check_launch(ctx, "vscalar_kernel");
    }
    if (!ki::aligned(a, esz)) return ki::set_error(ctx, KI_ERR_ARG, "vload/vstore: element-misaligned array");
    int rc;
    switch (esz) {
        case 1: rc = dispatch_vload_n<1>(store, nitem, a, idx, rebase, v, s); break;
        case 2: rc = dispatch_vload_n<2>(store, nitem, a, idx, rebase, v, s); break;
        case 4: rc = dispatch_vload_n<4>(store, nitem, a, idx, rebase, v, s); break;
        case 8: rc = dispatch_vload_n<8>(store, nitem, a, idx, rebase, v, s); break;
        default: rc = dispatch_vload_n<16>(store, nitem, a, idx, rebase, v, s); break;
    }
    if (rc) return ki::set_error(ctx, rc, "vload/vstore: unsupported shape");
    return ki::check_launch(ctx, "vload/vstore kernel");
}

// ---- @access / @fence ---------------------------------------------------------------------------------
using ki::Order;
using ki::Scope;

template <class T>
__device__ void do_store(T* p, T v, int scope, int order) {
    if (order == KI_ORDER_WEAK) ki::store<Order::Weak>(p, v);
    else if (order == KI_ORDER_VOLATILE) ki::store<Order::Volatile>(p, v);
    else if (order == KI_ORDER_RELAXED) {
        if (scope == KI_SCOPE_WORKGROUP) ki::store<Order::Relaxed, Scope::Workgroup>(p, v);
        else if (scope == KI_SCOPE_SYSTEM) ki::store<Order::Relaxed, Scope::System>(p, v);
        else ki::store<Order::Relaxed, Scope::Device>(p, v);
    } else {
        if (scope == KI_SCOPE_WORKGROUP) ki::store<Order::Release, Scope::Workgroup>(p, v);
        else if (scope == KI_SCOPE_SYSTEM) ki::store<Order::Release, Scope::System>(p, v);
        else ki::store<Order::Release, Scope::Device>(p, v);
    }
}

template <class T>
__device__ T do_load(const T* p, int scope, int order) {
    if (order == KI_ORDER_WEAK) return ki::load<Order::Weak>(p);
    if (order == KI_ORDER_VOLATILE) return ki::load<Order::Volatile>(p);
    if (order == KI_ORDER_RELAXED) {
        if (scope == KI_SCOPE_WORKGROUP) return ki::load<Order::Relaxed, Scope::Workgroup>(p);
        if (scope == KI_SCOPE_SYSTEM) return ki::load<Order::Relaxed, Scope::System>(p);
        return ki::load<Order::Relaxed, Scope::Device>(p);
    }
    if (scope == KI_SCOPE_WORKGROUP) return ki::load<Order::Acquire, Scope::Workgroup>(p);
    if (scope == KI_SCOPE_SYSTEM) return ki::load<Order::Acquire, Scope::System>(p);
    return ki::load<Order::Acquire, Scope::Device>(p);
}

__device__ void do_fence(int scope, int order) {
    const bool sc = (order == KI_ORDER_SEQCST);
    if (scope == KI_SCOPE_WORKGROUP) {
        if (sc) ki::fence<Scope::Workgroup, Order::SeqCst>();
        else ki::fence<Scope::Workgroup, Order::AcqRel>();
    } else if (scope == KI_SCOPE_SYSTEM) {
        if (sc) ki::fence<Scope::System, Order::SeqCst>();
        else ki::fence<Scope::System, Order::AcqRel>();
    } else {
        if (sc) ki::fence<Scope::Device, Order::SeqCst>();
        else ki::fence<Scope::Device, Order::AcqRel>();
    }
}

template <class T>
__global__ void access_kernel(int scope, int so, int lo, int fs, int fo, T* slot, const T* value, T* readback) {
    do_store<T>(slot, *value, scope, so);
    do_fence(fs, fo);
    *readback = do_load<T>(slot, scope, lo);
}

template <class T>
void launch_access(int scope, int so, int lo, int fs, int fo, void* slot, const void* value, void* rb,
                   cudaStream_t s) {
    access_kernel<T><<<1, 1, 0, s>>>(scope, so, lo, fs, fo, (T*)slot, (const T*)value, (T*)rb);
}

// ---- release / acquire message passing with bounded waits ------------------------------------------
__global__ void message_pass_kernel(int64_t* data, uint32_t* flag, int64_t* seen, int64_t payload, int produce,
                                    uint64_t timeout_ns, uint32_t* status) {
    if (threadIdx.x != 0) return;
    if (blockIdx.x == 0) {
        if (produce) {
            data[0] = payload;                                        // plain store
            ki::store<Order::Release, Scope::Device>(flag, 1u);       // @access Flag[1] = 1
        }
        return;
    }
    const uint64_t t0 = ki::globaltimer_ns();
    bool ok = true;
    while (ki::load<Order::Acquire, Scope::Device>(flag) != 1u) {   // @access Acquire Flag[1]
        if (ki::globaltimer_ns() - t0 > timeout_ns) {
            ok = false;
            break;
        }
        __nanosleep(100);
    }
    if (ok) {
        seen[blockIdx.x] = data[0];
    } else {
        seen[blockIdx.x] = -1;
        atomicOr(status, (uint32_t)KI_DEV_TIMEOUT);
    }
}

}  // namespace

extern "C" {

int ki_warp_shfl(ki_ctx* ctx, int dir, const void* d_src, void* d_dst, size_t elem_bytes, size_t n, int src,
                 void* stream) {
    KI_CHECK_CTX(ctx);
    if (dir < KI_SHFL_UP || dir > KI_SHFL_IDX) return ki::set_error(ctx, KI_ERR_ARG, "shfl: bad direction");
    if (elem_bytes == 0 || elem_bytes > 64) return ki::set_error(ctx, KI_ERR_ARG, "shfl: element size 1..64");
    if (n % 32) return ki::set_error(ctx, KI_ERR_ARG, "shfl: n must be a multiple of 32");
    if (n == 0) return KI_OK;
    if (!d_src || !d_dst) return ki::set_error(ctx, KI_ERR_ARG, "shfl: null pointer");
    if (dir == KI_SHFL_IDX && (src < 0 || src > 31)) return ki::set_error(ctx, KI_ERR_ARG, "shfl: lane 0..31");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    const int nw = (int)((elem_bytes + 3) / 4);
    if (nw <= 1) launch_shfl<1>(dir, d_src, d_dst, elem_bytes, n, src, s);
    else if (nw == 2) launch_shfl<2>(dir, d_src, d_dst, elem_bytes, n, src, s);
    else if (nw <= 4) launch_shfl<4>(dir, d_src, d_dst, elem_bytes, n, src, s);
    else if (nw <= 8) launch_shfl<8>(dir, d_src, d_dst, elem_bytes, n, src, s);
    else launch_shfl<16>(dir, d_src, d_dst, elem_bytes, n, src, s);
    return ki::check_launch(ctx, "warp_shfl_kernel");
}

int ki_warp_reduce(ki_ctx* ctx, int op, int dtype, const void* d_src, void* d_dst, size_t n, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n % 32) return ki::set_error(ctx, KI_ERR_ARG, "warpreduce: n must be a multiple of 32");
    if (n == 0) return KI_OK;
    if (!d_src || !d_dst || dtype_size(dtype) == 0) return ki::set_error(ctx, KI_ERR_ARG, "warpreduce: bad argument");
    KI_GUARD(ctx);
    int rc = dispatch_dtype(dtype, op, false, 0, d_src, d_dst, n, ki::as_stream(stream));
    if (rc) return ki::set_error(ctx, rc, "warpreduce: unsupported op/dtype");
    return ki::check_launch(ctx, "warp_scan_kernel");
}

int ki_warp_fold(ki_ctx* ctx, int op, int dtype, int form, const void* d_src, void* d_dst, size_t n, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n % 32) return ki::set_error(ctx, KI_ERR_ARG, "warpfold: n must be a multiple of 32");
    if (form != 0 && form != 1) return ki::set_error(ctx, KI_ERR_ARG, "warpfold: form 0 (xor) or 1 (down)");
    if (n == 0) return KI_OK;
    if (!d_src || !d_dst || dtype_size(dtype) == 0) return ki::set_error(ctx, KI_ERR_ARG, "warpfold: bad argument");
    KI_GUARD(ctx);
    int rc = dispatch_dtype(dtype, op, true, form, d_src, d_dst, n, ki::as_stream(stream));
    if (rc) return ki::set_error(ctx, rc, "warpfold: unsupported op/dtype");
    return ki::check_launch(ctx, "warp_fold_kernel");
}

int ki_warp_vote(ki_ctx* ctx, int mode, const uint8_t* d_pred, uint32_t* d_out, size_t n, void* stream) {
    KI_CHECK_CTX(ctx);
    if (mode < KI_VOTE_ALL || mode > KI_VOTE_BALLOT) return ki::set_error(ctx, KI_ERR_ARG, "vote: bad mode");
    if (n % 32) return ki::set_error(ctx, KI_ERR_ARG, "vote: n must be a multiple of 32");
    if (n == 0) return KI_OK;
    if (!d_pred || !d_out) return ki::set_error(ctx, KI_ERR_ARG, "vote: null pointer");
    KI_GUARD(ctx);
    warp_vote_kernel<<<(unsigned)((n + kThreads - 1) / kThreads), kThreads, 0, ki::as_stream(stream)>>>(mode, d_pred,
                                                                                                   d_out, n);
    return ki::check_launch(ctx, "warp_vote_kernel");
}

int ki_vload(ki_ctx* ctx, const void* d_a, size_t elem_bytes, int64_t idx, int nitem, int rebase, void* d_out,
             void* stream) {
    return vload_vstore(ctx, false, const_cast<void*>(d_a), elem_bytes, idx, nitem, rebase, d_out, stream);
}

int ki_vstore(ki_ctx* ctx, void* d_a, size_t elem_bytes, int64_t idx, int nitem, int rebase, const void* d_values,
              void* stream) {
    return vload_vstore(ctx, true, d_a, elem_bytes, idx, nitem, rebase, const_cast<void*>(d_values), stream);
}

int ki_access_roundtrip(ki_ctx* ctx, int dtype, int scope, int store_order, int load_order, int fence_scope,
                        int fence_order, void* d_slot, const void* d_value, void* d_readback, void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_slot || !d_value || !d_readback || dtype_size(dtype) == 0)
        return ki::set_error(ctx, KI_ERR_ARG, "access: bad argument");
    if (scope < KI_SCOPE_DEFAULT || scope > KI_SCOPE_SYSTEM || fence_scope < KI_SCOPE_DEFAULT ||
        fence_scope > KI_SCOPE_SYSTEM)
        return ki::set_error(ctx, KI_ERR_ARG, "access: bad scope");
    // Validation of src/macros.jl:203-207 and :217-233.
    auto scopeless = [](int o) { return o == KI_ORDER_WEAK || o == KI_ORDER_VOLATILE; };
    if (store_order == KI_ORDER_DEFAULT) store_order = KI_ORDER_RELEASE;
    if (load_order == KI_ORDER_DEFAULT) load_order = KI_ORDER_ACQUIRE;
    if (fence_order == KI_ORDER_DEFAULT) fence_order = KI_ORDER_ACQREL;
    if (store_order == KI_ORDER_ACQREL || store_order == KI_ORDER_SEQCST || load_order == KI_ORDER_ACQREL ||
        load_order == KI_ORDER_SEQCST)
        return ki::set_error(ctx, KI_ERR_ARG,
                             "AcqRel and SeqCst are not valid orderings for loads and stores; use @fence instead.");
    if (store_order == KI_ORDER_ACQUIRE || load_order == KI_ORDER_RELEASE)
        return ki::set_error(ctx, KI_ERR_ARG, "Acquire is a load ordering and Release a store ordering.");
    if (scope != KI_SCOPE_DEFAULT && (scopeless(store_order) || scopeless(load_order)))
        return ki::set_error(ctx, KI_ERR_ARG, "Cannot specify a scope with Weak or Volatile ordering.");
    if (fence_order == KI_ORDER_WEAK || fence_order == KI_ORDER_VOLATILE || fence_order == KI_ORDER_RELAXED)
        return ki::set_error(ctx, KI_ERR_ARG,
                             "Fences allows synchronizing orderings: Acquire, Release, AcqRel, or SeqCst.");
    if (!ki::aligned(d_slot, dtype_size(dtype))) return ki::set_error(ctx, KI_ERR_ARG, "access: misaligned slot");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    const int sc = scope, so = store_order, lo = load_order, fs = fence_scope, fo = fence_order;
    switch (dtype) {
        case KI_I8: launch_access<int8_t>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        case KI_U8: launch_access<uint8_t>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        case KI_I16: launch_access<int16_t>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        case KI_U16: launch_access<uint16_t>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        case KI_I32: launch_access<int32_t>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        case KI_U32: launch_access<uint32_t>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        case KI_I64: launch_access<int64_t>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        case KI_U64: launch_access<uint64_t>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        case KI_F32: launch_access<float>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
        default: launch_access<double>(sc, so, lo, fs, fo, d_slot, d_value, d_readback, s); break;
    }
    return ki::check_launch(ctx, "access_kernel");
}

int ki_flag_message_pass(ki_ctx* ctx, int64_t* d_data, uint32_t* d_flag, int64_t* d_seen, int nblocks,
                         int64_t payload, int produce, uint64_t timeout_ns, void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_data || !d_flag || !d_seen || nblocks < 2 || nblocks > ctx->sm_count || timeout_ns == 0)
        return ki::set_error(ctx, KI_ERR_ARG, "message_pass: bad argument (2 <= nblocks <= SM count)");
    KI_GUARD(ctx);
    message_pass_kernel<<<nblocks, 32, 0, ki::as_stream(stream)>>>(d_data, d_flag, d_seen, payload, produce,
                                                                  timeout_ns, ctx->d_status);
    return ki::check_launch(ctx, "message_pass_kernel");
}

}  // extern "C"

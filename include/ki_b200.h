/*
 * ki_b200.h -- C ABI of libki_b200.so: device-wide primitives for NVIDIA B200 (sm_100a) with the
 * semantics of epilliat/KernelIntrinsics.jl v0.1.6 and the Julia Base operations its intrinsics
 * are used to build.
 *
 * Conventions
 *   - Every pointer argument named d_* or documented as "device" is a device pointer on the
 *     context's device; sizes are in elements unless the name says bytes.
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream).  All calls are
 *     stream-ordered and asynchronous; none synchronises unless documented.
 *   - Every call returns a ki_status.  Errors detected on the device (a bounded wait that ran out)
 *     are latched in a device status word and reported by ki_ctx_check().
 *   - No C++ exception crosses this boundary.  No call allocates after the context's scratch has
 *     grown to the largest problem seen (scratch grows on first use of a size).
 *   - One context per (device, host thread).  Calls of the same operation through one context
 *     must be ordered on one stream; they share that operation's scratch.
 *
 * Reference interfaces replaced (file:line in the reference project):
 *   the reference's plugin boundary is a set of Julia stubs that each GPU backend overrides
 *   (src/scopes_orderings.jl:151-154, src/warp.jl:111-112, src/vectorization.jl:426-448,
 *   src/KernelIntrinsics.jl:19-21; CUDA overrides in the ext/CUDA directory).  Those run per thread inside a
 *   user kernel; this ABI exposes the device-wide operations built from them, plus one entry per
 *   intrinsic family that runs it over whole warps of an array so hosts can test it.
 */
#ifndef KI_B200_H
#define KI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ki_ctx ki_ctx;

typedef enum ki_status {
    KI_OK = 0,
    KI_ERR_ARG = 1,         /* invalid argument (the reference raises ArgumentError) */
    KI_ERR_CUDA = 2,        /* a CUDA runtime call failed; see ki_last_error_string */
    KI_ERR_TIMEOUT = 3,     /* a bounded device-side wait ran out (lookback flag, mbarrier) */
    KI_ERR_UNSUPPORTED = 4, /* device is not sm_100 / feature not available */
    KI_ERR_NOMEM = 5,       /* scratch allocation failed */
    KI_ERR_NCCL = 6         /* an NCCL call of a communicator failed; see ki_last_error_string */
} ki_status;

/* Scopes and orderings: src/scopes_orderings.jl:13-120 (Workgroup/Device/System;
 * Weak/Volatile/Relaxed/Acquire/Release/AcqRel/SeqCst). */
typedef enum { KI_SCOPE_DEFAULT = 0, KI_SCOPE_WORKGROUP = 1, KI_SCOPE_DEVICE = 2, KI_SCOPE_SYSTEM = 3 } ki_scope;
typedef enum {
    KI_ORDER_DEFAULT = 0,
    KI_ORDER_WEAK = 1,
    KI_ORDER_VOLATILE = 2,
    KI_ORDER_RELAXED = 3,
    KI_ORDER_ACQUIRE = 4,
    KI_ORDER_RELEASE = 5,
    KI_ORDER_ACQREL = 6,
    KI_ORDER_SEQCST = 7
} ki_order;

/* Shuffle directions (src/warp.jl:16-64) and vote modes (src/warp.jl:66-106). */
typedef enum { KI_SHFL_UP = 0, KI_SHFL_DOWN = 1, KI_SHFL_XOR = 2, KI_SHFL_IDX = 3 } ki_dir;
typedef enum { KI_VOTE_ALL = 0, KI_VOTE_ANY = 1, KI_VOTE_UNI = 2, KI_VOTE_BALLOT = 3 } ki_mode;

/* Element types and binary operators (warp-level and device-wide entry points). */
typedef enum {
    KI_I8 = 0, KI_U8 = 1, KI_I16 = 2, KI_U16 = 3, KI_I32 = 4, KI_U32 = 5,
    KI_I64 = 6, KI_U64 = 7, KI_F32 = 8, KI_F64 = 9
} ki_dtype;
typedef enum {
    KI_OP_ADD = 0, KI_OP_MAX = 1, KI_OP_MIN = 2, KI_OP_OR = 3, KI_OP_AND = 4, KI_OP_XOR = 5, KI_OP_MUL = 6
} ki_op;

/* ---- library / context ------------------------------------------------------------------- */

int ki_version(void);
const char* ki_status_string(int status);

/* Device queries (src/device.jl:1-19, ext/CUDA/device.jl:4-13, get_warpsize
 * src/KernelIntrinsics.jl:19).  Devices are 0-based here; the Julia/Python mirrors are 1-based. */
int ki_device_count(int* count);
int ki_device_info(int device, int* sm_count, int* warp_size, int* cc_major, int* cc_minor);

int ki_ctx_create(int device, ki_ctx** out);
int ki_ctx_destroy(ki_ctx* ctx);
/* Message of the context's last error; with ctx = NULL, of the calling thread's last failed call that
 * had no context to hold it (a communicator whose set-up failed). */
const char* ki_last_error_string(const ki_ctx* ctx);
/* Synchronises `stream`, returns KI_ERR_TIMEOUT if any device-side wait of this context ran out
 * since the last check (and clears the latch), KI_ERR_CUDA on an asynchronous CUDA error. */
int ki_ctx_check(ki_ctx* ctx, void* stream);
/* Limit of every device-side wait of this context (default 2 s). */
int ki_ctx_set_wait_timeout_ns(ki_ctx* ctx, uint64_t ns);

/* ---- (a1/a2) vectorised copy: vload_multi / vstore_multi! over a whole range --------------
 * Replaces: src/vectorization.jl:306-420 (patterns, vload_multi, vstore_multi!),
 * ext/CUDA/vectorization.jl:5-27 (_vload_batch, _vstore_batch!, _vload_norebase, _vstore_norebase!).
 * Semantics of copyto!(dst, src) on nbytes bytes; any byte alignment of dst and src.
 * dst and src must not overlap (KI_ERR_ARG). */
int ki_vcopy(ki_ctx* ctx, void* dst, const void* src, size_t nbytes, void* stream);
/* copyto! between two HOST buffers through the device: the bytes cross to the device in chunks,
 * are copied there by the same kernel as ki_vcopy and come back, with both copy directions and the
 * kernel overlapped (chunks cycle over device staging slots owned by the context).  Asynchronous
 * with respect to the host when both buffers are page-locked (cudaHostAlloc / cudaHostRegister);
 * the copy is complete when `stream` is.  dst and src must not overlap (KI_ERR_ARG).  Not
 * re-entrant on one context: two calls in flight on different streams share the staging slots. */
int ki_vcopy_host(ki_ctx* ctx, void* dst, const void* src, size_t nbytes, void* stream);

/* ---- strided copies: copyto! between strided views ------------------------------------------
 * Replaces: the AbstractArray fallbacks of vload / vstore! (src/vectorization.jl:202-211, 290-297;
 * _vload_batch / _vstore_batch!, :426-448), which move a strided view element by element.
 * ki_vcopy_2d: height rows of width bytes; row r goes from src + r*spitch to dst + r*dpitch (bytes).
 * Any byte alignment and any pitch >= width (a block of a column-major array: one row per column).
 * The two ranges must not overlap (KI_ERR_ARG).  width or height 0: nothing to do. */
int ki_vcopy_2d(ki_ctx* ctx, void* dst, size_t dpitch, const void* src, size_t spitch, size_t width_bytes,
                size_t height, void* stream);
/* ki_vcopy_strided: dst[i*dst_stride] = src[i*src_stride] for i < count, elements of elem_bytes
 * (1 to 65536: plain types and structs of any size, e.g. 12-byte structs, which the reference moves
 * field by field) with strides in elements of either sign (view(x, n:-2:1)); both pointers aligned
 * to the largest power of two (at most 16) that divides elem_bytes; src_stride 0 broadcasts one
 * element; the ranges must not overlap. */
int ki_vcopy_strided(ki_ctx* ctx, void* dst, int64_t dst_stride, const void* src, int64_t src_stride,
                     size_t elem_bytes, size_t count, void* stream);

/* ---- (a3) grid-wide reduce (@warpfold, src/warp.jl:273-282) ---------------------------------
 * sum(x) of n Float32 values, accumulated in Float64 across threads; writes the Float32 result to
 * d_out_f32 and/or the Float64 result to d_out_f64 (either may be NULL, not both).  n == 0 gives 0.
 * Deterministic: the same n and device give the same bits on every call. */
int ki_reduce_sum_f32(ki_ctx* ctx, const float* d_x, size_t n, float* d_out_f32, double* d_out_f64,
                      void* stream);
/* sum of Int64 with two's-complement wrap-around (the shard total of the sharded scan). */
int ki_reduce_sum_i64(ki_ctx* ctx, const int64_t* d_x, size_t n, int64_t* d_out, void* stream);
/* Device-wide reduce for any of the reference's fold operators that Base names (@warpfold takes any
 * op, src/warp.jl:273-282; the device-wide result is Base.sum / prod / maximum / minimum /
 * reduce(|, &, xor)).  op: KI_OP_ADD, KI_OP_MUL, KI_OP_MAX, KI_OP_MIN, KI_OP_OR, KI_OP_AND, KI_OP_XOR;
 * dtype: KI_I8 ... KI_U64, KI_F32, KI_F64 (the bitwise operators take integers only).
 * d_out receives one value of the result type: for KI_OP_ADD and KI_OP_MUL integers narrower than
 * 64 bits widen to Int64 / UInt64 (Base.add_sum, Base.mul_prod), 64-bit integers wrap, Float32 stays
 * Float32 (accumulated in Float64), Float64 stays Float64; for the other operators the input type
 * (KI_OP_MAX / KI_OP_MIN: NaN propagates, +0.0 > -0.0, as Base.max / Base.min).  n = 0: KI_OP_ADD
 * writes zero, KI_OP_MUL one, the others return KI_ERR_ARG (Base throws on an empty maximum).
 * Deterministic for a given n and device. */
int ki_reduce(ki_ctx* ctx, int op, int dtype, const void* d_x, size_t n, void* d_out, void* stream);
/* Element maps applied before a fold or a predicate, in the element type as Base computes them
 * (abs(typemin(Int8)) == typemin(Int8); abs2 wraps on integers; abs is the identity on unsigned). */
typedef enum { KI_MAP_IDENTITY = 0, KI_MAP_ABS = 1, KI_MAP_ABS2 = 2 } ki_map;
/* mapreduce(f, op, x): Base.sum(abs2, x), maximum(abs, x) and the like.  With KI_MAP_IDENTITY it is
 * ki_reduce; with KI_MAP_ABS or KI_MAP_ABS2 op is KI_OP_ADD, KI_OP_MAX or KI_OP_MIN, the result type
 * that of ki_reduce for (op, dtype), and the map runs in the element type before the widening. */
int ki_mapreduce(ki_ctx* ctx, int map, int op, int dtype, const void* d_x, size_t n, void* d_out, void* stream);
/* Segmented reduce: one ki_reduce per row of a row-major rows x cols matrix whose rows start ld
 * elements apart (ld >= cols; a column-major Julia matrix reduced along dims=1 has rows = its
 * columns).  d_out receives rows values of ki_reduce's result type.  cols = 0: KI_OP_ADD writes
 * zeros, KI_OP_MUL ones, the others return KI_ERR_ARG.  Deterministic for a given shape and device. */
int ki_reduce_rows(ki_ctx* ctx, int op, int dtype, const void* d_x, size_t rows, size_t cols, size_t ld,
                   void* d_out, void* stream);

/* ---- (a4/a5) single-pass decoupled-lookback inclusive scan ----------------------------------
 * Replaces: @warpreduce (src/warp.jl:226-237) for the in-warp scan, @access / @fence
 * (src/macros.jl:198-282, ext/CUDA/scopes_ordering.jl:89-193) for the tile flags.
 * out[i] = seed + in[0] + ... + in[i] with Int64 wrap-around (Base.cumsum; seed = 0).
 * in == out is allowed (in place).  Tile flags use st.release.gpu / ld.acquire.gpu; waits are
 * bounded by the context's timeout. */
int ki_scan_inclusive_i64(ki_ctx* ctx, const int64_t* d_in, int64_t* d_out, size_t n, int64_t seed,
                          void* stream);
/* The same scan with its seed read from device memory (*d_seed, one Int64) when the kernel starts, so
 * a seed computed on the device (a sum of other shards' totals, the last value of a previous chunk)
 * needs no round trip through the host. */
int ki_scan_inclusive_i64_dseed(ki_ctx* ctx, const int64_t* d_in, int64_t* d_out, size_t n, const int64_t* d_seed,
                                void* stream);
/* cumsum of HOST buffers through the device (Base.cumsum of an Array): 16 MiB chunks cross to the
 * device, are scanned there (each chunk seeded on the device with the previous chunk's last value)
 * and come back, both copy directions and the scans overlapped over staging slots owned by the
 * context (the pipeline of ki_vcopy_host; the two are not re-entrant on one context).  Asynchronous
 * with respect to the host when both buffers are page-locked; complete when `stream` is.  h_in ==
 * h_out is allowed; other overlaps return KI_ERR_ARG. */
int ki_scan_inclusive_i64_host(ki_ctx* ctx, const int64_t* h_in, int64_t* h_out, size_t n, int64_t seed,
                               void* stream);
/* Device-wide scan for any of those operators and types (@warpreduce takes any op,
 * src/warp.jl:226-237; the device-wide result is Base.cumsum / accumulate(op, x; init)).
 * op, dtype and the result type as for ki_reduce; d_out holds n values of the result type.
 * exclusive = 0: out[i] = op(init, in[0], ..., in[i]); exclusive != 0: out[i] = op(init, in[0], ...,
 * in[i-1]), out[0] = init.  h_init: host pointer to one value of the result type, or NULL for the
 * operator's identity (0 for + | xor, 1 for *, all ones for &, the lowest value for max, the highest
 * for min).  in == out is allowed when the input
 * and result types have the same size; other overlaps return KI_ERR_ARG.  Float sums accumulate in
 * Float64 (within 1e-5*log2(n) of a Float64 scan), Float32 products too.  Int64 + with a seed is
 * ki_scan_inclusive_i64. */
int ki_scan(ki_ctx* ctx, int op, int dtype, int exclusive, const void* d_in, void* d_out, size_t n,
            const void* h_init, void* stream);
/* Segmented scan: one ki_scan per row of a rows x cols row-major matrix, every row starting from
 * h_init (Base.accumulate(op, A; dims) along the contiguous dimension: cumsum(A; dims=1) of a
 * column-major Julia matrix has rows = its columns).  Row r is read at d_in + r*ld_in and written at
 * d_out + r*ld_out (elements of the input and of the result type; ld >= cols when rows > 1).
 * Operators, types, result types and exclusive as ki_scan; in place when the input and result
 * types have the same size and ld_in == ld_out. */
int ki_scan_rows(ki_ctx* ctx, int op, int dtype, int exclusive, const void* d_in, size_t ld_in, void* d_out,
                 size_t ld_out, size_t rows, size_t cols, const void* h_init, void* stream);

/* Allocation-free scan.  No counterpart in the reference.
 * For callers that cannot allocate device memory: hosts whose device memory belongs to another
 * allocator (a pool that must not be bypassed or grown), loops that forbid allocation after
 * start-up, code that must not stall the device as cudaMalloc may.  Same result as ki_scan_inclusive_i64, but needs no context and calls no cudaMalloc,
 * cudaFree or allocating routine: its tile-status scratch is a static device array sized for
 * n <= KI_SCAN_NOALLOC_MAX_N (about 400 KiB, held by every GPU that loads the library until exit).
 * n beyond that returns KI_ERR_ARG.  Uses the calling thread's current device and CUDA context.  The
 * first call in each CUDA context (each device's primary context, a context re-created after
 * cudaDeviceReset, any other context) runs a one-time set-up: cudaGetSymbolAddress of the array
 * (which also loads the module under lazy loading), cudaDeviceGetAttribute (SM count) and
 * cudaFuncSetAttribute (shared memory); make that first call before any stream capture.  Every call
 * reads the current context's ID (cudaSetDevice binds the primary context first if none is
 * current).  Every call shares the array, which keeps the last call's contents (each
 * call clears its tile flags first); calls that overlap on the GPU race.  A bounded wait that runs
 * out is not reported (use the context API where that matters). */
#define KI_SCAN_NOALLOC_MAX_N (1ull << 28)
int ki_scan_inclusive_i64_noalloc(const int64_t* d_in, int64_t* d_out, size_t n, int64_t seed, void* stream);

/* ---- (a6) order-preserving stream compaction (@vote Ballot, ext/CUDA/shuffle_vote.jl:23-34) --
 * Keeps x[i] > threshold in order: out_vals[j] = x[i_j], out_idx[j] = i_j + index_base (Int32;
 * index_base = 1 gives findall's 1-based indices).  *d_count (device, uint64) receives the count.
 * out_vals and out_idx must hold n entries (either may be NULL).  Requires
 * index_base + n - 1 <= INT32_MAX and index_base >= INT32_MIN. */
int ki_compact_gt_f32(ki_ctx* ctx, const float* d_x, size_t n, float threshold, float* d_out_vals,
                      int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, void* stream);
/* Compaction for any comparison predicate and element type (the same @vote Ballot pipeline):
 * filter(v -> v op t, x) and findall(v -> v op t, x) with op one of ki_pred, IEEE comparisons for
 * floats (a NaN is never kept except by KI_PRED_NE), dtype KI_I32, KI_U32, KI_I64, KI_U64, KI_F32 or
 * KI_F64, h_thr a host pointer to one value of dtype; d_out_vals holds values of dtype, d_out_idx
 * Int32 indices starting at index_base; either output may be NULL. */
typedef enum { KI_PRED_GT = 0, KI_PRED_GE = 1, KI_PRED_LT = 2, KI_PRED_LE = 3, KI_PRED_EQ = 4, KI_PRED_NE = 5 } ki_pred;
int ki_compact(ki_ctx* ctx, int pred, int dtype, const void* d_x, size_t n, const void* h_thr, void* d_out_vals,
               int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, void* stream);
/* Fused map-then-compact: keeps x[i] with map(x[i]) pred threshold (filter(v -> abs(v) > t, x) and
 * its findall); the kept elements are written as they are, not mapped.  map: a ki_map (with
 * KI_MAP_IDENTITY it is ki_compact); the threshold is compared with the mapped value in the element
 * type.  Null d_out_vals and d_out_idx give count(v -> map(v) pred t, x) in d_count. */
int ki_compact_map(ki_ctx* ctx, int map, int pred, int dtype, const void* d_x, size_t n, const void* h_thr,
                   void* d_out_vals, int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, void* stream);

/* ---- (e) several GPUs: communicators and range-sharded operations ---------------------------
 * Replaces: device enumeration and selection (src/device.jl:1-19, ext/CUDA/device.jl:4-13) and the
 * System scope of @access / @fence (ext/CUDA/scopes_ordering.jl:13), from which the reference's users
 * build multi-GPU code.  A communicator ties one rank to one GPU.  Rank r owns a contiguous shard of
 * the global array (ki_comm_shard_range gives the default split); the sharded operations below are
 * collective: every rank calls the same operations in the same order, each on its own shard, and
 * the calls of one communicator are ordered on one stream.  Only one 8-byte value per rank crosses
 * between the GPUs per operation, pushed into every peer's exchange buffer with plain peer stores
 * (st.release.sys) and awaited with bounded ld.acquire.sys loads by a one-warp exchange kernel on
 * the caller's stream; no host round trip.  A wait that runs out latches KI_ERR_TIMEOUT in the communicator's
 * context (ki_comm_get_ctx + ki_ctx_check); the communicator is then unusable: ki_comm_abort it.
 * Ranks must be on distinct GPUs (two ranks on one GPU would wait on one another). */
typedef struct ki_comm ki_comm;
#define KI_COMM_MAX_RANKS 64
typedef struct { char internal[128]; } ki_comm_id;  /* an ncclUniqueId */
typedef enum { KI_XCHG_AUTO = 0, KI_XCHG_PEER = 1, KI_XCHG_NCCL = 2 } ki_exchange;
/* Contiguous shard [*lo, *lo + *count) of rank `rank` of n elements: the first n % nranks ranks hold
 * one element more.  Host only. */
int ki_comm_shard_range(size_t n, int nranks, int rank, size_t* lo, size_t* count);
/* The split that gives every rank of ki_scan_inclusive_i64_sharded the same bytes to move: ranks
 * below the last read their shard twice (phase 1 sum, phase 2 scan: 24 B per element) and the last
 * rank once (its total is never needed: 16 B per element), so the last rank gets 3/2 of a share;
 * boundaries at n*2r/(2*nranks + 1) rounded down to a multiple of 256 elements.  Host only. */
int ki_comm_scan_shard_range(size_t n, int nranks, int rank, size_t* lo, size_t* count);
/* One process (or host thread) per GPU: one rank calls ki_comm_get_id and hands the id to the others
 * (any host channel), then every rank calls ki_comm_init_rank with its own device (0-based) and rank.
 * NCCL (libnccl.so.2, loaded at run time) exchanges the ranks' buffer handles once; with
 * KI_XCHG_AUTO or KI_XCHG_PEER the operations then run on peer memory without NCCL, with
 * KI_XCHG_NCCL (or KI_XCHG_AUTO when peer mappings fail) each exchange is an ncclAllGather of the
 * 8-byte values on the caller's stream.  Set-up and tear-down waits are bounded on the host (120 s);
 * on timeout the NCCL communicator is aborted and KI_ERR_TIMEOUT returned.  KI_ERR_UNSUPPORTED: no
 * NCCL library, or two ranks on one GPU. */
int ki_comm_get_id(ki_comm_id* id);
int ki_comm_init_rank(int device, int nranks, int rank, const ki_comm_id* id, int exchange, ki_comm** out);
/* One host thread driving ndev GPUs (devs: distinct 0-based devices, all peer-capable, else
 * KI_ERR_UNSUPPORTED): comms[i] is rank i on devs[i].  No NCCL.  Issue each operation on every rank
 * before the next operation (operation-major) and before waiting on any of them: a rank's first
 * call of an operation allocates that operation's scratch, and a device allocation may wait for the
 * GPU's pending work, which includes an exchange that only completes once every rank has issued it. */
int ki_comm_create(int ndev, const int* devs, ki_comm** comms);
/* Collective for communicators from ki_comm_init_rank (a bounded barrier, then unmap and free);
 * for ki_comm_create's, destroy every rank's communicator once all their work is complete. */
int ki_comm_destroy(ki_comm* comm);
/* Local tear-down without the barrier, for a communicator whose peers failed or left. */
int ki_comm_abort(ki_comm* comm);
int ki_comm_info(const ki_comm* comm, int* nranks, int* rank, int* device, int* exchange);
/* The communicator's own context: ki_ctx_check / ki_ctx_set_wait_timeout_ns on it. */
int ki_comm_get_ctx(ki_comm* comm, ki_ctx** ctx);
/* sum of all ranks' Float32 shards: each rank's Float64 partial (ki_reduce_sum_f32) is exchanged and
 * the partials are added in rank order, so every rank gets the same bits. */
int ki_reduce_sum_f32_sharded(ki_comm* comm, const float* d_x, size_t n_local, float* d_out_f32, double* d_out_f64,
                              void* stream);
/* cumsum of the concatenated Int64 shards (any contiguous split): rank r writes its slice.  Phase 1
 * sums the shard (ki_reduce_sum_i64; skipped on the last rank, whose total nobody needs), the totals
 * are exchanged, phase 2 is ki_scan_inclusive_i64_dseed seeded on the device with the sum of the
 * lower ranks' totals.  With one rank it is ki_scan_inclusive_i64. */
int ki_scan_inclusive_i64_sharded(ki_comm* comm, const int64_t* d_in, int64_t* d_out, size_t n_local, void* stream);
/* ki_scan_inclusive_i64_sharded with this rank's shard in HOST memory (h_in, h_out, 8-byte aligned;
 * page-locked for asynchrony): phase 1 brings the shard to the device in 16 MiB chunks and sums each
 * as it lands, the totals are exchanged, phase 2 scans the chunks in place (seeded on the device)
 * and sends each back as soon as it is done.  The device copy of the shard lives in the
 * communicator's scratch.  With one rank it is ki_scan_inclusive_i64_host. */
int ki_scan_inclusive_i64_sharded_host(ki_comm* comm, const int64_t* h_in, int64_t* h_out, size_t n_local,
                                       void* stream);
/* filter/findall of the concatenated Float32 shards: rank r compacts its shard (ki_compact_gt_f32 with
 * index_base = the 1-based global index of its first element for findall) into its own outputs; the
 * counts are exchanged and *d_offset receives where rank r's kept elements start in the global result
 * (the sum of the lower ranks' counts), *d_total the global count (device uint64; d_count, d_offset,
 * d_total may be NULL).  The ranks' outputs concatenated in rank order are the global result. */
int ki_compact_gt_f32_sharded(ki_comm* comm, const float* d_x, size_t n_local, float threshold, float* d_out_vals,
                              int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, uint64_t* d_offset,
                              uint64_t* d_total, void* stream);

/* ---- (a8) fp8 e4m3 GEMM on tcgen05 / TMEM ---------------------------------------------------
 * No counterpart in the reference.  C = (scale_a * scale_b) * A * B with A: M x K row-major e4m3,
 * B: K x N row-major e4m3, C: M x N row-major Float32, Float32 accumulation.
 * M, N multiples of 128 and 256, K a multiple of 128, pointers 16-byte aligned (KI_ERR_ARG). */
int ki_gemm_e4m3_f32(ki_ctx* ctx, const uint8_t* d_A, const uint8_t* d_B, float* d_C, int M, int N, int K,
                     float scale_a, float scale_b, void* stream);

/* ---- warp-level intrinsics over whole warps of an array -------------------------------------
 * Element i of the array is lane i % 32 of warp i / 32; n must be a multiple of 32.           */

/* @shfl (src/warp.jl:114-192): any element size 1..64 bytes (moved as 32-bit words, the
 * reference's _shfl_recurse decomposition).  `src` is the offset (Up/Down), the lane mask (Xor)
 * or the 0-BASED source lane (Idx). */
int ki_warp_shfl(ki_ctx* ctx, int dir, const void* d_src, void* d_dst, size_t elem_bytes, size_t n, int src,
                 void* stream);
/* @warpreduce (src/warp.jl:226-237): inclusive scan per warp with Up shuffles. */
int ki_warp_reduce(ki_ctx* ctx, int op, int dtype, const void* d_src, void* d_dst, size_t n, void* stream);
/* @warpfold (src/warp.jl:273-282).  form 0: xor butterfly, every lane holds the total;
 * form 1: the reference's Down fold exactly (lane 1 holds the total, others partial folds). */
int ki_warp_fold(ki_ctx* ctx, int op, int dtype, int form, const void* d_src, void* d_dst, size_t n,
                 void* stream);
/* @vote (src/warp.jl:311-315; ext/CUDA/shuffle_vote.jl:23-34): d_pred is one byte per lane
 * (nonzero = true); d_out is one uint32 per lane: 0/1 for All/AnyLane/Uni, the mask for Ballot. */
int ki_warp_vote(ki_ctx* ctx, int mode, const uint8_t* d_pred, uint32_t* d_out, size_t n, void* stream);

/* vload / vstore! (src/vectorization.jl:135-300) run by one device thread.
 * rebase != 0: idx is a 0-based block index (elements idx*nitem ..); otherwise a 0-based element
 * index.  elem_bytes 1,2,4,8,16 use vector accesses with the runtime alignment check and the
 * generate_partN patterns; other sizes use the scalar path.  nitem in {1,2,4,8,16}. */
int ki_vload(ki_ctx* ctx, const void* d_a, size_t elem_bytes, int64_t idx, int nitem, int rebase, void* d_out,
             void* stream);
int ki_vstore(ki_ctx* ctx, void* d_a, size_t elem_bytes, int64_t idx, int nitem, int rebase,
              const void* d_values, void* stream);

/* @access / @fence (src/macros.jl:198-282; ext/CUDA/scopes_ordering.jl:29-193), one device thread:
 * stores *d_value into *d_slot with (scope, store_order), issues fence(fence_scope, fence_order)
 * (KI_SCOPE_DEFAULT / KI_ORDER_DEFAULT give @fence's defaults, Device and AcqRel), then loads
 * *d_slot with (scope, load_order) into *d_readback.  Orderings default as @access does (Release
 * for the store, Acquire for the load).  Invalid combinations give KI_ERR_ARG under the
 * reference's validation rules.  dtype: any ki_dtype. */
int ki_access_roundtrip(ki_ctx* ctx, int dtype, int scope, int store_order, int load_order, int fence_scope,
                        int fence_order, void* d_slot, const void* d_value, void* d_readback, void* stream);
/* Release/acquire message passing: block 0 writes `payload` to d_data[0] and release-stores 1 to
 * *d_flag (only when produce != 0); blocks 1..nblocks-1 spin with bounded acquire loads until the
 * flag is 1 and copy d_data[0] into d_seen[block].  A consumer whose wait runs out (produce == 0,
 * or timeout_ns elapsed) writes -1 and latches KI_ERR_TIMEOUT for ki_ctx_check. */
int ki_flag_message_pass(ki_ctx* ctx, int64_t* d_data, uint32_t* d_flag, int64_t* d_seen, int nblocks,
                         int64_t payload, int produce, uint64_t timeout_ns, void* stream);

/* ---- synthetic input generators (bit-identical to the host generators) ---------------------
 * Element i of stream `seed` is splitmix64's (i+1)-th output: mix64(seed + (i+1)*0x9E3779B97F4A7C15). */
int ki_fill_uniform_f32(ki_ctx* ctx, uint64_t seed, float* d_out, size_t n, void* stream);   /* (r>>40)*2^-24 */
int ki_fill_int_range_i64(ki_ctx* ctx, uint64_t seed, int64_t lo, int64_t hi, int64_t* d_out, size_t n,
                          void* stream);                                                         /* r%(hi-lo+1)+lo */
int ki_fill_bytes(ki_ctx* ctx, uint64_t seed, uint8_t* d_out, size_t n, void* stream);       /* byte i%8 of word i/8 */
int ki_fill_normal_f32(ki_ctx* ctx, uint64_t seed, float* d_out, size_t n, void* stream);    /* Box-Muller */
int ki_fill_e4m3_uniform(ki_ctx* ctx, uint64_t seed, float scale, uint8_t* d_out, size_t n,
                         void* stream);                                          /* e4m3((2u-1)*scale) */

#ifdef __cplusplus
}
#endif

#endif /* KI_B200_H */

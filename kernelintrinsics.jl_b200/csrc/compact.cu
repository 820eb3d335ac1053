// compact.cu -- order-preserving stream compaction: filter(x -> x > t, x) and findall.
//
// One CTA per 4096-element tile (256 threads); the tile index comes from an atomic ticket taken
// when the CTA starts (predecessors always run; a tile's count depends only on its own data).
// A full, 16-byte-aligned tile arrives in shared memory by one 16 KiB 1-D TMA bulk copy.  Warp w
// owns elements [512w, 512w+512) as 4 rows; in row j lane l holds the float4 at 128j + 4l
// (conflict-free 16-byte shared loads).  For each of the 4 components the warp takes a @vote Ballot
// (ext/CUDA/shuffle_vote.jl:23-34, vote.sync ballot -> UInt32), and an element's rank inside its row
// is
//     sum over components c of popc(ballot_c & lanes_below) + (kept components before it in its lane)
// which keeps source order (lane-major, then component).  Warp counts are scanned by warp 0 with
// @warpreduce, the tile count is published at once and goes through the decoupled lookback
// (ki/lookback.cuh), and the kept values and their indices are packed in shared memory, shifted by
// the output's alignment residue so that the copy-out uses coalesced 16-byte stores into
// [tile prefix, tile prefix + tile count).
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 4096;
constexpr int kWarpSpan = kTile / kWarps;  // 512
constexpr int kRows = kWarpSpan / 128;     // 4 rows of 32 lanes x float4
constexpr size_t kBufBytes = kTile * sizeof(float);              // 16 KiB
constexpr size_t kStageElems = kTile + 4;                        // room for the alignment shift
constexpr size_t kSmemBytes = kBufBytes + kStageElems * 8;
#ifndef KI_COMPACT_LOOKBACK_K
#define KI_COMPACT_LOOKBACK_K 1
#endif
constexpr int kLookbackK = KI_COMPACT_LOOKBACK_K;  // lookback window of 32*K tiles per round trip

struct CompactArgs {
    const float* x;
    size_t n;
    float thr;
    float* out_vals;
    int32_t* out_idx;
    int64_t index_base;
    uint64_t* d_count;
    ki::TileStatus st;
    unsigned long long* ticket;
    uint32_t* status;
    uint64_t timeout_ns;
    int tma_in;   // x is 16-byte aligned
    int vec_out;  // out_vals and out_idx are 16-byte aligned (or absent)
};

__global__ void __launch_bounds__(kThreads) compact_gt_f32_kernel(CompactArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ int warp_cnt[kWarps];
    __shared__ int warp_excl[kWarps];
    __shared__ int tile_cnt;
    __shared__ int64_t tile_excl;
    __shared__ unsigned long long tile_id;

    float* sb = reinterpret_cast<float*>(smem_raw);
    float* stage_v = reinterpret_cast<float*>(smem_raw + kBufBytes);
    int32_t* stage_i = reinterpret_cast<int32_t*>(smem_raw + kBufBytes + kStageElems * 4);
    const int tid = threadIdx.x;
    const int w = tid >> 5;
    const unsigned lane = tid & 31;
    const uint64_t ntiles = (a.n + kTile - 1) / kTile;
    if (tid == 0) {
        tile_id = atomicAdd(a.ticket, 1ull);
        ki::mbar_init(&bar, 1);
        ki::fence_mbar_init();
    }
    __syncthreads();
    const uint64_t t = tile_id;
    const size_t first = (size_t)t * kTile;
    const int count = (int)min((size_t)kTile, a.n - first);
    const int wofs = w * kWarpSpan;
    if (a.tma_in && count == kTile) {
        if (tid == 0) {
            ki::mbar_arrive_expect_tx(&bar, (uint32_t)kBufBytes);
            ki::bulk_g2s(sb, a.x + first, (uint32_t)kBufBytes, &bar);
        }
        if (!ki::mbar_wait_bounded(&bar, 0, a.status, a.timeout_ns))
            ki::mbar_wait_bounded(&bar, 0, a.status, a.timeout_ns);  // never leave a copy in flight
    } else {
        for (int i = tid; i < kTile; i += kThreads) sb[i] = (i < count) ? a.x[first + i] : 0.0f;
        __syncthreads();
    }

    // predicates (elements past the end never pass) and ballots
    const unsigned below = (1u << lane) - 1u;  // lanes with a lower index
    float4 v[kRows];
    unsigned pbits = 0;  // bit 4j+c
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        v[j] = reinterpret_cast<const float4*>(sb + wofs)[32 * j + lane];
        const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int i = wofs + 128 * j + 4 * (int)lane + c;
            if (i < count && e[c] > a.thr) pbits |= 1u << (4 * j + c);
        }
    }
    int rank0[kRows];  // kept elements of the row before this lane
    int row_cnt[kRows];
    int wcount = 0;
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        rank0[j] = 0;
        row_cnt[j] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const unsigned bal = ki::ballot((pbits >> (4 * j + c)) & 1u);
            rank0[j] += __popc(bal & below);
            row_cnt[j] += __popc(bal);
        }
        wcount += row_cnt[j];
    }
    if (lane == 0) warp_cnt[w] = wcount;
    __syncthreads();

    if (w == 0) {
        const int c = (lane < (unsigned)kWarps) ? warp_cnt[lane] : 0;
        const int inc = ki::warpreduce(c, ki::Add{});
        if (lane < (unsigned)kWarps) warp_excl[lane] = inc - c;
        const int agg = __shfl_sync(0xffffffffu, inc, kWarps - 1);
        if (lane == 0) ki::publish_aggregate(a.st, t, agg, 0);
        const int64_t ex = ki::decoupled_lookback<kLookbackK>(a.st, t, agg, 0, a.status, a.timeout_ns);
        if (lane == 0) {
            tile_excl = ex;
            tile_cnt = agg;
            if (t == ntiles - 1 && a.d_count) *a.d_count = (uint64_t)(ex + agg);
        }
    }
    __syncthreads();

    // pack the kept elements in source order, shifted by the output alignment residue
    const int64_t tex = tile_excl;
    const int shift = (int)(tex & 3);
    int pos = warp_excl[w] + shift;
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        int r = pos + rank0[j];
        const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if ((pbits >> (4 * j + c)) & 1u) {
                stage_v[r] = e[c];
                stage_i[r] = (int32_t)((int64_t)(first + wofs + 128 * j + 4 * lane + c) + a.index_base);
                ++r;
            }
        }
        pos += row_cnt[j];
    }
    __syncthreads();

    // copy out [tex, tex + cnt): staged element k sits at stage[k + shift]
    const int cnt = tile_cnt;
    if (a.vec_out) {
        const int to_boundary = (4 - shift) & 3;  // elements before the first 16-byte boundary
        const int head = to_boundary < cnt ? to_boundary : cnt;
        if (tid < head) {
            if (a.out_vals) a.out_vals[tex + tid] = stage_v[shift + tid];
            if (a.out_idx) a.out_idx[tex + tid] = stage_i[shift + tid];
        }
        const int nvec = (cnt - head) >> 2;
        const int s0 = shift + head;  // multiple of 4
        for (int q = tid; q < nvec; q += kThreads) {
            if (a.out_vals)
                __stcs(reinterpret_cast<float4*>(a.out_vals + tex + head) + q,
                       reinterpret_cast<const float4*>(stage_v + s0)[q]);
            if (a.out_idx)
                __stcs(reinterpret_cast<int4*>(a.out_idx + tex + head) + q,
                       reinterpret_cast<const int4*>(stage_i + s0)[q]);
        }
        const int t0 = head + 4 * nvec;
        if (tid < cnt - t0) {
            if (a.out_vals) a.out_vals[tex + t0 + tid] = stage_v[shift + t0 + tid];
            if (a.out_idx) a.out_idx[tex + t0 + tid] = stage_i[shift + t0 + tid];
        }
    } else {
        for (int k = tid; k < cnt; k += kThreads) {
            if (a.out_vals) a.out_vals[tex + k] = stage_v[shift + k];
            if (a.out_idx) a.out_idx[tex + k] = stage_i[shift + k];
        }
    }
}

}  // namespace

extern "C" int ki_compact_gt_f32(ki_ctx* ctx, const float* d_x, size_t n, float threshold, float* d_out_vals,
                                 int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "compact: null input");
    if (n > 0 && !ki::aligned(d_x, 4)) return ki::set_error(ctx, KI_ERR_ARG, "compact: misaligned Float32 input");
    if ((d_out_vals && !ki::aligned(d_out_vals, 4)) || (d_out_idx && !ki::aligned(d_out_idx, 4)))
        return ki::set_error(ctx, KI_ERR_ARG, "compact: misaligned output");
    if (index_base < INT32_MIN || (n > 0 && index_base + (int64_t)n - 1 > (int64_t)INT32_MAX))
        return ki::set_error(ctx, KI_ERR_ARG, "compact: indices do not fit Int32");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    if (n == 0) {
        if (d_count) KI_CUDA(ctx, cudaMemsetAsync(d_count, 0, sizeof(uint64_t), s));
        return KI_OK;
    }
    const size_t ntiles = (n + kTile - 1) / kTile;
    const size_t words_off = 256;
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_COMPACT, words_off + ntiles * 24, &base);
    if (rc) return rc;
    char* b = static_cast<char*>(base);
    KI_CUDA(ctx, cudaMemsetAsync(b, 0, words_off + ntiles * sizeof(uint64_t), s));
    KI_CUDA(ctx, cudaFuncSetAttribute(compact_gt_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kSmemBytes));
    CompactArgs a;
    a.x = d_x;
    a.n = n;
    a.thr = threshold;
    a.out_vals = d_out_vals;
    a.out_idx = d_out_idx;
    a.index_base = index_base;
    a.d_count = d_count;
    a.st.words = reinterpret_cast<uint64_t*>(b + words_off);
    a.st.aggs = reinterpret_cast<int64_t*>(b + words_off + ntiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(b + words_off + ntiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(b);
    a.status = ctx->d_status;
    a.timeout_ns = ctx->wait_timeout_ns;
    a.tma_in = ki::aligned(d_x, 16);
    a.vec_out = (!d_out_vals || ki::aligned(d_out_vals, 16)) && (!d_out_idx || ki::aligned(d_out_idx, 16));
    compact_gt_f32_kernel<<<(unsigned)ntiles, kThreads, kSmemBytes, s>>>(a);
    return ki::check_launch(ctx, "compact_gt_f32_kernel launch");
}

// compact.cu -- order-preserving stream compaction: filter(x -> x > t, x) and findall.
//
// One CTA per 4096-element tile, tiles handed out by an atomic ticket.  Warp w owns elements
// [512w, 512w+512) of the tile as 4 rows; in row j lane l holds the float4 at 128j + 4l.  For each
// of the 4 components the warp takes a @vote Ballot (ext/CUDA/shuffle_vote.jl:23-34, vote.sync
// ballot -> UInt32), and an element's rank inside its row is
//     sum over components c of popc(ballot_c & lanes_below) + (kept components before it in its lane)
// which keeps source order (lane-major, then component).  Warp counts are scanned by warp 0 with
// @warpreduce, the tile count goes through the decoupled lookback (ki/lookback.cuh, release/acquire
// flags), and every kept element is written at tile prefix + warp prefix + row prefix + rank.
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 4096;
constexpr int kWarpSpan = kTile / kWarps;  // 512
constexpr int kRows = kWarpSpan / 128;     // 4 rows of 32 lanes x float4

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
    int vec_ok;  // x is 16-byte aligned
};

__global__ void __launch_bounds__(kThreads) compact_gt_f32_kernel(CompactArgs a) {
    __shared__ int64_t warp_cnt[kWarps];
    __shared__ int64_t warp_excl[kWarps];
    __shared__ int64_t tile_excl;
    __shared__ unsigned long long tile_id;

    const int tid = threadIdx.x;
    const int w = tid >> 5;
    const unsigned lane = tid & 31;
    if (tid == 0) tile_id = atomicAdd(a.ticket, 1ull);
    __syncthreads();
    const uint64_t t = tile_id;
    const size_t first = (size_t)t * kTile;
    const size_t count = min((size_t)kTile, a.n - first);
    const size_t wfirst = first + (size_t)w * kWarpSpan;

    float4 v[kRows];
    if (a.vec_ok && count == kTile) {
        const float4* xv = reinterpret_cast<const float4*>(a.x + wfirst);
#pragma unroll
        for (int j = 0; j < kRows; ++j) v[j] = __ldcs(xv + 32 * j + lane);
    } else {
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            float e[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const size_t i = (size_t)w * kWarpSpan + 128 * j + 4 * lane + c;
                e[c] = (i < count) ? a.x[first + i] : 0.0f;
            }
            v[j] = make_float4(e[0], e[1], e[2], e[3]);
        }
    }

    // predicates: elements past the end never pass
    unsigned pbits = 0;  // bit 4j+c
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const size_t i = (size_t)w * kWarpSpan + 128 * j + 4 * lane + c;
            if (i < count && e[c] > a.thr) pbits |= 1u << (4 * j + c);
        }
    }
    unsigned ballots[kRows][4];
    int row_cnt[kRows];
    int wcount = 0;
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        row_cnt[j] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            ballots[j][c] = ki::ballot((pbits >> (4 * j + c)) & 1u);
            row_cnt[j] += __popc(ballots[j][c]);
        }
        wcount += row_cnt[j];
    }
    if (lane == 0) warp_cnt[w] = wcount;
    __syncthreads();

    if (w == 0) {
        const int64_t c = (lane < (unsigned)kWarps) ? warp_cnt[lane] : 0;
        const int64_t inc = ki::warpreduce(c, ki::WrapAdd{});
        if (lane < (unsigned)kWarps) warp_excl[lane] = inc - c;
        const int64_t agg = __shfl_sync(0xffffffffu, inc, kWarps - 1);
        const int64_t ex = ki::decoupled_lookback(a.st, t, agg, 0, a.status, a.timeout_ns);
        if (lane == 0) {
            tile_excl = ex;
            if (t == gridDim.x - 1 && a.d_count) *a.d_count = (uint64_t)(ex + agg);
        }
    }
    __syncthreads();

    const unsigned below = (1u << lane) - 1u;  // lanes with a lower index
    int64_t pos = tile_excl + warp_excl[w];
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        int rank = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) rank += __popc(ballots[j][c] & below);
        const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if ((pbits >> (4 * j + c)) & 1u) {
                const size_t o = (size_t)(pos + rank);
                if (a.out_vals) a.out_vals[o] = e[c];
                if (a.out_idx) {
                    const int64_t src = (int64_t)(wfirst + 128 * j + 4 * lane + c);
                    a.out_idx[o] = (int32_t)(src + a.index_base);
                }
                ++rank;
            }
        }
        pos += row_cnt[j];
    }
}

}  // namespace

extern "C" int ki_compact_gt_f32(ki_ctx* ctx, const float* d_x, size_t n, float threshold, float* d_out_vals,
                                 int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "compact: null input");
    if (n > 0 && !ki::aligned(d_x, 4)) return ki::set_error(ctx, KI_ERR_ARG, "compact: misaligned Float32 input");
    if (index_base < INT32_MIN || (n > 0 && index_base + (int64_t)n - 1 > (int64_t)INT32_MAX))
        return ki::set_error(ctx, KI_ERR_ARG, "compact: indices do not fit Int32");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    if (n == 0) {
        if (d_count) KI_CUDA(ctx, cudaMemsetAsync(d_count, 0, sizeof(uint64_t), s));
        return KI_OK;
    }
    const size_t ntiles = (n + kTile - 1) / kTile;
    const size_t flags_off = 256;
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_COMPACT, flags_off + ntiles * 24, &base);
    if (rc) return rc;
    char* b = static_cast<char*>(base);
    KI_CUDA(ctx, cudaMemsetAsync(b, 0, flags_off + ntiles * sizeof(uint64_t), s));
    CompactArgs a;
    a.x = d_x;
    a.n = n;
    a.thr = threshold;
    a.out_vals = d_out_vals;
    a.out_idx = d_out_idx;
    a.index_base = index_base;
    a.d_count = d_count;
    a.st.flags = reinterpret_cast<uint64_t*>(b + flags_off);
    a.st.aggs = reinterpret_cast<int64_t*>(b + flags_off + ntiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(b + flags_off + ntiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(b);
    a.status = ctx->d_status;
    a.timeout_ns = ctx->wait_timeout_ns;
    a.vec_ok = ki::aligned(d_x, 16);
    compact_gt_f32_kernel<<<(unsigned)ntiles, kThreads, 0, s>>>(a);
    return ki::check_launch(ctx, "compact_gt_f32_kernel launch");
}

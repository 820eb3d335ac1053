// compact.cu -- ki_compact_gt_f32, ki_compact and ki_compact_map (kernel in compact.cuh).
#include "compact.cuh"

extern "C" int ki_compact_gt_f32(ki_ctx* ctx, const float* d_x, size_t n, float threshold, float* d_out_vals,
                                 int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, void* stream) {
    KI_CHECK_CTX(ctx);
    int rc = check_common(ctx, d_x, n, index_base);
    if (rc) return rc;
    KI_GUARD(ctx);
    return compact_run<float, PGt>(ctx, d_x, n, &threshold, d_out_vals, d_out_idx, index_base, d_count,
                                   ki::as_stream(stream));
}

extern "C" int ki_compact(ki_ctx* ctx, int pred, int dtype, const void* d_x, size_t n, const void* h_thr,
                          void* d_out_vals, int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, void* stream) {
    KI_CHECK_CTX(ctx);
    if (!h_thr) return ki::set_error(ctx, KI_ERR_ARG, "compact: null threshold");
    int rc = check_common(ctx, d_x, n, index_base);
    if (rc) return rc;
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    return compact_dtype(ctx, pred, dtype, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
}

extern "C" int ki_compact_map(ki_ctx* ctx, int map, int pred, int dtype, const void* d_x, size_t n, const void* h_thr,
                              void* d_out_vals, int32_t* d_out_idx, int64_t index_base, uint64_t* d_count,
                              void* stream) {
    if (map == KI_MAP_IDENTITY)
        return ki_compact(ctx, pred, dtype, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, stream);
    KI_CHECK_CTX(ctx);
    if (!h_thr) return ki::set_error(ctx, KI_ERR_ARG, "compact: null threshold");
    int rc = check_common(ctx, d_x, n, index_base);
    if (rc) return rc;
    KI_GUARD(ctx);
    return ki_compact_mapped(ctx, map, pred, dtype, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count,
                             ki::as_stream(stream));
}

// compact_map_abs2.cu -- the abs2 instances of the fused map-then-compact (compact_map.cu).
#include "compact.cuh"

__attribute__((visibility("hidden"))) int ki_compact_abs2(ki_ctx* ctx, int pred, int dtype, const void* d_x, size_t n,
                                                          const void* h_thr, void* d_out_vals, int32_t* d_out_idx,
                                                          int64_t index_base, uint64_t* d_count, cudaStream_t s) {
    return compact_dtype<ki::MapAbs2>(ctx, pred, dtype, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
}

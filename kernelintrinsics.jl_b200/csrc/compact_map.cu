// compact_map.cu -- fused map-then-compact: filter(v -> abs(v) op t, x) and filter(v -> abs2(v) op t,
// x) (and their findall), the compaction kernel of compact.cuh with the map inside the predicate.
// The kept elements are written as they are in x, not mapped.  The abs2 instances are in
// compact_map_abs2.cu (a file per map keeps the builds parallel).
#include "compact.cuh"

__attribute__((visibility("hidden"))) int ki_compact_abs2(ki_ctx* ctx, int pred, int dtype, const void* d_x, size_t n,
                                                          const void* h_thr, void* d_out_vals, int32_t* d_out_idx,
                                                          int64_t index_base, uint64_t* d_count, cudaStream_t s);

int ki_compact_mapped(ki_ctx* ctx, int map, int pred, int dtype, const void* d_x, size_t n, const void* h_thr,
                      void* d_out_vals, int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, cudaStream_t s) {
    switch (map) {
        case KI_MAP_ABS:
            return compact_dtype<ki::MapAbs>(ctx, pred, dtype, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_MAP_ABS2:
            return ki_compact_abs2(ctx, pred, dtype, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "compact: unknown map");
    }
}

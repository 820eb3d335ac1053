// reduce_map.cu -- mapreduce(abs, op, x) and mapreduce(abs2, op, x) for op in +, max, min: the
// reduce kernel of reduce.cuh with the map applied to each element before it is lifted into the
// accumulation type (the map in the element type, as Base computes abs / abs2).
#include "reduce.cuh"

namespace {

template <class M>
int reduce_map_op(ki_ctx* ctx, int op, int dtype, const void* d_x, size_t n, void* d_out, cudaStream_t s) {
    switch (op) {
        case KI_OP_ADD: return reduce_dtype<ki::JAdd, M>(ctx, dtype, d_x, n, d_out, s);
        case KI_OP_MAX: return reduce_dtype<ki::JMax, M>(ctx, dtype, d_x, n, d_out, s);
        case KI_OP_MIN: return reduce_dtype<ki::JMin, M>(ctx, dtype, d_x, n, d_out, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "mapreduce: with a map, op must be KI_OP_ADD, KI_OP_MAX or KI_OP_MIN");
    }
}

}  // namespace

int ki_reduce_mapped(ki_ctx* ctx, int map, int op, int dtype, const void* d_x, size_t n, void* d_out, cudaStream_t s) {
    switch (map) {
        case KI_MAP_ABS: return reduce_map_op<ki::MapAbs>(ctx, op, dtype, d_x, n, d_out, s);
        case KI_MAP_ABS2: return reduce_map_op<ki::MapAbs2>(ctx, op, dtype, d_x, n, d_out, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "mapreduce: unknown map");
    }
}

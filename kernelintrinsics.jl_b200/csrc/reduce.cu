// reduce.cu -- ki_reduce_sum_f32, ki_reduce_sum_i64, ki_reduce and ki_mapreduce (kernel in reduce.cuh).
#include "reduce.cuh"

extern "C" int ki_reduce_sum_f32(ki_ctx* ctx, const float* d_x, size_t n, float* d_out_f32, double* d_out_f64,
                                 void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_out_f32 && !d_out_f64) return ki::set_error(ctx, KI_ERR_ARG, "reduce: no output");
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "reduce: null input");
    if (n > 0 && !ki::aligned(d_x, 4)) return ki::set_error(ctx, KI_ERR_ARG, "reduce: misaligned Float32 input");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    if (n == 0) {
        if (d_out_f32) KI_CUDA(ctx, cudaMemsetAsync(d_out_f32, 0, sizeof(float), s));
        if (d_out_f64) KI_CUDA(ctx, cudaMemsetAsync(d_out_f64, 0, sizeof(double), s));
        return KI_OK;
    }
    return launch_reduce<float, ki::JAdd>(ctx, d_x, n, d_out_f32, d_out_f64, s);
}

extern "C" int ki_reduce_sum_i64(ki_ctx* ctx, const int64_t* d_x, size_t n, int64_t* d_out, void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_out) return ki::set_error(ctx, KI_ERR_ARG, "reduce: no output");
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "reduce: null input");
    if (n > 0 && !ki::aligned(d_x, 8)) return ki::set_error(ctx, KI_ERR_ARG, "reduce: misaligned Int64 input");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    if (n == 0) {
        KI_CUDA(ctx, cudaMemsetAsync(d_out, 0, sizeof(int64_t), s));
        return KI_OK;
    }
    return launch_reduce<int64_t, ki::JAdd>(ctx, d_x, n, d_out, nullptr, s);
}

extern "C" int ki_reduce(ki_ctx* ctx, int op, int dtype, const void* d_x, size_t n, void* d_out, void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_out) return ki::set_error(ctx, KI_ERR_ARG, "reduce: no output");
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "reduce: null input");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    switch (op) {
        case KI_OP_ADD: return reduce_dtype<ki::JAdd>(ctx, dtype, d_x, n, d_out, s);
        case KI_OP_MAX: return reduce_dtype<ki::JMax>(ctx, dtype, d_x, n, d_out, s);
        case KI_OP_MIN: return reduce_dtype<ki::JMin>(ctx, dtype, d_x, n, d_out, s);
        case KI_OP_MUL: return reduce_dtype<ki::JMul>(ctx, dtype, d_x, n, d_out, s);
        case KI_OP_OR: return reduce_dtype<ki::JOr>(ctx, dtype, d_x, n, d_out, s);
        case KI_OP_AND: return reduce_dtype<ki::JAnd>(ctx, dtype, d_x, n, d_out, s);
        case KI_OP_XOR: return reduce_dtype<ki::JXor>(ctx, dtype, d_x, n, d_out, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "reduce: unknown operator");
    }
}

extern "C" int ki_mapreduce(ki_ctx* ctx, int map, int op, int dtype, const void* d_x, size_t n, void* d_out,
                            void* stream) {
    if (map == KI_MAP_IDENTITY) return ki_reduce(ctx, op, dtype, d_x, n, d_out, stream);
    KI_CHECK_CTX(ctx);
    if (!d_out) return ki::set_error(ctx, KI_ERR_ARG, "mapreduce: no output");
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "mapreduce: null input");
    KI_GUARD(ctx);
    return ki_reduce_mapped(ctx, map, op, dtype, d_x, n, d_out, ki::as_stream(stream));
}

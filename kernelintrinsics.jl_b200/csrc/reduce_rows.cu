// reduce_rows.cu -- ki_reduce_rows (the segmented reduce; kernels in reduce_rows.cuh) and its + and *
// instances.
#include "reduce_rows.cuh"

KI_ROWS_ENTRY(ki_rows_add) { return rows_op<ki::JAdd>(ctx, dtype, d_x, rows, cols, ld, d_out, s); }
KI_ROWS_ENTRY(ki_rows_mul) { return rows_op<ki::JMul>(ctx, dtype, d_x, rows, cols, ld, d_out, s); }

extern "C" int ki_reduce_rows(ki_ctx* ctx, int op, int dtype, const void* d_x, size_t rows, size_t cols, size_t ld,
                              void* d_out, void* stream) {
    KI_CHECK_CTX(ctx);
    if (rows == 0) return KI_OK;
    if (!d_out || (cols > 0 && !d_x)) return ki::set_error(ctx, KI_ERR_ARG, "reduce_rows: null pointer");
    if (ld < cols) return ki::set_error(ctx, KI_ERR_ARG, "reduce_rows: leading dimension smaller than cols");
    // empty rows: + and * give their identity (the kernel reads nothing); the others have none (Base throws)
    if (cols == 0 && op != KI_OP_ADD && op != KI_OP_MUL)
        return ki::set_error(ctx, KI_ERR_ARG, "reduce_rows: reducing empty rows with an operator that has no identity");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    switch (op) {
        case KI_OP_ADD: return ki_rows_add(ctx, dtype, d_x, rows, cols, ld, d_out, s);
        case KI_OP_MUL: return ki_rows_mul(ctx, dtype, d_x, rows, cols, ld, d_out, s);
        case KI_OP_MAX: return ki_rows_max(ctx, dtype, d_x, rows, cols, ld, d_out, s);
        case KI_OP_MIN: return ki_rows_min(ctx, dtype, d_x, rows, cols, ld, d_out, s);
        case KI_OP_OR: return ki_rows_or(ctx, dtype, d_x, rows, cols, ld, d_out, s);
        case KI_OP_AND: return ki_rows_and(ctx, dtype, d_x, rows, cols, ld, d_out, s);
        case KI_OP_XOR: return ki_rows_xor(ctx, dtype, d_x, rows, cols, ld, d_out, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "reduce_rows: unknown operator");
    }
}

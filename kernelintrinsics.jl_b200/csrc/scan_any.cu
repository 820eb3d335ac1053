// scan_any.cu -- ki_scan and ki_scan_rows (the device-wide and the segmented generic scan; kernels in
// scan_any.cuh) and their + and * instances.
#include "scan_any.cuh"

KI_SCAN_ANY_ENTRY(ki_scan_any_add) { return scan_op<ki::JAdd>(ctx, dtype, excl, d_in, d_out, sh, h_init, s); }
KI_SCAN_ANY_ENTRY(ki_scan_any_mul) { return scan_op<ki::JMul>(ctx, dtype, excl, d_in, d_out, sh, h_init, s); }

namespace {

int scan_dispatch(ki_ctx* ctx, int op, int dtype, bool excl, const void* d_in, void* d_out, const ScanShape& sh,
                  const void* h_init, cudaStream_t s) {
    switch (op) {
        case KI_OP_ADD: return ki_scan_any_add(ctx, dtype, excl, d_in, d_out, sh, h_init, s);
        case KI_OP_MUL: return ki_scan_any_mul(ctx, dtype, excl, d_in, d_out, sh, h_init, s);
        case KI_OP_MAX: return ki_scan_any_max(ctx, dtype, excl, d_in, d_out, sh, h_init, s);
        case KI_OP_MIN: return ki_scan_any_min(ctx, dtype, excl, d_in, d_out, sh, h_init, s);
        case KI_OP_OR: return ki_scan_any_or(ctx, dtype, excl, d_in, d_out, sh, h_init, s);
        case KI_OP_AND: return ki_scan_any_and(ctx, dtype, excl, d_in, d_out, sh, h_init, s);
        case KI_OP_XOR: return ki_scan_any_xor(ctx, dtype, excl, d_in, d_out, sh, h_init, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "scan: unknown operator");
    }
}

}  // namespace

extern "C" int ki_scan(ki_ctx* ctx, int op, int dtype, int exclusive, const void* d_in, void* d_out, size_t n,
                       const void* h_init, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_in || !d_out) return ki::set_error(ctx, KI_ERR_ARG, "scan: null pointer");
    KI_GUARD(ctx);
    const ScanShape sh{1, n, n, n};
    return scan_dispatch(ctx, op, dtype, exclusive != 0, d_in, d_out, sh, h_init, ki::as_stream(stream));
}

extern "C" int ki_scan_rows(ki_ctx* ctx, int op, int dtype, int exclusive, const void* d_in, size_t ld_in,
                            void* d_out, size_t ld_out, size_t rows, size_t cols, const void* h_init, void* stream) {
    KI_CHECK_CTX(ctx);
    if (rows == 0 || cols == 0) return KI_OK;
    if (!d_in || !d_out) return ki::set_error(ctx, KI_ERR_ARG, "scan_rows: null pointer");
    if (rows > 1 && (ld_in < cols || ld_out < cols))
        return ki::set_error(ctx, KI_ERR_ARG, "scan_rows: a leading dimension is smaller than cols");
    KI_GUARD(ctx);
    const ScanShape sh{rows, cols, ld_in, ld_out};
    return scan_dispatch(ctx, op, dtype, exclusive != 0, d_in, d_out, sh, h_init, ki::as_stream(stream));
}

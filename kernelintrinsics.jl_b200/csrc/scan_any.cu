// scan_any.cu -- ki_scan (the device-wide generic scan; kernel in scan_any.cuh) and its + family.
#include "scan_any.cuh"

KI_SCAN_ANY_ENTRY(ki_scan_any_add) { return scan_op<ki::JAdd>(ctx, dtype, excl, d_in, d_out, n, h_init, s); }
KI_SCAN_ANY_ENTRY(ki_scan_any_mul) { return scan_op<ki::JMul>(ctx, dtype, excl, d_in, d_out, n, h_init, s); }

extern "C" int ki_scan(ki_ctx* ctx, int op, int dtype, int exclusive, const void* d_in, void* d_out, size_t n,
                       const void* h_init, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_in || !d_out) return ki::set_error(ctx, KI_ERR_ARG, "scan: null pointer");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    const bool excl = exclusive != 0;
    switch (op) {
        case KI_OP_ADD: return ki_scan_any_add(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        case KI_OP_MUL: return ki_scan_any_mul(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        case KI_OP_MAX: return ki_scan_any_max(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        case KI_OP_MIN: return ki_scan_any_min(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        case KI_OP_OR: return ki_scan_any_or(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        case KI_OP_AND: return ki_scan_any_and(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        case KI_OP_XOR: return ki_scan_any_xor(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "scan: unknown operator");
    }
}

// scan_any_bits.cu -- the |, & and xor instances of the generic scan (scan_any.cuh), integers only.
#include "scan_any.cuh"

KI_SCAN_ANY_ENTRY(ki_scan_any_or) { return scan_op<ki::JOr>(ctx, dtype, excl, d_in, d_out, sh, h_init, s); }
KI_SCAN_ANY_ENTRY(ki_scan_any_and) { return scan_op<ki::JAnd>(ctx, dtype, excl, d_in, d_out, sh, h_init, s); }
KI_SCAN_ANY_ENTRY(ki_scan_any_xor) { return scan_op<ki::JXor>(ctx, dtype, excl, d_in, d_out, sh, h_init, s); }

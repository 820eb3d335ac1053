// scan_any_maxmin.cu -- the max and min instances of the generic scan (scan_any.cuh).
#include "scan_any.cuh"

KI_SCAN_ANY_ENTRY(ki_scan_any_max) { return scan_op<ki::JMax>(ctx, dtype, excl, d_in, d_out, sh, h_init, s); }
KI_SCAN_ANY_ENTRY(ki_scan_any_min) { return scan_op<ki::JMin>(ctx, dtype, excl, d_in, d_out, sh, h_init, s); }

// reduce_rows_bits.cu -- the |, & and xor instances of the segmented reduce (reduce_rows.cuh).
#include "reduce_rows.cuh"

KI_ROWS_ENTRY(ki_rows_or) { return rows_op<ki::JOr>(ctx, dtype, d_x, rows, cols, ld, d_out, s); }
KI_ROWS_ENTRY(ki_rows_and) { return rows_op<ki::JAnd>(ctx, dtype, d_x, rows, cols, ld, d_out, s); }
KI_ROWS_ENTRY(ki_rows_xor) { return rows_op<ki::JXor>(ctx, dtype, d_x, rows, cols, ld, d_out, s); }

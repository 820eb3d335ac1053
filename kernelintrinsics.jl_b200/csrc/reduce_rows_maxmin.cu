// reduce_rows_maxmin.cu -- the max and min instances of the segmented reduce (reduce_rows.cuh).
#include "reduce_rows.cuh"

KI_ROWS_ENTRY(ki_rows_max) { return rows_op<ki::JMax>(ctx, dtype, d_x, rows, cols, ld, d_out, s); }
KI_ROWS_ENTRY(ki_rows_min) { return rows_op<ki::JMin>(ctx, dtype, d_x, rows, cols, ld, d_out, s); }

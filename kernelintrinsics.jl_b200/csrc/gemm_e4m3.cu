// gemm_e4m3.cu -- fp8 e4m3 GEMM on tcgen05 / TMEM (being written).
#include "ki/common.cuh"

extern "C" int ki_gemm_e4m3_f32(ki_ctx* ctx, const uint8_t* d_A, const uint8_t* d_B, float* d_C, int M, int N, int K,
                                float scale_a, float scale_b, void* stream) {
    (void)d_A; (void)d_B; (void)d_C; (void)M; (void)N; (void)K; (void)scale_a; (void)scale_b; (void)stream;
    KI_CHECK_CTX(ctx);
    return ki::set_error(ctx, KI_ERR_UNSUPPORTED, "gemm_e4m3: not built yet");
}

// linear.cu -- C ABI of the q4_0 linear layers (include/velo_cuda.h):
// weight repack and the tcgen05 dequant-fused GEMM.
#include "kernels/q4gemm.h"
#include "runtime/context.h"

using velo::fail;

extern "C" {

size_t velo_cuda_q4_0_repacked_bytes(int32_t N, int32_t K) {
    if (N <= 0 || K <= 0 || K % 32) return 0;
    return velo::q4_repacked_bytes(N, K);
}

int32_t velo_cuda_q4_0_repack(velo_cuda_ctx* c, const void* src, const void* src_b, int32_t N,
                              int32_t K, void* dst) {
    velo::clear_last_error();
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (N <= 0 || K <= 0 || K % 32)
        return fail(VELO_ERR_INVALID_ARGUMENT, "q4_0 repack: N = %d, K = %d (K must be a positive multiple of 32)", N, K);
    if (!src || !dst || (src_b && N % 2))
        return fail(VELO_ERR_INVALID_ARGUMENT, "q4_0 repack: NULL buffer or odd N for a gate/up pair");
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    VELO_CUDA_TRY(velo::launch_q4_repack(static_cast<const uint8_t*>(src),
                                         static_cast<const uint8_t*>(src_b), src_b != nullptr, N, K,
                                         static_cast<uint8_t*>(dst), c->stream));
    return VELO_OK;
}

int32_t velo_cuda_gemm_q4_0(velo_cuda_ctx* c, const void* w, const void* x, int32_t M, int32_t N,
                            int32_t K, void* y, int32_t ldy, int32_t mode) {
    velo::Range nvtx_range("velo.gemm_q4_0");
    velo::clear_last_error();
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (M < 0 || N <= 0 || K <= 0 || K % 32)
        return fail(VELO_ERR_INVALID_ARGUMENT, "q4_0 GEMM: M = %d, N = %d, K = %d", M, N, K);
    if (mode < velo::kEpiStoreF32 || mode > velo::kEpiStoreBF16)
        return fail(VELO_ERR_INVALID_ARGUMENT, "q4_0 GEMM: epilogue mode %d unknown", mode);
    if (mode == velo::kEpiSwiGLU && N % 2)
        return fail(VELO_ERR_INVALID_ARGUMENT, "q4_0 GEMM: SwiGLU needs an even N (gate + up)");
    const int out_cols = mode == velo::kEpiSwiGLU ? N / 2 : N;
    if (ldy < out_cols) return fail(VELO_ERR_INVALID_ARGUMENT, "q4_0 GEMM: ldy %d < %d", ldy, out_cols);
    if (M == 0) return VELO_OK;
    if (!w || !x || !y) return fail(VELO_ERR_INVALID_ARGUMENT, "q4_0 GEMM: NULL buffer");
    if ((uintptr_t)x % 16 || (uintptr_t)w % 16)
        return fail(VELO_ERR_INVALID_ARGUMENT, "q4_0 GEMM: activations and weights must be 16-byte aligned");
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    velo::Q4GemmArgs a{};
    a.w = static_cast<const uint8_t*>(w);
    a.N = N;
    a.K = K;
    a.M = M;
    a.y = y;
    a.ldy = ldy;
    a.mode = mode;
    a.err = c->err_flag;
    VELO_CUDA_TRY(velo::launch_q4_gemm(a, static_cast<const __half*>(x), c->sm_count, c->stream));
    return VELO_OK;
}

}  // extern "C"

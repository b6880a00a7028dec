// gemm.cu -- prefill GEMM entry (tokens > 16).
//
// Interim path: the token dimension is processed in groups of 16 by the GEMV
// kernel (same numerics as the prefill contract: f16 activations, f16
// weights, f32 accumulation on the tensor cores). f16 activations are widened
// to f32 in the context scratch first (exact).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace ef {

__global__ void f16_to_f32_kernel(const __half *__restrict__ src, float *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __half2float(src[i]);
}

int launch_gemm(ef_ctx *ctx, const ef_weight *w, const void *x, int x_type, int M, float *y) {
    const float *xf = (const float *)x;
    if (x_type == EF_F16) {
        const int64_t n = (int64_t)M * w->k;
        if (int rc = ensure_scratch(ctx, 1, (size_t)n * 4)) return rc;
        int64_t blocks = (n + 255) / 256;
        if (blocks > 148 * 32) blocks = 148 * 32;
        f16_to_f32_kernel<<<(int)blocks, 256, 0, ctx->stream>>>((const __half *)x, (float *)ctx->scratch[1], n);
        if (int rc = check_cuda(ctx, cudaGetLastError(), "gemm f16->f32")) return rc;
        xf = (const float *)ctx->scratch[1];
    }
    for (int t0 = 0; t0 < M; t0 += 16) {
        const int mt = M - t0 < 16 ? M - t0 : 16;
        float *ys[1] = {y + (int64_t)t0 * w->rows};
        if (int rc = launch_gemv(ctx, &w, 1, nullptr, xf + (int64_t)t0 * w->k, mt, ys)) return rc;
    }
    return EF_OK;
}

}  // namespace ef

// internal.h -- host-side objects behind the opaque C handles.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/elffuss_cuda.h"

struct ef_buf {
    void *ptr = nullptr;
    size_t size = 0;
    uint64_t seq = 0;     // allocation sequence number (pool marks)
};

struct ef_weight {
    int type = 0;
    int64_t rows = 0, k = 0;          // logical shape
    int64_t rowgroups = 0, nchunks = 0;
    int tile_bytes = 0, chunk_k = 0;
    size_t bytes = 0;                 // device bytes of the repacked tiles
    uint8_t *dev = nullptr;
};

struct ef_ctx {
    int device = 0;
    int sm_count = 148;
    cudaStream_t own = nullptr;
    cudaStream_t stream = nullptr;
    std::string err;
    std::vector<ef_buf *> pool;       // live ef_alloc buffers, in allocation order
    uint64_t seq = 0;
    // Persistent device scratch owned by the context (grown on demand):
    // slot 0 holds the GEMV's f16 activation fragments, slot 1 the GEMM's
    // converted activations. A first call of a new, larger shape grows them
    // (cudaMalloc), so that call must come before any stream capture.
    void *scratch[2] = {nullptr, nullptr};
    size_t scratch_bytes[2] = {0, 0};
};

namespace ef {

int set_err(ef_ctx *ctx, int code, const char *fmt, ...);
int check_cuda(ef_ctx *ctx, cudaError_t e, const char *what);
int ensure_scratch(ef_ctx *ctx, int slot, size_t bytes);

// weights.cu
int launch_repack(ef_ctx *ctx, int type, const uint8_t *dev_gguf, int64_t rows, int64_t k,
                  ef_weight *w);
int launch_unpack(ef_ctx *ctx, const ef_weight *w, uint8_t *dev_gguf);
int launch_dequant(ef_ctx *ctx, const ef_weight *w, int64_t row0, int64_t nrows, float *out);

// gemv.cu
struct GemvPlan {
    int kslices;    // CTAs along k (one thread-block cluster)
    int cps;        // chunks per k-slice
    int rowblocks;  // CTAs along rows (8 rowgroups = 128 rows each)
    int nt;         // 8-token tiles (1 or 2)
    int warps;      // rowgroups (warps) per CTA
};
GemvPlan gemv_plan(int sm_count, int64_t rowgroups, int64_t nchunks, int M, const int ctas_per_sm[2]);
int launch_gemv(ef_ctx *ctx, const ef_weight *const *ws, int n, const ef_weight *w_up,
                const float *x, int M, float *const *ys);

// gemm.cu
int launch_gemm(ef_ctx *ctx, const ef_weight *w, const void *x, int x_type, int M, float *y);

}  // namespace ef

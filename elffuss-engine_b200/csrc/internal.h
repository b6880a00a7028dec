// internal.h -- host-side objects behind the opaque C handles.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>
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
    // slot 0 holds the GEMV's activation data, slot 1 the GEMM's converted
    // activations, slot 2 the decode attention's per-split partial results,
    // slot 3 the top-k kernel's per-chunk candidates. A first call of a new,
    // larger shape grows them (cudaMalloc), so that call must come before any
    // stream capture.
    static constexpr int kScratchSlots = 4;
    void *scratch[kScratchSlots] = {nullptr, nullptr, nullptr, nullptr};
    size_t scratch_bytes[kScratchSlots] = {0, 0, 0, 0};
    std::vector<void *> retired;      // outgrown scratch buffers, freed with the context
    uint64_t launches = 0;            // kernels this context has launched (diagnostic counter)
    // Programmatic dependent launch: each kernel may be scheduled while the
    // previous one on the stream finishes; it waits for that kernel's results
    // (griddepcontrol.wait) before reading them.
    bool pdl = false;
    // Set only on the stack context of ef_gemv_noalloc: scratch must never
    // grow (ensure_scratch reports EF_ERR_RANGE instead of allocating).
    bool no_alloc = false;
};

namespace ef {

int set_err(ef_ctx *ctx, int code, const char *fmt, ...);
int check_cuda(ef_ctx *ctx, cudaError_t e, const char *what);

// Launch `kern` on the context's stream (with the programmatic-dependent-
// launch attribute when ctx->pdl), counting it.
template <typename... KArgs, typename... Args>
int launch_on(ef_ctx *ctx, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, const char *what,
              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ctx->pdl ? 1 : 0;
    ctx->launches++;
    return check_cuda(ctx, cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what);
}
int ensure_scratch(ef_ctx *ctx, int slot, size_t bytes, bool zero = false);

// weights.cu
int launch_repack(ef_ctx *ctx, int type, const uint8_t *dev_gguf, int64_t rows, int64_t k,
                  ef_weight *w);
int launch_unpack(ef_ctx *ctx, const ef_weight *w, uint8_t *dev_gguf);
int launch_dequant(ef_ctx *ctx, const ef_weight *w, int64_t row0, int64_t nrows, float *out);
int launch_gather(ef_ctx *ctx, const ef_weight *w, const int *ids, int tokens, float *out);
int launch_gather_norm(ef_ctx *ctx, const ef_weight *w, const int *ids, int tokens, const float *wn, float eps,
                       float *x, float *nrm);

// model.cu / comm.cu: a row of n floats per CTA of T = min(256, n/4) threads
// with V float4 each, n = 4 * T * V, V in {1, 2, 4, 8}; 0 when n has no such
// split (n a multiple of 128 up to 8192).
inline int norm_v(int n, int &threads) {
    if (n < 128 || n % 128) return 0;
    threads = n / 4 < 256 ? n / 4 : 256;
    if (n % (4 * threads)) return 0;
    const int v = n / (4 * threads);
    return v == 1 || v == 2 || v == 4 || v == 8 ? v : 0;
}

// gemv.cu
// Row-parallel output of a tensor-parallel GEMV (comm.cu): instead of y, the
// kernel stores its rows, each word stamped with this call's number
// e = *epoch + 1 as one 8-byte store (e << 32 | word), into slot
// [e & 1][rank] of every rank's exchange data region.
struct GemvPush {
    int n = 0, rank = 0;                      // ranks (0 = off), this rank
    int64_t slot_bytes = 0;                   // bytes of a stamped slot
    uint8_t *data[EF_TP_MAX_RANKS] = {};      // each rank's data region [2][n][slot_bytes]
    const uint32_t *epoch = nullptr;          // this rank's count of finished calls
};
struct GemvPlan {
    int64_t ctas;      // rowblocks x kslices
    int kslices;       // CTAs (one cluster) per rowblock, each a contiguous k-slice
    int phase_chunks;  // chunks of activation data staged in shared memory at a time
    int whole;         // 1: the slice's chunks staged once at the start
    int xs_bytes;      // shared memory for activation data
    int xs_half;       // bytes of one phase buffer
};
GemvPlan gemv_plan(int64_t rowblocks, int64_t nchunks, int xb, bool fused, int ks);
int launch_gemv(ef_ctx *ctx, const ef_weight *const *ws, int n, const ef_weight *w_up,
                const float *x, int M, float *const *ys, const GemvPush *push = nullptr);

// gemm.cu
int gemm_status(ef_ctx *ctx);
int gemm_set_wait_limit(ef_ctx *ctx, int polls);
int launch_gemm(ef_ctx *ctx, const ef_weight *w, const void *x, int x_type, int M, float *y);

}  // namespace ef

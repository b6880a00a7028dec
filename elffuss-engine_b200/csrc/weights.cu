// weights.cu -- one-time device repack of GGUF tensors into rowgroup tiles, its
// inverse, and the bit-exact dequant test hook.
//
// The reference repacks on the CPU at load time (js/repack.js:153-199
// reordenaBloques, only Q8_0/Q4_0) and keeps a byte-exact inverse for its tests
// (vuelveAlGGUF, js/repack.js:201-219). Here the permutation runs on the GPU,
// one thread per GGUF block, for every hot-path type; see common.cuh for the
// tile layout.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "gen/iq_grids.h"
#include "internal.h"

namespace ef {

__device__ const int8_t g_grid_iq2xxs_i8[EF_GRID_IQ2XXS_ENTRIES * 8] = {EF_GRID_IQ2XXS_I8_INIT};
__device__ const int8_t g_grid_iq1s_i8[EF_GRID_IQ1S_ENTRIES * 8] = {EF_GRID_IQ1S_I8_INIT};

// Thread per GGUF block of the padded tensor (rowgroups*16 rows x
// nchunks*blocks_per_chunk blocks). Padding blocks are written as zeros.
__global__ void ef_repack_kernel(int type, const uint8_t *__restrict__ src, int64_t rows, int64_t bpr,
                              int64_t rowgroups, int64_t nchunks, int bpc, int bb, int tile_bytes,
                              uint8_t *__restrict__ dst) {
    const int64_t bpr_pad = nchunks * bpc;
    const int64_t total = rowgroups * RG_ROWS * bpr_pad;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / bpr_pad, b = i % bpr_pad;
        uint8_t blk[256];
        if (row < rows && b < bpr) {
            const uint8_t *s = src + (row * bpr + b) * bb;
            for (int j = 0; j < bb; j++) blk[j] = s[j];
        } else {
            for (int j = 0; j < bb; j++) blk[j] = 0;
        }
        const int64_t rg = row / RG_ROWS, c = b / bpc;
        uint8_t *T = dst + (rg * nchunks + c) * tile_bytes;
        scatter_block(type, blk, (int)(row % RG_ROWS), (int)(b % bpc), T);
    }
}

// Thread per GGUF block of the logical tensor: gather back the original bytes.
__global__ void ef_unpack_kernel(int type, const uint8_t *__restrict__ src, int64_t rows, int64_t bpr,
                              int64_t nchunks, int bpc, int bb, int tile_bytes,
                              uint8_t *__restrict__ dst) {
    const int64_t total = rows * bpr;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / bpr, b = i % bpr;
        const int64_t rg = row / RG_ROWS, c = b / bpc;
        const uint8_t *T = src + (rg * nchunks + c) * tile_bytes;
        uint8_t blk[256];
        gather_block(type, T, (int)(row % RG_ROWS), (int)(b % bpc), blk);
        uint8_t *d = dst + (row * bpr + b) * bb;
        for (int j = 0; j < bb; j++) d[j] = blk[j];
    }
}

// Thread per GGUF block of rows [row0, row0+nrows): gather, then decode with
// the reference's f32 arithmetic (common.cuh decode_block).
__global__ void ef_dequant_kernel(int type, const uint8_t *__restrict__ src, int64_t row0, int64_t nrows,
                               int64_t bpr, int64_t nchunks, int bpc, int bb, int be, int tile_bytes,
                               int64_t k, float *__restrict__ out) {
    const int8_t *grid = type == EF_IQ2_XXS ? g_grid_iq2xxs_i8 : g_grid_iq1s_i8;
    const int64_t total = nrows * bpr;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = row0 + i / bpr, b = i % bpr;
        const int64_t rg = row / RG_ROWS, c = b / bpc;
        const uint8_t *T = src + (rg * nchunks + c) * tile_bytes;
        uint8_t blk[256];
        float v[256];
        gather_block(type, T, (int)(row % RG_ROWS), (int)(b % bpc), blk);
        decode_block(type, blk, grid, v);
        float *o = out + (row - row0) * k + b * be;
        for (int j = 0; j < be; j++) o[j] = v[j];
    }
}

// Thread per GGUF block of `tokens` rows chosen by device-side ids (the
// reference's quant.gather, js/ops.js:1104-1118 / gatherShader
// kernels.wgsl.js:1199): out[t][:] = dequant(W)[ids[t]][:]. Ids outside
// [0, rows) produce a row of zeros.
__global__ void ef_gather_kernel(int type, const uint8_t *__restrict__ src, const int *__restrict__ ids, int tokens,
                              int64_t rows, int64_t bpr, int64_t nchunks, int bpc, int bb, int be, int tile_bytes,
                              int64_t k, float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const int8_t *grid = type == EF_IQ2_XXS ? g_grid_iq2xxs_i8 : g_grid_iq1s_i8;
    const int64_t total = (int64_t)tokens * bpr;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / bpr, b = i % bpr;
        const int64_t row = ids[t];
        float *o = out + t * k + b * be;
        if (row < 0 || row >= rows) {
            for (int j = 0; j < be; j++) o[j] = 0.f;
            continue;
        }
        const int64_t rg = row / RG_ROWS, c = b / bpc;
        const uint8_t *T = src + (rg * nchunks + c) * tile_bytes;
        uint8_t blk[256];
        float v[256];
        gather_block(type, T, (int)(row % RG_ROWS), (int)(b % bpc), blk);
        decode_block(type, blk, grid, v);
        for (int j = 0; j < be; j++) o[j] = v[j];
    }
}

// F2 (js/ops.fusion.js:152-165, kernels.fusion.wgsl.js:143-200): CTA per
// token: the embedding row as ef_gather_kernel decodes it (same blocks, same
// bits) into shared memory and x, then nrm = x * rsqrt(mean(x^2) + eps) * w.
__global__ void ef_gather_norm_kernel(int type, const uint8_t *__restrict__ src, const int *__restrict__ ids,
                                   int64_t rows, int64_t bpr, int64_t nchunks, int bpc, int be, int tile_bytes,
                                   int64_t k, const float *__restrict__ wn, float eps, float *__restrict__ x,
                                   float *__restrict__ nrm) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float rowbuf[];
    __shared__ float red[32];
    const int8_t *grid = type == EF_IQ2_XXS ? g_grid_iq2xxs_i8 : g_grid_iq1s_i8;
    const int t = blockIdx.x;
    const int64_t row = ids[t];
    const bool valid = row >= 0 && row < rows;
    for (int64_t b = threadIdx.x; b < bpr; b += blockDim.x) {
        float *o = rowbuf + b * be;
        if (!valid) {
            for (int j = 0; j < be; j++) o[j] = 0.f;
            continue;
        }
        const int64_t rg = row / RG_ROWS, c = b / bpc;
        const uint8_t *T = src + (rg * nchunks + c) * tile_bytes;
        uint8_t blk[256];
        float v[256];
        gather_block(type, T, (int)(row % RG_ROWS), (int)(b % bpc), blk);
        decode_block(type, blk, grid, v);
        for (int j = 0; j < be; j++) o[j] = v[j];
    }
    __syncthreads();
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) ss += rowbuf[i] * rowbuf[i];
    const float scale = rsqrtf(block_sum(ss, red) / (float)k + eps);
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
        x[(int64_t)t * k + i] = rowbuf[i];
        nrm[(int64_t)t * k + i] = rowbuf[i] * scale * wn[i];
    }
}

static int grid_for(int64_t total) {
    int64_t g = (total + 255) / 256;
    if (g > 148 * 64) g = 148 * 64;
    if (g < 1) g = 1;
    return (int)g;
}

int launch_repack(ef_ctx *ctx, int type, const uint8_t *dev_gguf, int64_t rows, int64_t k,
                  ef_weight *w) {
    TypeGeo geo;
    if (!geo_of(type, geo)) return set_err(ctx, EF_ERR_TYPE, "repack: unsupported type %d", type);
    const int bpc = geo.chunk_k / geo.block_elems;
    const int64_t bpr = k / geo.block_elems;
    const int64_t total = w->rowgroups * RG_ROWS * w->nchunks * bpc;
    ctx->launches++;
    ef_repack_kernel<<<grid_for(total), 256, 0, ctx->stream>>>(type, dev_gguf, rows, bpr, w->rowgroups,
                                                            w->nchunks, bpc, geo.block_bytes,
                                                            geo.tile_bytes, w->dev);
    return check_cuda(ctx, cudaGetLastError(), "repack launch");
}

int launch_unpack(ef_ctx *ctx, const ef_weight *w, uint8_t *dev_gguf) {
    TypeGeo geo;
    geo_of(w->type, geo);
    const int bpc = geo.chunk_k / geo.block_elems;
    const int64_t bpr = w->k / geo.block_elems;
    ctx->launches++;
    ef_unpack_kernel<<<grid_for(w->rows * bpr), 256, 0, ctx->stream>>>(
        w->type, w->dev, w->rows, bpr, w->nchunks, bpc, geo.block_bytes, geo.tile_bytes, dev_gguf);
    return check_cuda(ctx, cudaGetLastError(), "unpack launch");
}

int launch_dequant(ef_ctx *ctx, const ef_weight *w, int64_t row0, int64_t nrows, float *out) {
    TypeGeo geo;
    geo_of(w->type, geo);
    const int bpc = geo.chunk_k / geo.block_elems;
    const int64_t bpr = w->k / geo.block_elems;
    // 256 f32 + 256 bytes of local state per thread: keep blocks small.
    ctx->launches++;
    ef_dequant_kernel<<<grid_for(nrows * bpr), 128, 0, ctx->stream>>>(
        w->type, w->dev, row0, nrows, bpr, w->nchunks, bpc, geo.block_bytes, geo.block_elems,
        geo.tile_bytes, w->k, out);
    return check_cuda(ctx, cudaGetLastError(), "dequant launch");
}

int launch_gather_norm(ef_ctx *ctx, const ef_weight *w, const int *ids, int tokens, const float *wn, float eps,
                       float *x, float *nrm) {
    TypeGeo geo;
    if (!geo_of(w->type, geo)) return set_err(ctx, EF_ERR_TYPE, "gather_rmsnorm: unsupported type %d", w->type);
    const size_t smem = (size_t)w->k * sizeof(float);
    if (smem > 200 * 1024) return set_err(ctx, EF_ERR_RANGE, "gather_rmsnorm: row of %lld exceeds shared memory",
                                          (long long)w->k);
    static std::atomic<unsigned long long> configured{0};
    if (ctx->device < 64 && !(configured.load() & (1ull << ctx->device))) {
        if (int rc = check_cuda(ctx, cudaFuncSetAttribute(ef_gather_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                          200 * 1024), "gather_rmsnorm smem attribute"))
            return rc;
        configured.fetch_or(1ull << ctx->device);
    }
    const int bpc = geo.chunk_k / geo.block_elems;
    const int64_t bpr = w->k / geo.block_elems;
    return launch_on(ctx, ef_gather_norm_kernel, tokens, 256, smem, "gather_rmsnorm launch", w->type,
                     (const uint8_t *)w->dev, ids, w->rows, bpr, w->nchunks, bpc, geo.block_elems, geo.tile_bytes, w->k,
                     wn, eps, x, nrm);
}

int launch_gather(ef_ctx *ctx, const ef_weight *w, const int *ids, int tokens, float *out) {
    TypeGeo geo;
    geo_of(w->type, geo);
    const int bpc = geo.chunk_k / geo.block_elems;
    const int64_t bpr = w->k / geo.block_elems;
    return launch_on(ctx, ef_gather_kernel, grid_for((int64_t)tokens * bpr), 128, 0, "gather launch", w->type,
                     (const uint8_t *)w->dev, ids, tokens, w->rows, bpr, w->nchunks, bpc, geo.block_bytes,
                     geo.block_elems, geo.tile_bytes, w->k, out);
}

}  // namespace ef

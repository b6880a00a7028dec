// api.cu -- the C ABI of include/elffuss_cuda.h: contexts, buffers, weights,
// argument checking and dispatch to the kernels.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace ef {

int set_err(ef_ctx *ctx, int code, const char *fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ctx->err = buf;
    }
    return code;
}

int check_cuda(ef_ctx *ctx, cudaError_t e, const char *what) {
    if (e == cudaSuccess) return EF_OK;
    return set_err(ctx, e == cudaErrorMemoryAllocation ? EF_ERR_OOM : EF_ERR_CUDA, "%s: %s (%s)", what,
                   cudaGetErrorString(e), cudaGetErrorName(e));
}

int ensure_scratch(ef_ctx *ctx, int slot, size_t bytes, bool zero) {
    if (ctx->scratch_bytes[slot] >= bytes) return EF_OK;
    if (ctx->no_alloc)
        return set_err(ctx, EF_ERR_RANGE, "scratch: %zu bytes needed, more than the allocation-free array", bytes);
    if (ctx->scratch[slot]) {
        // Queued work or a CUDA graph captured earlier may still use the old
        // buffer: it is kept until the context is destroyed.
        ctx->retired.push_back(ctx->scratch[slot]);
        ctx->scratch[slot] = nullptr;
        ctx->scratch_bytes[slot] = 0;
    }
    size_t sz = std::max(bytes, (size_t)1 << 20);
    int rc = check_cuda(ctx, cudaMalloc(&ctx->scratch[slot], sz), "scratch alloc");
    if (rc) return rc;
    ctx->scratch_bytes[slot] = sz;
    if (zero) return check_cuda(ctx, cudaMemsetAsync(ctx->scratch[slot], 0, sz, ctx->stream), "scratch zero");
    return EF_OK;
}

static int use_device(ef_ctx *ctx) { return check_cuda(ctx, cudaSetDevice(ctx->device), "cudaSetDevice"); }

static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace ef

using namespace ef;

extern "C" {

int ef_version(void) { return EF_ABI_VERSION; }

int ef_type_info(int type, int *block_elems, int *block_bytes) {
    TypeGeo g;
    if (!geo_of(type, g)) return EF_ERR_TYPE;
    if (block_elems) *block_elems = g.block_elems;
    if (block_bytes) *block_bytes = g.block_bytes;
    return EF_OK;
}

int ef_ctx_create(int device, ef_ctx **out) {
    if (!out) return EF_ERR_INVALID;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return EF_ERR_CUDA;
    ef_ctx *c = new ef_ctx();
    c->device = device;
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return EF_ERR_CUDA;
    }
    c->stream = c->own;
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
    const char *pdl = getenv("EF_PDL");
    c->pdl = !(pdl && pdl[0] == '0');
    *out = c;
    return EF_OK;
}

int ef_ctx_destroy(ef_ctx *ctx) {
    if (!ctx) return EF_ERR_INVALID;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (ef_buf *b : ctx->pool) {
        cudaFree(b->ptr);
        delete b;
    }
    for (int i = 0; i < ef_ctx::kScratchSlots; i++)
        if (ctx->scratch[i]) cudaFree(ctx->scratch[i]);
    for (void *p : ctx->retired) cudaFree(p);
    if (ctx->own) cudaStreamDestroy(ctx->own);
    delete ctx;
    return EF_OK;
}

int ef_ctx_set_stream(ef_ctx *ctx, void *stream) {
    if (!ctx) return EF_ERR_INVALID;
    ctx->stream = (cudaStream_t)stream;   // NULL = the CUDA default (legacy) stream
    return EF_OK;
}

int ef_ctx_set_pdl(ef_ctx *ctx, int on) {
    if (!ctx) return EF_ERR_INVALID;
    ctx->pdl = on != 0;
    return EF_OK;
}

void *ef_ctx_stream(const ef_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int ef_stream_sync(ef_ctx *ctx) {
    if (!ctx) return EF_ERR_INVALID;
    return check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "stream sync");
}

const char *ef_last_error(const ef_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

uint64_t ef_ctx_launch_count(const ef_ctx *ctx) { return ctx ? ctx->launches : 0; }

// ---------------------------------------------------------------- buffers --
int ef_alloc(ef_ctx *ctx, size_t bytes, ef_buf **out) {
    if (!ctx || !out) return EF_ERR_INVALID;
    if (bytes == 0) return set_err(ctx, EF_ERR_INVALID, "ef_alloc: zero bytes");
    if (int rc = use_device(ctx)) return rc;
    void *p = nullptr;
    // sizes rounded to 256 like the reference pool (js/ops.js:242-253)
    if (int rc = check_cuda(ctx, cudaMalloc(&p, (bytes + 255) & ~(size_t)255), "ef_alloc")) return rc;
    ef_buf *b = new ef_buf();
    b->ptr = p;
    b->size = bytes;
    b->seq = ++ctx->seq;
    ctx->pool.push_back(b);
    *out = b;
    return EF_OK;
}

int ef_free(ef_ctx *ctx, ef_buf *buf) {
    if (!ctx || !buf) return EF_ERR_INVALID;
    auto it = std::find(ctx->pool.begin(), ctx->pool.end(), buf);
    if (it == ctx->pool.end()) return set_err(ctx, EF_ERR_INVALID, "ef_free: buffer not owned by this context");
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(buf->ptr);
    ctx->pool.erase(it);
    delete buf;
    return EF_OK;
}

void *ef_buf_ptr(const ef_buf *buf) { return buf ? buf->ptr : nullptr; }
size_t ef_buf_size(const ef_buf *buf) { return buf ? buf->size : 0; }

int ef_upload(ef_ctx *ctx, ef_buf *buf, size_t off, const void *host, size_t n) {
    if (!ctx || !buf || (!host && n)) return EF_ERR_INVALID;
    if (off > buf->size || n > buf->size - off)
        return set_err(ctx, EF_ERR_RANGE, "ef_upload: [%zu, +%zu) outside buffer of %zu", off, n, buf->size);
    if (int rc = use_device(ctx)) return rc;
    return check_cuda(ctx, cudaMemcpyAsync((char *)buf->ptr + off, host, n, cudaMemcpyHostToDevice, ctx->stream),
                      "ef_upload");
}

int ef_download(ef_ctx *ctx, const ef_buf *buf, size_t off, void *host, size_t n) {
    if (!ctx || !buf || (!host && n)) return EF_ERR_INVALID;
    if (off > buf->size || n > buf->size - off)
        return set_err(ctx, EF_ERR_RANGE, "ef_download: [%zu, +%zu) outside buffer of %zu", off, n, buf->size);
    if (int rc = use_device(ctx)) return rc;
    if (int rc = check_cuda(ctx, cudaMemcpyAsync(host, (const char *)buf->ptr + off, n, cudaMemcpyDeviceToHost,
                                                 ctx->stream), "ef_download"))
        return rc;
    return check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "ef_download sync");
}

int ef_scratch_mark(ef_ctx *ctx, uint64_t *mark) {
    if (!ctx || !mark) return EF_ERR_INVALID;
    *mark = ctx->seq;
    return EF_OK;
}

int ef_scratch_release(ef_ctx *ctx, uint64_t mark, ef_buf *const *live, int nlive) {
    if (!ctx || nlive < 0 || (nlive && !live)) return EF_ERR_INVALID;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    std::vector<ef_buf *> keep;
    for (ef_buf *b : ctx->pool) {
        bool is_live = b->seq <= mark;
        for (int i = 0; i < nlive && !is_live; i++) is_live = live[i] == b;
        if (is_live) {
            keep.push_back(b);
        } else {
            cudaFree(b->ptr);
            delete b;
        }
    }
    ctx->pool.swap(keep);
    return EF_OK;
}

// ---------------------------------------------------------------- weights --
static int check_shape(ef_ctx *ctx, int type, int64_t rows, int64_t k, TypeGeo &g) {
    if (!geo_of(type, g)) return set_err(ctx, EF_ERR_TYPE, "unsupported quant type %d", type);
    if (rows <= 0 || k <= 0) return set_err(ctx, EF_ERR_SHAPE, "bad shape rows=%lld k=%lld", (long long)rows,
                                            (long long)k);
    if (k % g.block_elems)
        return set_err(ctx, EF_ERR_SHAPE, "k=%lld is not a multiple of %d", (long long)k, g.block_elems);
    return EF_OK;
}

static int new_weight(ef_ctx *ctx, int type, int64_t rows, int64_t k, const TypeGeo &g, ef_weight **out) {
    ef_weight *w = new ef_weight();
    w->type = type;
    w->rows = rows;
    w->k = k;
    w->rowgroups = (rows + RG_ROWS - 1) / RG_ROWS;
    w->nchunks = (k + g.chunk_k - 1) / g.chunk_k;
    w->tile_bytes = g.tile_bytes;
    w->chunk_k = g.chunk_k;
    w->bytes = (size_t)w->rowgroups * w->nchunks * g.tile_bytes;
    int rc = check_cuda(ctx, cudaMalloc(&w->dev, w->bytes), "weight alloc");
    if (rc) {
        delete w;
        return rc;
    }
    *out = w;
    return EF_OK;
}

int ef_weight_load_device(ef_ctx *ctx, int type, const void *dev_gguf, int64_t rows, int64_t k,
                          ef_weight **out) {
    if (!ctx || !dev_gguf || !out) return EF_ERR_INVALID;
    TypeGeo g;
    if (int rc = check_shape(ctx, type, rows, k, g)) return rc;
    if (int rc = use_device(ctx)) return rc;
    ef_weight *w = nullptr;
    if (int rc = new_weight(ctx, type, rows, k, g, &w)) return rc;
    if (int rc = launch_repack(ctx, type, (const uint8_t *)dev_gguf, rows, k, w)) {
        cudaFree(w->dev);
        delete w;
        return rc;
    }
    // Kernels launched with programmatic dependent launch read weights before
    // they wait for the kernel ahead of them: the repacked tiles must be in
    // memory before any later launch.
    if (int rc = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "weight repack")) {
        cudaFree(w->dev);
        delete w;
        return rc;
    }
    *out = w;
    return EF_OK;
}

int ef_weight_load(ef_ctx *ctx, int type, const void *host_gguf, int64_t rows, int64_t k, ef_weight **out) {
    if (!ctx || !host_gguf || !out) return EF_ERR_INVALID;
    TypeGeo g;
    if (int rc = check_shape(ctx, type, rows, k, g)) return rc;
    if (int rc = use_device(ctx)) return rc;
    const size_t n = (size_t)rows * (k / g.block_elems) * g.block_bytes;
    void *tmp = nullptr;
    if (int rc = check_cuda(ctx, cudaMalloc(&tmp, n), "weight staging alloc")) return rc;
    int rc = check_cuda(ctx, cudaMemcpyAsync(tmp, host_gguf, n, cudaMemcpyHostToDevice, ctx->stream),
                        "weight upload");
    if (!rc) rc = ef_weight_load_device(ctx, type, tmp, rows, k, out);
    cudaStreamSynchronize(ctx->stream);   // staging buffer is read by the repack
    cudaFree(tmp);
    return rc;
}

int ef_weight_load_slice(ef_ctx *ctx, int type, const void *host_gguf, int64_t rows, int64_t k, int64_t row0,
                         int64_t nrows, int64_t k0, int64_t nk, ef_weight **out) {
    if (!ctx || !host_gguf || !out) return EF_ERR_INVALID;
    TypeGeo g;
    if (int rc = check_shape(ctx, type, rows, k, g)) return rc;
    if (row0 < 0 || nrows <= 0 || row0 + nrows > rows || k0 < 0 || nk <= 0 || k0 + nk > k)
        return set_err(ctx, EF_ERR_RANGE, "slice rows [%lld,+%lld) k [%lld,+%lld) outside %lldx%lld",
                       (long long)row0, (long long)nrows, (long long)k0, (long long)nk, (long long)rows,
                       (long long)k);
    if (k0 % g.block_elems || nk % g.block_elems)
        return set_err(ctx, EF_ERR_SHAPE, "slice k0=%lld nk=%lld not multiples of %d", (long long)k0,
                       (long long)nk, g.block_elems);
    const int64_t bpr = k / g.block_elems, b0 = k0 / g.block_elems, nb = nk / g.block_elems;
    std::vector<uint8_t> part((size_t)nrows * nb * g.block_bytes);
    const uint8_t *src = (const uint8_t *)host_gguf;
    for (int64_t r = 0; r < nrows; r++)
        memcpy(part.data() + (size_t)r * nb * g.block_bytes, src + ((row0 + r) * bpr + b0) * g.block_bytes,
               (size_t)nb * g.block_bytes);
    return ef_weight_load(ctx, type, part.data(), nrows, nk, out);
}

int ef_weight_load_shard(ef_ctx *ctx, int type, const void *host_gguf, int64_t rows, int64_t k, int shard_axis,
                         int rank, int nranks, ef_weight **out) {
    if (!ctx || !host_gguf || !out) return EF_ERR_INVALID;
    if (nranks < 1 || rank < 0 || rank >= nranks || (shard_axis != 0 && shard_axis != 1))
        return set_err(ctx, EF_ERR_INVALID, "shard: axis %d, rank %d of %d", shard_axis, rank, nranks);
    TypeGeo g;
    if (int rc = check_shape(ctx, type, rows, k, g)) return rc;
    if (shard_axis == 0) {   // column-parallel: a range of output rows
        if (rows % nranks) return set_err(ctx, EF_ERR_SHAPE, "shard: %lld rows over %d ranks", (long long)rows, nranks);
        const int64_t n = rows / nranks;
        return ef_weight_load_slice(ctx, type, host_gguf, rows, k, rank * n, n, 0, k, out);
    }
    // row-parallel: a range of input columns, whole blocks
    if (k % ((int64_t)nranks * g.block_elems))
        return set_err(ctx, EF_ERR_SHAPE, "shard: k=%lld is not %d ranks x whole blocks of %d", (long long)k, nranks,
                       g.block_elems);
    const int64_t n = k / nranks;
    return ef_weight_load_slice(ctx, type, host_gguf, rows, k, 0, rows, rank * n, n, out);
}

int ef_weight_free(ef_ctx *ctx, ef_weight *w) {
    if (!ctx || !w) return EF_ERR_INVALID;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(w->dev);
    delete w;
    return EF_OK;
}

int ef_weight_info(const ef_weight *w, int *type, int64_t *rows, int64_t *k, size_t *bytes) {
    if (!w) return EF_ERR_INVALID;
    if (type) *type = w->type;
    if (rows) *rows = w->rows;
    if (k) *k = w->k;
    if (bytes) *bytes = w->bytes;
    return EF_OK;
}

int ef_weight_unpack(ef_ctx *ctx, const ef_weight *w, void *dev_gguf_out) {
    if (!ctx || !w || !dev_gguf_out) return EF_ERR_INVALID;
    if (int rc = use_device(ctx)) return rc;
    return launch_unpack(ctx, w, (uint8_t *)dev_gguf_out);
}

// -------------------------------------------------------------- operators --
int ef_dequant(ef_ctx *ctx, const ef_weight *w, int64_t row0, int64_t nrows, float *out) {
    if (!ctx || !w || !out) return EF_ERR_INVALID;
    if (row0 < 0 || nrows <= 0 || row0 + nrows > w->rows)
        return set_err(ctx, EF_ERR_RANGE, "dequant rows [%lld,+%lld) outside %lld rows", (long long)row0,
                       (long long)nrows, (long long)w->rows);
    if (int rc = use_device(ctx)) return rc;
    return launch_dequant(ctx, w, row0, nrows, out);
}

int ef_gather(ef_ctx *ctx, const ef_weight *w, const int *dev_ids, int tokens, float *out) {
    if (!ctx || !w || !dev_ids || !out) return EF_ERR_INVALID;
    if (tokens < 1) return set_err(ctx, EF_ERR_SHAPE, "gather: tokens=%d < 1", tokens);
    if (int rc = use_device(ctx)) return rc;
    return launch_gather(ctx, w, dev_ids, tokens, out);
}

int ef_gather_rmsnorm(ef_ctx *ctx, const ef_weight *w, const int *dev_ids, int tokens, const float *w_norm, float eps,
                      float *x, float *nrm) {
    if (!ctx || !w || !dev_ids || !w_norm || !x || !nrm) return EF_ERR_INVALID;
    if (tokens < 1 || tokens > 65535) return set_err(ctx, EF_ERR_SHAPE, "gather_rmsnorm: tokens=%d", tokens);
    if (int rc = use_device(ctx)) return rc;
    return launch_gather_norm(ctx, w, dev_ids, tokens, w_norm, eps, x, nrm);
}

static int check_gemv(ef_ctx *ctx, const ef_weight *w, const float *x, int M, const void *y) {
    if (!w || !x || !y) return set_err(ctx, EF_ERR_INVALID, "gemv: null argument");
    if (M < 1) return set_err(ctx, EF_ERR_SHAPE, "gemv: M=%d < 1", M);
    if (M > 16) return EF_NOT_APPLICABLE;
    if (!aligned16(x)) return set_err(ctx, EF_ERR_INVALID, "gemv: x must be 16-byte aligned");
    return EF_OK;
}

int ef_gemv(ef_ctx *ctx, const ef_weight *w, const float *x, int M, float *y) {
    if (!ctx) return EF_ERR_INVALID;
    if (int rc = check_gemv(ctx, w, x, M, y)) return rc;
    if (int rc = use_device(ctx)) return rc;
    float *ys[1] = {y};
    return launch_gemv(ctx, &w, 1, nullptr, x, M, ys);
}

int ef_gemv_swiglu(ef_ctx *ctx, const ef_weight *wg, const ef_weight *wu, const float *x, int M, float *y) {
    if (!ctx) return EF_ERR_INVALID;
    if (int rc = check_gemv(ctx, wg, x, M, y)) return rc;
    if (!wu) return set_err(ctx, EF_ERR_INVALID, "gemv_swiglu: null up weight");
    if (wu->type != wg->type || wu->rows != wg->rows || wu->k != wg->k)
        return set_err(ctx, EF_ERR_MISMATCH, "gemv_swiglu: gate and up differ in type or shape");
    if (int rc = use_device(ctx)) return rc;
    float *ys[1] = {y};
    return launch_gemv(ctx, &wg, 1, wu, x, M, ys);
}

int ef_gemv_sections(ef_ctx *ctx, const ef_weight *const *ws, int n, const float *x, int M, float *const *ys) {
    if (!ctx) return EF_ERR_INVALID;
    if (!ws || !ys || n < 1 || n > 4) return set_err(ctx, EF_ERR_INVALID, "gemv_sections: n=%d (1..4)", n);
    for (int i = 0; i < n; i++) {
        if (int rc = check_gemv(ctx, ws[i], x, M, ys[i])) return rc;
        if (ws[i]->type != ws[0]->type || ws[i]->k != ws[0]->k)
            return set_err(ctx, EF_ERR_MISMATCH, "gemv_sections: all sections need the same type and k");
    }
    if (int rc = use_device(ctx)) return rc;
    return launch_gemv(ctx, ws, n, nullptr, x, M, ys);
}

int ef_gemm(ef_ctx *ctx, const ef_weight *w, const void *x, int x_type, int M, float *y, uint32_t flags) {
    if (!ctx) return EF_ERR_INVALID;
    if (!w || !x || !y) return set_err(ctx, EF_ERR_INVALID, "gemm: null argument");
    if (M < 1) return set_err(ctx, EF_ERR_SHAPE, "gemm: M=%d < 1", M);
    if (x_type != EF_F16 && x_type != EF_F32) return set_err(ctx, EF_ERR_TYPE, "gemm: x_type %d", x_type);
    if (flags) return set_err(ctx, EF_ERR_INVALID, "gemm: flags must be 0");
    if (!aligned16(x) || !aligned16(y)) return set_err(ctx, EF_ERR_INVALID, "gemm: x and y must be 16-byte aligned");
    if (int rc = use_device(ctx)) return rc;
    return launch_gemm(ctx, w, x, x_type, M, y);
}

int ef_gemm_status(ef_ctx *ctx) {
    if (!ctx) return EF_ERR_INVALID;
    if (int rc = use_device(ctx)) return rc;
    return gemm_status(ctx);
}

int ef_gemm_set_wait_limit(ef_ctx *ctx, int polls) {
    if (!ctx) return EF_ERR_INVALID;
    if (int rc = use_device(ctx)) return rc;
    return gemm_set_wait_limit(ctx, polls);
}

int ef_matmul(ef_ctx *ctx, const ef_weight *w, const float *x, int tokens, float *y) {
    if (!ctx) return EF_ERR_INVALID;
    if (tokens <= 16) return ef_gemv(ctx, w, x, tokens, y);
    return ef_gemm(ctx, w, x, EF_F32, tokens, y, 0);
}

}  // extern "C"

// comm.cu -- the tensor-parallel decode's small collectives over NVLink peer
// memory (sm_100a): one-shot all-reduce (sum) and all-gather between the
// ranks of one node, one process per GPU.
//
// The reference runs on one device and has no collectives; these are the
// exchanges of a Megatron-style split of the decode step (row-parallel
// attn_output / ffn_down / shortconv.out_proj outputs summed over the ranks,
// the sharded head's argmax pairs gathered).
//
// Design: every rank maps every other rank's exchange buffer (CUDA IPC, plain
// peer stores -- no multicast). A call is TP_CTAS CTAs per GPU, CTA b owning
// one contiguous part of the data: it stores its part into slot
// [parity][rank] of every rank's buffer (its own included), publishes it with
// a system-scope release store of its epoch into each rank's flag [b][rank],
// waits (bounded) until every rank's flag [b][.] in its own buffer has
// reached that epoch (acquire), then reads the slots in rank order -- the sum
// is the same on every rank, bit for bit. Epochs count calls per CTA index
// and live in device memory, so calls can be captured in a CUDA graph and
// replayed. Two slot parities: a CTA can be at most one call ahead of the
// same CTA on any other rank, so it never overwrites words still being read.
// A wait that runs out sets the buffer's error word, skips the read and
// returns; every later call returns at once, and the host reads the status.
//
// Fused form (ef_gemv_allreduce_norm): the row-parallel GEMV itself stores its
// output rows into slot [parity][rank] of a second data region of every rank
// and each of its CTAs adds 1 to counter [parity][rank] of every rank
// (gemv.cu, GemvPush); ef_tp_norm_kernel waits until every rank's counter has
// reached the GEMV's CTA count, sums the slots in rank order and applies the
// post-norm + residual + next norm of the decoder. Its last CTA clears the
// parity's counters and advances the call counter that gives the parity. A
// rank can be at most one call ahead of another here too, so it only ever
// writes the other parity's slots and counters.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "internal.h"

constexpr int TP_CTAS = 32;          // CTAs per call (fixed: the per-CTA epochs must stay in step)
constexpr size_t TP_CTRL_BYTES = 4096;

struct ef_tp {
    int rank = 0, nranks = 1, device = 0;
    size_t slot_bytes = 0;           // per rank per parity
    size_t data_bytes = 0;           // 2 * nranks * slot_bytes
    // [2][nranks][slot_bytes] data (collectives) | [2][nranks][slot_bytes] data (fused GEMV) | control:
    // flags u32 [TP_CTAS][nranks] | epoch u32 [TP_CTAS] | error u32 | counters u32 [2][nranks] |
    // fused call counter u32 | CTAs done u32
    uint8_t *buf = nullptr;
    uint8_t *peer[EF_TP_MAX_RANKS] = {};
    bool opened[EF_TP_MAX_RANKS] = {};
    int64_t timeout_ns = 2000000000;
};

namespace ef {

struct TpArgs {
    uint8_t *peer[EF_TP_MAX_RANKS];
    int rank, nranks;
    int64_t slot_bytes, data_bytes, timeout_ns;   // the control block is at 2 * data_bytes
};

// control block words of a rank's buffer
struct TpCtl {
    uint32_t *flags, *epoch, *error, *ctr, *fepoch, *fdone;
};
__host__ __device__ inline TpCtl tp_ctl(uint8_t *buf, int64_t data_bytes, int nranks) {
    TpCtl c;
    c.flags = reinterpret_cast<uint32_t *>(buf + 2 * data_bytes);
    c.epoch = c.flags + TP_CTAS * nranks;
    c.error = c.epoch + TP_CTAS;
    c.ctr = c.error + 1;
    c.fepoch = c.ctr + 2 * nranks;
    c.fdone = c.fepoch + 1;
    return c;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// SUM: dst[i] = sum over ranks r (in order) of rank r's src[i], n floats.
// !SUM: dst[r * n + i] = rank r's src[i], n 4-byte words.
template <bool SUM>
__global__ void __launch_bounds__(256) ef_tp_kernel(const TpArgs a, const uint32_t *__restrict__ src, int64_t n,
                                                 uint32_t *__restrict__ dst) {
    pdl_trigger();
    pdl_wait();
    __shared__ uint32_t ep, bad;
    const int cb = blockIdx.x;
    uint8_t *mine = a.peer[a.rank];
    const TpCtl ctl = tp_ctl(mine, a.data_bytes, a.nranks);
    uint32_t *flags = ctl.flags, *epoch = ctl.epoch, *error = ctl.error;
    if (threadIdx.x == 0) {
        bad = *(volatile uint32_t *)error;
        ep = *(volatile uint32_t *)(epoch + cb) + 1;
    }
    __syncthreads();
    if (bad) return;
    // this CTA's part: [i0, i1), in whole 16-byte pieces except at the end
    const int64_t per = ((n + TP_CTAS - 1) / TP_CTAS + 3) / 4 * 4;
    const int64_t i0 = cb * per < n ? cb * per : n, i1 = i0 + per < n ? i0 + per : n;
    const int parity = ep & 1;
    const int64_t off = ((int64_t)parity * a.nranks + a.rank) * a.slot_bytes;
    const bool vec = ((uintptr_t)src % 16) == 0;
    for (int r = 0; r < a.nranks; r++) {
        uint32_t *d = reinterpret_cast<uint32_t *>(a.peer[r] + off);
        int64_t i = i0;
        if (vec) {
            const int64_t nv = (i1 - i0) / 4;
            for (int64_t j = threadIdx.x; j < nv; j += blockDim.x)
                reinterpret_cast<uint4 *>(d + i0)[j] = reinterpret_cast<const uint4 *>(src + i0)[j];
            i = i0 + 4 * nv;
        }
        for (int64_t j = i + threadIdx.x; j < i1; j += blockDim.x) d[j] = src[j];
    }
    // the CTA barrier orders every thread's stores before the flag stores,
    // and a release is cumulative over what happens before it
    __syncthreads();
    if (threadIdx.x < a.nranks) {
        uint32_t *f = tp_ctl(a.peer[threadIdx.x], a.data_bytes, a.nranks).flags + cb * a.nranks + a.rank;
        st_release_sys(f, ep);
    }
    // wait for every rank's part of this call (bounded)
    if (threadIdx.x < a.nranks) {
        const uint64_t t0 = global_ns();
        while ((int32_t)(ld_acquire_sys(flags + cb * a.nranks + threadIdx.x) - ep) < 0) {
            if ((int64_t)(global_ns() - t0) > a.timeout_ns) {
                atomicExch(error, 1u + threadIdx.x);
                bad = 1;
                break;
            }
            __nanosleep(20);
        }
    }
    __syncthreads();
    if (bad) return;
    const uint8_t *slots = mine + (int64_t)parity * a.nranks * a.slot_bytes;
    if (SUM) {
        float *df = reinterpret_cast<float *>(dst);
        for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
            float s = 0.f;
            for (int r = 0; r < a.nranks; r++) s += reinterpret_cast<const float *>(slots + r * a.slot_bytes)[i];
            df[i] = s;
        }
    } else {
        for (int r = 0; r < a.nranks; r++) {
            const uint32_t *sr = reinterpret_cast<const uint32_t *>(slots + r * a.slot_bytes);
            for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) dst[r * n + i] = sr[i];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *(volatile uint32_t *)(epoch + cb) = ep;
}

// Consumer of the fused row-parallel GEMV: row blockIdx.x of o = sum over
// ranks (in order) of the slots; then x += rmsnorm(o) * w_post (or += o without
// w_post) and nrm = rmsnorm(x) * w_next, as ef_norm_add_norm_kernel.
template <int V>
__global__ void __launch_bounds__(256) ef_tp_norm_kernel(const TpArgs a, uint32_t expected,
                                                      const float *__restrict__ w_post, float *__restrict__ x,
                                                      const float *__restrict__ w_next, int n, float eps,
                                                      float *__restrict__ nrm) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    __shared__ uint32_t par, ep, bad;
    uint8_t *mine = a.peer[a.rank];
    const TpCtl ctl = tp_ctl(mine, a.data_bytes, a.nranks);
    if (threadIdx.x == 0) {
        bad = *(volatile uint32_t *)ctl.error;
        ep = *(volatile uint32_t *)ctl.fepoch;
        par = ep & 1;
    }
    __syncthreads();
    if (bad) return;
    if (threadIdx.x < a.nranks) {
        const uint32_t *c = ctl.ctr + par * a.nranks + threadIdx.x;
        const uint64_t t0 = global_ns();
        while (ld_acquire_sys(c) < expected) {
            if ((int64_t)(global_ns() - t0) > a.timeout_ns) {
                atomicExch(ctl.error, 1u + threadIdx.x);
                bad = 1;
                break;
            }
            __nanosleep(20);
        }
    }
    __syncthreads();
    if (bad) return;
    const int64_t row = (int64_t)blockIdx.x * (n / 4);
    const uint8_t *slots = mine + a.data_bytes + (int64_t)par * a.nranks * a.slot_bytes;
    float4 *x4 = reinterpret_cast<float4 *>(x) + row;
    float4 *n4 = reinterpret_cast<float4 *>(nrm) + row;
    const float4 *wp = reinterpret_cast<const float4 *>(w_post), *wn = reinterpret_cast<const float4 *>(w_next);
    float4 ov[V], xv[V];
#pragma unroll
    for (int j = 0; j < V; j++) {
        const int i = threadIdx.x + blockDim.x * j;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < a.nranks; r++) {
            const float4 v = reinterpret_cast<const float4 *>(slots + r * a.slot_bytes)[row + i];
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        ov[j] = s;
        xv[j] = x4[i];
    }
    float s1 = 1.f;
    if (w_post) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < V; j++) ss += ov[j].x * ov[j].x + ov[j].y * ov[j].y + ov[j].z * ov[j].z + ov[j].w * ov[j].w;
        s1 = rsqrtf(block_sum(ss, red) / (float)n + eps);
    }
    float ss2 = 0.f;
#pragma unroll
    for (int j = 0; j < V; j++) {
        const int i = threadIdx.x + blockDim.x * j;
        const float4 w4 = w_post ? wp[i] : make_float4(1.f, 1.f, 1.f, 1.f);
        xv[j].x += ov[j].x * s1 * w4.x;
        xv[j].y += ov[j].y * s1 * w4.y;
        xv[j].z += ov[j].z * s1 * w4.z;
        xv[j].w += ov[j].w * s1 * w4.w;
        ss2 += xv[j].x * xv[j].x + xv[j].y * xv[j].y + xv[j].z * xv[j].z + xv[j].w * xv[j].w;
        x4[i] = xv[j];
    }
    const float s2 = rsqrtf(block_sum(ss2, red) / (float)n + eps);
#pragma unroll
    for (int j = 0; j < V; j++) {
        const int i = threadIdx.x + blockDim.x * j;
        const float4 w4 = wn[i];
        n4[i] = make_float4(xv[j].x * s2 * w4.x, xv[j].y * s2 * w4.y, xv[j].z * s2 * w4.z, xv[j].w * s2 * w4.w);
    }
    // the last CTA clears this parity's counters and advances the call counter
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(ctl.fdone, 1u) == gridDim.x - 1) {
            for (int r = 0; r < a.nranks; r++) ctl.ctr[par * a.nranks + r] = 0;
            *ctl.fdone = 0;
            __threadfence();
            *(volatile uint32_t *)ctl.fepoch = ep + 1;
        }
    }
}

static TpArgs tp_args(ef_tp *tp) {
    TpArgs a = {};
    for (int r = 0; r < tp->nranks; r++) a.peer[r] = tp->peer[r];
    a.rank = tp->rank;
    a.nranks = tp->nranks;
    a.slot_bytes = (int64_t)tp->slot_bytes;
    a.data_bytes = (int64_t)tp->data_bytes;
    a.timeout_ns = tp->timeout_ns;
    return a;
}

static int tp_launch(ef_ctx *ctx, ef_tp *tp, bool sum, const void *src, int64_t words, void *dst) {
    TpArgs a = {};
    for (int r = 0; r < tp->nranks; r++) {
        if (!tp->peer[r]) return set_err(ctx, EF_ERR_INVALID, "tp: rank %d is not connected", r);
        a.peer[r] = tp->peer[r];
    }
    a.rank = tp->rank;
    a.nranks = tp->nranks;
    a.slot_bytes = (int64_t)tp->slot_bytes;
    a.data_bytes = (int64_t)tp->data_bytes;
    a.timeout_ns = tp->timeout_ns;
    if (sum)
        return launch_on(ctx, ef_tp_kernel<true>, TP_CTAS, 256, 0, "allreduce launch", a, (const uint32_t *)src, words,
                         (uint32_t *)dst);
    return launch_on(ctx, ef_tp_kernel<false>, TP_CTAS, 256, 0, "allgather launch", a, (const uint32_t *)src, words,
                     (uint32_t *)dst);
}

}  // namespace ef

using namespace ef;

extern "C" {

int ef_tp_create(ef_ctx *ctx, int rank, int nranks, size_t max_bytes, double timeout_s, ef_tp **out) {
    if (!ctx || !out || nranks < 1 || nranks > EF_TP_MAX_RANKS || rank < 0 || rank >= nranks || max_bytes == 0 ||
        !(timeout_s > 0))
        return ctx ? set_err(ctx, EF_ERR_INVALID, "tp_create: bad arguments") : EF_ERR_INVALID;
    if (int rc = check_cuda(ctx, cudaSetDevice(ctx->device), "set device")) return rc;
    ef_tp *tp = new ef_tp();
    tp->rank = rank;
    tp->nranks = nranks;
    tp->device = ctx->device;
    tp->slot_bytes = (max_bytes + 255) / 256 * 256;
    tp->data_bytes = 2 * (size_t)nranks * tp->slot_bytes;
    tp->timeout_ns = (int64_t)(timeout_s * 1e9);
    const size_t total = 2 * tp->data_bytes + TP_CTRL_BYTES;
    int rc = check_cuda(ctx, cudaMalloc(&tp->buf, total), "tp buffer alloc");
    if (!rc) rc = check_cuda(ctx, cudaMemset(tp->buf, 0, total), "tp buffer clear");
    if (rc) {
        if (tp->buf) cudaFree(tp->buf);
        delete tp;
        return rc;
    }
    tp->peer[rank] = tp->buf;
    *out = tp;
    return EF_OK;
}

int ef_tp_handle(ef_ctx *ctx, const ef_tp *tp, void *handle_out) {
    if (!ctx || !tp || !handle_out) return ctx ? set_err(ctx, EF_ERR_INVALID, "tp_handle: bad arguments") : EF_ERR_INVALID;
    cudaIpcMemHandle_t h;
    if (int rc = check_cuda(ctx, cudaIpcGetMemHandle(&h, tp->buf), "ipc handle")) return rc;
    static_assert(sizeof(h) == EF_TP_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    return EF_OK;
}

int ef_tp_connect(ef_ctx *ctx, ef_tp *tp, const void *handles) {
    if (!ctx || !tp || !handles) return ctx ? set_err(ctx, EF_ERR_INVALID, "tp_connect: bad arguments") : EF_ERR_INVALID;
    if (int rc = check_cuda(ctx, cudaSetDevice(tp->device), "set device")) return rc;
    for (int r = 0; r < tp->nranks; r++) {
        if (r == tp->rank || tp->opened[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *)handles + (size_t)r * EF_TP_HANDLE_BYTES, sizeof(h));
        void *p = nullptr;
        if (int rc = check_cuda(ctx, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "ipc open"))
            return rc;
        tp->peer[r] = (uint8_t *)p;
        tp->opened[r] = true;
    }
    return EF_OK;
}

int ef_allreduce_sum(ef_ctx *ctx, ef_tp *tp, float *buf, int64_t n) {
    if (!ctx || !tp || !buf || n < 1) return ctx ? set_err(ctx, EF_ERR_INVALID, "allreduce: bad arguments") : EF_ERR_INVALID;
    if ((size_t)n * 4 > tp->slot_bytes)
        return set_err(ctx, EF_ERR_RANGE, "allreduce: %lld floats exceed the %zu-byte slot", (long long)n,
                       tp->slot_bytes);
    return tp_launch(ctx, tp, true, buf, n, buf);
}

int ef_allgather(ef_ctx *ctx, ef_tp *tp, const void *src, int64_t bytes, void *dst) {
    if (!ctx || !tp || !src || !dst || bytes < 4 || bytes % 4)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "allgather: bad arguments") : EF_ERR_INVALID;
    if ((size_t)bytes > tp->slot_bytes)
        return set_err(ctx, EF_ERR_RANGE, "allgather: %lld bytes exceed the %zu-byte slot", (long long)bytes,
                       tp->slot_bytes);
    return tp_launch(ctx, tp, false, src, bytes / 4, dst);
}

int ef_gemv_allreduce_norm(ef_ctx *ctx, ef_tp *tp, const ef_weight *w, const float *x, int M, const float *w_post,
                           float *x_resid, const float *w_next, float eps, float *nrm) {
    if (!ctx || !tp || !w || !x || !x_resid || !w_next || !nrm || M < 1 || M > 16)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "gemv_allreduce_norm: bad arguments") : EF_ERR_INVALID;
    for (int r = 0; r < tp->nranks; r++)
        if (!tp->peer[r]) return set_err(ctx, EF_ERR_INVALID, "tp: rank %d is not connected", r);
    if ((size_t)M * w->rows * 4 > tp->slot_bytes)
        return set_err(ctx, EF_ERR_RANGE, "gemv_allreduce_norm: %d x %lld floats exceed the %zu-byte slot", M,
                       (long long)w->rows, tp->slot_bytes);
    int th = 0;
    const int v = norm_v((int)w->rows, th);
    if (!v || w->rows > 8192)
        return set_err(ctx, EF_ERR_SHAPE, "gemv_allreduce_norm: %lld rows (a multiple of 128 up to 8192)",
                       (long long)w->rows);
    const TpArgs a = tp_args(tp);
    GemvPush push;
    push.n = tp->nranks;
    push.rank = tp->rank;
    push.slot_bytes = (int64_t)tp->slot_bytes;
    for (int r = 0; r < tp->nranks; r++) {
        push.data[r] = tp->peer[r] + tp->data_bytes;
        push.ctr[r] = tp_ctl(tp->peer[r], (int64_t)tp->data_bytes, tp->nranks).ctr;
    }
    push.epoch = tp_ctl(tp->buf, (int64_t)tp->data_bytes, tp->nranks).fepoch;
    int64_t ctas = 0;
    float *ys[1] = {nrm};    // (not written: the output goes to the ranks' slots)
    if (int rc = launch_gemv(ctx, &w, 1, nullptr, x, M, ys, &push, &ctas)) return rc;
    const uint32_t expected = (uint32_t)ctas;
    switch (v) {
    case 1: return launch_on(ctx, ef_tp_norm_kernel<1>, M, th, 0, "tp norm launch", a, expected, w_post, x_resid, w_next,
                             (int)w->rows, eps, nrm);
    case 2: return launch_on(ctx, ef_tp_norm_kernel<2>, M, th, 0, "tp norm launch", a, expected, w_post, x_resid, w_next,
                             (int)w->rows, eps, nrm);
    case 4: return launch_on(ctx, ef_tp_norm_kernel<4>, M, th, 0, "tp norm launch", a, expected, w_post, x_resid, w_next,
                             (int)w->rows, eps, nrm);
    default: return launch_on(ctx, ef_tp_norm_kernel<8>, M, th, 0, "tp norm launch", a, expected, w_post, x_resid,
                              w_next, (int)w->rows, eps, nrm);
    }
}

int ef_tp_status(ef_ctx *ctx, const ef_tp *tp) {
    if (!ctx || !tp) return ctx ? set_err(ctx, EF_ERR_INVALID, "tp_status: bad arguments") : EF_ERR_INVALID;
    uint32_t err = 0;
    const TpCtl c = tp_ctl(tp->buf, (int64_t)tp->data_bytes, tp->nranks);
    if (int rc = check_cuda(ctx, cudaMemcpy(&err, c.error, 4, cudaMemcpyDeviceToHost), "tp status read"))
        return rc;
    if (err) return set_err(ctx, EF_ERR_TIMEOUT, "tp: rank %d did not arrive in time", (int)err - 1);
    return EF_OK;
}

int ef_tp_destroy(ef_ctx *ctx, ef_tp *tp) {
    if (!tp) return EF_ERR_INVALID;
    cudaSetDevice(tp->device);
    if (ctx) cudaStreamSynchronize(ctx->stream);
    for (int r = 0; r < tp->nranks; r++)
        if (tp->opened[r]) cudaIpcCloseMemHandle(tp->peer[r]);
    cudaFree(tp->buf);
    delete tp;
    return EF_OK;
}

}  // extern "C"

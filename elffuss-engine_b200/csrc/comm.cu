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
// peer stores -- no multicast). Every word travels stamped: one 8-byte store
// of (epoch << 32 | word), so the data is its own flag -- the reader polls
// the words themselves until each carries this call's epoch, with no release
// fence and no separate flag store after the data (one NVLink crossing per
// exchange instead of data + fence round trip + flag). A call is TP_CTAS
// CTAs per GPU, CTA b owning one contiguous part of the data: it stores its
// part, stamped, into slot [parity][rank] of every other rank's buffer, then
// reads every other rank's slot words of its part (bounded wait on each
// stamp) and combines them with its own source words in rank order -- the
// sum is the same on every rank, bit for bit. Epochs count calls per CTA
// index (every call runs every CTA, so they are all equal) and live in device
// memory, so calls can be captured in a CUDA graph and replayed. Two slot
// parities: a rank that writes call e+2 into a slot has seen every rank's
// data of call e+1, which each rank wrote only after its call e had ended,
// so no word is overwritten while it is still read; a stale word carries an
// older epoch and is never taken for a new one. A wait that runs out sets the
// buffer's error word, skips the output and returns; every later call
// returns at once, and the host reads the status.
//
// Fused form (ef_gemv_allreduce_norm): the row-parallel GEMV itself stores its
// output rows, stamped with the fused call counter, into slot [parity][rank]
// of a second data region of every rank (gemv.cu, GemvPush);
// ef_tp_norm_kernel waits until every word of its row carries that counter,
// sums the slots in rank order and applies the post-norm + residual + next
// norm of the decoder. Its last CTA advances the call counter.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

constexpr int TP_CTAS = 32;          // CTAs per call (fixed: the per-CTA epochs must stay in step)
constexpr size_t TP_CTRL_BYTES = 4096;

struct ef_tp {
    int rank = 0, nranks = 1, device = 0;
    size_t slot_bytes = 0;           // payload bytes per rank per parity (stamped: twice that)
    size_t data_bytes = 0;           // 2 * nranks * 2 * slot_bytes
    // [2][nranks][2 * slot_bytes] data (collectives) | [2][nranks][2 * slot_bytes] data (fused GEMV) |
    // control: epoch u32 [TP_CTAS] | error u32 | fused call counter u32 | CTAs done u32
    uint8_t *buf = nullptr;
    uint8_t *peer[EF_TP_MAX_RANKS] = {};
    bool opened[EF_TP_MAX_RANKS] = {};
    int64_t timeout_ns = 2000000000;
};

namespace ef {

struct TpArgs {
    uint8_t *peer[EF_TP_MAX_RANKS];
    int rank, nranks;
    int64_t slot_bytes, data_bytes, timeout_ns;   // stamped slot bytes; the control block is at 2 * data_bytes
};

// control block words of a rank's buffer
struct TpCtl {
    uint32_t *epoch, *error, *fepoch, *fdone;
};
__host__ __device__ inline TpCtl tp_ctl(uint8_t *buf, int64_t data_bytes) {
    TpCtl c;
    c.epoch = reinterpret_cast<uint32_t *>(buf + 2 * data_bytes);
    c.error = c.epoch + TP_CTAS;
    c.fepoch = c.error + 1;
    c.fdone = c.fepoch + 1;
    return c;
}

// stamped words: (epoch << 32 | word), one single-copy-atomic 8-byte access each
__device__ __forceinline__ void st_stamped(uint64_t *p, uint32_t w, uint32_t ep) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(((uint64_t)ep << 32) | w) : "memory");
}
__device__ __forceinline__ void st_stamped2(uint64_t *p, uint32_t w0, uint32_t w1, uint32_t ep) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(((uint64_t)ep << 32) | w0),
                 "l"(((uint64_t)ep << 32) | w1)
                 : "memory");
}
__device__ __forceinline__ uint64_t ld_stamped(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ld_stamped2(const uint64_t *p, uint64_t &v0, uint64_t &v1) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// The word at p once its stamp is ep. Bounded: once `late` is set (by this
// wait or an earlier one of the thread) it returns at once.
__device__ __forceinline__ uint32_t wait_stamped(const uint64_t *p, uint32_t ep, uint64_t t0, int64_t limit,
                                                 bool &late) {
    uint64_t v = ld_stamped(p);
    while ((uint32_t)(v >> 32) != ep && !late) {
        if ((int64_t)(global_ns() - t0) > limit) late = true;
        v = ld_stamped(p);
    }
    return (uint32_t)v;
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
    const TpCtl ctl = tp_ctl(mine, a.data_bytes);
    if (threadIdx.x == 0) {
        bad = *(volatile uint32_t *)ctl.error;
        ep = *(volatile uint32_t *)(ctl.epoch + cb) + 1;
    }
    __syncthreads();
    if (bad) return;
    const uint32_t e = ep;
    // this CTA's part: [i0, i1), in whole 16-byte pieces except at the end
    const int64_t per = ((n + TP_CTAS - 1) / TP_CTAS + 3) / 4 * 4;
    const int64_t i0 = cb * per < n ? cb * per : n, i1 = i0 + per < n ? i0 + per : n;
    const int parity = e & 1;
    const int64_t off = ((int64_t)parity * a.nranks + a.rank) * a.slot_bytes;
    const bool vec = ((uintptr_t)src % 16) == 0;
    for (int r = 0; r < a.nranks; r++) {
        if (r == a.rank) continue;
        uint64_t *d = reinterpret_cast<uint64_t *>(a.peer[r] + off);
        int64_t i = i0;
        if (vec) {
            const int64_t nv = (i1 - i0) / 4;
            for (int64_t j = threadIdx.x; j < nv; j += blockDim.x) {
                const uint4 v = reinterpret_cast<const uint4 *>(src + i0)[j];
                st_stamped2(d + i0 + 4 * j, v.x, v.y, e);
                st_stamped2(d + i0 + 4 * j + 2, v.z, v.w, e);
            }
            i = i0 + 4 * nv;
        }
        for (int64_t j = i + threadIdx.x; j < i1; j += blockDim.x) st_stamped(d + j, src[j], e);
    }
    // every thread's reads of src above before any thread's writes of dst (in place)
    __syncthreads();
    const uint64_t t0 = global_ns();
    bool late = false;
    int who = -1;                           // the first rank whose words did not arrive in time
    const uint64_t *slots = reinterpret_cast<const uint64_t *>(mine + (int64_t)parity * a.nranks * a.slot_bytes);
    const int64_t sw = a.slot_bytes / 8;    // stamped words per slot
    if (SUM) {
        float *df = reinterpret_cast<float *>(dst);
        for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
            float s = 0.f;
            for (int r = 0; r < a.nranks; r++) {
                s += __uint_as_float(r == a.rank ? src[i] : wait_stamped(slots + r * sw + i, e, t0, a.timeout_ns, late));
                if (late && who < 0) who = r;
            }
            if (!late) df[i] = s;
        }
    } else {
        for (int r = 0; r < a.nranks; r++)
            for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
                const uint32_t w = r == a.rank ? src[i] : wait_stamped(slots + r * sw + i, e, t0, a.timeout_ns, late);
                if (late && who < 0) who = r;
                if (!late) dst[r * n + i] = w;
            }
    }
    if (__syncthreads_or(late)) {
        if (late) atomicExch(ctl.error, 1u + (uint32_t)who);
        return;
    }
    if (threadIdx.x == 0) *(volatile uint32_t *)(ctl.epoch + cb) = e;
}

// The four words at p (16-byte aligned) once every stamp is ep; bounded like
// wait_stamped.
__device__ __forceinline__ float4 wait_stamped4(const uint64_t *p, uint32_t ep, uint64_t t0, int64_t limit,
                                                bool &late) {
    uint64_t v0, v1, v2, v3;
    for (;;) {
        ld_stamped2(p, v0, v1);
        ld_stamped2(p + 2, v2, v3);
        const bool ok = (uint32_t)(v0 >> 32) == ep && (uint32_t)(v1 >> 32) == ep && (uint32_t)(v2 >> 32) == ep &&
                        (uint32_t)(v3 >> 32) == ep;
        if (ok || late) break;
        if ((int64_t)(global_ns() - t0) > limit) late = true;
    }
    return make_float4(__uint_as_float((uint32_t)v0), __uint_as_float((uint32_t)v1), __uint_as_float((uint32_t)v2),
                       __uint_as_float((uint32_t)v3));
}

// Consumer of the fused row-parallel GEMV: row blockIdx.x of o = sum over
// ranks (in order) of the slots; then x += rmsnorm(o) * w_post (or += o without
// w_post) and nrm = rmsnorm(x) * w_next, as ef_norm_add_norm_kernel.
// It works as soon as it is scheduled, without waiting for the GEMV's grid to
// complete (which includes the acknowledgement of the GEMV's stores to the
// other ranks): the GEMV's rows arrive stamped, and everything else it reads
// (the call counter, x, the norm weights) was written by kernels that had
// completed before the GEMV passed its own wait, which it does before it lets
// this kernel be scheduled. It waits for the GEMV's completion only before it
// exits, so that completion stays transitive for the kernels after it.
template <int V>
__global__ void __launch_bounds__(256) ef_tp_norm_kernel(const TpArgs a, const float *__restrict__ w_post,
                                                      float *__restrict__ x, const float *__restrict__ w_next, int n,
                                                      float eps, float *__restrict__ nrm) {
    pdl_trigger();
    __shared__ float red[32];
    __shared__ uint32_t ep, bad;
    uint8_t *mine = a.peer[a.rank];
    const TpCtl ctl = tp_ctl(mine, a.data_bytes);
    if (threadIdx.x == 0) {
        bad = *(volatile uint32_t *)ctl.error;
        ep = *(volatile uint32_t *)ctl.fepoch + 1;   // this call's number (the GEMV's stamp)
    }
    __syncthreads();
    if (bad) {
        pdl_wait();
        return;
    }
    const uint32_t e = ep;
    const int64_t row = (int64_t)blockIdx.x * (n / 4);
    const uint64_t *slots =
        reinterpret_cast<const uint64_t *>(mine + a.data_bytes + (int64_t)(e & 1) * a.nranks * a.slot_bytes);
    const int64_t sw = a.slot_bytes / 8;    // stamped words per slot
    float4 *x4 = reinterpret_cast<float4 *>(x) + row;
    float4 *n4 = reinterpret_cast<float4 *>(nrm) + row;
    const float4 *wp = reinterpret_cast<const float4 *>(w_post), *wn = reinterpret_cast<const float4 *>(w_next);
    const uint64_t t0 = global_ns();
    bool late = false;
    int who = -1;
    float4 ov[V], xv[V];
#pragma unroll
    for (int j = 0; j < V; j++) {
        const int i = threadIdx.x + blockDim.x * j;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < a.nranks; r++) {
            const float4 v = wait_stamped4(slots + r * sw + 4 * (row + i), e, t0, a.timeout_ns, late);
            if (late && who < 0) who = r;
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        ov[j] = s;
        xv[j] = x4[i];
    }
    if (__syncthreads_or(late)) {
        if (late) atomicExch(ctl.error, 1u + (uint32_t)who);
        pdl_wait();
        return;
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
    // the last CTA advances the call counter
    __syncthreads();
    if (threadIdx.x == 0) {
        if (atomicAdd(ctl.fdone, 1u) == gridDim.x - 1) {
            *ctl.fdone = 0;
            *(volatile uint32_t *)ctl.fepoch = e;
        }
    }
    pdl_wait();                      // the GEMV has completed before this kernel does
}

// Consumer of the fused row-sharded GEMV (ef_gemv_allgather): dst[r * n + i]
// = rank r's y[i] (n = M x its rows), read from the ranks' stamped slots of
// the fused region; bounded waits as above. Like ef_tp_norm_kernel it works as
// soon as it is scheduled and waits for the GEMV's completion only before it
// exits; its last CTA advances the fused call counter.
__global__ void __launch_bounds__(256) ef_tp_gather_kernel(const TpArgs a, int64_t n, float *__restrict__ dst) {
    pdl_trigger();
    __shared__ uint32_t ep, bad;
    uint8_t *mine = a.peer[a.rank];
    const TpCtl ctl = tp_ctl(mine, a.data_bytes);
    if (threadIdx.x == 0) {
        bad = *(volatile uint32_t *)ctl.error;
        ep = *(volatile uint32_t *)ctl.fepoch + 1;   // this call's number (the GEMV's stamp)
    }
    __syncthreads();
    if (bad) {
        pdl_wait();
        return;
    }
    const uint32_t e = ep;
    const uint64_t *slots =
        reinterpret_cast<const uint64_t *>(mine + a.data_bytes + (int64_t)(e & 1) * a.nranks * a.slot_bytes);
    const int64_t sw = a.slot_bytes / 8;    // stamped words per slot
    const uint64_t t0 = global_ns();
    bool late = false;
    int who = -1;
    const int64_t total = (int64_t)a.nranks * n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / n);
        const uint32_t w = wait_stamped(slots + r * sw + (i - (int64_t)r * n), e, t0, a.timeout_ns, late);
        if (late) {
            if (who < 0) who = r;
            break;
        }
        dst[i] = __uint_as_float(w);
    }
    if (__syncthreads_or(late)) {
        if (late) atomicExch(ctl.error, 1u + (uint32_t)who);
        pdl_wait();
        return;
    }
    if (threadIdx.x == 0) {
        if (atomicAdd(ctl.fdone, 1u) == gridDim.x - 1) {
            *ctl.fdone = 0;
            *(volatile uint32_t *)ctl.fepoch = e;
        }
    }
    pdl_wait();                      // the GEMV has completed before this kernel does
}

static TpArgs tp_args(ef_tp *tp) {
    TpArgs a = {};
    for (int r = 0; r < tp->nranks; r++) a.peer[r] = tp->peer[r];
    a.rank = tp->rank;
    a.nranks = tp->nranks;
    a.slot_bytes = 2 * (int64_t)tp->slot_bytes;
    a.data_bytes = (int64_t)tp->data_bytes;
    a.timeout_ns = tp->timeout_ns;
    return a;
}

static int tp_connected(ef_ctx *ctx, const ef_tp *tp) {
    for (int r = 0; r < tp->nranks; r++)
        if (!tp->peer[r]) return set_err(ctx, EF_ERR_INVALID, "tp: rank %d is not connected", r);
    return EF_OK;
}

static int tp_launch(ef_ctx *ctx, ef_tp *tp, bool sum, const void *src, int64_t words, void *dst) {
    if (int rc = tp_connected(ctx, tp)) return rc;
    const TpArgs a = tp_args(tp);
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
    tp->data_bytes = 2 * (size_t)nranks * 2 * tp->slot_bytes;
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
    if (int rc = tp_connected(ctx, tp)) return rc;
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
    push.slot_bytes = a.slot_bytes;
    for (int r = 0; r < tp->nranks; r++) push.data[r] = tp->peer[r] + tp->data_bytes;
    push.epoch = tp_ctl(tp->buf, (int64_t)tp->data_bytes).fepoch;
    float *ys[1] = {nrm};    // (not written: the output goes to the ranks' slots)
    if (int rc = launch_gemv(ctx, &w, 1, nullptr, x, M, ys, &push)) return rc;
    switch (v) {
    case 1: return launch_on(ctx, ef_tp_norm_kernel<1>, M, th, 0, "tp norm launch", a, w_post, x_resid, w_next,
                             (int)w->rows, eps, nrm);
    case 2: return launch_on(ctx, ef_tp_norm_kernel<2>, M, th, 0, "tp norm launch", a, w_post, x_resid, w_next,
                             (int)w->rows, eps, nrm);
    case 4: return launch_on(ctx, ef_tp_norm_kernel<4>, M, th, 0, "tp norm launch", a, w_post, x_resid, w_next,
                             (int)w->rows, eps, nrm);
    default: return launch_on(ctx, ef_tp_norm_kernel<8>, M, th, 0, "tp norm launch", a, w_post, x_resid, w_next,
                              (int)w->rows, eps, nrm);
    }
}

int ef_gemv_allgather(ef_ctx *ctx, ef_tp *tp, const ef_weight *w, const float *x, int M, float *yall) {
    if (!ctx || !tp || !w || !x || !yall || M < 1 || M > 16)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "gemv_allgather: bad arguments") : EF_ERR_INVALID;
    if (int rc = tp_connected(ctx, tp)) return rc;
    const int64_t n = (int64_t)M * w->rows;
    if ((size_t)n * 4 > tp->slot_bytes)
        return set_err(ctx, EF_ERR_RANGE, "gemv_allgather: %d x %lld floats exceed the %zu-byte slot", M,
                       (long long)w->rows, tp->slot_bytes);
    const TpArgs a = tp_args(tp);
    GemvPush push;
    push.n = tp->nranks;
    push.rank = tp->rank;
    push.slot_bytes = a.slot_bytes;
    for (int r = 0; r < tp->nranks; r++) push.data[r] = tp->peer[r] + tp->data_bytes;
    push.epoch = tp_ctl(tp->buf, (int64_t)tp->data_bytes).fepoch;
    float *ys[1] = {yall};   // (not written by the GEMV: its output goes to the ranks' slots)
    if (int rc = launch_gemv(ctx, &w, 1, nullptr, x, M, ys, &push)) return rc;
    const int64_t total = (int64_t)tp->nranks * n;
    const int ctas = (int)std::min<int64_t>(128, std::max<int64_t>(1, (total + 2047) / 2048));
    return launch_on(ctx, ef_tp_gather_kernel, ctas, 256, 0, "tp gather launch", a, n, yall);
}

int ef_tp_status(ef_ctx *ctx, const ef_tp *tp) {
    if (!ctx || !tp) return ctx ? set_err(ctx, EF_ERR_INVALID, "tp_status: bad arguments") : EF_ERR_INVALID;
    uint32_t err = 0;
    const TpCtl c = tp_ctl(tp->buf, (int64_t)tp->data_bytes);
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

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
    // [2][nranks][slot_bytes] data | flags u32 [TP_CTAS][nranks] | epoch u32 [TP_CTAS] | error u32
    uint8_t *buf = nullptr;
    uint8_t *peer[EF_TP_MAX_RANKS] = {};
    bool opened[EF_TP_MAX_RANKS] = {};
    int64_t timeout_ns = 2000000000;
};

namespace ef {

struct TpArgs {
    uint8_t *peer[EF_TP_MAX_RANKS];
    int rank, nranks;
    int64_t slot_bytes, data_bytes, timeout_ns;
};

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
__global__ void __launch_bounds__(256) tp_kernel(const TpArgs a, const uint32_t *__restrict__ src, int64_t n,
                                                 uint32_t *__restrict__ dst) {
    pdl_trigger();
    pdl_wait();
    __shared__ uint32_t ep, bad;
    const int cb = blockIdx.x;
    uint8_t *mine = a.peer[a.rank];
    uint32_t *flags = reinterpret_cast<uint32_t *>(mine + a.data_bytes);          // [TP_CTAS][nranks]
    uint32_t *epoch = flags + TP_CTAS * a.nranks, *error = epoch + TP_CTAS;
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
        uint32_t *f = reinterpret_cast<uint32_t *>(a.peer[threadIdx.x] + a.data_bytes) + cb * a.nranks + a.rank;
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
        return launch_on(ctx, tp_kernel<true>, TP_CTAS, 256, 0, "allreduce launch", a, (const uint32_t *)src, words,
                         (uint32_t *)dst);
    return launch_on(ctx, tp_kernel<false>, TP_CTAS, 256, 0, "allgather launch", a, (const uint32_t *)src, words,
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
    const size_t total = tp->data_bytes + TP_CTRL_BYTES;
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

int ef_tp_status(ef_ctx *ctx, const ef_tp *tp) {
    if (!ctx || !tp) return ctx ? set_err(ctx, EF_ERR_INVALID, "tp_status: bad arguments") : EF_ERR_INVALID;
    uint32_t err = 0;
    const size_t at = tp->data_bytes + 4 * ((size_t)TP_CTAS * tp->nranks + TP_CTAS);
    if (int rc = check_cuda(ctx, cudaMemcpy(&err, tp->buf + at, 4, cudaMemcpyDeviceToHost), "tp status read"))
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

// gemm.cu -- prefill GEMM on the 5th-generation tensor cores (sm_100a).
//
//   y[t][r] = sum_k f16(dequant(W)[r][k]) * f16(x[t][k])      f32 accumulate
//
// The reference's prefill kernel (GEMM2 "exacto", js/kernels.gemm2.wgsl.js:
// 12-23,174-240) dequantises a tile of W to f16 in shared memory and
// multiplies it with f16 activations, accumulating in f32. Here the same
// contract runs as a tcgen05 pipeline:
//
//   producer (1 thread):  cp.async.bulk of the repacked weight tiles (8
//                         rowgroup tiles of 2176 B = 128 rows x 128 k) and a
//                         TMA load (128B swizzle, no multicast) of the f16
//                         activation tile, completing on one mbarrier;
//   dequant (4 warps):    one thread per weight row expands its 128 quants to
//                         f16(d*q) and writes them in the K-major 128B-swizzle
//                         layout the MMA reads (A operand, double-buffered);
//   MMA (1 thread):       tcgen05.mma.kind::f16, M=128 (weight rows) x N=BN
//                         (tokens) x K=16, accumulator in tensor memory;
//   epilogue (4 warps):   tcgen05.ld of the accumulator, coalesced f32 stores
//                         of y[token][row].
// Every wait on an mbarrier is bounded: past the limit the kernel records an
// error code, stops issuing work and still releases its tensor memory.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace ef {

constexpr int GM_BM = 128;     // weight rows per CTA tile (MMA M)
constexpr int GM_BK = 128;     // k per pipeline step (one Q8_0 rowgroup tile)
constexpr int GM_THREADS = 192;
constexpr uint32_t GM_WAIT_LIMIT = 1u << 24;   // try_wait polls before giving up (about a second)

__device__ int g_gemm_error;   // nonzero after a bounded wait gave up

// ------------------------------------------------------------ PTX wrappers --
// (mbarrier and bulk-copy helpers are in common.cuh)
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity, GM_WAIT_LIMIT)) return true;
    atomicExch(&g_gemm_error, 1);
    return false;
}
__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte-swizzled operand: 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);         // start address
    d |= (uint64_t)1 << 16;                          // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;                // stride byte offset
    d |= (uint64_t)1 << 46;                          // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                          // layout: 128B swizzle
    return d;
}
__device__ __forceinline__ void umma_f16(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

template <int BN>
__global__ void __launch_bounds__(GM_THREADS, 1)
    gemm_q8_0_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                     int64_t nchunks, int64_t rows, int M, float *__restrict__ y) {
    constexpr int S = 3;                                 // raw (W + X) pipeline stages
    constexpr int WRAW = 8 * 2176;                       // 8 rowgroup tiles
    constexpr int XBYTES = 2 * BN * 128;                 // two 64-k boxes of BN rows x 128 B
    constexpr int ABYTES = 2 * GM_BM * 128;              // two 64-k atoms of 128 rows x 128 B
    constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(GM_BM >> 4) << 24);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled operand tiles
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *xs = smem;                                  // S x XBYTES
    uint8_t *as = xs + S * XBYTES;                       // 2 x ABYTES
    uint8_t *ws = as + 2 * ABYTES;                       // S x WRAW
    uint64_t *bars = reinterpret_cast<uint64_t *>(ws + S * WRAW);
    uint64_t *full = bars, *empty = bars + S, *afull = bars + 2 * S, *aempty = bars + 2 * S + 2;
    uint64_t *tfull = bars + 2 * S + 4;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2 * S + 5);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rb = blockIdx.x;                       // 8 rowgroups = 128 rows
    const int n0 = blockIdx.y * BN;                      // first token
    const int nk = (int)nchunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&afull[b], 128);
            mbar_init(&aempty[b], 1);
        }
        mbar_init(tfull, 1);
        mbar_init_fence();
    }
    if (warp == 1) {   // tensor memory: BN f32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {   // ---------------------------------------- producer
            const int64_t nrg = rowgroups - rb * 8 < 8 ? rowgroups - rb * 8 : 8;
            const uint32_t tx = (uint32_t)(nrg * 2176 + XBYTES);
            for (int ks = 0; ks < nk && ok; ks++) {
                const int s = ks % S;
                if (ks >= S) ok = mbar_wait(&empty[s], ((ks / S) - 1) & 1);
                if (!ok) break;
                mbar_expect_tx(&full[s], tx);
                for (int i = 0; i < nrg; i++)
                    bulk_g2s(ws + s * WRAW + i * 2176, W + ((rb * 8 + i) * nchunks + ks) * 2176, 2176, &full[s]);
                tma_2d(xs + s * XBYTES, &xmap, ks * GM_BK, n0, &full[s]);
                tma_2d(xs + s * XBYTES + BN * 128, &xmap, ks * GM_BK + 64, n0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // --------------------------------------------- MMA
            for (int ks = 0; ks < nk && ok; ks++) {
                const int s = ks % S, b = ks & 1;
                ok = mbar_wait(&full[s], (ks / S) & 1) && mbar_wait(&afull[b], (ks >> 1) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(as + b * ABYTES), b0 = smem_u32(xs + s * XBYTES);
#pragma unroll
                for (int j = 0; j < GM_BK / 16; j++) {
                    const uint32_t ao = (j >> 2) * (GM_BM * 128) + (j & 3) * 32;
                    const uint32_t bo = (j >> 2) * (BN * 128) + (j & 3) * 32;
                    umma_f16(tmem, sw128_desc(a0 + ao), sw128_desc(b0 + bo), IDESC, (ks | j) != 0);
                }
                umma_commit(&empty[s]);    // X (and W raw) stage reusable when these MMAs finish
                umma_commit(&aempty[b]);   // A buffer reusable
            }
            umma_commit(tfull);            // accumulator complete
        }
    } else {
        // ------------------------------------------------ dequant (128 threads)
        const int r = threadIdx.x - 64;                  // weight row within the tile
        const int rl = r & 15, g = rl & 7, hs = rl >> 3, rg_in = r >> 4;
        const bool have = rb * 8 + rg_in < rowgroups;
        for (int ks = 0; ks < nk && ok; ks++) {
            const int s = ks % S, b = ks & 1;
            ok = mbar_wait(&full[s], (ks / S) & 1);
            if (ok && ks >= 2) ok = mbar_wait(&aempty[b], ((ks >> 1) - 1) & 1);
            if (!ok) break;
            const uint8_t *T = ws + s * WRAW + rg_in * 2176;
            uint8_t *A = as + b * ABYTES;
#pragma unroll
            for (int t = 0; t < 4; t++) {   // block t of the row: k = 32t .. 32t+31
                uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
                uint32_t dd = 0;
                if (have) {
                    q0 = *reinterpret_cast<const uint4 *>(T + (2 * hs) * 512 + (4 * g + t) * 16);
                    q1 = *reinterpret_cast<const uint4 *>(T + (2 * hs + 1) * 512 + (4 * g + t) * 16);
                    const uint32_t sc = *reinterpret_cast<const uint32_t *>(T + 2048 + (4 * g + t) * 4);
                    dd = prmt(sc, 0, hs ? 0x3232 : 0x1010);   // (d, d)
                }
                const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                uint32_t h[16];
#pragma unroll
                for (int i = 0; i < 8; i++) {   // 4 quants (biased by 128) -> 2 x half2 f16(d*q)
                    h[2 * i] = hmul2u(hsub2u(prmt(w[i], 0x64646464u, 0x5140), 0x64806480u), dd);
                    h[2 * i + 1] = hmul2u(hsub2u(prmt(w[i], 0x64646464u, 0x7362), 0x64806480u), dd);
                }
                // 32 f16 = four 16-byte chunks at k = 32t .. 32t+31: atom t>>1,
                // chunk (4*(t&1) + c) XOR (row & 7) of the row's 128 bytes
                uint8_t *rowp = A + (t >> 1) * (GM_BM * 128) + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int chunk = (4 * (t & 1) + c) ^ (r & 7);
                    *reinterpret_cast<uint4 *>(rowp + chunk * 16) =
                        make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
                }
            }
            fence_proxy_async();   // generic-proxy writes -> visible to the tensor core
            mbar_arrive(&afull[b]);
        }
        // ------------------------------------------------------------ epilogue
        if (ok) ok = mbar_wait(tfull, 0);
        tc_fence_after();
        if (ok) {
            const int quad = warp & 3;                   // TMEM lanes 32*quad .. +31
            const int64_t row = rb * GM_BM + quad * 32 + lane;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t v[32];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                      "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                      "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
                      "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
                      "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (row < rows) {
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const int tok = n0 + c0 + j;
                        if (tok < M) y[(int64_t)tok * rows + row] = __uint_as_float(v[j]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    }
}

// f32 -> f16 activations (round to nearest even), for x given in f32.
__global__ void f32_to_f16_kernel(const float *__restrict__ src, __half *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}
__global__ void f16_to_f32_kernel(const __half *__restrict__ src, float *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __half2float(src[i]);
}

// ------------------------------------------------------------------ host ---
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

template <int BN> static size_t gemm_smem() {
    static_assert(BN == 128, "the 256-token tile does not fit 227 KB of shared memory with this pipeline");
    constexpr int S = 3;
    return 1024 + (size_t)S * (2 * BN * 128) + 2 * (2 * GM_BM * 128) + (size_t)S * 8 * 2176 + 256;
}

template <int BN>
static int launch_q8_0(ef_ctx *ctx, const ef_weight *w, const __half *xh, int M, float *y) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_err(ctx, EF_ERR_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)w->k, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)w->k * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)BN};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)xh, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_err(ctx, EF_ERR_CUDA, "gemm: tensor map encode failed (%d)", (int)cr);
    auto kern = gemm_q8_0_kernel<BN>;
    const size_t smem = gemm_smem<BN>();
    static unsigned long long configured = 0;
    if (ctx->device < 64 && !(configured & (1ull << ctx->device))) {
        if (int rc = check_cuda(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                "gemm smem attribute"))
            return rc;
        configured |= 1ull << ctx->device;
    }
    dim3 grid((unsigned)((w->rowgroups + 7) / 8), (unsigned)((M + BN - 1) / BN));
    ctx->launches++;
    kern<<<grid, GM_THREADS, smem, ctx->stream>>>(map, w->dev, w->rowgroups, w->nchunks, w->rows, M, y);
    return check_cuda(ctx, cudaGetLastError(), "gemm launch");
}

int launch_gemm(ef_ctx *ctx, const ef_weight *w, const void *x, int x_type, int M, float *y) {
    if (w->type == EF_Q8_0 && w->k % 8 == 0) {
        // tcgen05 path: activations as f16 [M][K] (converted from f32 if needed)
        const __half *xh = (const __half *)x;
        if (x_type == EF_F32) {
            const int64_t n = (int64_t)M * w->k;
            if (int rc = ensure_scratch(ctx, 1, (size_t)n * 2)) return rc;
            int64_t blocks = (n + 255) / 256;
            if (blocks > 148 * 32) blocks = 148 * 32;
            ctx->launches++;
            f32_to_f16_kernel<<<(int)blocks, 256, 0, ctx->stream>>>((const float *)x, (__half *)ctx->scratch[1], n);
            if (int rc = check_cuda(ctx, cudaGetLastError(), "gemm f32->f16")) return rc;
            xh = (const __half *)ctx->scratch[1];
        }
        return launch_q8_0<128>(ctx, w, xh, M, y);
    }
    // Other types: the token dimension in groups of 16 through the GEMV
    // kernel (same numerics contract: f16 activations, f32 accumulation).
    const float *xf = (const float *)x;
    if (x_type == EF_F16) {
        const int64_t n = (int64_t)M * w->k;
        if (int rc = ensure_scratch(ctx, 1, (size_t)n * 4)) return rc;
        int64_t blocks = (n + 255) / 256;
        if (blocks > 148 * 32) blocks = 148 * 32;
        ctx->launches++;
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

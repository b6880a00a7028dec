// gemm.cu -- prefill GEMM on the 5th-generation tensor cores (sm_100a).
//
//   y[t][r] = sum_k f16(dequant(W)[r][k]) * f16(x[t][k])      f32 accumulate
//
// The reference's prefill kernel (GEMM2 "exacto", js/kernels.gemm2.wgsl.js:
// 12-23,174-240) dequantises a tile of W to f16 and multiplies it with f16
// activations, accumulating in f32. Here the same contract runs as a tcgen05
// pipeline. CTA tile: 128 weight rows (MMA M) x 256 tokens (MMA N).
//
//   producer (1 thread):  per stage of 256 k, one cp.async.bulk per rowgroup
//                         of its repacked chunk tiles (2 x 2176 B for Q8_0,
//                         2 x 1152 B for Q4_0, one 256-k tile of 2304 /
//                         3360 / 2816 / 1344 B for Q4_K / Q6_K / Q5_K / Q2_K:
//                         a rowgroup's chunks are contiguous), 2-4 stages as
//                         shared memory allows; and TMA loads (128B swizzle,
//                         into this CTA only) of the f16 activations, 64 k x
//                         256 tokens per box (4 boxes in flight);
//   dequant (2 x 4 warps): thread = weight row = tensor-memory lane; the two
//                         groups take alternate stages, expand the 256
//                         quants of their row to f16 weights and store them
//                         into tensor memory (tcgen05.st), where the MMA
//                         reads the A operand (one buffer per group);
//   MMA (1 thread):       tcgen05.mma.kind::f16, A from tensor memory, B from
//                         shared memory, M=128 x N=256 x K=16, accumulator in
//                         tensor memory (256 columns);
//   epilogue (8 warps):   tcgen05.ld of the accumulator, coalesced f32 stores
//                         of y[token][row] (each group half of the tokens).
// Keeping A out of shared memory leaves shared-memory bandwidth to the TMA
// writes and the MMA's B reads: about 160 B/clock per SM at full tensor rate
// against 420 for an A operand staged in shared memory at N=128.
// Every wait on an mbarrier is bounded: past the limit the kernel records an
// error code, stops issuing work and still releases its tensor memory.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "gen/iq_grids.h"
#include "internal.h"

namespace ef {

constexpr int GM_BM = 128;     // weight rows per CTA tile (MMA M)
constexpr int GM_BN = 256;     // tokens per CTA tile (MMA N)
constexpr int GM_BKX = 64;     // k per activation stage (one 128-byte swizzle atom)
constexpr int GM_SX = 4;       // activation stages
constexpr uint32_t GM_WAIT_LIMIT = 1u << 24;   // try_wait polls before giving up (about a second)

__device__ int g_gemm_error;   // nonzero after a bounded wait gave up
// Polls a pipeline wait makes before it gives up (GM_WAIT_LIMIT unless a test
// lowers it through ef_gemm_set_wait_limit). The waits that let a CTA's own
// copies and MMAs drain before it exits always use GM_WAIT_LIMIT.
__device__ uint32_t g_gemm_wait_limit = GM_WAIT_LIMIT;

// i-quant codebooks as f16 (8 weights of an entry per 16 bytes, in weight order)
__device__ const __align__(16) uint16_t g_gm_grid_iq2xxs[EF_GRID_IQ2XXS_ENTRIES * 8] = {EF_GRID_IQ2XXS_F16_INIT};
__device__ const __align__(16) uint16_t g_gm_grid_iq1s[EF_GRID_IQ1S_ENTRIES * 8] = {EF_GRID_IQ1S_F16_INIT};

// ------------------------------------------------------------ PTX wrappers --
// (mbarrier and bulk-copy helpers are in common.cuh)
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit) {
    if (mbar_wait_bounded(bar, parity, limit)) return true;
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

__device__ __forceinline__ void umma_f16_ts(uint32_t dtmem, uint32_t atmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(dtmem),
        "r"(atmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 16 consecutive 32-bit tensor-memory columns of this thread's lane
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// Tensor memory: accumulator in columns [0, 256), A buffers in [256, 384) and
// [384, 512) (256 k of f16 pairs each); 512 columns allocated.
constexpr uint32_t GM_TMEM_COLS = 512;
constexpr uint32_t GM_TMEM_A = 256;
constexpr int GM_KW = 256;              // k per pipeline stage (one A buffer)
constexpr int GM_SMEM_MAX = 232448;     // dynamic shared memory a CTA may opt into

// Weight tile of a rowgroup (16 rows x CK k, one repacked chunk) and where its
// scales / row headers start.
template <int TYPE> struct GmTile;
template <> struct GmTile<EF_Q8_0> { static constexpr int BYTES = 2176, SC = 2048, CK = 128; };
template <> struct GmTile<EF_Q4_0> { static constexpr int BYTES = 1152, SC = 1024, CK = 128; };
template <> struct GmTile<EF_Q4_K> { static constexpr int BYTES = 2304, SC = 2048, CK = 256; };
template <> struct GmTile<EF_Q6_K> { static constexpr int BYTES = 3360, SC = 3072, CK = 256; };
template <> struct GmTile<EF_Q5_K> { static constexpr int BYTES = 2816, SC = 2560, CK = 256; };
template <> struct GmTile<EF_Q2_K> { static constexpr int BYTES = 1344, SC = 1024, CK = 256; };
template <> struct GmTile<EF_IQ2_XXS> { static constexpr int BYTES = 1056, SC = 1024, CK = 256; };   // SC: d
template <> struct GmTile<EF_IQ1_S> { static constexpr int BYTES = 800, SC = 768, CK = 256; };        // SC: d
// shared-memory codebook bytes: IQ2_XXS grid (256 x 16) + sign masks (128 x 16); IQ1_S grid (2048 x 16)
template <int TYPE> __host__ __device__ constexpr int gm_tab() {
    return TYPE == EF_IQ2_XXS ? 384 * 16 : TYPE == EF_IQ1_S ? 2048 * 16 : 0;
}
// Threads: producer, MMA, and 2 x 4 dequant / epilogue warps per chunk tile of
// a stage (two tiles of 128 k for Q8_0 / Q4_0, dequantised in parallel by the
// two halves of each group; one 256-k tile for the other types).
template <int TYPE> __host__ __device__ constexpr int gm_threads() { return 64 + 256 * (GM_KW / GmTile<TYPE>::CK); }
// weight stages (each 8 rowgroups x GM_KW) that fit beside the activation ring, at most 4
template <int TYPE> __host__ __device__ constexpr int gm_sw() {
    constexpr int per = 8 * (GM_KW / GmTile<TYPE>::CK) * GmTile<TYPE>::BYTES;
    constexpr int n = (GM_SMEM_MAX - 1024 - GM_SX * GM_BN * 128 - 256 - gm_tab<TYPE>()) / per;
    return n > 4 ? 4 : n;
}

template <int TYPE>
__device__ __forceinline__ void gemm_body(const CUtensorMap &xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                                          int64_t nchunks, int64_t rows, int64_t kdim, int M, float *__restrict__ y) {
    constexpr int TB = GmTile<TYPE>::BYTES, SCO = GmTile<TYPE>::SC, CK = GmTile<TYPE>::CK;
    constexpr int CPS = GM_KW / CK;                      // chunks per stage (contiguous per rowgroup)
    constexpr int NTHR = gm_threads<TYPE>();             // 2 x 4 dequant warps per chunk of a stage
    constexpr int SW = gm_sw<TYPE>();
    constexpr int NBOX = GM_KW / GM_BKX, ACOLS = GM_KW / 2;
    constexpr int WRAW = 8 * CPS * TB;                   // 8 rowgroups x CPS chunk tiles
    constexpr int XBYTES = GM_BN * 128;                  // one 64-k box of 256 rows x 128 B
    constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(GM_BN >> 3) << 17) | ((uint32_t)(GM_BM >> 4) << 24);
    static_assert(SW >= 2, "two weight stages at least (one per dequant group)");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled activation tiles
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *xs = smem;                                  // GM_SX x XBYTES
    uint8_t *ws = xs + GM_SX * XBYTES;                   // SW x WRAW
    uint64_t *bars = reinterpret_cast<uint64_t *>(ws + SW * WRAW);
    uint64_t *xfull = bars, *xempty = bars + GM_SX;
    uint64_t *wfull = bars + 2 * GM_SX, *wempty = bars + 2 * GM_SX + SW;
    uint64_t *afull = bars + 2 * GM_SX + 2 * SW, *aempty = afull + 2, *tfull = afull + 4;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(tfull + 1);
    uint4 *tab = reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(bars) + 256);   // i-quant codebooks

    // Programmatic dependent launch: the next kernel may be scheduled at once
    // (it cannot share this CTA's SM, whose shared memory this one fills);
    // the previous kernel's results are read (activations, by the producer's
    // TMA) and y is written (epilogue) only after griddepcontrol.wait. The
    // set-up, the weight copies and their dequantisation do not depend on it.
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rb = blockIdx.x;                       // 8 rowgroups = 128 rows
    const int n0 = blockIdx.y * GM_BN;                   // first token
    const int nk = (int)((nchunks + CPS - 1) / CPS);     // stages along k
    // chunks in stage kk, and the activation boxes it needs (none wholly past k)
    auto chunks_of = [&](int kk) {
        const int64_t c = nchunks - (int64_t)kk * CPS;
        return c < CPS ? (int)c : CPS;
    };
    auto boxes_of = [&](int kk) {
        const int64_t b = (kdim - (int64_t)kk * GM_KW + GM_BKX - 1) / GM_BKX;
        return b < NBOX ? (int)b : NBOX;
    };

    if constexpr (TYPE == EF_IQ2_XXS) {   // grid, then the sign masks (7 stored bits + even parity)
        const uint4 *src = reinterpret_cast<const uint4 *>(g_gm_grid_iq2xxs);
        for (int i = threadIdx.x; i < 256; i += NTHR) tab[i] = src[i];
        for (int i = threadIdx.x; i < 128; i += NTHR) {
            const uint32_t s8 = (uint32_t)i | ((uint32_t)(__popc(i) & 1) << 7);
            uint32_t w[4];
#pragma unroll
            for (int p = 0; p < 4; p++) w[p] = (((s8 >> (2 * p)) & 1u) << 15) | (((s8 >> (2 * p + 1)) & 1u) << 31);
            tab[256 + i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    } else if constexpr (TYPE == EF_IQ1_S) {
        const uint4 *src = reinterpret_cast<const uint4 *>(g_gm_grid_iq1s);
        for (int i = threadIdx.x; i < 2048; i += NTHR) tab[i] = src[i];
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < GM_SX; s++) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], 1);
        }
        for (int s = 0; s < SW; s++) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], 128 * CPS);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&afull[b], 128 * CPS);
            mbar_init(&aempty[b], 1);
        }
        mbar_init(tfull, 1);
        mbar_init_fence();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(GM_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t lim = g_gemm_wait_limit;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {   // ---------------------------------------- producer
            const int64_t nrg = rowgroups - rb * 8 < 8 ? rowgroups - rb * 8 : 8;
            int wi = 0, xi = 0;                          // copies issued
            // weight stage kk -> slot kk % SW (refilled once the dequant
            // warps have consumed stage kk - SW)
            auto issue_w = [&](int kk) {
                const int sw = kk % SW;
                if (kk >= SW) ok = mbar_wait(&wempty[sw], ((kk / SW) - 1) & 1, lim);
                if (!ok) return;
                const int nc = chunks_of(kk);
                mbar_expect_tx(&wfull[sw], (uint32_t)(nrg * nc * TB));
                for (int i = 0; i < nrg; i++)
                    bulk_g2s(ws + sw * WRAW + i * (CPS * TB), W + ((rb * 8 + i) * nchunks + (int64_t)kk * CPS) * TB,
                             (uint32_t)(nc * TB), &wfull[sw]);
                wi++;
            };
            for (int kk = 0; kk < SW && kk < nk && ok; kk++) issue_w(kk);
            pdl_wait();                                  // the activations come from the kernel before
            for (int kk = 0; kk < nk && ok; kk++) {
                const int nb = boxes_of(kk);
                for (int h = 0; h < nb && ok; h++) {
                    const int sx = xi % GM_SX;
                    if (xi >= GM_SX) ok = mbar_wait(&xempty[sx], ((xi / GM_SX) - 1) & 1, lim);
                    if (!ok) break;
                    mbar_expect_tx(&xfull[sx], XBYTES);
                    tma_2d(xs + sx * XBYTES, &xmap, kk * GM_KW + h * GM_BKX, n0, &xfull[sx]);
                    xi++;
                }
                if (ok && kk + SW < nk) issue_w(kk + SW);
            }
            if (!ok) {   // a wait gave up: let this thread's copies still in flight land first
                for (int j = wi > SW ? wi - SW : 0; j < wi; j++)
                    mbar_wait_bounded(&wfull[j % SW], (j / SW) & 1, GM_WAIT_LIMIT);
                for (int j = xi > GM_SX ? xi - GM_SX : 0; j < xi; j++)
                    mbar_wait_bounded(&xfull[j % GM_SX], (j / GM_SX) & 1, GM_WAIT_LIMIT);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // --------------------------------------------- MMA
            int xc = 0;                              // activation boxes consumed
            for (int kk = 0; kk < nk && ok; kk++) {
                const int b = kk & 1;
                ok = mbar_wait(&afull[b], (kk >> 1) & 1, lim);
                if (!ok) break;
                tc_fence_after();
                const uint32_t abuf = tmem + GM_TMEM_A + ACOLS * b;
                const int nb = boxes_of(kk);
                for (int h = 0; h < nb && ok; h++) {
                    const int sx = xc % GM_SX;
                    ok = mbar_wait(&xfull[sx], (xc / GM_SX) & 1, lim);
                    if (!ok) break;
                    xc++;
                    tc_fence_after();
                    const uint32_t b0 = smem_u32(xs + sx * XBYTES);
#pragma unroll
                    for (int j = 0; j < GM_BKX / 16; j++)
                        umma_f16_ts(tmem, abuf + 32 * h + 8 * j, sw128_desc(b0 + 32 * j), IDESC, (kk | h | j) != 0);
                    umma_commit(&xempty[sx]);   // activation stage reusable when these MMAs finish
                }
                umma_commit(&aempty[b]);       // A buffer reusable
            }
            umma_commit(tfull);                // accumulator complete
            // Whether or not a wait gave up, every MMA issued above must finish
            // before tensor memory is freed and the CTA's shared memory is
            // released (the epilogue warps skip their wait after a failure).
            mbar_wait_bounded(tfull, 0, GM_WAIT_LIMIT);
        }
    } else {
        // ------------------------ dequant (2 groups of 4 warps = 128 rows each,
        // per chunk of a stage) Group G handles the stages kk = G, G+2, ... (A
        // buffer G); with two chunks per stage, half h of the group the chunk h.
        // Thread = weight row r = tensor-memory lane: warp w
        // owns lanes 32*(w%4) .. +31. Row r of the tile is row g + 8hs of rowgroup r>>4;
        // its block t (32 quants) is two 16-byte parts of fragment lane 4g+t
        // and its f16 scale sits at 2048 + 4(4g+t) + 2hs. The four blocks are
        // read in a lane-staggered order, so one 128-bit shared load by the 32
        // lanes touches each bank group four times (no conflicts).
        const int quad = warp & 3, grp = ((warp - 2) >> 2) & 1, half = (warp - 2) >> 3;
        const int r = quad * 32 + lane;
        const int rl = r & 15, g = rl & 7, hs = rl >> 3, rg_in = r >> 4;
        const bool have = rb * 8 + rg_in < rowgroups;
        const uint32_t tlane = (uint32_t)(quad * 32) << 16;
        for (int kk = grp; kk < nk && ok; kk += 2) {
            const int sw = kk % SW, b = kk & 1;
            ok = mbar_wait(&wfull[sw], (kk / SW) & 1, lim);
            if (ok && kk >= 2) ok = mbar_wait(&aempty[b], ((kk >> 1) - 1) & 1, lim);
            if (!ok) break;
            tc_fence_after();
            const int nc = CPS == 1 ? 1 : chunks_of(kk);
#pragma unroll 1
            for (int ch = half; ch < nc; ch += CPS) {
            const uint8_t *T = ws + sw * WRAW + rg_in * (CPS * TB) + ch * TB;
            const uint32_t abuf = tmem + tlane + GM_TMEM_A + ACOLS * b + (CK / 2) * ch;
            if constexpr (TYPE == EF_Q6_K) {
                // Row r = g + 8hs: for lane column t and step s (32 weights) a
                // low-nibble word at part 2hs + (s>>2), offset 4(s&3) of lane
                // 4g+t (byte b: k = 32s + 4t + b in bits 0-3, 32s + 16 + 4t + b
                // in bits 4-7); for step pair sp a high-bit word at part 4 + hs,
                // offset 4sp (byte b: bits 0-1 / 2-3 = halves 0 / 1 of step 2sp,
                // 4-5 / 6-7 = those of step 2sp+1); 16 int8 scales at 3072 + 16 rl
                // (one per 16 weights); f16 d at 3328 + 4g + 2hs.
                uint4 lo[4][2], hi[4], scv = make_uint4(0, 0, 0, 0);
                uint32_t dbits = 0;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const uint8_t *P = T + (4 * g + t) * 16;
                    lo[t][0] = have ? *reinterpret_cast<const uint4 *>(P + (2 * hs) * 512) : make_uint4(0, 0, 0, 0);
                    lo[t][1] = have ? *reinterpret_cast<const uint4 *>(P + (2 * hs + 1) * 512) : make_uint4(0, 0, 0, 0);
                    hi[t] = have ? *reinterpret_cast<const uint4 *>(P + (4 + hs) * 512) : make_uint4(0, 0, 0, 0);
                }
                if (have) {
                    scv = *reinterpret_cast<const uint4 *>(T + SCO + 16 * rl);
                    dbits = *reinterpret_cast<const unsigned short *>(T + 3328 + 4 * g + 2 * hs);
                }
                const float d = __half2float(__ushort_as_half((unsigned short)dbits));
                const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
                auto wd = [](const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; };
#pragma unroll
                for (int st = 0; st < 8; st++) {
                    // f16(d * sc) of sub-blocks 2st (half 0) and 2st+1 (half 1)
                    const int s0 = (int)(int8_t)((scw[st >> 1] >> (16 * (st & 1))) & 0xFF);
                    const int s1 = (int)(int8_t)((scw[st >> 1] >> (16 * (st & 1) + 8)) & 0xFF);
                    const uint32_t d0 = (uint32_t)__half_as_ushort(__float2half_rn(d * (float)s0)) * 0x10001u;
                    const uint32_t d1 = (uint32_t)__half_as_ushort(__float2half_rn(d * (float)s1)) * 0x10001u;
                    uint32_t h[16];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        const uint32_t w = wd(lo[t][st >> 2], st & 3), hw = wd(hi[t], st >> 1);
                        const uint32_t g0 = (st & 1) ? hw : hw << 4, g1 = (st & 1) ? hw >> 2 : hw << 2;
                        const uint32_t q0 = (w & 0x0F0F0F0Fu) | (g0 & 0x30303030u);          // k = 32st + 4t + b
                        const uint32_t q1 = ((w >> 4) & 0x0F0F0F0Fu) | (g1 & 0x30303030u);   // k = 32st + 16 + 4t + b
                        // (1024 + q) - (1024 + 32) = q - 32, exact in f16
                        h[2 * t] = hmul2u(hsub2u(prmt(q0, 0x64646464u, 0x5140), 0x64206420u), d0);
                        h[2 * t + 1] = hmul2u(hsub2u(prmt(q0, 0x64646464u, 0x7362), 0x64206420u), d0);
                        h[8 + 2 * t] = hmul2u(hsub2u(prmt(q1, 0x64646464u, 0x5140), 0x64206420u), d1);
                        h[9 + 2 * t] = hmul2u(hsub2u(prmt(q1, 0x64646464u, 0x7362), 0x64206420u), d1);
                    }
                    tmem_st16(abuf + 16 * st, h);   // k = 32st .. 32st+31 as 16 f16 pairs
                }
            } else if constexpr (TYPE == EF_Q5_K) {
                // Row r = g + 8hs: lane column t holds the 64 weights 64t..: qs
                // bytes 0..31 at parts 2hs, 2hs+1 of lane 4g+t (low nibble:
                // weight 64t + b, sub-block 2t; high nibble: 64t + 32 + b,
                // sub-block 2t+1), their fifth bits as two words (bit l of
                // weight 64t + l / 64t + 32 + l) at part 4, offset 8hs; the row's
                // header (d, dmin, scale_min_k4 bytes) at 2560 + 16 rl.
                uint4 qs[4][2], hdr = make_uint4(0, 0, 0, 0);
                uint2 fb[4];
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const uint8_t *P = T + (4 * g + t) * 16;
                    qs[t][0] = have ? *reinterpret_cast<const uint4 *>(P + (2 * hs) * 512) : make_uint4(0, 0, 0, 0);
                    qs[t][1] = have ? *reinterpret_cast<const uint4 *>(P + (2 * hs + 1) * 512) : make_uint4(0, 0, 0, 0);
                    fb[t] = have ? *reinterpret_cast<const uint2 *>(P + 4 * 512 + 8 * hs) : make_uint2(0, 0);
                }
                if (have) hdr = *reinterpret_cast<const uint4 *>(T + SCO + 16 * rl);
                const uint32_t hw[4] = {hdr.x, hdr.y, hdr.z, hdr.w};
                auto hbyte = [&](int i) { return (int)((hw[i >> 2] >> (8 * (i & 3))) & 0xFF); };
                const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFF)));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
#pragma unroll
                for (int t = 0; t < 4; t++) {
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        const int sb = 2 * t + u;
                        int sc, mn;
                        if (sb < 4) {
                            sc = hbyte(4 + sb) & 63;
                            mn = hbyte(8 + sb) & 63;
                        } else {
                            sc = (hbyte(8 + sb) & 0xF) | ((hbyte(sb) >> 6) << 4);
                            mn = (hbyte(8 + sb) >> 4) | ((hbyte(4 + sb) >> 6) << 4);
                        }
                        const uint32_t d2 = f16x2_bcast(d * (float)sc), m2 = f16x2_bcast(-(dmin * (float)mn));
                        const uint32_t bits = u ? fb[t].y : fb[t].x;
                        uint32_t h[16];
#pragma unroll
                        for (int w = 0; w < 8; w++) {   // weights 64t + 32u + 4w .. +3
                            const uint32_t raw = wsel(qs[t][w >> 2], w & 3);
                            const uint32_t q = ((u ? raw >> 4 : raw) & 0x0F0F0F0Fu) | (spread4((bits >> (4 * w)) & 0xF) << 4);
                            h[2 * w] = f16_pair_dm(q, 0x5140, d2, m2);
                            h[2 * w + 1] = f16_pair_dm(q, 0x7362, d2, m2);
                        }
                        tmem_st16(abuf + 32 * t + 16 * u, h);   // k = 64t + 32u .. +31 as 16 f16 pairs
                    }
                }
            } else if constexpr (TYPE == EF_Q2_K) {
                // Row r = g + 8hs: lane column t holds the 64 weights 64t.. =
                // sub-blocks 4t..4t+3 of 16 weights: part hs of lane 4g+t, word
                // w (sub-block 4t + w), byte c, bits 2s'..2s'+1 = the 2-bit q of
                // weight 64t + 16w + 4s' + c; the sub-blocks' scale bytes (low
                // nibble sc, high nibble m) at 1024 + 8(4g+t) + 4hs; the row's
                // f16 d, dmin at 1280 + 4 rl.
                uint4 qv[4];
                uint32_t scb[4], dmw = 0;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    qv[t] = have ? *reinterpret_cast<const uint4 *>(T + hs * 512 + (4 * g + t) * 16) : make_uint4(0, 0, 0, 0);
                    scb[t] = have ? *reinterpret_cast<const uint32_t *>(T + SCO + 8 * (4 * g + t) + 4 * hs) : 0u;
                }
                if (have) dmw = *reinterpret_cast<const uint32_t *>(T + 1280 + 4 * rl);
                const float d = __half2float(__ushort_as_half((unsigned short)(dmw & 0xFFFF)));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(dmw >> 16)));
#pragma unroll
                for (int t = 0; t < 4; t++) {
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        uint32_t h[16];
#pragma unroll
                        for (int ww = 0; ww < 2; ww++) {
                            const int w = 2 * hf + ww;
                            const uint32_t sc = (scb[t] >> (8 * w)) & 0xFF;
                            const uint32_t d2 = f16x2_bcast(d * (float)(sc & 15));
                            const uint32_t m2 = f16x2_bcast(-(dmin * (float)(sc >> 4)));
                            const uint32_t word = wsel(qv[t], w);
#pragma unroll
                            for (int sp = 0; sp < 4; sp++) {   // weights 64t + 16w + 4sp .. +3
                                const uint32_t q = (word >> (2 * sp)) & 0x03030303u;
                                h[8 * ww + 2 * sp] = f16_pair_dm(q, 0x5140, d2, m2);
                                h[8 * ww + 2 * sp + 1] = f16_pair_dm(q, 0x7362, d2, m2);
                            }
                        }
                        tmem_st16(abuf + 32 * t + 16 * hf, h);   // k = 64t + 32hf .. +31
                    }
                }
            } else if constexpr (TYPE == EF_IQ2_XXS) {
                // Row r = g + 8hs: lane column t holds 32-blocks 2t, 2t+1
                // (weights 64t..): their GGUF bytes at part hs of lane 4g+t, per
                // block u a word of four grid indices and a word of four 7-bit
                // sign indices with the 4-bit scale on top; f16 d at
                // 1024 + 4g + 2hs. Weight 8l + j of a block = db * grid * sign
                // (kernels.wgsl.js:368-396), db = f16(d * (0.5 + s) / 4).
                uint4 qv[4];
                uint32_t dbits = 0;
#pragma unroll
                for (int t = 0; t < 4; t++)
                    qv[t] = have ? *reinterpret_cast<const uint4 *>(T + hs * 512 + (4 * g + t) * 16) : make_uint4(0, 0, 0, 0);
                if (have) dbits = *reinterpret_cast<const unsigned short *>(T + SCO + 4 * g + 2 * hs);
                const float d = __half2float(__ushort_as_half((unsigned short)dbits));
                const uint4 *grid = tab, *sgn = tab + 256;
#pragma unroll
                for (int t = 0; t < 4; t++) {
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        const uint32_t a0 = u ? qv[t].z : qv[t].x, a1 = u ? qv[t].w : qv[t].y;
                        const uint32_t db = f16x2_bcast(d * (0.5f + (float)(a1 >> 28)) * 0.25f);
                        uint32_t h[16];
#pragma unroll
                        for (int l = 0; l < 4; l++) {
                            const uint4 G = grid[(a0 >> (8 * l)) & 0xFF], S = sgn[(a1 >> (7 * l)) & 127];
                            h[4 * l] = hmul2u(G.x ^ S.x, db);
                            h[4 * l + 1] = hmul2u(G.y ^ S.y, db);
                            h[4 * l + 2] = hmul2u(G.z ^ S.z, db);
                            h[4 * l + 3] = hmul2u(G.w ^ S.w, db);
                        }
                        tmem_st16(abuf + 32 * t + 16 * u, h);   // k = 64t + 32u .. +31
                    }
                }
            } else if constexpr (TYPE == EF_IQ1_S) {
                // Row r = g + 8hs: lane column t holds 32-blocks 2t, 2t+1: their
                // qs bytes (one word per block) at 16(4g+t) + 8hs, their qh
                // halves at 512 + 8(4g+t) + 4hs; f16 d at 768 + 4g + 2hs. Weight
                // 8l + j = dl * (grid + delta) (kernels.wgsl.js:805-822), grid
                // entry qs byte l | qh bits 3l..3l+2 << 8, delta -/+ 1/8 by qh
                // bit 15, dl = f16(d * (2 * qh[12..14] + 1)).
                uint2 qs[4];
                uint32_t qh[4], dbits = 0;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    qs[t] = have ? *reinterpret_cast<const uint2 *>(T + (4 * g + t) * 16 + 8 * hs) : make_uint2(0, 0);
                    qh[t] = have ? *reinterpret_cast<const uint32_t *>(T + 512 + (4 * g + t) * 8 + 4 * hs) : 0u;
                }
                if (have) dbits = *reinterpret_cast<const unsigned short *>(T + SCO + 4 * g + 2 * hs);
                const float d = __half2float(__ushort_as_half((unsigned short)dbits));
#pragma unroll
                for (int t = 0; t < 4; t++) {
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        const uint32_t q = u ? qs[t].y : qs[t].x, hh = (qh[t] >> (16 * u)) & 0xFFFFu;
                        const uint32_t del = (hh & 0x8000u) ? 0xB000B000u : 0x30003000u;   // -/+ 0.125
                        const uint32_t dl = f16x2_bcast(d * (float)(2u * ((hh >> 12) & 7u) + 1u));
                        uint32_t h[16];
#pragma unroll
                        for (int l = 0; l < 4; l++) {
                            const uint4 G = tab[((q >> (8 * l)) & 0xFF) | (((hh >> (3 * l)) & 7) << 8)];
                            h[4 * l] = hmul2u(hadd2u(G.x, del), dl);   // grid + delta exact in f16
                            h[4 * l + 1] = hmul2u(hadd2u(G.y, del), dl);
                            h[4 * l + 2] = hmul2u(hadd2u(G.z, del), dl);
                            h[4 * l + 3] = hmul2u(hadd2u(G.w, del), dl);
                        }
                        tmem_st16(abuf + 32 * t + 16 * u, h);   // k = 64t + 32u .. +31
                    }
                }
            } else if constexpr (TYPE == EF_Q4_K) {
                // Row r: header (d, dmin, scale_min_k4 bytes) at 2048 + 16 rl; the
                // qs bytes [4t, 4t+4) and [16+4t, 16+4t+4) of group j in lane
                // 4g+t's part 2hs + (j>>1) at offset 8(j&1). Low nibbles of group
                // j are k = 64j + l (sub-block 2j), high nibbles k = 64j + 32 + l.
                uint4 hdr = make_uint4(0, 0, 0, 0);
                uint2 pc[4][4];
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int tt = 0; tt < 4; tt++)
                        pc[j][tt] = have ? *reinterpret_cast<const uint2 *>(T + (2 * hs + (j >> 1)) * 512 +
                                                                           (4 * g + tt) * 16 + 8 * (j & 1))
                                         : make_uint2(0, 0);
                if (have) hdr = *reinterpret_cast<const uint4 *>(T + SCO + 16 * rl);
                const uint32_t hw[4] = {hdr.x, hdr.y, hdr.z, hdr.w};
                auto hbyte = [&](int i) { return (int)((hw[i >> 2] >> (8 * (i & 3))) & 0xFF); };
                const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFF)));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
#pragma unroll
                for (int j = 0; j < 4; j++) {
#pragma unroll
                    for (int u = 0; u < 2; u++) {           // u = 0: sub-block 2j (low nibbles), 1: 2j+1
                        const int sb = 2 * j + u;
                        int sc, mn;
                        if (sb < 4) {
                            sc = hbyte(4 + sb) & 63;
                            mn = hbyte(8 + sb) & 63;
                        } else {
                            sc = (hbyte(8 + sb) & 0xF) | ((hbyte(sb) >> 6) << 4);
                            mn = (hbyte(8 + sb) >> 4) | ((hbyte(4 + sb) >> 6) << 4);
                        }
                        const __half dh = __float2half_rn(d * (float)sc), mh = __float2half_rn(-(dmin * (float)mn));
                        const uint32_t d2 = (uint32_t)__half_as_ushort(dh) * 0x10001u;
                        const uint32_t m2 = (uint32_t)__half_as_ushort(mh) * 0x10001u;
                        uint32_t h[16];
#pragma unroll
                        for (int tt = 0; tt < 4; tt++) {
#pragma unroll
                            for (int v = 0; v < 2; v++) {   // v = 0: bytes 4tt.., 1: 16+4tt..
                                const uint32_t w = pc[j][tt].x * (v == 0) + pc[j][tt].y * (v == 1);
                                const uint32_t q = u ? (w >> 4) & 0x0F0F0F0Fu : w & 0x0F0F0F0Fu;
                                const int c = 8 * v + 2 * tt;          // column of k = 64j + 32u + 16v + 4tt
                                uint32_t r0, r1;
                                const uint32_t q0 = hsub2u(prmt(q, 0x64646464u, 0x5140), 0x64006400u);
                                const uint32_t q1 = hsub2u(prmt(q, 0x64646464u, 0x7362), 0x64006400u);
                                asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r0) : "r"(q0), "r"(d2), "r"(m2));
                                asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r1) : "r"(q1), "r"(d2), "r"(m2));
                                h[c] = r0;
                                h[c + 1] = r1;
                            }
                        }
                        tmem_st16(abuf + 32 * j + 16 * u, h);   // k = 64j + 32u .. +31 as 16 f16 pairs
                    }
                }
            } else {
            // Q8_0: block t = parts 2hs, 2hs+1 of lane 4g+t; Q4_0: part hs of
            // lane 4g+t (word j = weights 8j..8j+7 at nibble slots 0,16,4,20,...)
            uint4 q0[4], q1[4];
            uint32_t sc[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int t = (i + (lane >> 1)) & 3;
                if (have) {
                    if (TYPE == EF_Q8_0) {
                        q0[i] = *reinterpret_cast<const uint4 *>(T + (2 * hs) * 512 + (4 * g + t) * 16);
                        q1[i] = *reinterpret_cast<const uint4 *>(T + (2 * hs + 1) * 512 + (4 * g + t) * 16);
                    } else {
                        q0[i] = *reinterpret_cast<const uint4 *>(T + hs * 512 + (4 * g + t) * 16);
                        q1[i] = q0[i];
                    }
                    sc[i] = *reinterpret_cast<const uint32_t *>(T + SCO + (4 * g + t) * 4);
                } else {
                    q0[i] = q1[i] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
                    sc[i] = 0;
                }
            }
            // tcgen05.st takes one column address for the whole warp: block t
            // is stored by all lanes at once, each picking it from the slot
            // its staggered load order put it in (i = (t - stagger) mod 4).
            const int stg = (lane >> 1) & 3;
#pragma unroll
            for (int t = 0; t < 4; t++) {
                uint4 a0 = q0[t & 3], a1 = q1[t & 3];
                uint32_t sct = sc[t & 3];
                if (stg == 1) { a0 = q0[(t + 3) & 3]; a1 = q1[(t + 3) & 3]; sct = sc[(t + 3) & 3]; }
                if (stg == 2) { a0 = q0[(t + 2) & 3]; a1 = q1[(t + 2) & 3]; sct = sc[(t + 2) & 3]; }
                if (stg == 3) { a0 = q0[(t + 1) & 3]; a1 = q1[(t + 1) & 3]; sct = sc[(t + 1) & 3]; }
                const uint32_t dd = prmt(sct, 0, hs ? 0x3232 : 0x1010);   // (d, d)
                uint32_t h[16];
                if (TYPE == EF_Q8_0) {
                    const uint32_t w[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
                    for (int j = 0; j < 8; j++) {   // 4 quants (biased by 128) -> 2 x half2 f16(d*q)
                        h[2 * j] = hmul2u(hsub2u(prmt(w[j], 0x64646464u, 0x5140), 0x64806480u), dd);
                        h[2 * j + 1] = hmul2u(hsub2u(prmt(w[j], 0x64646464u, 0x7362), 0x64806480u), dd);
                    }
                } else {
                    const uint32_t w[4] = {a0.x, a0.y, a0.z, a0.w};
#pragma unroll
                    for (int j = 0; j < 4; j++)     // 8 nibbles -> 4 x half2 f16(d*(q-8)), k order
#pragma unroll
                        for (int u = 0; u < 4; u++)
                            h[4 * j + u] = hmul2u(hsub2u(((w[j] >> (4 * u)) & 0x000F000Fu) | 0x64006400u, 0x64086408u),
                                                  dd);
                }
                tmem_st16(abuf + 16 * t, h);   // k = 32t .. 32t+31 as 16 f16 pairs
            }
            }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(&afull[b]);
            // The raw stage is released only after the tensor-memory stores
            // that consume every value read from it. Released right after the
            // shared loads, the next bulk copy into the stage may overtake
            // loads that the compiler scheduled later (wrong Q4_K results when
            // a weight producer of its own refilled stages at once).
            mbar_arrive(&wempty[sw]);
        }
        // ------------------------------------------------------------ epilogue
        if (ok) ok = mbar_wait(tfull, 0, lim);
        tc_fence_after();
        pdl_wait();                  // (long since satisfied: y is written after the kernel before)
        if (ok) {
            const int64_t row = rb * GM_BM + quad * 32 + lane;
            constexpr int EC = GM_BN / (2 * CPS);   // accumulator columns per epilogue group
            const int eg = grp + 2 * half;
#pragma unroll 1
            for (int c0 = eg * EC; c0 < (eg + 1) * EC; c0 += 32) {
                if (n0 + c0 >= M) break;
                uint32_t v[32];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                      "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                      "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
                      "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
                      "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(tmem + tlane + (uint32_t)c0));
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GM_TMEM_COLS) : "memory");
    }
}

// f32 -> f16 activations (round to nearest even), for x given in f32.
__global__ void __launch_bounds__(gm_threads<EF_Q8_0>(), 1)
    ef_gemm_q8_0_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                     int64_t nchunks, int64_t rows, int64_t k, int M, float *__restrict__ y) {
    gemm_body<EF_Q8_0>(xmap, W, rowgroups, nchunks, rows, k, M, y);
}
__global__ void __launch_bounds__(gm_threads<EF_Q4_K>(), 1)
    ef_gemm_q4_k_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                     int64_t nchunks, int64_t rows, int64_t k, int M, float *__restrict__ y) {
    gemm_body<EF_Q4_K>(xmap, W, rowgroups, nchunks, rows, k, M, y);
}
__global__ void __launch_bounds__(gm_threads<EF_Q6_K>(), 1)
    ef_gemm_q6_k_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                     int64_t nchunks, int64_t rows, int64_t k, int M, float *__restrict__ y) {
    gemm_body<EF_Q6_K>(xmap, W, rowgroups, nchunks, rows, k, M, y);
}
__global__ void __launch_bounds__(gm_threads<EF_Q5_K>(), 1)
    ef_gemm_q5_k_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                     int64_t nchunks, int64_t rows, int64_t k, int M, float *__restrict__ y) {
    gemm_body<EF_Q5_K>(xmap, W, rowgroups, nchunks, rows, k, M, y);
}
__global__ void __launch_bounds__(gm_threads<EF_Q2_K>(), 1)
    ef_gemm_q2_k_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                     int64_t nchunks, int64_t rows, int64_t k, int M, float *__restrict__ y) {
    gemm_body<EF_Q2_K>(xmap, W, rowgroups, nchunks, rows, k, M, y);
}
__global__ void __launch_bounds__(gm_threads<EF_IQ2_XXS>(), 1)
    ef_gemm_iq2_xxs_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                        int64_t nchunks, int64_t rows, int64_t k, int M, float *__restrict__ y) {
    gemm_body<EF_IQ2_XXS>(xmap, W, rowgroups, nchunks, rows, k, M, y);
}
__global__ void __launch_bounds__(gm_threads<EF_IQ1_S>(), 1)
    ef_gemm_iq1_s_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                      int64_t nchunks, int64_t rows, int64_t k, int M, float *__restrict__ y) {
    gemm_body<EF_IQ1_S>(xmap, W, rowgroups, nchunks, rows, k, M, y);
}
__global__ void __launch_bounds__(gm_threads<EF_Q4_0>(), 1)
    ef_gemm_q4_0_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t rowgroups,
                     int64_t nchunks, int64_t rows, int64_t k, int M, float *__restrict__ y) {
    gemm_body<EF_Q4_0>(xmap, W, rowgroups, nchunks, rows, k, M, y);
}

__global__ void ef_f32_to_f16_kernel(const float *__restrict__ src, __half *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}
__global__ void ef_f16_to_f32_kernel(const __half *__restrict__ src, float *__restrict__ dst, int64_t n) {
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

template <int TYPE> static size_t gemm_smem() {
    return 1024 + (size_t)GM_SX * (GM_BN * 128) +
           (size_t)gm_sw<TYPE>() * 8 * (GM_KW / GmTile<TYPE>::CK) * GmTile<TYPE>::BYTES + 256 + gm_tab<TYPE>();
}

template <int TYPE>
static int launch_tc(ef_ctx *ctx, const ef_weight *w, const __half *xh, int M, float *y) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_err(ctx, EF_ERR_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)w->k, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)w->k * 2};
    const cuuint32_t box[2] = {GM_BKX, (cuuint32_t)GM_BN};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)xh, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_err(ctx, EF_ERR_CUDA, "gemm: tensor map encode failed (%d)", (int)cr);
    auto kern = TYPE == EF_Q8_0   ? ef_gemm_q8_0_kernel
                : TYPE == EF_Q4_0 ? ef_gemm_q4_0_kernel
                : TYPE == EF_Q4_K ? ef_gemm_q4_k_kernel
                : TYPE == EF_Q5_K ? ef_gemm_q5_k_kernel
                : TYPE == EF_Q2_K ? ef_gemm_q2_k_kernel
                : TYPE == EF_IQ2_XXS ? ef_gemm_iq2_xxs_kernel
                : TYPE == EF_IQ1_S   ? ef_gemm_iq1_s_kernel
                                     : ef_gemm_q6_k_kernel;
    const size_t smem = gemm_smem<TYPE>();
    static std::atomic<unsigned long long> configured{0};   // one bit per device
    if (ctx->device < 64 && !(configured.load() & (1ull << ctx->device))) {
        if (int rc = check_cuda(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                "gemm smem attribute"))
            return rc;
        configured.fetch_or(1ull << ctx->device);
    }
    dim3 grid((unsigned)((w->rowgroups + 7) / 8), (unsigned)((M + GM_BN - 1) / GM_BN));
    return launch_on(ctx, kern, grid, dim3(gm_threads<TYPE>()), smem, "gemm launch", map, (const uint8_t *)w->dev,
                     w->rowgroups, w->nchunks, w->rows, w->k, M, y);
}

// Reads and clears the flag a bounded pipeline wait sets when it gives up.
int gemm_status(ef_ctx *ctx) {
    int flag = 0;
    if (int rc = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "gemm status sync")) return rc;
    if (int rc = check_cuda(ctx, cudaMemcpyFromSymbol(&flag, g_gemm_error, sizeof(int)), "gemm status read"))
        return rc;
    if (!flag) return EF_OK;
    const int zero = 0;
    if (int rc = check_cuda(ctx, cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int)), "gemm status clear"))
        return rc;
    return set_err(ctx, EF_ERR_TIMEOUT, "gemm: a pipeline wait gave up; outputs since the last check are invalid");
}

// Sets the poll count of the pipeline waits (negative: the default, about a
// second; 0: every wait gives up without polling).
int gemm_set_wait_limit(ef_ctx *ctx, int polls) {
    const uint32_t v = polls < 0 ? GM_WAIT_LIMIT : (uint32_t)polls;
    if (int rc = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "gemm wait limit sync")) return rc;
    return check_cuda(ctx, cudaMemcpyToSymbol(g_gemm_wait_limit, &v, sizeof(v)), "gemm wait limit set");
}

int launch_gemm(ef_ctx *ctx, const ef_weight *w, const void *x, int x_type, int M, float *y) {
    // The activation tensor map needs rows of a multiple of 16 bytes (k % 8 == 0),
    // which every GGUF block size (32 or 256 weights) gives.
    if (w->k % 8 == 0) {
        // tcgen05 path: activations as f16 [M][K] (converted from f32 if needed)
        const __half *xh = (const __half *)x;
        if (x_type == EF_F32) {
            const int64_t n = (int64_t)M * w->k;
            if (int rc = ensure_scratch(ctx, 1, (size_t)n * 2)) return rc;
            int64_t blocks = (n + 255) / 256;
            if (blocks > 148 * 32) blocks = 148 * 32;
            ctx->launches++;
            ef_f32_to_f16_kernel<<<(int)blocks, 256, 0, ctx->stream>>>((const float *)x, (__half *)ctx->scratch[1], n);
            if (int rc = check_cuda(ctx, cudaGetLastError(), "gemm f32->f16")) return rc;
            xh = (const __half *)ctx->scratch[1];
        }
        if (w->type == EF_Q8_0) return launch_tc<EF_Q8_0>(ctx, w, xh, M, y);
        if (w->type == EF_Q4_0) return launch_tc<EF_Q4_0>(ctx, w, xh, M, y);
        if (w->type == EF_Q4_K) return launch_tc<EF_Q4_K>(ctx, w, xh, M, y);
        if (w->type == EF_Q5_K) return launch_tc<EF_Q5_K>(ctx, w, xh, M, y);
        if (w->type == EF_Q2_K) return launch_tc<EF_Q2_K>(ctx, w, xh, M, y);
        if (w->type == EF_IQ2_XXS) return launch_tc<EF_IQ2_XXS>(ctx, w, xh, M, y);
        if (w->type == EF_IQ1_S) return launch_tc<EF_IQ1_S>(ctx, w, xh, M, y);
        if (w->type == EF_Q6_K) return launch_tc<EF_Q6_K>(ctx, w, xh, M, y);
    }
    // Otherwise the token dimension in groups of 16 through the GEMV kernel
    // (same numerics contract: f16 activations, f32 accumulation).
    const float *xf = (const float *)x;
    if (x_type == EF_F16) {
        const int64_t n = (int64_t)M * w->k;
        if (int rc = ensure_scratch(ctx, 1, (size_t)n * 4)) return rc;
        int64_t blocks = (n + 255) / 256;
        if (blocks > 148 * 32) blocks = 148 * 32;
        ctx->launches++;
        ef_f16_to_f32_kernel<<<(int)blocks, 256, 0, ctx->stream>>>((const __half *)x, (float *)ctx->scratch[1], n);
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

// gemv.cu -- decode GEMV over repacked GGUF tiles, 1..16 tokens (sm_100a).
//
//   y[t][r] = sum_k dequant(W)[r][k] * x[t][k]        (js/ops.js:827-829)
//   swiglu:  y = silu(Wg.x) * (Wu.x)                   (kernels.gemv.wgsl.js:434-437)
//   sections: several W sharing x and k, one output each (js/ops.gemv.js:192-215)
//
// Design (B200). The GEMV is HBM-bound: every weight byte is read once and
// must be turned into tensor-core operands with as few instructions as
// possible, and enough bytes must be in flight to cover DRAM latency.
//
//  * Weights: each warp owns one 16-row rowgroup and streams its tiles through
//    a private ring of cp.async (LDGSTS, L2-only) shared-memory slots, several
//    tiles ahead of the math. The hardware wait (cp.async.wait_group) needs no
//    spin loop.
//  * Math: quants are expanded IN REGISTERS to f16 A fragments of
//    mma.sync.m16n8k16 (A = 16 weight rows x 16 k, B = 16 k x 8 tokens, f32
//    accumulate). Register-sourced MMA is the right tensor instruction for a
//    GEMV: tcgen05.mma reads A from shared or tensor memory, which would add a
//    store and a read of every dequantised weight.
//  * Activations: a small prep kernel converts x once per call into f16 B
//    fragments (zero-padded to 8/16 tokens) plus, for Q4_K, the per-sub-block
//    sums needed by the "-m*sum(x)" term; each CTA copies its k-slice of that
//    buffer into shared memory with cp.async. The GEMV is launched with
//    programmatic dependent launch, so its weight prefetch overlaps the prep.
//  * Work split: CTA = WARPS rowgroups x one k-slice; the k-slices of a
//    rowblock form one thread-block cluster whose partial sums are added
//    through distributed shared memory in rank order (deterministic, no
//    atomics). A small cost model picks WARPS and the k-split for load
//    balance over the 148 SMs.
//
// Numerics: quants are exact small integers in f16 and the per-block scales
// are applied in f16 with one rounding per weight -- Q8_0: f16(d*q); Q4_K:
// f16(f16(d*sc)*q) with -f16(dmin*m)*sum(x) as one more MMA; IQ2_XXS:
// f16(db)*grid*sign; IQ1_S: f16(dl)*(grid+delta) -- because the 16 k-columns of
// one MMA belong to four different blocks. Q6_K: sc*(q-32) is exact in f16 and
// the superblock d is applied in f32 on the accumulator. x is rounded to f16.
// Products are exact and summed in f32 by the tensor cores.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <stdio.h>
#include <stdlib.h>

#include <algorithm>

#include "common.cuh"
#include "gen/iq_grids.h"
#include "internal.h"

namespace cg = cooperative_groups;

namespace ef {

__device__ const __align__(16) uint16_t g_grid_iq2xxs_f16[EF_GRID_IQ2XXS_ENTRIES * 8] = {EF_GRID_IQ2XXS_F16_INIT};
__device__ const __align__(16) uint16_t g_grid_iq1s_f16[EF_GRID_IQ1S_ENTRIES * 8] = {EF_GRID_IQ1S_F16_INIT};

constexpr uint32_t H2_1024 = 0x64006400u;   // half2(1024, 1024)
constexpr uint32_t H2_1152 = 0x64806480u;   // half2(1152, 1152)
constexpr uint32_t H2_2080 = 0x68106810u;   // half2(2080, 2080)
constexpr int MAX_XS_BYTES = 32 * 1024;     // shared memory for one phase of x fragments
constexpr int RING_PER_WARP = 7 * 1024;     // bytes of weight tiles per warp ring

struct GemvArgs {
    const uint8_t *w[4];      // repacked tiles of each section
    const uint8_t *w_up;      // SwiGLU partner of w[0] (same geometry)
    float *y[4];
    int64_t rows[4];
    int64_t rowgroups[4];
    int rb_end[4];            // cumulative rowblocks per section
    int nmat;
    const uint8_t *xf;        // x data from gemv_xprep: nchunks x xb bytes (5..16 tokens)
    int M;
    int64_t nchunks;
    int cps;                  // chunks per k-slice
    int kslices;
    int phase_chunks;         // chunks of x fragments in shared memory at a time
    int xb;                   // bytes of x data per chunk (f16_xbytes / i8_xbytes)
    const float *x;           // f32 activations [M][K] (fused staging)
    int64_t K;
};

// ---------------------------------------------------------------- traits ---
// STEPS = k16 steps per chunk; inv maps a k-quad (4 consecutive weights of the
// chunk) to the lane column t and the step s that consume it; I8 = the type
// runs on the 8-bit tensor cores with 8-bit activation planes (Q4_K).
template <int TYPE> struct Tr;
template <> struct Tr<EF_Q8_0> {
    static constexpr int CHUNK = 128, STEPS = 8, TILE = 2176, I8 = 0;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 3; s = kq & 7; }
};
template <> struct Tr<EF_Q4_K> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 2304, I8 = 1;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = 2 * (kq & 7) + ((kq >> 3) & 1); }
};
template <> struct Tr<EF_Q6_K> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 3360, I8 = 0;
    __device__ static void inv(int kq, int &t, int &s) {
        t = 2 * (kq >> 5) + ((kq >> 2) & 1);
        s = 4 * ((kq >> 3) & 3) + (kq & 3);
    }
};
template <> struct Tr<EF_IQ2_XXS> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 1056, I8 = 0;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = kq & 15; }
};
template <> struct Tr<EF_IQ1_S> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 800, I8 = 0;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = kq & 15; }
};
// bytes of f16 x fragments per chunk for M tokens: STEPS x M x 4 lanes x 8 B
template <int TYPE> __host__ __device__ inline int f16_xbytes(int M) { return Tr<TYPE>::STEPS * M * 32; }
// bytes of 8-bit x data per 256-weight chunk for M tokens (I8 types):
// two int8 planes (high and residual) of B fragments, each
// [8 sub-blocks][M tokens][4 lanes][8 B]; [M][4] f16 pairs of sub-block sums;
// [M] f32 scales; rounded up to 16.
__host__ __device__ inline int i8_xbytes(int M) { return (532 * M + 15) & ~15; }

__device__ __forceinline__ uint32_t wsel(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
// Tile reads: the tiles sit in the warp's shared-memory ring (see the kernel).
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

// Asynchronous global -> shared copies (LDGSTS, L2 only).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
template <int TILE>
__device__ __forceinline__ void copy_tile(uint8_t *dst, const uint8_t *src, int lane) {
#pragma unroll
    for (int p = lane; p < TILE / 16; p += 32) cp_async16(dst + 16 * p, src + 16 * p);
}

// x data of one chunk for the f16 types: B fragments [step][token][lane t]
// (8 B each), tokens 0..M-1 only; lanes whose token is >= M feed zeros.
struct XF {
    const uint8_t *xc;
    int M;
    uint32_t vmask;   // bit nt: token nt*8 + g of this lane exists
};
template <int NT>
__device__ __forceinline__ XF make_xf(const uint8_t *xc, int M, int lane) {
    uint32_t v = 0;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) v |= (uint32_t)(nt * 8 + (lane >> 2) < M) << nt;
    return XF{xc, M, v};
}
template <int NT>
__device__ __forceinline__ void mma_step(float (&acc)[NT][4], const XF &xf, int s, int lane, uint32_t a0,
                                         uint32_t a1, uint32_t a2, uint32_t a3) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const uint2 b = (xf.vmask >> nt) & 1
                            ? *reinterpret_cast<const uint2 *>(xf.xc + (s * xf.M + nt * 8) * 32 + lane * 8)
                            : make_uint2(0u, 0u);
        mma16816(acc[nt], a0, a1, a2, a3, b.x, b.y);
    }
}

__device__ __forceinline__ uint32_t dup_h2(float v) {
    const uint32_t b = __half_as_ushort(__float2half_rn(v));
    return b | (b << 16);
}

// ------------------------------------------------------------------ Q8_0 ---
// lane (g,t) holds block t of rows g and g+8 (biased bytes q+128) and their f16 d.
struct RawQ8 { uint4 q[4]; uint32_t sc; };
__device__ __forceinline__ void load_raw(RawQ8 &r, const uint8_t *T, int lane) {
#pragma unroll
    for (int p = 0; p < 4; p++) r.q[p] = lds128(T + p * 512 + lane * 16);
    r.sc = lds32(T + 2048 + lane * 4);
}
template <int NT>
__device__ __forceinline__ void compute(const RawQ8 &r, const uint8_t *xc, int M, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
    const XF xsc = make_xf<NT>(xc, M, lane);
    const uint32_t dg = prmt(r.sc, 0, 0x1010), dg8 = prmt(r.sc, 0, 0x3232);
#pragma unroll
    for (int s = 0; s < 8; s++) {
        const uint32_t wg = wsel(r.q[s >> 2], s & 3), wg8 = wsel(r.q[2 + (s >> 2)], s & 3);
        // (1024 + q + 128) - 1152 = q exactly; then one rounding of d*q
        const uint32_t a0 = hmul2u(hsub2u(prmt(wg, 0x64646464u, 0x5140), H2_1152), dg);
        const uint32_t a2 = hmul2u(hsub2u(prmt(wg, 0x64646464u, 0x7362), H2_1152), dg);
        const uint32_t a1 = hmul2u(hsub2u(prmt(wg8, 0x64646464u, 0x5140), H2_1152), dg8);
        const uint32_t a3 = hmul2u(hsub2u(prmt(wg8, 0x64646464u, 0x7362), H2_1152), dg8);
        mma_step<NT>(acc, xsc, s, lane, a0, a1, a2, a3);
    }
}

// ------------------------------------------------------------------ Q4_K ---
struct RawQ4K { uint4 q[4]; uint4 hg, hg8; };
__device__ __forceinline__ void load_raw(RawQ4K &r, const uint8_t *T, int lane) {
#pragma unroll
    for (int p = 0; p < 4; p++) r.q[p] = lds128(T + p * 512 + lane * 16);
    const int g = lane >> 2;
    r.hg = lds128(T + 2048 + g * 16);
    r.hg8 = lds128(T + 2048 + (g + 8) * 16);
}
// 8-bit tensor-core MMA: D = A(16x32 u8, row) * B(32x8 s8, col), s32.
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
// (-f16(dmin*m_2t), -f16(dmin*m_2t+1)) of lane column t from a verbatim 16-byte
// Q4_K header (scale_min_k4, kernels.wgsl.js:94-104, for j = 2t, 2t+1).
__device__ __forceinline__ uint32_t q4k_negmin(const uint4 &h, int t) {
    const uint32_t nmm = prmt(h.x, 0, 0x3232) ^ 0x80008000u;
    const int sh = 16 * (t & 1);
    const uint32_t p0 = (h.y >> sh) & 0xFFFF, p1 = (h.z >> sh) & 0xFFFF, p2 = (h.w >> sh) & 0xFFFF;
    const uint32_t mp = t < 2 ? (p1 & 0x3F3F) : (((p2 >> 4) & 0x0F0F) | ((p1 >> 2) & 0x3030));
    (void)p0;
    return hmul2u(hsub2u(prmt(mp, 0x64646464u, 0x4140), H2_1024), nmm);
}
// Q4_K on the 8-bit tensor cores. The prep kernel writes x per 256-weight
// chunk and token as x = dx * (qh + ql / 256) with two int8 planes (qh =
// round(x/dx), dx = max|x|/127; ql = round(256 * residual)), i.e. about 16
// significant bits, finer than f16. Per 32-weight sub-block: the raw nibbles
// are the A operand (one LOP3 per 4 weights), one m16n8k32 MMA per plane, and
// the 6-bit sub-block scale is applied to the exact integer results; d*dx once
// per superblock in f32; -dmin*m*sum(x) is one f16 MMA per superblock.
template <int NT>
__device__ __forceinline__ void compute(const RawQ4K &r, const uint8_t *xc, int M, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
    const int g = lane >> 2, t = lane & 3;
    // 6-bit scales of sub-blocks 0..7 of rows g and g+8, one byte each
    const uint32_t sgl = r.hg.y & 0x3F3F3F3Fu, sgh = (r.hg.w & 0x0F0F0F0Fu) | ((r.hg.y >> 2) & 0x30303030u);
    const uint32_t shl = r.hg8.y & 0x3F3F3F3Fu, shh = (r.hg8.w & 0x0F0F0F0Fu) | ((r.hg8.y >> 2) & 0x30303030u);
    int si[NT][4], sl[NT][4];
    bool tv[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        si[nt][0] = si[nt][1] = si[nt][2] = si[nt][3] = 0;
        sl[nt][0] = sl[nt][1] = sl[nt][2] = sl[nt][3] = 0;
        tv[nt] = nt * 8 + g < M;
    }
    const uint8_t *fr = xc + g * 32 + t * 8;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint4 &pg = r.q[j >> 1], &ph = r.q[2 + (j >> 1)];
        const uint32_t g0 = (j & 1) ? pg.z : pg.x, g1 = (j & 1) ? pg.w : pg.y;
        const uint32_t h0 = (j & 1) ? ph.z : ph.x, h1 = (j & 1) ? ph.w : ph.y;
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            const int sub = 2 * j + hf;
            const uint32_t a0 = (hf ? g0 >> 4 : g0) & 0x0F0F0F0Fu, a2 = (hf ? g1 >> 4 : g1) & 0x0F0F0F0Fu;
            const uint32_t a1 = (hf ? h0 >> 4 : h0) & 0x0F0F0F0Fu, a3 = (hf ? h1 >> 4 : h1) & 0x0F0F0F0Fu;
            const int scg = (int)(((sub < 4 ? sgl : sgh) >> (8 * (sub & 3))) & 0xFF);
            const int sch = (int)(((sub < 4 ? shl : shh) >> (8 * (sub & 3))) & 0xFF);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const uint8_t *f = fr + (sub * M + nt * 8) * 32;
                const uint2 b = tv[nt] ? *reinterpret_cast<const uint2 *>(f) : make_uint2(0u, 0u);
                const uint2 bl = tv[nt] ? *reinterpret_cast<const uint2 *>(f + 256 * M) : make_uint2(0u, 0u);
                int d[4], e[4];
                imma16832(d, a0, a1, a2, a3, b.x, b.y);
                imma16832(e, a0, a1, a2, a3, bl.x, bl.y);
                si[nt][0] += scg * d[0];
                si[nt][1] += scg * d[1];
                si[nt][2] += sch * d[2];
                si[nt][3] += sch * d[3];
                sl[nt][0] += scg * e[0];
                sl[nt][1] += scg * e[1];
                sl[nt][2] += sch * e[2];
                sl[nt][3] += sch * e[3];
            }
        }
    }
    const float dg = h2f(r.hg.x & 0xFFFF), dh = h2f(r.hg8.x & 0xFFFF);
    const float *dxp = reinterpret_cast<const float *>(xc + 528 * M);
    const uint32_t gnm = q4k_negmin(r.hg, t), hnm = q4k_negmin(r.hg8, t);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int tk0 = nt * 8 + 2 * t, tk1 = tk0 + 1;
        const float dx0 = tk0 < M ? dxp[tk0] : 0.f, dx1 = tk1 < M ? dxp[tk1] : 0.f;
        acc[nt][0] = fmaf(dg * dx0, fmaf((float)sl[nt][0], 1.f / 256.f, (float)si[nt][0]), acc[nt][0]);
        acc[nt][1] = fmaf(dg * dx1, fmaf((float)sl[nt][1], 1.f / 256.f, (float)si[nt][1]), acc[nt][1]);
        acc[nt][2] = fmaf(dh * dx0, fmaf((float)sl[nt][2], 1.f / 256.f, (float)si[nt][2]), acc[nt][2]);
        acc[nt][3] = fmaf(dh * dx1, fmaf((float)sl[nt][3], 1.f / 256.f, (float)si[nt][3]), acc[nt][3]);
        const uint32_t mf = tv[nt] ? *reinterpret_cast<const uint32_t *>(xc + 512 * M + (nt * 8 + g) * 16 + t * 4) : 0u;
        mma16816(acc[nt], gnm, hnm, 0u, 0u, mf, 0u);
    }
}

// ------------------------------------------------------------------ Q6_K ---
struct RawQ6K { uint4 q[6]; uint2 scg, scg8; uint32_t d; };
__device__ __forceinline__ void load_raw(RawQ6K &r, const uint8_t *T, int lane) {
#pragma unroll
    for (int p = 0; p < 6; p++) r.q[p] = lds128(T + p * 512 + lane * 16);
    const int g = lane >> 2, n = (lane & 3) >> 1;
    r.scg = lds64(T + 3072 + g * 16 + 8 * n);
    r.scg8 = lds64(T + 3072 + (g + 8) * 16 + 8 * n);
    r.d = lds32(T + 3328 + 4 * g);
}
__device__ __forceinline__ uint32_t q6_pair(uint32_t nw, int nsh, uint32_t hw, int hsh, uint32_t sc2) {
    const uint32_t lo = lop3_and_or(nw >> nsh, 0x000F000Fu, H2_1024);
    const uint32_t hs = hsh >= 0 ? (hw >> hsh) : (hw << -hsh);
    const uint32_t hi = lop3_and_or(hs, 0x00300030u, H2_1024);
    // (1024 + lo) - (2080 - (1024 + 16 hi)) = lo + 16 hi - 32; times sc: all exact
    return hmul2u(hsub2u(lo, hsub2u(H2_2080, hi)), sc2);
}
template <int NT>
__device__ __forceinline__ void compute(const RawQ6K &r, const uint8_t *xc, int M, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
    const XF xsc = make_xf<NT>(xc, M, lane);
    const int lh = lane & 1;
    float tmp[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) tmp[nt][0] = tmp[nt][1] = tmp[nt][2] = tmp[nt][3] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        // int8 scale sc[8n + 2i + lh] of each row, as (sc, sc) in f16
        const int idx = 2 * i + lh;
        const uint32_t swg = (idx < 4 ? r.scg.x : r.scg.y) ^ 0x80808080u;
        const uint32_t swg8 = (idx < 4 ? r.scg8.x : r.scg8.y) ^ 0x80808080u;
        const uint32_t sel = 0x4040u | (uint32_t)(idx & 3) | ((uint32_t)(idx & 3) << 8);
        const uint32_t scg = hsub2u(prmt(swg, 0x64646464u, sel), H2_1152);
        const uint32_t scg8 = hsub2u(prmt(swg8, 0x64646464u, sel), H2_1152);
        const int nsb = (i >> 1) * 8;
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const uint32_t nwg = wsel(r.q[i & 1], jj), nwg8 = wsel(r.q[3 + (i & 1)], jj);
            const uint32_t hwg = wsel(r.q[2], i), hwg8 = wsel(r.q[5], i);
            const int h0 = 4 * jj - 4, h1 = 4 * jj - 2;
            const uint32_t a0 = q6_pair(nwg, nsb, hwg, h0, scg);
            const uint32_t a2 = q6_pair(nwg, nsb + 4, hwg, h1, scg);
            const uint32_t a1 = q6_pair(nwg8, nsb, hwg8, h0, scg8);
            const uint32_t a3 = q6_pair(nwg8, nsb + 4, hwg8, h1, scg8);
            mma_step<NT>(tmp, xsc, 4 * i + jj, lane, a0, a1, a2, a3);
        }
    }
    // the superblock d is common to the 4 lane columns of a row: apply in f32
    const float dg = h2f(r.d & 0xFFFF), dg8 = h2f(r.d >> 16);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        acc[nt][0] = fmaf(dg, tmp[nt][0], acc[nt][0]);
        acc[nt][1] = fmaf(dg, tmp[nt][1], acc[nt][1]);
        acc[nt][2] = fmaf(dg8, tmp[nt][2], acc[nt][2]);
        acc[nt][3] = fmaf(dg8, tmp[nt][3], acc[nt][3]);
    }
}

// --------------------------------------------------------------- IQ2_XXS ---
struct RawIQ2 { uint4 q[2]; uint32_t d; };
__device__ __forceinline__ void load_raw(RawIQ2 &r, const uint8_t *T, int lane) {
    r.q[0] = lds128(T + lane * 16);
    r.q[1] = lds128(T + 512 + lane * 16);
    r.d = lds32(T + 1024 + 4 * (lane >> 2));
}
template <int NT>
__device__ __forceinline__ void compute(const RawIQ2 &r, const uint8_t *xc, int M, float (&acc)[NT][4], int lane,
                                        const uint4 *grid, const uint4 *sgn) {
    const XF xsc = make_xf<NT>(xc, M, lane);
    const float dg = h2f(r.d & 0xFFFF), dg8 = h2f(r.d >> 16);
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const uint32_t a0g = u ? r.q[0].z : r.q[0].x, a1g = u ? r.q[0].w : r.q[0].y;
        const uint32_t a0h = u ? r.q[1].z : r.q[1].x, a1h = u ? r.q[1].w : r.q[1].y;
        // db = d * (0.5 + s) * 0.25 (kernels.wgsl.js:377), as f16 pairs
        const uint32_t bg = dup_h2(dg * (0.5f + (float)(a1g >> 28)) * 0.25f);
        const uint32_t bh = dup_h2(dg8 * (0.5f + (float)(a1h >> 28)) * 0.25f);
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint4 G = grid[(a0g >> (8 * l)) & 0xFF], S = sgn[(a1g >> (7 * l)) & 127];
            const uint4 H = grid[(a0h >> (8 * l)) & 0xFF], Sh = sgn[(a1h >> (7 * l)) & 127];
            mma_step<NT>(acc, xsc, 8 * u + 2 * l, lane, hmul2u(G.x ^ S.x, bg), hmul2u(H.x ^ Sh.x, bh),
                         hmul2u(G.y ^ S.y, bg), hmul2u(H.y ^ Sh.y, bh));
            mma_step<NT>(acc, xsc, 8 * u + 2 * l + 1, lane, hmul2u(G.z ^ S.z, bg), hmul2u(H.z ^ Sh.z, bh),
                         hmul2u(G.w ^ S.w, bg), hmul2u(H.w ^ Sh.w, bh));
        }
    }
}

// ----------------------------------------------------------------- IQ1_S ---
struct RawIQ1 { uint4 qs; uint2 qh; uint32_t d; };
__device__ __forceinline__ void load_raw(RawIQ1 &r, const uint8_t *T, int lane) {
    r.qs = lds128(T + lane * 16);
    r.qh = lds64(T + 512 + lane * 8);
    r.d = lds32(T + 768 + 4 * (lane >> 2));
}
template <int NT>
__device__ __forceinline__ void compute(const RawIQ1 &r, const uint8_t *xc, int M, float (&acc)[NT][4], int lane,
                                        const uint4 *grid, const uint4 *) {
    const XF xsc = make_xf<NT>(xc, M, lane);
    const float dg = h2f(r.d & 0xFFFF), dg8 = h2f(r.d >> 16);
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const uint32_t qsg = u ? r.qs.y : r.qs.x, qsh = u ? r.qs.w : r.qs.z;
        const uint32_t qhg = (r.qh.x >> (16 * u)) & 0xFFFF, qhh = (r.qh.y >> (16 * u)) & 0xFFFF;
        const uint32_t delg = (qhg & 0x8000u) ? 0xB000B000u : 0x30003000u;   // -/+ 0.125
        const uint32_t delh = (qhh & 0x8000u) ? 0xB000B000u : 0x30003000u;
        // dl = d * (2 * ((qh >> 12) & 7) + 1) (kernels.wgsl.js:809), as f16 pairs
        const uint32_t lg = dup_h2(dg * (float)(2u * ((qhg >> 12) & 7u) + 1u));
        const uint32_t lh = dup_h2(dg8 * (float)(2u * ((qhh >> 12) & 7u) + 1u));
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint4 G = grid[((qsg >> (8 * l)) & 0xFF) | (((qhg >> (3 * l)) & 7) << 8)];
            const uint4 H = grid[((qsh >> (8 * l)) & 0xFF) | (((qhh >> (3 * l)) & 7) << 8)];
            // grid + delta is exact in f16; one rounding for the product with dl
            mma_step<NT>(acc, xsc, 8 * u + 2 * l, lane, hmul2u(hadd2u(G.x, delg), lg),
                         hmul2u(hadd2u(H.x, delh), lh), hmul2u(hadd2u(G.y, delg), lg),
                         hmul2u(hadd2u(H.y, delh), lh));
            mma_step<NT>(acc, xsc, 8 * u + 2 * l + 1, lane, hmul2u(hadd2u(G.z, delg), lg),
                         hmul2u(hadd2u(H.z, delh), lh), hmul2u(hadd2u(G.w, delg), lg),
                         hmul2u(hadd2u(H.w, delh), lh));
        }
    }
}

template <int TYPE> struct RawOf;
template <> struct RawOf<EF_Q8_0> { using T = RawQ8; };
template <> struct RawOf<EF_Q4_K> { using T = RawQ4K; };
template <> struct RawOf<EF_Q6_K> { using T = RawQ6K; };
template <> struct RawOf<EF_IQ2_XXS> { using T = RawIQ2; };
template <> struct RawOf<EF_IQ1_S> { using T = RawIQ1; };

template <int TYPE> struct TableBytes { static constexpr int v = 0; };
template <> struct TableBytes<EF_IQ2_XXS> { static constexpr int v = 256 * 16 + 128 * 16; };
template <> struct TableBytes<EF_IQ1_S> { static constexpr int v = 2048 * 16; };

// ------------------------------------------------------------- x staging ---
// Chunks [c, c + n) of x (f32 [M][K]) are written as the activation data the
// compute functions read, to `dst` (chunk i at dst + i * xb), by the threads
// [tid, tid + nthreads) -- either one CTA (the fused, single-kernel path used
// for up to 4 tokens) or the whole grid of the prep kernel (5..16 tokens).
//
// f16 types: per chunk, B fragments [step][token][lane t] (8 B: the pairs
// (k, k+1), (k+2, k+3) of the k-quad that (t, step) consumes), tokens 0..M-1.
template <int TYPE>
__device__ __forceinline__ void stage_f16(const float *__restrict__ x, int M, int64_t K, int64_t c, int n,
                                          uint8_t *dst, int xb, int tid, int nthreads) {
    using TR = Tr<TYPE>;
    constexpr int QPC = TR::CHUNK / 4;
    const int per_chunk = M * QPC;
    for (int i = tid; i < n * per_chunk; i += nthreads) {
        const int cc = i / per_chunk, rem = i - cc * per_chunk;
        const int token = rem / QPC, kq = rem - token * QPC;
        const int64_t k = (c + cc) * TR::CHUNK + 4 * kq;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < K) v = __ldg(reinterpret_cast<const float4 *>(x + token * K + k));
        int t, st;
        TR::inv(kq, t, st);
        *reinterpret_cast<uint2 *>(dst + (int64_t)cc * xb + ((st * M + token) * 4 + t) * 8) =
            make_uint2(pack_h2(v.x, v.y), pack_h2(v.z, v.w));
    }
}
// Q4_K (8-bit MMA): per 256-weight chunk and token x = dx * (qh + ql/256),
// dx = max|x|/127, qh = rne(x/dx), ql = rne(256 * (x/dx - qh)), both int8, as
// B fragments [plane][sub-block][token][lane t][b0 b1]; then the f16 sums of x
// over each 32-weight sub-block as pairs (2t, 2t+1) per (token, t); then dx per
// token. One warp per (chunk, token); lane l holds weights 8l .. 8l+7.
__device__ __forceinline__ void stage_i8(const float *__restrict__ x, int M, int64_t K, int64_t c, int n,
                                         uint8_t *dst, int xb, int tid, int nthreads) {
    const int lane = tid & 31;
    for (int w = tid >> 5; w < n * M; w += nthreads >> 5) {
        const int cc = w / M, token = w - cc * M;
        const int64_t k0 = (c + cc) * 256 + 8 * lane;
        float v[8];
        if (k0 < K) {
            const float4 p = __ldg(reinterpret_cast<const float4 *>(x + token * K + k0));
            const float4 q = __ldg(reinterpret_cast<const float4 *>(x + token * K + k0 + 4));
            v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w; v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
        } else {
            for (int i = 0; i < 8; i++) v[i] = 0.f;
        }
        float amax = 0.f, sum = 0.f;
        for (int i = 0; i < 8; i++) {
            amax = fmaxf(amax, fabsf(v[i]));
            sum += v[i];
        }
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        const float dx = amax / 127.f, inv = amax > 0.f ? 127.f / amax : 0.f;
        uint32_t wq[2], wl[2];
        for (int h = 0; h < 2; h++) {
            uint32_t word = 0, wlo = 0;
            for (int i = 0; i < 4; i++) {
                const float u = v[4 * h + i] * inv;
                const float qh = fminf(fmaxf(rintf(u), -127.f), 127.f);
                const int ql = (int)fminf(fmaxf(rintf((u - qh) * 256.f), -127.f), 127.f);
                word |= (uint32_t)((int)qh & 0xFF) << (8 * i);
                wlo |= (uint32_t)(ql & 0xFF) << (8 * i);
            }
            wq[h] = word;
            wl[h] = wlo;
        }
        uint8_t *base = dst + (int64_t)cc * xb;
        const int sub = lane >> 2, kk = 8 * (lane & 3);                  // k within the sub-block
        const int tA = (kk & 15) >> 2, off = kk >= 16 ? 4 : 0;          // fragment lane and half
        uint8_t *fr = base + (sub * M + token) * 32;
        *reinterpret_cast<uint32_t *>(fr + tA * 8 + off) = wq[0];
        *reinterpret_cast<uint32_t *>(fr + (tA + 1) * 8 + off) = wq[1];
        *reinterpret_cast<uint32_t *>(fr + 256 * M + tA * 8 + off) = wl[0];
        *reinterpret_cast<uint32_t *>(fr + 256 * M + (tA + 1) * 8 + off) = wl[1];
        if ((lane & 3) == 0)
            *reinterpret_cast<__half *>(base + 512 * M + token * 16 + (sub >> 1) * 4 + (sub & 1) * 2) =
                __float2half_rn(sum);
        if (lane == 0) *reinterpret_cast<float *>(base + 528 * M + token * 4) = dx;
    }
}
template <int TYPE>
__device__ __forceinline__ void stage_x(const float *x, int M, int64_t K, int64_t c, int n, uint8_t *dst, int xb,
                                        int tid, int nthreads) {
    if (Tr<TYPE>::I8) stage_i8(x, M, K, c, n, dst, xb, tid, nthreads);
    else stage_f16<TYPE>(x, M, K, c, n, dst, xb, tid, nthreads);
}

// Prep kernel (5..16 tokens): all chunks into global scratch. Launched with
// programmatic dependent launch: it lets the GEMV that follows start (and
// prefetch weights) at once, and waits for the kernel before it (which may
// have produced x, or still read the scratch) before touching memory.
template <int TYPE>
__global__ void gemv_xprep(const float *__restrict__ x, int M, int64_t K, int64_t nchunks, int xb,
                           uint8_t *__restrict__ xf) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    stage_x<TYPE>(x, M, K, 0, (int)nchunks, xf, xb, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

// ------------------------------------------------------------- epilogue ----
template <int NT, bool SWIGLU>
__device__ __forceinline__ void write_out(const float (&acc)[NT][4], const float (&acc2)[NT][4], float *y,
                                          int64_t rows, int M, int64_t rg, int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int64_t r0 = rg * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int tk0 = nt * 8 + 2 * t, tk1 = tk0 + 1;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (SWIGLU) {
                const float gt = acc[nt][j];
                v[j] = gt / (1.0f + expf(-gt)) * acc2[nt][j];   // silu(g) * u
            } else {
                v[j] = acc[nt][j];
            }
        }
        if (r0 < rows) {
            if (tk0 < M) y[(int64_t)tk0 * rows + r0] = v[0];
            if (tk1 < M) y[(int64_t)tk1 * rows + r0] = v[1];
        }
        if (r1 < rows) {
            if (tk0 < M) y[(int64_t)tk0 * rows + r1] = v[2];
            if (tk1 < M) y[(int64_t)tk1 * rows + r1] = v[3];
        }
    }
}

// ---------------------------------------------------------------- kernel ---
// Shared memory: [weight rings: WARPS x NMAT x ST tiles][x fragments of one
// phase][codebooks][cluster partial sums].
template <int TYPE, bool SW> struct Stages {
    static constexpr int raw = RING_PER_WARP / ((SW ? 2 : 1) * Tr<TYPE>::TILE);
    static constexpr int v = raw < 2 ? 2 : raw > 6 ? 6 : raw;
};
template <int WARPS> struct MinBlocks { static constexpr int v = WARPS == 8 ? 2 : 4; };

// FUSED: the CTA stages its own x slice from f32 x (up to 4 tokens: one
// kernel per call); otherwise it copies the slice the prep kernel wrote.
template <int TYPE, int NT, bool SWIGLU, int WARPS, bool FUSED>
__global__ void __launch_bounds__(WARPS * 32, MinBlocks<WARPS>::v) gemv_kernel(const GemvArgs a) {
    using TR = Tr<TYPE>;
    using Raw = typename RawOf<TYPE>::T;
    constexpr int NMAT = SWIGLU ? 2 : 1;
    constexpr int ST = Stages<TYPE, SWIGLU>::v;
    constexpr int TILE = TR::TILE;
    const int FB = a.xb;
    extern __shared__ __align__(16) uint8_t smem[];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = blockIdx.x, rb = blockIdx.y;
    int m = 0;
    while (m + 1 < a.nmat && rb >= a.rb_end[m]) m++;
    const int rb_local = rb - (m ? a.rb_end[m - 1] : 0);
    const int64_t rg = (int64_t)rb_local * WARPS + warp;
    const bool active = rg < a.rowgroups[m];
    const int c0 = ks * a.cps;
    const int nc = (int)min((int64_t)a.cps, a.nchunks - c0);

    constexpr int RING = WARPS * NMAT * ST * TILE;
    uint8_t *ring = smem + warp * NMAT * ST * TILE;
    uint8_t *xs = smem + RING;
    const int xs_bytes = a.phase_chunks * FB;
    uint4 *grid = reinterpret_cast<uint4 *>(smem + RING + xs_bytes);
    uint4 *sgn = grid + 256;
    float *red = reinterpret_cast<float *>(smem + RING + xs_bytes + TableBytes<TYPE>::v);

    // Weight stream: chunk cc of this warp goes to ring slot cc % ST by
    // cp.async; one commit group per chunk (empty groups keep the count).
    const int64_t tile0 = active ? (rg * a.nchunks + c0) * (int64_t)TILE : 0;
    const uint8_t *Tm = a.w[m] + tile0;
    const uint8_t *Tu = SWIGLU ? a.w_up + tile0 : nullptr;
    auto issue = [&](int cc) {
        if (active && cc < nc) {
            copy_tile<TILE>(ring + (cc % ST) * TILE, Tm + (int64_t)cc * TILE, lane);
            if (SWIGLU) copy_tile<TILE>(ring + (ST + cc % ST) * TILE, Tu + (int64_t)cc * TILE, lane);
        }
        cp_commit();
    };
#pragma unroll
    for (int s0 = 0; s0 < ST - 1; s0++) issue(s0);

    // codebooks -> shared memory (f16 entries; IQ2_XXS also the sign masks:
    // 7 stored sign bits + even parity -> XOR masks on f16 pairs)
    if (TYPE == EF_IQ2_XXS) {
        const uint4 *src = reinterpret_cast<const uint4 *>(g_grid_iq2xxs_f16);
        for (int i = threadIdx.x; i < 256; i += blockDim.x) grid[i] = src[i];
        for (int i = threadIdx.x; i < 128; i += blockDim.x) {
            const uint32_t s8 = (uint32_t)i | ((uint32_t)(__popc(i) & 1) << 7);
            uint32_t w[4];
            for (int p = 0; p < 4; p++)
                w[p] = (((s8 >> (2 * p)) & 1u) << 15) | (((s8 >> (2 * p + 1)) & 1u) << 31);
            sgn[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    } else if (TYPE == EF_IQ1_S) {
        const uint4 *src = reinterpret_cast<const uint4 *>(g_grid_iq1s_f16);
        for (int i = threadIdx.x; i < 2048; i += blockDim.x) grid[i] = src[i];
    }

    float acc[NT][4], acc2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[nt][j] = acc2[nt][j] = 0.f;

    // x is produced by the kernel before this one (the prep kernel, or the
    // caller's previous kernel): wait for it only now, after the weight prefetch.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int p0 = 0; p0 < nc; p0 += a.phase_chunks) {
        const int pc = min(a.phase_chunks, nc - p0);
        if (p0) __syncthreads();   // every warp is done with the previous phase
        if (FUSED) {
            stage_x<TYPE>(a.x, a.M, a.K, c0 + p0, pc, xs, FB, threadIdx.x, blockDim.x);
        } else {
            const uint8_t *src = a.xf + (int64_t)(c0 + p0) * FB;
            for (int i = threadIdx.x; i < pc * FB / 16; i += blockDim.x) cp_async16(xs + 16 * i, src + 16 * i);
            cp_commit();
            cp_wait<0>();   // the x phase (and the weight tiles issued before it)
        }
        __syncthreads();
        for (int cl = 0; cl < pc; cl++) {
            const int cc = p0 + cl;
            __syncwarp();          // every lane is done reading the slot refilled next
            issue(cc + ST - 1);
            cp_wait<ST - 1>();     // this thread's copies of chunk cc have landed
            __syncwarp();          // ... and every other lane's
            if (active) {
                const uint8_t *xc = xs + cl * FB;
                Raw r;
                load_raw(r, ring + (cc % ST) * TILE, lane);
                compute<NT>(r, xc, a.M, acc, lane, grid, sgn);
                if (SWIGLU) {
                    Raw u;
                    load_raw(u, ring + (ST + cc % ST) * TILE, lane);
                    compute<NT>(u, xc, a.M, acc2, lane, grid, sgn);
                }
            }
        }
    }
    cp_wait<0>();
    // The weight stream is done: the next kernel in the stream may launch now
    // (programmatic dependent launch) and prefetch its weights while this one
    // reduces and writes y. Triggering earlier lets waiting CTAs of the next
    // kernel hold SM resources that this kernel still needs.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (a.kslices == 1) {
        if (active) write_out<NT, SWIGLU>(acc, acc2, a.y[m], a.rows[m], a.M, rg, lane);
        return;
    }
    // k-slices of this rowblock are one cluster: add partials in rank order.
    float *mine = red + ((warp * NMAT) * NT * 32 + lane) * 4;
#pragma unroll
    for (int mm = 0; mm < NMAT; mm++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int j = 0; j < 4; j++) mine[((mm * NT + nt) * 32) * 4 + j] = mm ? acc2[nt][j] : acc[nt][j];
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (warp % a.kslices == ks && active) {
        float s1[NT][4], s2[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int j = 0; j < 4; j++) s1[nt][j] = s2[nt][j] = 0.f;
        for (int rk = 0; rk < a.kslices; rk++) {
            const float *src = cluster.map_shared_rank(mine, rk);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const float4 v = *reinterpret_cast<const float4 *>(src + (nt * 32) * 4);
                s1[nt][0] += v.x; s1[nt][1] += v.y; s1[nt][2] += v.z; s1[nt][3] += v.w;
                if (SWIGLU) {
                    const float4 u = *reinterpret_cast<const float4 *>(src + ((NT + nt) * 32) * 4);
                    s2[nt][0] += u.x; s2[nt][1] += u.y; s2[nt][2] += u.z; s2[nt][3] += u.w;
                }
            }
        }
        write_out<NT, SWIGLU>(s1, s2, a.y[m], a.rows[m], a.M, rg, lane);
    }
    cluster.sync();   // keep this CTA's shared memory alive until all ranks have read it
}

// ------------------------------------------------------------------ host ---
// Pick the CTA shape. Measured on B200 (sweeps over width x k-split for the
// benchmark shapes): long-lived warps that stream many tiles beat short CTAs
// even when some SMs stay idle, because every CTA pays a pipeline start, an
// activation staging and a cluster reduction. So: 8 rowgroups per CTA and the
// smallest k-split that puts at least 3/4 of the SMs to work (4 rowgroups
// when the rows are too few even for that).
GemvPlan gemv_plan(int sm_count, int64_t rowgroups, int64_t nchunks, int M, const int ctas_per_sm[2]) {
    (void)ctas_per_sm;
    GemvPlan best = {};
    const int64_t want = (3LL * sm_count + 3) / 4;
    best.warps = 8;
    int64_t rowblocks = (rowgroups + 7) / 8;
    if (rowblocks * std::min<int64_t>(8, nchunks) < want) {
        best.warps = 4;
        rowblocks = (rowgroups + 3) / 4;
    }
    int64_t ks = 1;
    while (ks < 8 && ks < nchunks && rowblocks * ks < want) ks++;
    best.cps = (int)((nchunks + ks - 1) / ks);
    best.kslices = (int)((nchunks + best.cps - 1) / best.cps);
    best.rowblocks = (int)rowblocks;
    best.nt = M <= 8 ? 1 : 2;
    return best;
}

// Programmatic dependent launch between consecutive kernels: off by default
// (measured on B200 over the mixed-shape benchmark sequence: the early-
// launched CTAs of the next GEMV hold shared memory and registers that the
// current one still needs, a net loss); EF_GEMV_PDL=1 turns it on.
static bool gemv_pdl() {
    const char *v = getenv("EF_GEMV_PDL");
    return v && v[0] == '1';
}

template <int TYPE, int NT, bool SWIGLU, int WARPS>
static size_t smem_bytes(int phase_chunks, int xb, int kslices) {
    constexpr int NMAT = SWIGLU ? 2 : 1;
    return (size_t)WARPS * NMAT * Stages<TYPE, SWIGLU>::v * Tr<TYPE>::TILE + (size_t)phase_chunks * xb +
           TableBytes<TYPE>::v + (kslices > 1 ? (size_t)WARPS * NMAT * NT * 32 * 16 : 0);
}

template <int TYPE, int NT, bool SWIGLU, int WARPS, bool FUSED>
static int launch_kernel(ef_ctx *ctx, GemvArgs &a, int grid_y) {
    auto kern = gemv_kernel<TYPE, NT, SWIGLU, WARPS, FUSED>;
    static unsigned long long configured = 0;   // per instantiation, one bit per device
    if (ctx->device < 64 && !(configured & (1ull << ctx->device))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e != cudaSuccess) return check_cuda(ctx, e, "gemv smem attribute");
        configured |= 1ull << ctx->device;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.kslices, grid_y, 1);
    cfg.blockDim = dim3(WARPS * 32, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes<TYPE, NT, SWIGLU, WARPS>(a.phase_chunks, a.xb, a.kslices);
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (gemv_pdl()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (a.kslices > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = a.kslices;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return check_cuda(ctx, cudaLaunchKernelEx(&cfg, kern, a), "gemv launch");
}

// Up to this many tokens each CTA stages its own x slice (one kernel per
// call); above it a prep kernel writes the slices once into context scratch.
constexpr int FUSED_MAX_TOKENS = 2;

template <int TYPE> static int x_bytes_per_chunk(int M) {
    return Tr<TYPE>::I8 ? i8_xbytes(M) : f16_xbytes<TYPE>(M);
}

template <int TYPE, int NT, bool SWIGLU>
static int launch_t(ef_ctx *ctx, GemvArgs &a, const ef_weight *const *ws, int n, const float *x) {
    a.xb = x_bytes_per_chunk<TYPE>(a.M);
    a.x = x;
    a.K = ws[0]->k;
    const bool fused = NT == 1 && a.M <= FUSED_MAX_TOKENS;
    if (!fused) {
        // x data for all chunks -> context scratch slot 0 (prep kernel, PDL)
        const size_t xbytes = (size_t)a.nchunks * a.xb;
        if (int rc = ensure_scratch(ctx, 0, xbytes)) return rc;
        a.xf = (const uint8_t *)ctx->scratch[0];
        const int64_t work = Tr<TYPE>::I8 ? a.nchunks * a.M * 32 : a.nchunks * a.M * (Tr<TYPE>::CHUNK / 4);
        int64_t blocks = (work + 255) / 256;
        if (blocks > 2LL * ctx->sm_count) blocks = 2LL * ctx->sm_count;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)blocks, 1, 1);
        cfg.blockDim = dim3(256, 1, 1);
        cfg.stream = ctx->stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = gemv_pdl() ? 1 : 0;
        if (int rc = check_cuda(ctx, cudaLaunchKernelEx(&cfg, gemv_xprep<TYPE>, x, a.M, a.K, a.nchunks, a.xb,
                                                        (uint8_t *)ctx->scratch[0]), "gemv xprep launch"))
            return rc;
    } else {
        a.xf = nullptr;
    }
    // how many CTAs of each width fit on one SM, then the cost model
    const int ph = std::max(1, std::min(8, MAX_XS_BYTES / a.xb));
    const int fit8 = (int)std::min<size_t>(2, 227 * 1024 / (smem_bytes<TYPE, NT, SWIGLU, 8>(ph, a.xb, 2) + 1024));
    const int fit4 = (int)std::min<size_t>(4, 227 * 1024 / (smem_bytes<TYPE, NT, SWIGLU, 4>(ph, a.xb, 2) + 1024));
    const int fits[2] = {std::max(fit8, 1), std::max(fit4, 1)};
    int64_t total_rg = 0;
    for (int i = 0; i < n; i++) total_rg += ws[i]->rowgroups;
    GemvPlan p = gemv_plan(ctx->sm_count, total_rg, a.nchunks, a.M, fits);
    // Tuning override for sweeps: EF_GEMV_PLAN="W:ks" (W = 4 or 8 rowgroups per
    // CTA, ks = k-slices, 1..8); ignored when it does not fit the shape.
    if (const char *ov = getenv("EF_GEMV_PLAN")) {
        int W = 0, ks = 0;
        if (sscanf(ov, "%d:%d", &W, &ks) == 2 && (W == 4 || W == 8) && ks >= 1 && ks <= 8 && ks <= a.nchunks) {
            p.warps = W;
            p.cps = (int)((a.nchunks + ks - 1) / ks);
            p.kslices = (int)((a.nchunks + p.cps - 1) / p.cps);
        }
    }
    a.cps = p.cps;
    a.kslices = p.kslices;
    a.phase_chunks = std::min(a.cps, MAX_XS_BYTES / a.xb);
    if (a.phase_chunks < 1) a.phase_chunks = 1;
    int grid_y = 0;
    for (int i = 0; i < n; i++) {
        grid_y += (int)((ws[i]->rowgroups + p.warps - 1) / p.warps);
        a.rb_end[i] = grid_y;
    }
    if (fused)
        return p.warps == 8 ? launch_kernel<TYPE, NT, SWIGLU, 8, true>(ctx, a, grid_y)
                            : launch_kernel<TYPE, NT, SWIGLU, 4, true>(ctx, a, grid_y);
    return p.warps == 8 ? launch_kernel<TYPE, NT, SWIGLU, 8, false>(ctx, a, grid_y)
                        : launch_kernel<TYPE, NT, SWIGLU, 4, false>(ctx, a, grid_y);
}

template <int TYPE>
static int launch_type(ef_ctx *ctx, GemvArgs &a, int nt, bool swiglu, const ef_weight *const *ws, int n,
                       const float *x) {
    if (swiglu)
        return nt == 1 ? launch_t<TYPE, 1, true>(ctx, a, ws, n, x) : launch_t<TYPE, 2, true>(ctx, a, ws, n, x);
    return nt == 1 ? launch_t<TYPE, 1, false>(ctx, a, ws, n, x) : launch_t<TYPE, 2, false>(ctx, a, ws, n, x);
}

int launch_gemv(ef_ctx *ctx, const ef_weight *const *ws, int n, const ef_weight *w_up, const float *x, int M,
                float *const *ys) {
    GemvArgs a = {};
    const ef_weight *w0 = ws[0];
    a.nmat = n;
    for (int i = 0; i < n; i++) {
        a.w[i] = ws[i]->dev;
        a.y[i] = ys[i];
        a.rows[i] = ws[i]->rows;
        a.rowgroups[i] = ws[i]->rowgroups;
    }
    a.w_up = w_up ? w_up->dev : nullptr;
    a.M = M;
    a.nchunks = w0->nchunks;
    const bool sw = w_up != nullptr;
    const int nt = M <= 8 ? 1 : 2;
    switch (w0->type) {
    case EF_Q8_0: return launch_type<EF_Q8_0>(ctx, a, nt, sw, ws, n, x);
    case EF_Q4_K: return launch_type<EF_Q4_K>(ctx, a, nt, sw, ws, n, x);
    case EF_Q6_K: return launch_type<EF_Q6_K>(ctx, a, nt, sw, ws, n, x);
    case EF_IQ2_XXS: return launch_type<EF_IQ2_XXS>(ctx, a, nt, sw, ws, n, x);
    case EF_IQ1_S: return launch_type<EF_IQ1_S>(ctx, a, nt, sw, ws, n, x);
    default: return set_err(ctx, EF_ERR_TYPE, "gemv: unsupported type %d", w0->type);
    }
}

}  // namespace ef

// ------------------------------------------------------ allocation-free GEMV --
// ef_gemv_noalloc: the decode GEMV for callers that must not allocate device
// memory. Its per-call activation fragments live in this file-scope array
// (NOALLOC_SCRATCH_BYTES, held by every GPU that loads the library until the
// process exits) instead of the context scratch that ef_gemv grows with
// cudaMalloc. Host code cannot use `g_noalloc_scratch` as an address (the name
// is a host-side shadow); the device address is looked up once per device with
// cudaGetSymbolAddress on the first call on that device.
namespace ef {

constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)1 << 20;   // 1 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// Bytes of activation data one GEMV call keeps in scratch (the same amount
// launch_t sizes its scratch for; calls of up to FUSED_MAX_TOKENS tokens keep
// it in shared memory and need none).
static size_t gemv_xfrag_bytes(int type, int64_t nchunks, int M) {
    size_t fb = 0;
    switch (type) {
    case EF_Q8_0: fb = (size_t)f16_xbytes<EF_Q8_0>(M); break;
    case EF_Q4_K: fb = (size_t)i8_xbytes(M); break;
    case EF_Q6_K: fb = (size_t)f16_xbytes<EF_Q6_K>(M); break;
    case EF_IQ2_XXS: fb = (size_t)f16_xbytes<EF_IQ2_XXS>(M); break;
    case EF_IQ1_S: fb = (size_t)f16_xbytes<EF_IQ1_S>(M); break;
    default: return 0;
    }
    return M <= FUSED_MAX_TOKENS ? 1 : (size_t)nchunks * fb;
}

}  // namespace ef

#include <mutex>

extern "C" int ef_gemv_noalloc(const ef_weight *w, const float *x, int M, float *y, void *cuda_stream) {
    using namespace ef;
    if (!w || !x || !y) return EF_ERR_INVALID;
    if (M < 1) return EF_ERR_SHAPE;
    if (M > 16) return EF_NOT_APPLICABLE;
    if (((uintptr_t)x & 15) != 0) return EF_ERR_INVALID;
    const size_t need = gemv_xfrag_bytes(w->type, w->nchunks, M);
    if (need == 0) return EF_ERR_TYPE;
    if (need > NOALLOC_SCRATCH_BYTES) return EF_ERR_RANGE;   // k too large for the static array
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return EF_ERR_CUDA;
    // once per device: the device address of the static array
    static std::mutex mu;
    static void *addr[64] = {nullptr};
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!addr[dev]) {
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return EF_ERR_CUDA;
            addr[dev] = p;
        }
    }
    // A context on the stack whose scratch slot 0 IS the static array (large
    // enough, checked above), so the shared launch path never allocates.
    ef_ctx tmp;
    tmp.device = dev;
    tmp.stream = (cudaStream_t)cuda_stream;
    if (cudaDeviceGetAttribute(&tmp.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return EF_ERR_CUDA;
    tmp.scratch[0] = addr[dev];
    tmp.scratch_bytes[0] = NOALLOC_SCRATCH_BYTES;
    float *ys[1] = {y};
    const int rc = launch_gemv(&tmp, &w, 1, nullptr, x, M, ys);
    tmp.scratch[0] = nullptr;   // not the context's to free
    return rc;
}

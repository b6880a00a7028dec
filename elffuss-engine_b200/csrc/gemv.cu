// gemv.cu -- decode GEMV over repacked GGUF tiles, 1..16 tokens (sm_100a).
//
//   y[t][r] = sum_k dequant(W)[r][k] * x[t][k]        (js/ops.js:827-829)
//   swiglu:  y = silu(Wg.x) * (Wu.x)                   (kernels.gemv.wgsl.js:434-437)
//   sections: several W sharing x and k, one output each (js/ops.gemv.js:192-215)
//
// Design (B200): the GEMV is HBM-bound, so every weight byte is read once with
// 128-bit streaming loads and turned into f16 operands IN REGISTERS, which feed
// the tensor cores through mma.sync.m16n8k16 (A = 16 weight rows x 16 k, B =
// 16 k x 8 tokens, f32 accumulate). Register-sourced MMA is the right tensor
// instruction here: tcgen05.mma takes A from shared or tensor memory, which
// would add a store + read of every dequantised weight for a kernel whose only
// job is to stream weights; with register operands a 16-token GEMV costs two
// MMAs per 256 weights and the dequant stays the only per-weight work.
//
// Work split: CTA = 8 warps = one "rowblock" of 8 rowgroups (128 rows); a warp
// owns one rowgroup. Along k the chunks are cut into `kslices` slices, one CTA
// each; the slices of a rowblock form one thread-block cluster and their
// partial sums are added through distributed shared memory in rank order
// (deterministic, no atomics, no global scratch). Activations of the CTA's
// k-slice are converted once to f16 and staged in shared memory already in
// B-fragment order, so a fragment is one conflict-free 64-bit shared load.
//
// Numerics: quants are exact small integers in f16; the block scales are
// applied in f16 (Q8_0: f16(d*q); Q4_K: f16(f16(d*sc)*q - f16(dmin*m));
// IQ2_XXS: f16(db)*grid*sign; IQ1_S: f16(dl)*(grid + delta); one rounding
// each) because the 16 k-columns of one MMA come from four different blocks;
// only a scale shared by the whole tile row (Q6_K's superblock d) is applied in
// f32 on the accumulator. x is rounded to f16. The products are exact and
// summed in f32 by the tensor cores.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

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
constexpr int WARPS = 8;                    // warps (rowgroups) per CTA
constexpr int MAX_XS_BYTES = 96 * 1024;     // shared memory for staged activations

struct GemvArgs {
    const uint8_t *w[4];      // repacked tiles of each section
    const uint8_t *w_up;      // SwiGLU partner of w[0] (same geometry)
    float *y[4];
    int64_t rows[4];
    int64_t rowgroups[4];
    int rb_end[4];            // cumulative rowblocks per section
    int nmat;
    const float *x;
    int M;
    int64_t K;
    int64_t nchunks;
    int cps;                  // chunks per k-slice
    int kslices;
    int phase_chunks;         // chunks staged in shared memory at a time
};

// ---------------------------------------------------------------- traits ---
// STEPS = k16 steps per chunk; inv maps a k-quad (4 consecutive weights of the
// chunk) to the lane column t and the step s that consume it.
template <int TYPE> struct Tr;
template <> struct Tr<EF_Q8_0> {
    static constexpr int CHUNK = 128, STEPS = 8, TILE = 2176;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 3; s = kq & 7; }
};
template <> struct Tr<EF_Q4_K> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 2304;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = 2 * (kq & 7) + ((kq >> 3) & 1); }
};
template <> struct Tr<EF_Q6_K> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 3360;
    __device__ static void inv(int kq, int &t, int &s) {
        t = 2 * (kq >> 5) + ((kq >> 2) & 1);
        s = 4 * ((kq >> 3) & 3) + (kq & 3);
    }
};
template <> struct Tr<EF_IQ2_XXS> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 1056;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = kq & 15; }
};
template <> struct Tr<EF_IQ1_S> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 800;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = kq & 15; }
};

__device__ __forceinline__ uint32_t wsel(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t ldg32(const void *p) { return __ldg((const unsigned int *)p); }
__device__ __forceinline__ uint2 ldg64(const void *p) { return __ldg((const uint2 *)p); }

template <int NT>
__device__ __forceinline__ void mma_step(float (&acc)[NT][4], const uint2 *xsc, int s, int lane, uint32_t a0,
                                         uint32_t a1, uint32_t a2, uint32_t a3) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const uint2 b = xsc[(s * NT + nt) * 32 + lane];
        mma16816(acc[nt], a0, a1, a2, a3, b.x, b.y);
    }
}

template <int NT>
__device__ __forceinline__ void scale_acc(float (&acc)[NT][4], float (&tmp)[NT][4], float sg, float sg8) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        acc[nt][0] = fmaf(sg, tmp[nt][0], acc[nt][0]);
        acc[nt][1] = fmaf(sg, tmp[nt][1], acc[nt][1]);
        acc[nt][2] = fmaf(sg8, tmp[nt][2], acc[nt][2]);
        acc[nt][3] = fmaf(sg8, tmp[nt][3], acc[nt][3]);
        tmp[nt][0] = tmp[nt][1] = tmp[nt][2] = tmp[nt][3] = 0.f;
    }
}

// ------------------------------------------------------------------ Q8_0 ---
struct RawQ8 { uint4 q[4]; uint32_t sc; };
__device__ __forceinline__ void load_raw(RawQ8 &r, const uint8_t *T, int lane) {
#pragma unroll
    for (int p = 0; p < 4; p++) r.q[p] = ldg_stream(T + p * 512 + lane * 16);
    r.sc = ldg32(T + 2048 + lane * 4);
}
template <int NT>
__device__ __forceinline__ void compute(const RawQ8 &r, const uint2 *xsc, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
    const uint32_t dg = prmt(r.sc, 0, 0x1010), dg8 = prmt(r.sc, 0, 0x3232);
#pragma unroll
    for (int s = 0; s < 8; s++) {
        const uint32_t wg = wsel(r.q[s >> 2], s & 3), wg8 = wsel(r.q[2 + (s >> 2)], s & 3);
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
    for (int p = 0; p < 4; p++) r.q[p] = ldg_stream(T + p * 512 + lane * 16);
    const int g = lane >> 2;
    r.hg = ldg_stream(T + 2048 + g * 16);
    r.hg8 = ldg_stream(T + 2048 + (g + 8) * 16);
}
// (d*sc_a, d*sc_b, -dmin*m_a, -dmin*m_b) as duplicated half2 for lane column t
// (sub-blocks 2t, 2t+1), from a verbatim 16-byte Q4_K header: scale_min_k4
// (kernels.wgsl.js:94-104) for j = 2t, 2t+1 without divergence.
__device__ __forceinline__ void q4k_scales(const uint4 &h, int t, uint32_t &d1a, uint32_t &d1b, uint32_t &nm1a,
                                           uint32_t &nm1b) {
    const uint32_t dd = prmt(h.x, 0, 0x1010), nmm = prmt(h.x, 0, 0x3232) ^ 0x80008000u;
    const int sh = 16 * (t & 1);
    const uint32_t p0 = (h.y >> sh) & 0xFFFF, p1 = (h.z >> sh) & 0xFFFF, p2 = (h.w >> sh) & 0xFFFF;
    uint32_t scp, mp;
    if (t < 2) {
        scp = p0 & 0x3F3F;
        mp = p1 & 0x3F3F;
    } else {
        scp = (p2 & 0x0F0F) | ((p0 >> 2) & 0x3030);
        mp = ((p2 >> 4) & 0x0F0F) | ((p1 >> 2) & 0x3030);
    }
    d1a = hmul2u(hsub2u(prmt(scp, 0x64646464u, 0x4040), H2_1024), dd);
    d1b = hmul2u(hsub2u(prmt(scp, 0x64646464u, 0x4141), H2_1024), dd);
    nm1a = hmul2u(hsub2u(prmt(mp, 0x64646464u, 0x4040), H2_1024), nmm);
    nm1b = hmul2u(hsub2u(prmt(mp, 0x64646464u, 0x4141), H2_1024), nmm);
}
template <int NT>
__device__ __forceinline__ void compute(const RawQ4K &r, const uint2 *xsc, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
    const int t = lane & 3;
    uint32_t ga, gb, gna, gnb, ha, hb, hna, hnb;
    q4k_scales(r.hg, t, ga, gb, gna, gnb);
    q4k_scales(r.hg8, t, ha, hb, hna, hnb);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t wg = wsel(r.q[i >> 2], i & 3), wg8 = wsel(r.q[2 + (i >> 2)], i & 3);
        {   // sub-block 2t: weights 64t + 4i .. +3
            const uint32_t a0 = hfma2u(hsub2u(lop3_and_or(wg, 0x000F000Fu, H2_1024), H2_1024), ga, gna);
            const uint32_t a2 = hfma2u(hsub2u(lop3_and_or(wg >> 4, 0x000F000Fu, H2_1024), H2_1024), ga, gna);
            const uint32_t a1 = hfma2u(hsub2u(lop3_and_or(wg8, 0x000F000Fu, H2_1024), H2_1024), ha, hna);
            const uint32_t a3 = hfma2u(hsub2u(lop3_and_or(wg8 >> 4, 0x000F000Fu, H2_1024), H2_1024), ha, hna);
            mma_step<NT>(acc, xsc, 2 * i, lane, a0, a1, a2, a3);
        }
        {   // sub-block 2t+1: weights 64t + 32 + 4i .. +3
            const uint32_t a0 = hfma2u(hsub2u(lop3_and_or(wg >> 8, 0x000F000Fu, H2_1024), H2_1024), gb, gnb);
            const uint32_t a2 = hfma2u(hsub2u(lop3_and_or(wg >> 12, 0x000F000Fu, H2_1024), H2_1024), gb, gnb);
            const uint32_t a1 = hfma2u(hsub2u(lop3_and_or(wg8 >> 8, 0x000F000Fu, H2_1024), H2_1024), hb, hnb);
            const uint32_t a3 = hfma2u(hsub2u(lop3_and_or(wg8 >> 12, 0x000F000Fu, H2_1024), H2_1024), hb, hnb);
            mma_step<NT>(acc, xsc, 2 * i + 1, lane, a0, a1, a2, a3);
        }
    }
}

// ------------------------------------------------------------------ Q6_K ---
struct RawQ6K { uint4 q[6]; uint2 scg, scg8; uint32_t d; };
__device__ __forceinline__ void load_raw(RawQ6K &r, const uint8_t *T, int lane) {
#pragma unroll
    for (int p = 0; p < 6; p++) r.q[p] = ldg_stream(T + p * 512 + lane * 16);
    const int g = lane >> 2, n = (lane & 3) >> 1;
    r.scg = ldg64(T + 3072 + g * 16 + 8 * n);
    r.scg8 = ldg64(T + 3072 + (g + 8) * 16 + 8 * n);
    r.d = ldg32(T + 3328 + 4 * g);
}
__device__ __forceinline__ uint32_t q6_pair(uint32_t nw, int nsh, uint32_t hw, int hsh, uint32_t sc2) {
    const uint32_t lo = lop3_and_or(nw >> nsh, 0x000F000Fu, H2_1024);
    const uint32_t hs = hsh >= 0 ? (hw >> hsh) : (hw << -hsh);
    const uint32_t hi = lop3_and_or(hs, 0x00300030u, H2_1024);
    // (1024 + lo) - (2080 - (1024 + 16 hi)) = lo + 16 hi - 32, all exact
    return hmul2u(hsub2u(lo, hsub2u(H2_2080, hi)), sc2);
}
template <int NT>
__device__ __forceinline__ void compute(const RawQ6K &r, const uint2 *xsc, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
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
    scale_acc<NT>(acc, tmp, h2f(r.d & 0xFFFF), h2f(r.d >> 16));
}

// --------------------------------------------------------------- IQ2_XXS ---
// The 32-block scales (db, dl) differ between the four lane columns t of one
// MMA step, so they are applied to the f16 operand before the MMA.
__device__ __forceinline__ uint32_t dup_h2(float v) {
    const __half h = __float2half_rn(v);
    const uint32_t b = __half_as_ushort(h);
    return b | (b << 16);
}
struct RawIQ2 { uint4 q[2]; uint32_t d; };
__device__ __forceinline__ void load_raw(RawIQ2 &r, const uint8_t *T, int lane) {
    r.q[0] = ldg_stream(T + lane * 16);
    r.q[1] = ldg_stream(T + 512 + lane * 16);
    r.d = ldg32(T + 1024 + 4 * (lane >> 2));
}
template <int NT>
__device__ __forceinline__ void compute(const RawIQ2 &r, const uint2 *xsc, float (&acc)[NT][4], int lane,
                                        const uint4 *grid, const uint4 *sgn) {
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
    r.qs = ldg_stream(T + lane * 16);
    r.qh = ldg64(T + 512 + lane * 8);
    r.d = ldg32(T + 768 + 4 * (lane >> 2));
}
template <int NT>
__device__ __forceinline__ void compute(const RawIQ1 &r, const uint2 *xsc, float (&acc)[NT][4], int lane,
                                        const uint4 *grid, const uint4 *) {
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
template <int TYPE, int NT, bool SWIGLU>
__global__ void __launch_bounds__(WARPS * 32) gemv_kernel(const GemvArgs a) {
    using TR = Tr<TYPE>;
    using Raw = typename RawOf<TYPE>::T;
    constexpr int QPC = TR::CHUNK / 4;          // k-quads per chunk
    constexpr int NMAT = SWIGLU ? 2 : 1;
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

    uint2 *xs = reinterpret_cast<uint2 *>(smem);
    const int xs_bytes = a.phase_chunks * TR::STEPS * NT * 32 * 8;
    uint4 *grid = reinterpret_cast<uint4 *>(smem + xs_bytes);
    uint4 *sgn = grid + 256;
    float *red = reinterpret_cast<float *>(smem + xs_bytes + TableBytes<TYPE>::v);

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

    const uint8_t *Wm = a.w[m];
    const uint8_t *Wu = a.w_up;
    for (int p0 = 0; p0 < nc; p0 += a.phase_chunks) {
        const int pc = min(a.phase_chunks, nc - p0);
        if (p0) __syncthreads();   // previous phase done with xs
        // stage x[:, chunks c0+p0 .. +pc) as f16 B fragments
        const int per_tok = pc * QPC;
        for (int idx = threadIdx.x; idx < 8 * NT * per_tok; idx += blockDim.x) {
            const int token = idx / per_tok, rem = idx - token * per_tok;
            const int cc = rem / QPC, kq = rem - cc * QPC;
            const int64_t kg = (int64_t)(c0 + p0 + cc) * TR::CHUNK + 4 * kq;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (token < a.M && kg < a.K) v = __ldg(reinterpret_cast<const float4 *>(a.x + token * a.K + kg));
            int t, s;
            TR::inv(kq, t, s);
            xs[((cc * TR::STEPS + s) * NT + (token >> 3)) * 32 + 4 * (token & 7) + t] =
                make_uint2(pack_h2(v.x, v.y), pack_h2(v.z, v.w));
        }
        __syncthreads();
        if (active && pc > 0) {
            const int64_t tile0 = (rg * a.nchunks + c0 + p0) * (int64_t)TR::TILE;
            const uint8_t *Tm = Wm + tile0;
            const uint8_t *Tu = SWIGLU ? Wu + tile0 : nullptr;
            Raw ra, rb2, ua, ub;
            load_raw(ra, Tm, lane);
            if (SWIGLU) load_raw(ua, Tu, lane);
            for (int cc = 0; cc < pc; cc += 2) {
                const bool more = cc + 1 < pc;
                if (more) {
                    load_raw(rb2, Tm + (cc + 1) * TR::TILE, lane);
                    if (SWIGLU) load_raw(ub, Tu + (cc + 1) * TR::TILE, lane);
                }
                const uint2 *xc = xs + cc * TR::STEPS * NT * 32;
                compute<NT>(ra, xc, acc, lane, grid, sgn);
                if (SWIGLU) compute<NT>(ua, xc, acc2, lane, grid, sgn);
                if (more) {
                    if (cc + 2 < pc) {
                        load_raw(ra, Tm + (cc + 2) * TR::TILE, lane);
                        if (SWIGLU) load_raw(ua, Tu + (cc + 2) * TR::TILE, lane);
                    }
                    const uint2 *xd = xc + TR::STEPS * NT * 32;
                    compute<NT>(rb2, xd, acc, lane, grid, sgn);
                    if (SWIGLU) compute<NT>(ub, xd, acc2, lane, grid, sgn);
                }
            }
        }
    }

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
GemvPlan gemv_plan(int sm_count, int64_t rowgroups, int64_t nchunks, int M) {
    GemvPlan p;
    p.nt = M <= 8 ? 1 : 2;
    p.rowblocks = (int)((rowgroups + WARPS - 1) / WARPS);
    const int64_t target = 2LL * sm_count;
    int64_t ks = (target + p.rowblocks - 1) / p.rowblocks;
    if (ks > 8) ks = 8;
    if (ks > nchunks) ks = nchunks;
    if (ks < 1) ks = 1;
    p.cps = (int)((nchunks + ks - 1) / ks);
    p.kslices = (int)((nchunks + p.cps - 1) / p.cps);
    return p;
}

template <int TYPE, int NT, bool SWIGLU>
static int launch_t(ef_ctx *ctx, GemvArgs &a, int total_rowblocks) {
    using TR = Tr<TYPE>;
    const int per_chunk = TR::STEPS * NT * 32 * 8;
    a.phase_chunks = a.cps;
    if (a.phase_chunks * per_chunk > MAX_XS_BYTES) a.phase_chunks = MAX_XS_BYTES / per_chunk;
    const int nmat = SWIGLU ? 2 : 1;
    const size_t smem = (size_t)a.phase_chunks * per_chunk + TableBytes<TYPE>::v +
                        (a.kslices > 1 ? (size_t)WARPS * nmat * NT * 32 * 16 : 0);
    auto kern = gemv_kernel<TYPE, NT, SWIGLU>;
    static unsigned long long configured = 0;   // per instantiation, one bit per device
    if (ctx->device < 64 && !(configured & (1ull << ctx->device))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return check_cuda(ctx, e, "gemv smem attribute");
        configured |= 1ull << ctx->device;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.kslices, total_rowblocks, 1);
    cfg.blockDim = dim3(WARPS * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.kslices;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.kslices > 1 ? 1 : 0;
    return check_cuda(ctx, cudaLaunchKernelEx(&cfg, kern, a), "gemv launch");
}

template <int TYPE>
static int launch_type(ef_ctx *ctx, GemvArgs &a, int nt, bool swiglu, int total_rowblocks) {
    if (swiglu)
        return nt == 1 ? launch_t<TYPE, 1, true>(ctx, a, total_rowblocks)
                       : launch_t<TYPE, 2, true>(ctx, a, total_rowblocks);
    return nt == 1 ? launch_t<TYPE, 1, false>(ctx, a, total_rowblocks)
                   : launch_t<TYPE, 2, false>(ctx, a, total_rowblocks);
}

int launch_gemv(ef_ctx *ctx, const ef_weight *const *ws, int n, const ef_weight *w_up, const float *x,
                int M, float *const *ys) {
    GemvArgs a = {};
    const ef_weight *w0 = ws[0];
    a.nmat = n;
    int64_t max_rg = 0;
    int total_rb = 0;
    for (int i = 0; i < n; i++) {
        a.w[i] = ws[i]->dev;
        a.y[i] = ys[i];
        a.rows[i] = ws[i]->rows;
        a.rowgroups[i] = ws[i]->rowgroups;
        total_rb += (int)((ws[i]->rowgroups + WARPS - 1) / WARPS);
        a.rb_end[i] = total_rb;
        if (ws[i]->rowgroups > max_rg) max_rg = ws[i]->rowgroups;
    }
    a.w_up = w_up ? w_up->dev : nullptr;
    a.x = x;
    a.M = M;
    a.K = w0->k;
    a.nchunks = w0->nchunks;
    // the plan sees the total rowblocks of all sections as one matrix
    GemvPlan p = gemv_plan(ctx->sm_count, (int64_t)total_rb * WARPS, w0->nchunks, M);
    a.cps = p.cps;
    a.kslices = p.kslices;
    const bool sw = w_up != nullptr;
    switch (w0->type) {
    case EF_Q8_0: return launch_type<EF_Q8_0>(ctx, a, p.nt, sw, total_rb);
    case EF_Q4_K: return launch_type<EF_Q4_K>(ctx, a, p.nt, sw, total_rb);
    case EF_Q6_K: return launch_type<EF_Q6_K>(ctx, a, p.nt, sw, total_rb);
    case EF_IQ2_XXS: return launch_type<EF_IQ2_XXS>(ctx, a, p.nt, sw, total_rb);
    case EF_IQ1_S: return launch_type<EF_IQ1_S>(ctx, a, p.nt, sw, total_rb);
    default: return set_err(ctx, EF_ERR_TYPE, "gemv: unsupported type %d", w0->type);
    }
}

}  // namespace ef

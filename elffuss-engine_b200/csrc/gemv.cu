// gemv.cu -- decode GEMV over repacked GGUF tiles, 1..16 tokens (sm_100a).
//
//   y[t][r] = sum_k dequant(W)[r][k] * x[t][k]        (js/ops.js:827-829)
//   swiglu:  y = silu(Wg.x) * (Wu.x)                   (kernels.gemv.wgsl.js:434-437)
//   sections: several W sharing x and k, one output each (js/ops.gemv.js:192-215)
//
// Design (B200). The GEMV is HBM-bound: every weight byte is read once and
// must become tensor-core operands with as few instructions as possible, while
// enough loads are in flight on every SM to cover DRAM latency.
//
//  * Work split: CTA = one rowblock (8 rowgroups of 16 rows) x one k-slice;
//    the k-slices of a rowblock form one thread-block cluster whose partial
//    sums are added through distributed shared memory in rank order
//    (deterministic, no atomics). The widest k-split (up to 8) whose
//    clusters all fit on the device at once is used.
//  * Weights: each warp streams the tiles of its rowgroup straight from HBM
//    into registers (128-bit non-allocating loads of the lane's fragment
//    parts), one tile ahead of the math. Measured on B200, loads into
//    registers from 16 warps per SM stream faster than shared-memory rings
//    filled by bulk (TMA) or per-lane asynchronous copies. Where the kernel
//    fits 128 registers, a CTA has 16 warps: two per rowgroup, taking
//    alternate chunks and merging their sums in shared memory at the end.
//  * Math: quants become tensor-core operands IN REGISTERS (register-sourced
//    mma.sync is the right tensor instruction for a GEMV: tcgen05.mma reads A
//    from shared or tensor memory, which would add a store and a read of every
//    dequantised weight). Q8_0, Q6_K and the i-quants run m16n8k16 f16 MMAs;
//    Q4_K runs m16n8k32 8-bit MMAs on the raw nibbles, with the 8 MMA columns
//    holding (token, sub-block) pairs for 1-4 tokens (i8_tq).
//  * Activations: converted once per call into the operand layout -- by each
//    CTA for its own chunks when there are 1-2 tokens (one kernel per call),
//    else by a small prep kernel into context scratch -- and staged in shared
//    memory, per phase of chunks when they do not fit at once.
//
// Numerics. f16 types: quants are exact small integers in f16 and the
// per-block scales are applied in f16 with one rounding per weight (Q8_0:
// f16(d*q); IQ2_XXS: f16(db)*grid*sign; IQ1_S: f16(dl)*(grid+delta)), because
// the 16 k-columns of one MMA belong to four different blocks; Q6_K:
// sc*(q-32) is exact in f16 and d is applied in f32 on the accumulator. x is
// rounded to f16. Products are exact and summed in f32 by the tensor cores.
// Q4_K: x per 256-weight chunk and token is x = dx*(xh + xl/256) with two int8
// planes (about 16 significant bits); the nibble products are exact integer
// sums, the 6-bit sub-block scales are applied to them in integers, and d*dx,
// dmin*m*sum(x) in f32.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "gen/iq_grids.h"
#include "internal.h"

namespace cg = cooperative_groups;

namespace ef {

__device__ const __align__(16) uint16_t g_grid_iq2xxs_f16[EF_GRID_IQ2XXS_ENTRIES * 8] = {EF_GRID_IQ2XXS_F16_INIT};
__device__ const __align__(16) uint16_t g_grid_iq1s_f16[EF_GRID_IQ1S_ENTRIES * 8] = {EF_GRID_IQ1S_F16_INIT};

constexpr uint32_t H2_1152 = 0x64806480u;   // half2(1152, 1152)
constexpr uint32_t H2_1032 = 0x64086408u;   // half2(1032, 1032)
constexpr int GV_WARPS = 8;                 // rowgroups (warps) per CTA = one rowblock
constexpr int MAX_XS_BYTES = 64 * 1024;     // shared memory for activation data


struct GemvArgs {
    const uint8_t *w[4];      // repacked tiles of each section
    const uint8_t *w_up;      // SwiGLU partner of w[0] (same geometry)
    float *y[4];
    int64_t rows[4];
    int64_t rowgroups[4];
    int rb_end[4];            // cumulative rowblocks per section
    int nmat;
    int M;
    int64_t nchunks;
    int kslices;              // CTAs (one cluster) per rowblock
    int phase_chunks;         // chunks of activation data in shared memory at a time
    int whole;                // the k-slice's chunks staged once (else phases)
    int xs_bytes;             // shared memory for activation data
    int xs_half;              // offset of the second phase buffer
    int xb;                   // bytes of activation data per chunk
    const uint8_t *xf;        // activation data from ef_gemv_xprep (3..16 tokens)
    const float *x;           // f32 activations [M][K] (1..2 tokens: staged by each CTA)
    int64_t K;
    GemvPush push;            // tensor-parallel row-parallel output (push.n = 0: write y)
    int64_t ctas;             // (host) CTAs of the launch
};

// ---------------------------------------------------------------- traits ---
// STEPS = k16 steps per chunk; inv maps a k-quad (4 consecutive weights of the
// chunk) to the lane column t and the step s that consume it (f16 types).
template <int TYPE> struct Tr;
template <> struct Tr<EF_Q8_0> {
    static constexpr int CHUNK = 128, STEPS = 8, TILE = 2176, I8 = 0;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 3; s = kq & 7; }
};
template <> struct Tr<EF_Q4_0> {   // the Q8_0 chunk and activation layout
    static constexpr int CHUNK = 128, STEPS = 8, TILE = 1152, I8 = 0;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 3; s = kq & 7; }
};
template <> struct Tr<EF_Q5_K> {   // lane t: weights 64t..64t+63, step s: 64t + 4s..+3
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 2816, I8 = 0;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = kq & 15; }
};
template <> struct Tr<EF_Q2_K> {   // the same lane ownership as Q5_K
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 1344, I8 = 0;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = kq & 15; }
};
template <> struct Tr<EF_Q4_K> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 2304, I8 = 1;
    __device__ static void inv(int kq, int &t, int &s) { t = kq >> 4; s = 2 * (kq & 7) + ((kq >> 3) & 1); }
};
template <> struct Tr<EF_Q6_K> {
    static constexpr int CHUNK = 256, STEPS = 16, TILE = 3360, I8 = 1;
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

// Activation layout of the 8-bit types (Q4_K, Q6_K). The 8 columns of the
// 8-bit MMA hold TQ tokens x (8 / TQ) sub-blocks: TQ = 1, 2, 4 for 1, 2, 3-4
// tokens (several sub-blocks share one MMA, each in its own columns, so the
// integer sub-block scales are applied once per group of MMAs), TQ = 8 for
// 5-16 tokens in NT tiles of 8.
__host__ __device__ inline int i8_tq(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }
__host__ __device__ inline int i8_nt(int M) { return M > 8 ? 2 : 1; }
// Per chunk: B fragments [..][lane][16 B: xh b0 b1, xl b0 b1] -- Q4_K:
// [ntile][TQ][lane] (32-weight sub-blocks); Q6_K: [2 TQ flushes][lane] for TQ
// <= 4, [ntile][8 steps][lane] for TQ = 8 (16-weight sub-blocks), then for TQ
// = 8 the f16 m16n8k16 B fragments of S/dx [ntile][lane][8 B]; then the f32
// sums of x over each sub-block [8 or 16][MP]; then dx [MP] (MP = NT * TQ
// padded tokens); rounded up to 16 bytes.
template <int TYPE> __host__ __device__ inline int i8_frag_bytes(int M) {
    const int tq = i8_tq(M), nt = i8_nt(M);
    if (TYPE == EF_Q6_K) return tq <= 4 ? 1024 * tq : 4352 * nt;   // tq = 8: + f16 sums S/dx as MMA B
    return 512 * tq * nt;
}
template <int TYPE> __host__ __device__ inline int i8_xbytes(int M) {
    const int mp = i8_tq(M) * i8_nt(M), subs = TYPE == EF_Q6_K ? 16 : 8;
    return (i8_frag_bytes<TYPE>(M) + 4 * (subs + 1) * mp + 15) & ~15;
}

// Shared-memory reads (activation data).
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
// Tile reads, straight from global memory into registers: quant parts are
// streamed (read once: no L1 allocation); scale bytes that the 4 lanes of a
// group share go through L1.
__device__ __forceinline__ uint4 ldq128(const uint8_t *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldq64(const uint8_t *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldq32(const uint8_t *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ldh128(const uint8_t *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldh64(const uint8_t *p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldh32(const uint8_t *p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// Asynchronous 16-byte global -> shared copies (LDGSTS, L2 only), for the
// activation phases.

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
    for (int p = 0; p < 4; p++) r.q[p] = ldq128(T + p * 512 + lane * 16);
    r.sc = ldq32(T + 2048 + lane * 4);
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

// ------------------------------------------------------------------ Q4_0 ---
// lane (g,t): part 0 / 1 = the 32 nibbles of block t of row g / g+8 (word j:
// weights 8j..8j+7 at the nibble slots of common.cuh q40_slot), the two rows'
// f16 d at 1024 + 4*lane.
struct RawQ40 { uint4 q[2]; uint32_t sc; };
__device__ __forceinline__ void load_raw(RawQ40 &r, const uint8_t *T, int lane) {
    r.q[0] = ldq128(T + lane * 16);
    r.q[1] = ldq128(T + 512 + lane * 16);
    r.sc = ldq32(T + 1024 + lane * 4);
}
template <int NT>
__device__ __forceinline__ void compute(const RawQ40 &r, const uint8_t *xc, int M, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
    const XF xsc = make_xf<NT>(xc, M, lane);
    const uint32_t dg = prmt(r.sc, 0, 0x1010), dg8 = prmt(r.sc, 0, 0x3232);
#pragma unroll
    for (int s = 0; s < 8; s++) {
        const int sh = 8 * (s & 1);
        const uint32_t wg = wsel(r.q[0], s >> 1), wg8 = wsel(r.q[1], s >> 1);
        // (1024 + q) - 1032 = q - 8 exactly; then one rounding of d*(q-8)
        const uint32_t a0 = hmul2u(hsub2u(((wg >> sh) & 0x000F000Fu) | 0x64006400u, H2_1032), dg);
        const uint32_t a2 = hmul2u(hsub2u(((wg >> (sh + 4)) & 0x000F000Fu) | 0x64006400u, H2_1032), dg);
        const uint32_t a1 = hmul2u(hsub2u(((wg8 >> sh) & 0x000F000Fu) | 0x64006400u, H2_1032), dg8);
        const uint32_t a3 = hmul2u(hsub2u(((wg8 >> (sh + 4)) & 0x000F000Fu) | 0x64006400u, H2_1032), dg8);
        mma_step<NT>(acc, xsc, s, lane, a0, a1, a2, a3);
    }
}

// --------------------------------------------------------- Q5_K / Q2_K ---
// f16 operands: f16_pair_dm (common.cuh) -- q as (1024 + q) - 1024 exactly,
// then one f16 fma with the sub-block's f16(d * sc) and -f16(dmin * m).

// Q5_K, lane (g,t): parts 0,1 / 2,3 = qs bytes 32t.. of rows g / g+8, part 4 =
// fifth-bit words (low, high sub-block) of both rows, the rows' verbatim
// 16-byte headers (d, dmin, scale_min_k4 bytes) at 2560 + 16 * row.
struct RawQ5K { uint4 q[5]; uint4 hg, hg8; };
__device__ __forceinline__ void load_raw(RawQ5K &r, const uint8_t *T, int lane) {
#pragma unroll
    for (int p = 0; p < 5; p++) r.q[p] = ldq128(T + p * 512 + lane * 16);
    const int g = lane >> 2;
    r.hg = ldh128(T + 2560 + g * 16);
    r.hg8 = ldh128(T + 2560 + (g + 8) * 16);
}
// f16 (d * sc, -dmin * m) of sub-block j of a Q5_K / Q4_K header (scale_min_k4)
__device__ __forceinline__ void q5_dm(const uint4 &h, int j, uint32_t &d2, uint32_t &negm2) {
    const uint32_t w[4] = {h.x, h.y, h.z, h.w};
    auto byte = [&](int i) { return (int)((w[i >> 2] >> (8 * (i & 3))) & 0xFF); };
    int sc, mn;
    if (j < 4) {
        sc = byte(4 + j) & 63;
        mn = byte(8 + j) & 63;
    } else {
        sc = (byte(8 + j) & 0xF) | ((byte(j) >> 6) << 4);
        mn = (byte(8 + j) >> 4) | ((byte(4 + j) >> 6) << 4);
    }
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    d2 = f16x2_bcast(d * (float)sc);
    negm2 = f16x2_bcast(-(dmin * (float)mn));
}
template <int NT>
__device__ __forceinline__ void compute(const RawQ5K &r, const uint8_t *xc, int M, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
    const XF xsc = make_xf<NT>(xc, M, lane);
    const int t = lane & 3;
    uint32_t dg[2], mg[2], dg8[2], mg8[2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
        q5_dm(r.hg, 2 * t + u, dg[u], mg[u]);
        q5_dm(r.hg8, 2 * t + u, dg8[u], mg8[u]);
    }
    const uint32_t hb[4] = {r.q[4].x, r.q[4].y, r.q[4].z, r.q[4].w};   // row g: lo, hi; row g+8: lo, hi
#pragma unroll
    for (int s = 0; s < 16; s++) {
        const int u = s >> 3, ls = s & 7;                                  // sub-block 2t+u, bytes 4ls..
        const uint32_t wg = wsel(r.q[ls >> 2], ls & 3), wg8 = wsel(r.q[2 + (ls >> 2)], ls & 3);
        const uint32_t ng = u ? (wg >> 4) & 0x0F0F0F0Fu : wg & 0x0F0F0F0Fu;
        const uint32_t ng8 = u ? (wg8 >> 4) & 0x0F0F0F0Fu : wg8 & 0x0F0F0F0Fu;
        const uint32_t q5 = ng | (spread4((hb[u] >> (4 * ls)) & 0xF) << 4);
        const uint32_t q58 = ng8 | (spread4((hb[2 + u] >> (4 * ls)) & 0xF) << 4);
        const uint32_t a0 = f16_pair_dm(q5, 0x5140, dg[u], mg[u]);
        const uint32_t a2 = f16_pair_dm(q5, 0x7362, dg[u], mg[u]);
        const uint32_t a1 = f16_pair_dm(q58, 0x5140, dg8[u], mg8[u]);
        const uint32_t a3 = f16_pair_dm(q58, 0x7362, dg8[u], mg8[u]);
        mma_step<NT>(acc, xsc, s, lane, a0, a1, a2, a3);
    }
}

// Q2_K, lane (g,t): part 0 / 1 = the 2-bit q of weights 64t.. of row g / g+8
// (word w, byte c, bits 2s'.. = weight 4(4w + s') + c), the four scale bytes
// of its sub-blocks per row at 1024 + 8 * lane, d and dmin per row at 1280.
struct RawQ2K { uint4 q[2]; uint2 sc; uint32_t dm, dm8; };
__device__ __forceinline__ void load_raw(RawQ2K &r, const uint8_t *T, int lane) {
    r.q[0] = ldq128(T + lane * 16);
    r.q[1] = ldq128(T + 512 + lane * 16);
    r.sc = ldq64(T + 1024 + lane * 8);
    const int g = lane >> 2;
    r.dm = ldh32(T + 1280 + 4 * g);
    r.dm8 = ldh32(T + 1280 + 4 * (g + 8));
}
template <int NT>
__device__ __forceinline__ void compute(const RawQ2K &r, const uint8_t *xc, int M, float (&acc)[NT][4], int lane,
                                        const uint4 *, const uint4 *) {
    const XF xsc = make_xf<NT>(xc, M, lane);
    const float d = __half2float(__ushort_as_half((unsigned short)(r.dm & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(r.dm >> 16)));
    const float d8 = __half2float(__ushort_as_half((unsigned short)(r.dm8 & 0xFFFF)));
    const float dmin8 = __half2float(__ushort_as_half((unsigned short)(r.dm8 >> 16)));
#pragma unroll
    for (int k = 0; k < 4; k++) {                                          // sub-block 4t + k: steps 4k..4k+3
        const int sc = (int)((r.sc.x >> (8 * k)) & 0xFF), sc8 = (int)((r.sc.y >> (8 * k)) & 0xFF);
        const uint32_t dd = f16x2_bcast(d * (float)(sc & 15)), mm = f16x2_bcast(-(dmin * (float)(sc >> 4)));
        const uint32_t dd8 = f16x2_bcast(d8 * (float)(sc8 & 15)), mm8 = f16x2_bcast(-(dmin8 * (float)(sc8 >> 4)));
#pragma unroll
        for (int sp = 0; sp < 4; sp++) {
            const int s = 4 * k + sp;
            const uint32_t qg = (wsel(r.q[0], k) >> (2 * sp)) & 0x03030303u;
            const uint32_t qg8 = (wsel(r.q[1], k) >> (2 * sp)) & 0x03030303u;
            const uint32_t a0 = f16_pair_dm(qg, 0x5140, dd, mm), a2 = f16_pair_dm(qg, 0x7362, dd, mm);
            const uint32_t a1 = f16_pair_dm(qg8, 0x5140, dd8, mm8), a3 = f16_pair_dm(qg8, 0x7362, dd8, mm8);
            mma_step<NT>(acc, xsc, s, lane, a0, a1, a2, a3);
        }
    }
}

// ------------------------------------------------------------------ Q4_K ---
// lane (g,t): for each 64-weight group j the bytes l = 4t..4t+3 and
// 16+4t..16+4t+3 of rows g and g+8 (low nibble: sub-block 2j, high nibble:
// sub-block 2j+1), and the verbatim 16-byte headers of rows g and g+8.
struct RawQ4K { uint4 q[4]; uint4 hg, hg8; };
__device__ __forceinline__ void load_raw(RawQ4K &r, const uint8_t *T, int lane) {
#pragma unroll
    for (int p = 0; p < 4; p++) r.q[p] = ldq128(T + p * 512 + lane * 16);
    const int g = lane >> 2;
    r.hg = ldh128(T + 2048 + g * 16);
    r.hg8 = ldh128(T + 2048 + (g + 8) * 16);
}
// 6-bit scales (sc) and mins (m) of one row, one per byte: sub-blocks 0..3
// and 4..7 (scale_min_k4, kernels.wgsl.js:94-104).
struct Q4Scales { uint32_t scl, sch, ml, mh; };
__device__ __forceinline__ Q4Scales q4k_scales(const uint4 &h) {
    Q4Scales s;
    s.scl = h.y & 0x3F3F3F3Fu;
    s.sch = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    s.ml = h.z & 0x3F3F3F3Fu;
    s.mh = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    return s;
}
// byte `b` of w as an integer
__device__ __forceinline__ int byte_of(uint32_t w, int b) { return (int)prmt(w, 0u, 0x4440u | (uint32_t)b); }

// A fragment of sub-block s (m16n8k32, u8): rows g, g+8; k = 4t.., 16+4t..
// The high-nibble sub-blocks (odd s) are taken as 16*q (mask 0xF0), so every
// integer product sum carries a factor 16 once even sub-blocks' scales are
// shifted by 4.
__device__ __forceinline__ void q4k_afrag(const RawQ4K &r, int s, uint32_t &a0, uint32_t &a1, uint32_t &a2,
                                          uint32_t &a3) {
    const int j = s >> 1;
    const uint4 &pg = r.q[j >> 1], &ph = r.q[2 + (j >> 1)];
    const uint32_t mask = (s & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
    a0 = ((j & 1) ? pg.z : pg.x) & mask;
    a1 = ((j & 1) ? ph.z : ph.x) & mask;
    a2 = ((j & 1) ? pg.w : pg.y) & mask;
    a3 = ((j & 1) ? ph.w : ph.y) & mask;
}

// Q4_K tile: acc[nt][i] (row g or g+8 by i>>1; lane column 2t + (i&1)) +=
//   d*dx*(sum_sub sc*sum_k q*(xh + xl/256)) - dmin*sum_sub m*S_sub
// with the column -> (sub-block, token) mapping of TQ (see i8_tq).
template <int TQ, int NT>
__device__ __forceinline__ void compute_q4k(const RawQ4K &r, const uint8_t *xc, float (&acc)[NT][4], int lane) {
    constexpr int FL = 8 / TQ;   // sub-blocks per MMA group (flush)
    constexpr int MP = NT * TQ;
    const int g = lane >> 2, t = lane & 3;
    const Q4Scales sg = q4k_scales(r.hg), sh = q4k_scales(r.hg8);
    const float *S = reinterpret_cast<const float *>(xc + 512 * TQ * NT);
    const float *DX = S + 8 * MP;
    int ih[NT][4], il[NT][4];
    float ms[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            ih[nt][i] = il[nt][i] = 0;
            ms[nt][i] = 0.f;
        }
    if constexpr (TQ == 8) {
        // one sub-block per MMA, all 8 columns are tokens
#pragma unroll
        for (int s = 0; s < 8; s++) {
            uint32_t a0, a1, a2, a3;
            q4k_afrag(r, s, a0, a1, a2, a3);
            const int shl = (s & 1) ? 0 : 4;
            const int scg = byte_of(s < 4 ? sg.scl : sg.sch, s & 3) << shl;
            const int sch = byte_of(s < 4 ? sh.scl : sh.sch, s & 3) << shl;
            const float mg = (float)byte_of(s < 4 ? sg.ml : sg.mh, s & 3);
            const float mh = (float)byte_of(s < 4 ? sh.ml : sh.mh, s & 3);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const uint4 b = lds128(xc + ((nt * 8 + s) * 32 + lane) * 16);
                int dh[4] = {0, 0, 0, 0}, dl[4] = {0, 0, 0, 0};
                imma16832(dh, a0, a1, a2, a3, b.x, b.y);
                imma16832(dl, a0, a1, a2, a3, b.z, b.w);
                ih[nt][0] += scg * dh[0];
                ih[nt][1] += scg * dh[1];
                ih[nt][2] += sch * dh[2];
                ih[nt][3] += sch * dh[3];
                il[nt][0] += scg * dl[0];
                il[nt][1] += scg * dl[1];
                il[nt][2] += sch * dl[2];
                il[nt][3] += sch * dl[3];
                const float2 sv = *reinterpret_cast<const float2 *>(S + s * MP + nt * 8 + 2 * t);
                ms[nt][0] = fmaf(mg, sv.x, ms[nt][0]);
                ms[nt][1] = fmaf(mg, sv.y, ms[nt][1]);
                ms[nt][2] = fmaf(mh, sv.x, ms[nt][2]);
                ms[nt][3] = fmaf(mh, sv.y, ms[nt][3]);
            }
        }
    } else {
        // B column g of this lane carries token g % TQ of sub-blocks with
        // s % FL == g / TQ: one 16-byte fragment per flush, zero otherwise.
        const int sgb = g / TQ;
#pragma unroll
        for (int f = 0; f < TQ; f++) {
            const uint4 xb = lds128(xc + (f * 32 + lane) * 16);
            // two independent MMA chains (even / odd steps) for latency; the
            // columns they fill are disjoint, so their sum is exact
            int dh[4] = {0, 0, 0, 0}, dl[4] = {0, 0, 0, 0}, eh[4] = {0, 0, 0, 0}, el[4] = {0, 0, 0, 0};
#pragma unroll
            for (int q = 0; q < FL; q++) {
                uint32_t a0, a1, a2, a3;
                q4k_afrag(r, f * FL + q, a0, a1, a2, a3);
                const uint32_t mk = q == sgb ? 0xFFFFFFFFu : 0u;
                if (q & 1) {
                    imma16832(eh, a0, a1, a2, a3, xb.x & mk, xb.y & mk);
                    imma16832(el, a0, a1, a2, a3, xb.z & mk, xb.w & mk);
                } else {
                    imma16832(dh, a0, a1, a2, a3, xb.x & mk, xb.y & mk);
                    imma16832(dl, a0, a1, a2, a3, xb.z & mk, xb.w & mk);
                }
            }
            if (FL > 1)
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    dh[i] += eh[i];
                    dl[i] += el[i];
                }
            // accumulator column 2t + c now holds sub-block f*FL + (2t+c)/TQ
            // of token (2t+c) % TQ
            int s0, s1, tok0;
            if (TQ == 1) {
                s0 = 2 * t;
                s1 = 2 * t + 1;
                tok0 = 0;
            } else if (TQ == 2) {
                s0 = s1 = 4 * f + t;
                tok0 = 0;
            } else {
                s0 = s1 = 2 * f + (t >> 1);
                tok0 = 2 * (t & 1);
            }
            const int sh0 = (s0 & 1) ? 0 : 4, sh1 = (s1 & 1) ? 0 : 4;
            const uint32_t wsg = s0 < 4 ? sg.scl : sg.sch, wsh = s0 < 4 ? sh.scl : sh.sch;
            const uint32_t wmg = s0 < 4 ? sg.ml : sg.mh, wmh = s0 < 4 ? sh.ml : sh.mh;
            const int scg0 = byte_of(wsg, s0 & 3) << sh0, scg1 = byte_of(wsg, s1 & 3) << sh1;
            const int sch0 = byte_of(wsh, s0 & 3) << sh0, sch1 = byte_of(wsh, s1 & 3) << sh1;
            ih[0][0] += scg0 * dh[0];
            ih[0][1] += scg1 * dh[1];
            ih[0][2] += sch0 * dh[2];
            ih[0][3] += sch1 * dh[3];
            il[0][0] += scg0 * dl[0];
            il[0][1] += scg1 * dl[1];
            il[0][2] += sch0 * dl[2];
            il[0][3] += sch1 * dl[3];
            const float mg0 = (float)byte_of(wmg, s0 & 3), mg1 = (float)byte_of(wmg, s1 & 3);
            const float mh0 = (float)byte_of(wmh, s0 & 3), mh1 = (float)byte_of(wmh, s1 & 3);
            float2 sv;
            if (TQ == 1) sv = *reinterpret_cast<const float2 *>(S + s0);               // S[s0][0], S[s1][0]
            else sv = *reinterpret_cast<const float2 *>(S + s0 * MP + tok0);          // S[s][tok0], S[s][tok0+1]
            ms[0][0] = fmaf(mg0, sv.x, ms[0][0]);
            ms[0][1] = fmaf(mg1, sv.y, ms[0][1]);
            ms[0][2] = fmaf(mh0, sv.x, ms[0][2]);
            ms[0][3] = fmaf(mh1, sv.y, ms[0][3]);
        }
    }
    // d*dx/16 and dmin per row, dx per lane column
    const float dg = h2f(r.hg.x & 0xFFFF), mng = h2f(r.hg.x >> 16);
    const float dh8 = h2f(r.hg8.x & 0xFFFF), mnh = h2f(r.hg8.x >> 16);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        float dx0, dx1;
        if (TQ == 1) {
            dx0 = dx1 = DX[0];
        } else {
            const int tk = TQ == 2 ? 0 : TQ == 4 ? 2 * (t & 1) : nt * 8 + 2 * t;
            const float2 d2 = *reinterpret_cast<const float2 *>(DX + tk);
            dx0 = d2.x;
            dx1 = d2.y;
        }
        const float k0 = dx0 * (1.f / 16.f), k1 = dx1 * (1.f / 16.f);
        const float v0 = fmaf((float)il[nt][0], 1.f / 256.f, (float)ih[nt][0]);
        const float v1 = fmaf((float)il[nt][1], 1.f / 256.f, (float)ih[nt][1]);
        const float v2 = fmaf((float)il[nt][2], 1.f / 256.f, (float)ih[nt][2]);
        const float v3 = fmaf((float)il[nt][3], 1.f / 256.f, (float)ih[nt][3]);
        acc[nt][0] = fmaf(-mng, ms[nt][0], fmaf(dg * k0, v0, acc[nt][0]));
        acc[nt][1] = fmaf(-mng, ms[nt][1], fmaf(dg * k1, v1, acc[nt][1]));
        acc[nt][2] = fmaf(-mnh, ms[nt][2], fmaf(dh8 * k0, v2, acc[nt][2]));
        acc[nt][3] = fmaf(-mnh, ms[nt][3], fmaf(dh8 * k1, v3, acc[nt][3]));
    }
}

// ------------------------------------------------------------------ Q6_K ---
// lane (g,t): parts 0,1 = low-nibble words of row g for steps 0-3, 4-7;
// parts 2,3 = the same for row g+8; parts 4,5 = high-bit words (one per pair
// of steps) of rows g and g+8; the rows' 16 int8 scales; d of both rows.
struct RawQ6K { uint4 q[6]; uint4 scg, scg8; uint32_t d; };
__device__ __forceinline__ void load_raw(RawQ6K &r, const uint8_t *T, int lane) {
#pragma unroll
    for (int p = 0; p < 6; p++) r.q[p] = ldq128(T + p * 512 + lane * 16);
    const int g = lane >> 2;
    r.scg = ldh128(T + 3072 + g * 16);
    r.scg8 = ldh128(T + 3072 + (g + 8) * 16);
    r.d = ldh32(T + 3328 + 4 * g);
}
// D (+)= A(16x16 u8, row) * B(16x8 s8, col), s32 accumulate (one 16-weight sub-block).
__device__ __forceinline__ void imma16816(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}
// u8 A fragment of 32-weight step s: 6-bit q = low nibble | high 2 bits << 4
// for rows g (a0: k 4t.., a2: k 16+4t..) and g+8 (a1, a3).
__device__ __forceinline__ void q6k_afrag(const RawQ6K &r, int s, uint32_t &a0, uint32_t &a1, uint32_t &a2,
                                          uint32_t &a3) {
    const uint32_t ng = wsel(r.q[s >> 2], s & 3), nh = wsel(r.q[2 + (s >> 2)], s & 3);
    const uint32_t hg = wsel(r.q[4], s >> 1), hh = wsel(r.q[5], s >> 1);
    // high fields per byte: bits 0-1 / 2-3 = even step halves 0 / 1, 4-5 / 6-7 = odd step
    const uint32_t g0 = (s & 1) ? hg : hg << 4, g1 = (s & 1) ? hg >> 2 : hg << 2;
    const uint32_t h0 = (s & 1) ? hh : hh << 4, h1 = (s & 1) ? hh >> 2 : hh << 2;
    a0 = lop3_and_or(g0, 0x30303030u, ng & 0x0F0F0F0Fu);
    a2 = lop3_and_or(g1, 0x30303030u, (ng >> 4) & 0x0F0F0F0Fu);
    a1 = lop3_and_or(h0, 0x30303030u, nh & 0x0F0F0F0Fu);
    a3 = lop3_and_or(h1, 0x30303030u, (nh >> 4) & 0x0F0F0F0Fu);
}
// signed int8 scale `i` (runtime) of a row's 16 scale bytes
__device__ __forceinline__ int q6_sc(const uint4 &v, int i) {
    const uint32_t b = (uint32_t)(i & 3), sgn = 8u | b;
    return (int)prmt(wsel(v, i >> 2), 0u, b | (sgn << 4) | (sgn << 8) | (sgn << 12));
}

// Q6_K tile: w = d * sc * (q - 32) over 16-weight sub-blocks:
//   acc += d * (dx * sum_sub sc * sum_k q * (xh + xl/256) - 32 * sum_sub sc * S_sub)
// TQ <= 4: the 8 MMA columns hold 8/TQ sub-blocks x TQ tokens; a lane's B
// fragment is nonzero in one step of each group (one of b0/b1). TQ = 8: one
// 16-k MMA per sub-block.
template <int TQ, int NT>
__device__ __forceinline__ void compute_q6k(const RawQ6K &r, const uint8_t *xc, float (&acc)[NT][4], int lane) {
    constexpr int MP = NT * TQ;
    const int g = lane >> 2, t = lane & 3;
    const float *S = reinterpret_cast<const float *>(xc + (TQ <= 4 ? 1024 * TQ : 4352 * NT));
    const float *DX = S + 16 * MP;
    int ih[NT][4], il[NT][4];
    float ms[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            ih[nt][i] = il[nt][i] = 0;
            ms[nt][i] = 0.f;
        }
    if constexpr (TQ == 8) {
#pragma unroll
        for (int s = 0; s < 8; s++) {
            uint32_t a0, a1, a2, a3;
            q6k_afrag(r, s, a0, a1, a2, a3);
            const int sg0 = q6_sc(r.scg, 2 * s), sg1 = q6_sc(r.scg, 2 * s + 1);
            const int sh0 = q6_sc(r.scg8, 2 * s), sh1 = q6_sc(r.scg8, 2 * s + 1);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const uint4 b = lds128(xc + ((nt * 8 + s) * 32 + lane) * 16);
                int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0}, e0[4] = {0, 0, 0, 0}, e1[4] = {0, 0, 0, 0};
                imma16816(d0, a0, a1, b.x);   // sub-block 2s, plane h
                imma16816(d1, a2, a3, b.y);   // sub-block 2s+1
                imma16816(e0, a0, a1, b.z);   // plane l
                imma16816(e1, a2, a3, b.w);
                ih[nt][0] += sg0 * d0[0] + sg1 * d1[0];
                ih[nt][1] += sg0 * d0[1] + sg1 * d1[1];
                ih[nt][2] += sh0 * d0[2] + sh1 * d1[2];
                ih[nt][3] += sh0 * d0[3] + sh1 * d1[3];
                il[nt][0] += sg0 * e0[0] + sg1 * e1[0];
                il[nt][1] += sg0 * e0[1] + sg1 * e1[1];
                il[nt][2] += sh0 * e0[2] + sh1 * e1[2];
                il[nt][3] += sh0 * e0[3] + sh1 * e1[3];
            }
        }
        // sum_sub sc * S_sub / dx for 16 rows x 8 tokens: one f16 MMA per tile
        // (int8 scales are exact in f16; A: sub-blocks 2t, 2t+1 and 8+2t, 9+2t)
        const uint32_t ma0 = pack_h2((float)q6_sc(r.scg, 2 * t), (float)q6_sc(r.scg, 2 * t + 1));
        const uint32_t ma1 = pack_h2((float)q6_sc(r.scg8, 2 * t), (float)q6_sc(r.scg8, 2 * t + 1));
        const uint32_t ma2 = pack_h2((float)q6_sc(r.scg, 8 + 2 * t), (float)q6_sc(r.scg, 9 + 2 * t));
        const uint32_t ma3 = pack_h2((float)q6_sc(r.scg8, 8 + 2 * t), (float)q6_sc(r.scg8, 9 + 2 * t));
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const uint2 b = lds64(xc + 4096 * NT + (nt * 32 + lane) * 8);
            mma16816(ms[nt], ma0, ma1, ma2, ma3, b.x, b.y);
        }
    } else {
        constexpr int FLS = 8 / TQ;          // sub-blocks per flush
        constexpr int SPF = FLS / 2;         // 32-weight steps per flush
        const int ql = (g / TQ) >> 1;        // step of the flush in which this lane's B fragment is nonzero
#pragma unroll
        for (int f = 0; f < 2 * TQ; f++) {
            const uint4 xb = lds128(xc + (f * 32 + lane) * 16);
            int dh[4] = {0, 0, 0, 0}, dl[4] = {0, 0, 0, 0}, eh[4] = {0, 0, 0, 0}, el[4] = {0, 0, 0, 0};
#pragma unroll
            for (int q = 0; q < SPF; q++) {
                uint32_t a0, a1, a2, a3;
                q6k_afrag(r, f * SPF + q, a0, a1, a2, a3);
                const uint32_t mk = (SPF == 1 || q == ql) ? 0xFFFFFFFFu : 0u;
                if (q & 1) {
                    imma16832(eh, a0, a1, a2, a3, xb.x & mk, xb.y & mk);
                    imma16832(el, a0, a1, a2, a3, xb.z & mk, xb.w & mk);
                } else {
                    imma16832(dh, a0, a1, a2, a3, xb.x & mk, xb.y & mk);
                    imma16832(dl, a0, a1, a2, a3, xb.z & mk, xb.w & mk);
                }
            }
            if (SPF > 1)
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    dh[i] += eh[i];
                    dl[i] += el[i];
                }
            // accumulator column 2t + c: sub-block f*FLS + (2t+c)/TQ, token (2t+c) % TQ
            int s0, s1, tok0;
            if (TQ == 1) {
                s0 = 8 * f + 2 * t;
                s1 = s0 + 1;
                tok0 = 0;
            } else if (TQ == 2) {
                s0 = s1 = 4 * f + t;
                tok0 = 0;
            } else {
                s0 = s1 = 2 * f + (t >> 1);
                tok0 = 2 * (t & 1);
            }
            const int sg0 = q6_sc(r.scg, s0), sg1 = q6_sc(r.scg, s1);
            const int sh0 = q6_sc(r.scg8, s0), sh1 = q6_sc(r.scg8, s1);
            ih[0][0] += sg0 * dh[0];
            ih[0][1] += sg1 * dh[1];
            ih[0][2] += sh0 * dh[2];
            ih[0][3] += sh1 * dh[3];
            il[0][0] += sg0 * dl[0];
            il[0][1] += sg1 * dl[1];
            il[0][2] += sh0 * dl[2];
            il[0][3] += sh1 * dl[3];
            float2 sv;
            if (TQ == 1) sv = *reinterpret_cast<const float2 *>(S + s0);               // S[s0][0], S[s0+1][0]
            else sv = *reinterpret_cast<const float2 *>(S + s0 * MP + tok0);          // S[s][tok0], S[s][tok0+1]
            ms[0][0] = fmaf((float)sg0, sv.x, ms[0][0]);
            ms[0][1] = fmaf((float)sg1, sv.y, ms[0][1]);
            ms[0][2] = fmaf((float)sh0, sv.x, ms[0][2]);
            ms[0][3] = fmaf((float)sh1, sv.y, ms[0][3]);
        }
    }
    const float dg = h2f(r.d & 0xFFFF), dh8 = h2f(r.d >> 16);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        float dx0, dx1;
        if (TQ == 1) {
            dx0 = dx1 = DX[0];
        } else {
            const int tk = TQ == 2 ? 0 : TQ == 4 ? 2 * (t & 1) : nt * 8 + 2 * t;
            const float2 d2 = *reinterpret_cast<const float2 *>(DX + tk);
            dx0 = d2.x;
            dx1 = d2.y;
        }
        const float v0 = fmaf((float)il[nt][0], 1.f / 256.f, (float)ih[nt][0]);
        const float v1 = fmaf((float)il[nt][1], 1.f / 256.f, (float)ih[nt][1]);
        const float v2 = fmaf((float)il[nt][2], 1.f / 256.f, (float)ih[nt][2]);
        const float v3 = fmaf((float)il[nt][3], 1.f / 256.f, (float)ih[nt][3]);
        if (TQ == 8) {   // ms holds sum sc * S / dx
            acc[nt][0] = fmaf(dg * dx0, fmaf(-32.f, ms[nt][0], v0), acc[nt][0]);
            acc[nt][1] = fmaf(dg * dx1, fmaf(-32.f, ms[nt][1], v1), acc[nt][1]);
            acc[nt][2] = fmaf(dh8 * dx0, fmaf(-32.f, ms[nt][2], v2), acc[nt][2]);
            acc[nt][3] = fmaf(dh8 * dx1, fmaf(-32.f, ms[nt][3], v3), acc[nt][3]);
        } else {
            acc[nt][0] = fmaf(dg, fmaf(dx0, v0, -32.f * ms[nt][0]), acc[nt][0]);
            acc[nt][1] = fmaf(dg, fmaf(dx1, v1, -32.f * ms[nt][1]), acc[nt][1]);
            acc[nt][2] = fmaf(dh8, fmaf(dx0, v2, -32.f * ms[nt][2]), acc[nt][2]);
            acc[nt][3] = fmaf(dh8, fmaf(dx1, v3, -32.f * ms[nt][3]), acc[nt][3]);
        }
    }
}

// --------------------------------------------------------------- IQ2_XXS ---
struct RawIQ2 { uint4 q[2]; uint32_t d; };
__device__ __forceinline__ void load_raw(RawIQ2 &r, const uint8_t *T, int lane) {
    r.q[0] = ldq128(T + lane * 16);
    r.q[1] = ldq128(T + 512 + lane * 16);
    r.d = ldh32(T + 1024 + 4 * (lane >> 2));
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
    r.qs = ldq128(T + lane * 16);
    r.qh = ldq64(T + 512 + lane * 8);
    r.d = ldh32(T + 768 + 4 * (lane >> 2));
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
template <> struct RawOf<EF_Q4_0> { using T = RawQ40; };
template <> struct RawOf<EF_Q5_K> { using T = RawQ5K; };
template <> struct RawOf<EF_Q2_K> { using T = RawQ2K; };
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
// [tid, tid + nthreads) -- either one CTA (1-2 tokens) or the whole grid of
// the prep kernel (3..16 tokens).
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
// 8-bit types: per 256-weight chunk and token x = dx * (xh + xl/256), dx =
// max|x|/127, xh = rne(x/dx), xl = rne(256 * (x/dx - xh)), both int8, as the
// B fragments of the column layout of i8_tq (tokens M..MP-1 are zero); the f32
// sums of x over each sub-block; dx. One warp per (chunk, token); lane l holds
// weights 8l .. 8l+7.
template <int TYPE>
__device__ __forceinline__ void stage_i8(const float *__restrict__ x, int M, int64_t K, int64_t c, int n,
                                         uint8_t *dst, int xb, int tid, int nthreads) {
    const int lane = tid & 31;
    const int tq = i8_tq(M), ntl = i8_nt(M), mp = tq * ntl;
    for (int w = tid >> 5; w < n * mp; w += nthreads >> 5) {
        const int cc = w / mp, token = w - cc * mp;
        const int64_t k0 = (c + cc) * 256 + 8 * lane;
        float v[8];
        if (token < M && k0 < K) {
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
        const float sum16 = sum + __shfl_xor_sync(0xffffffffu, sum, 1);
        const float sum32 = sum16 + __shfl_xor_sync(0xffffffffu, sum16, 2);
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
        float *S = reinterpret_cast<float *>(base + i8_frag_bytes<TYPE>(M));
        const int nt = token >> 3, tk = token & 7;            // n-tile, token within it
        if (TYPE == EF_Q4_K) {
            const int fl = 8 / tq;
            const int sub = lane >> 2, kk = 8 * (lane & 3);   // 32-weight sub-block, k within it
            const int n_col = (sub % fl) * tq + (tq == 8 ? tk : token);   // B column
            const int f = sub / fl;                           // fragment index of that lane
            const int tb = (kk & 15) >> 2, reg = kk >> 4;     // lane t of the B fragment, b0 or b1
            uint8_t *fr0 = base + ((nt * tq + f) * 32 + 4 * n_col + tb) * 16 + reg * 4;
            uint8_t *fr1 = fr0 + 16;
            *reinterpret_cast<uint32_t *>(fr0) = wq[0];
            *reinterpret_cast<uint32_t *>(fr0 + 8) = wl[0];
            *reinterpret_cast<uint32_t *>(fr1) = wq[1];
            *reinterpret_cast<uint32_t *>(fr1 + 8) = wl[1];
            if ((lane & 3) == 0) S[sub * mp + token] = sum32;
            if (lane == 0) S[8 * mp + token] = dx;
        } else {
            // Q6_K: 16-weight sub-block sig = lane >> 1 is half sig & 1 (b0 or
            // b1) of 32-weight step sig >> 1; the lane's 8 weights are the
            // k-quads of B-fragment lanes t = 2(lane&1), 2(lane&1)+1.
            const int sig = lane >> 1, half = sig & 1, tb = 2 * (lane & 1);
            if (tq <= 4) {
                const int fls = 8 / tq;                       // sub-blocks per flush
                const int n_col = (sig % fls) * tq + token, f = sig / fls;
                uint8_t *fr0 = base + (f * 32 + 4 * n_col + tb) * 16;
                uint8_t *fr1 = fr0 + 16;
                // the other half of each entry is zero: one sub-block per lane and flush
                *reinterpret_cast<uint2 *>(fr0) = half ? make_uint2(0u, wq[0]) : make_uint2(wq[0], 0u);
                *reinterpret_cast<uint2 *>(fr0 + 8) = half ? make_uint2(0u, wl[0]) : make_uint2(wl[0], 0u);
                *reinterpret_cast<uint2 *>(fr1) = half ? make_uint2(0u, wq[1]) : make_uint2(wq[1], 0u);
                *reinterpret_cast<uint2 *>(fr1 + 8) = half ? make_uint2(0u, wl[1]) : make_uint2(wl[1], 0u);
            } else {
                uint8_t *fr0 = base + ((nt * 8 + (sig >> 1)) * 32 + 4 * tk + tb) * 16 + half * 4;
                uint8_t *fr1 = fr0 + 16;
                *reinterpret_cast<uint32_t *>(fr0) = wq[0];
                *reinterpret_cast<uint32_t *>(fr0 + 8) = wl[0];
                *reinterpret_cast<uint32_t *>(fr1) = wq[1];
                *reinterpret_cast<uint32_t *>(fr1 + 8) = wl[1];
            }
            if ((lane & 1) == 0) {
                S[sig * mp + token] = sum16;
                if (tq == 8) {   // S/dx (|S/dx| <= 16 * 127) as f16, B fragment of the sub-block-sum MMA
                    const float sd = amax > 0.f ? sum16 * inv : 0.f;
                    __half *hb = reinterpret_cast<__half *>(base + 4096 * ntl + (nt * 32 + 4 * tk + ((sig & 7) >> 1)) * 8 +
                                                            (sig >> 3) * 4) + (sig & 1);
                    *hb = __float2half_rn(sd);
                }
            }
            if (lane == 0) S[16 * mp + token] = dx;
        }
    }
}
template <int TYPE>
__device__ __forceinline__ void stage_x(const float *x, int M, int64_t K, int64_t c, int n, uint8_t *dst, int xb,
                                        int tid, int nthreads) {
    if (Tr<TYPE>::I8) stage_i8<TYPE>(x, M, K, c, n, dst, xb, tid, nthreads);
    else stage_f16<TYPE>(x, M, K, c, n, dst, xb, tid, nthreads);
}

// Prep kernel (3..16 tokens): all chunks into global scratch. When launched
// with programmatic dependent launch it lets the GEMV that follows start at
// once, and waits for the kernel before it (which may have produced x, or
// still read the scratch) before touching memory.
template <int TYPE>
__global__ void ef_gemv_xprep(const float *__restrict__ x, int M, int64_t K, int64_t nchunks, int xb,
                           uint8_t *__restrict__ xf) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    stage_x<TYPE>(x, M, K, 0, (int)nchunks, xf, xb, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

// ------------------------------------------------------- result columns ----
// After a segment, the accumulators of the 4 lanes t of a group are reduced
// over the lanes that hold the same token (i8_tq column layouts); then
// for_owned visits each (row, token) value exactly once, on its owner lane:
// f(nt, i, row within the rowgroup, token).
template <int TQ, int NT>
__device__ __forceinline__ void reduce_cols(float (&acc)[NT][4]) {
    if constexpr (TQ == 1) {
        acc[0][0] += acc[0][1];
        acc[0][2] += acc[0][3];
        acc[0][0] += __shfl_xor_sync(0xffffffffu, acc[0][0], 1);
        acc[0][2] += __shfl_xor_sync(0xffffffffu, acc[0][2], 1);
        acc[0][0] += __shfl_xor_sync(0xffffffffu, acc[0][0], 2);
        acc[0][2] += __shfl_xor_sync(0xffffffffu, acc[0][2], 2);
    } else if constexpr (TQ == 2) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            acc[0][i] += __shfl_xor_sync(0xffffffffu, acc[0][i], 1);
            acc[0][i] += __shfl_xor_sync(0xffffffffu, acc[0][i], 2);
        }
    } else if constexpr (TQ == 4) {
#pragma unroll
        for (int i = 0; i < 4; i++) acc[0][i] += __shfl_xor_sync(0xffffffffu, acc[0][i], 2);
    }
}
template <int TQ, int NT, typename F>
__device__ __forceinline__ void for_owned(int lane, F &&f) {
    const int g = lane >> 2, t = lane & 3;
    if constexpr (TQ == 1) {
        if (t == 0) {
            f(0, 0, g, 0);
            f(0, 2, g + 8, 0);
        }
    } else if constexpr (TQ == 2) {
        if (t == 0)
#pragma unroll
            for (int i = 0; i < 4; i++) f(0, i, g + 8 * (i >> 1), i & 1);
    } else if constexpr (TQ == 4) {
        if (t < 2)
#pragma unroll
            for (int i = 0; i < 4; i++) f(0, i, g + 8 * (i >> 1), 2 * t + (i & 1));
    } else {
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) f(nt, i, g + 8 * (i >> 1), nt * 8 + 2 * t + (i & 1));
    }
}
template <bool SWIGLU> __device__ __forceinline__ float out_value(float gate, float up) {
    if (SWIGLU) return gate / (1.0f + expf(-gate)) * up;   // silu(g) * u
    return gate;
}

// ---------------------------------------------------------------- kernel ---
// CTA = one rowblock (8 rowgroups) x one k-slice [c0, c1) of its chunks; the
// ks k-slices of a rowblock form one thread-block cluster and add their sums
// through distributed shared memory, in rank order (deterministic, no
// atomics). KH = warps per rowgroup: with KH = 2 a CTA has 16 warps and the
// two warps of a rowgroup take alternate chunks, merging their sums through
// shared memory at the end.
template <int NT, int KH> struct CombineBytes {
    static constexpr int v = KH == 2 ? GV_WARPS * 32 * NT * 4 * 4 : 0;
};
// cluster reduction: [rowgroup slot][k-slice][matrix][token][16 rows] f32
template <bool SW> constexpr int reduce_bytes(int ks) { return GV_WARPS * ks * (SW ? 2 : 1) * 16 * 16 * 4; }
// Shared memory: [activation data: the slice's chunks, or one or two phase
// buffers][codebooks][pair-combine buffer][cluster-reduction buffer].
template <int TYPE, int NT, bool SWIGLU, int KH>
static size_t gemv_smem(int xs_bytes, int ks) {
    return (size_t)xs_bytes + TableBytes<TYPE>::v + CombineBytes<NT, KH>::v + (ks > 1 ? reduce_bytes<SWIGLU>(ks) : 0);
}

// TQ: Q4_K column layout (8 for the f16 types); NT: 8-token tiles; FUSED: the
// CTA stages its own activation data from f32 x (1-2 tokens); KH: warps per
// rowgroup (1 or 2).
// Launch-phase trace (only in builds with -DEF_GEMV_TRACE, a separate library
// for measurement): thread 0 of each CTA records the global timer and its
// SM's cycle counter at kernel entry, after the wait for the previous kernel,
// once the activation data is staged, after the weight stream and at exit,
// into the buffer set by ef_gemv_trace_set (12 words per CTA: block, SM, 5
// times in ns, 5 cycle counts).
#ifdef EF_GEMV_TRACE
__device__ unsigned long long *g_trace = nullptr;
__device__ unsigned int g_trace_n = 0, g_trace_cap = 0;
#define EF_TRACE_MARK(i)                                               \
    do {                                                               \
        if (threadIdx.x == 0) {                                        \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(tg[i]));  \
            tc[i] = clock64();                                         \
        }                                                              \
    } while (0)
#else
#define EF_TRACE_MARK(i) \
    do {                 \
    } while (0)
#endif

template <int TYPE, int TQ, int NT, bool SWIGLU, bool FUSED, int KH>
__global__ void __launch_bounds__(GV_WARPS * KH * 32, 1) ef_gemv_kernel(const GemvArgs a) {
#ifdef EF_GEMV_TRACE
    unsigned long long tg[5] = {}, tc[5] = {};
#endif
    EF_TRACE_MARK(0);
    using TR = Tr<TYPE>;
    using Raw = typename RawOf<TYPE>::T;
    constexpr int W = GV_WARPS;
    constexpr int NMAT = SWIGLU ? 2 : 1;
    constexpr int TILE = TR::TILE;
    static_assert(KH == 1 || !SWIGLU, "SwiGLU runs one warp per rowgroup");
    extern __shared__ __align__(128) uint8_t smem[];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wr = warp % W, kh = warp / W;   // rowgroup slot, k-half
    const int FB = a.xb;
    uint8_t *xs = smem;
    uint4 *grid = reinterpret_cast<uint4 *>(xs + a.xs_bytes);
    uint4 *sgn = grid + 256;
    float *comb = reinterpret_cast<float *>(xs + a.xs_bytes + TableBytes<TYPE>::v);
    float *red = reinterpret_cast<float *>(xs + a.xs_bytes + TableBytes<TYPE>::v + CombineBytes<NT, KH>::v);

    // codebooks -> shared memory (f16 entries; IQ2_XXS also the sign masks:
    // 7 stored sign bits + even parity -> XOR masks on f16 pairs). Visible to
    // all warps after the first activation barrier.
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

    const int nc = (int)a.nchunks, ks = a.kslices;
    const int rb = blockIdx.x / ks, ksi = blockIdx.x - rb * ks;
    const int c0 = (int)((int64_t)ksi * nc / ks), c1 = (int)((int64_t)(ksi + 1) * nc / ks);
    int m = 0;
    while (m + 1 < a.nmat && rb >= a.rb_end[m]) m++;
    int64_t rg = (int64_t)(rb - (m ? a.rb_end[m - 1] : 0)) * W + wr;
    const bool active = rg < a.rowgroups[m];

    // every rank of the cluster has started once this barrier phase completes
    // (waited for before the first distributed shared memory store)
    if (ks > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

    // ---- weight stream: this warp's chunks c0+kh, c0+kh+KH, ... < c1, each
    // tile loaded into registers one tile ahead of the math
    const int64_t tile0 = active ? (rg * nc + c0 + kh) * (int64_t)TILE : 0;
    const uint8_t *ip = a.w[m] + tile0;
    const uint8_t *ipu = SWIGLU ? a.w_up + tile0 : nullptr;
    int ic = c0 + kh;
    auto fetch = [&](Raw &r, Raw &ru) {
        if (ic < c1 && active) {
            load_raw(r, ip, lane);
            if (SWIGLU) load_raw(ru, ipu, lane);
            ip += KH * TILE;
            if (SWIGLU) ipu += KH * TILE;
        }
        ic += KH;
    };
    Raw q0, q0u;
    fetch(q0, q0u);

    // ---- activation data ---------------------------------------------------
    // whole: the slice's chunks staged once (1-2 tokens, when they fit); else
    // phases of at most phase_chunks chunks, copied from the prep kernel's
    // buffer one phase ahead into two alternating buffers (or, FUSED, staged
    // in place). x is produced by the kernel before this one: with
    // programmatic dependent launch, wait for it only now.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    EF_TRACE_MARK(1);
    auto copy_phase = [&](int c, uint8_t *dst) {   // prep buffer -> shared, async
        const int len = min(a.phase_chunks, c1 - c);
        const uint8_t *src = a.xf + (int64_t)c * FB;
        for (int i = threadIdx.x; i < len * FB / 16; i += blockDim.x) cp_async16(dst + 16 * i, src + 16 * i);
    };
    int ph_i = 0;
    if (a.whole) {
        stage_x<TYPE>(a.x, a.M, a.K, c0, c1 - c0, xs, FB, threadIdx.x, blockDim.x);
        __syncthreads();
    } else if (!FUSED) {
        copy_phase(c0, xs);
        cp_commit();
    }

    float acc[NT][4], acc2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = acc2[nt][i] = 0.f;

    EF_TRACE_MARK(2);                // (phases: staging continues inside the stream)
#pragma unroll 1
    for (int p0 = c0; p0 < c1;) {    // activation phases
        int p1;
        const uint8_t *xbase;        // activation data of chunk p0
        if (a.whole) {
            p1 = c1;
            xbase = xs;
        } else {
            p1 = min(c1, p0 + a.phase_chunks);
            __syncthreads();         // every warp is done with the previous phase
            if (FUSED) {
                stage_x<TYPE>(a.x, a.M, a.K, p0, p1 - p0, xs, FB, threadIdx.x, blockDim.x);
                xbase = xs;
            } else {
                if (p1 < c1) copy_phase(p1, xs + ((ph_i + 1) & 1) * a.xs_half);
                cp_commit();
                cp_wait<1>();        // this thread's copies of this phase have landed
                xbase = xs + (ph_i & 1) * a.xs_half;
                ph_i++;
            }
            __syncthreads();
        }
        // this warp's chunks of the phase: c = c0 + kh (mod KH)
        int c = p0;
        if (KH > 1) c += ((c0 + kh - p0) % KH + KH) % KH;
#pragma unroll 1
        for (; c < p1; c += KH) {
            Raw r = q0, ru = q0u;
            fetch(q0, q0u);          // the next tile's loads go out before this tile's math
            if (active) {
                const uint8_t *xc = xbase + (c - (a.whole ? c0 : p0)) * FB;
                if constexpr (TYPE == EF_Q4_K) compute_q4k<TQ, NT>(r, xc, acc, lane);
                else if constexpr (TYPE == EF_Q6_K) compute_q6k<TQ, NT>(r, xc, acc, lane);
                else compute<NT>(r, xc, a.M, acc, lane, grid, sgn);
                if (SWIGLU) {
                    if constexpr (TYPE == EF_Q4_K) compute_q4k<TQ, NT>(ru, xc, acc2, lane);
                    else if constexpr (TYPE == EF_Q6_K) compute_q6k<TQ, NT>(ru, xc, acc2, lane);
                    else compute<NT>(ru, xc, a.M, acc2, lane, grid, sgn);
                }
            }
        }
        p0 = p1;
    }
    if (!FUSED) cp_wait<0>();
    EF_TRACE_MARK(3);
    // The weight stream is done: with programmatic dependent launch the next
    // kernel may start now.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // ---- the two warps of a rowgroup ----
    if constexpr (KH == 2) {
        float4 *cb = reinterpret_cast<float4 *>(comb) + (wr * 32 + lane) * NT;
        if (kh == 1) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++) cb[nt] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
        }
        asm volatile("bar.sync %0, 64;" ::"r"(1 + wr) : "memory");
        if (kh == 0) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const float4 o = cb[nt];
                acc[nt][0] += o.x;
                acc[nt][1] += o.y;
                acc[nt][2] += o.z;
                acc[nt][3] += o.w;
            }
        }
    }
    const int M = a.M;
    const int64_t rows = a.rows[m];
    float *y = a.y[m];
    // output element [tok][r]: y, or every rank's exchange slot (tensor
    // parallel), stamped with this call's number
    const int npush = a.push.n;
    const uint32_t call = npush ? *(volatile const uint32_t *)a.push.epoch + 1 : 0;
    const int64_t slot_off = ((int64_t)(call & 1) * npush + a.push.rank) * a.push.slot_bytes;
    auto put = [&](int tok, int64_t r, float v) {
        const int64_t idx = (int64_t)tok * rows + r;
        if (!npush) {
            y[idx] = v;
        } else {
            const uint64_t word = ((uint64_t)call << 32) | __float_as_uint(v);
            for (int p = 0; p < npush; p++)
                asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(
                                 reinterpret_cast<uint64_t *>(a.push.data[p] + slot_off) + idx),
                             "l"(word)
                             : "memory");
        }
    };
    if (kh == 0 && active) {
        reduce_cols<TQ, NT>(acc);
        if (SWIGLU) reduce_cols<TQ, NT>(acc2);
    }
    if (ks == 1) {
        if (kh == 0 && active)
            for_owned<TQ, NT>(lane, [&](int nt, int i, int row, int tok) {
                const int64_t r = rg * 16 + row;
                if (tok < M && r < rows) put(tok, r, out_value<SWIGLU>(acc[nt][i], acc2[nt][i]));
            });
    } else {
        // ---- k-slices of this rowblock (one cluster), added in rank order:
        // rowgroup wr is finished by rank wr % ks; every slice stores its
        // partial sums into slot [wr][its rank] of that rank's shared memory
        // (distributed shared memory stores), one cluster barrier (release /
        // acquire) makes them visible, and the owner reads only its own
        // shared memory after it -- so no rank touches another's shared
        // memory once the barrier is passed, and each may exit when done.
        // (The barrier at the start of the kernel guarantees every rank has
        // started before its shared memory is written.)
        cg::cluster_group cluster = cg::this_cluster();
        const int owner = wr % ks;
        float *slot = red + ((size_t)wr * ks + ksi) * NMAT * 256;
        float *dst = owner == ksi ? slot : cluster.map_shared_rank(slot, owner);
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
        if (kh == 0 && active)
            for_owned<TQ, NT>(lane, [&](int nt, int i, int row, int tok) {
                if (tok < M) {
                    dst[tok * 16 + row] = acc[nt][i];
                    if (SWIGLU) dst[256 + tok * 16 + row] = acc2[nt][i];
                }
            });
        cluster.sync();
        if (kh == 0 && active && owner == ksi) {
            for (int i = lane; i < 16 * M; i += 32) {
                float s1 = 0.f, s2 = 0.f;
                for (int rk = 0; rk < ks; rk++) {
                    const float *src = red + ((size_t)wr * ks + rk) * NMAT * 256;
                    s1 += src[i];
                    if (SWIGLU) s2 += src[256 + i];
                }
                const int64_t r = rg * 16 + (i & 15);
                if (r < rows) put(i >> 4, r, out_value<SWIGLU>(s1, s2));
            }
        }
    }
#ifdef EF_GEMV_TRACE
    __syncthreads();
    EF_TRACE_MARK(4);
    if (threadIdx.x == 0) {
        const unsigned slot = atomicAdd(&g_trace_n, 1u);
        if (g_trace && slot < g_trace_cap) {
            unsigned long long *o = g_trace + (size_t)slot * 12;
            unsigned sm;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
            o[0] = blockIdx.x;
            o[1] = sm;
            for (int i = 0; i < 5; i++) {
                o[2 + i] = tg[i];
                o[7 + i] = tc[i];
            }
        }
    }
#endif
}

// ------------------------------------------------------------------ host ---
// Work split: CTA = 8 rowgroups (one rowblock) x one k-slice, the k-slices of
// a rowblock in one thread-block cluster. Activation data: with 1-2 tokens
// the slice's chunks at once when they fit, else phases (two buffers when a
// prep kernel supplies the data).
GemvPlan gemv_plan(int64_t rowblocks, int64_t nchunks, int xb, bool fused, int ks) {
    GemvPlan p = {};
    p.kslices = ks;
    p.ctas = rowblocks * ks;
    const int64_t slice = (nchunks + ks - 1) / ks;
    if (fused && slice * xb <= MAX_XS_BYTES) {
        p.whole = 1;
        p.phase_chunks = (int)slice;
        p.xs_bytes = (int)(slice * xb);
        p.xs_half = 0;
    } else {
        const int budget = fused ? MAX_XS_BYTES : MAX_XS_BYTES / 2;
        p.whole = 0;
        p.phase_chunks = (int)std::max<int64_t>(1, std::min<int64_t>(slice, budget / xb));
        p.xs_half = p.phase_chunks * xb;
        p.xs_bytes = fused ? p.xs_half : 2 * p.xs_half;
    }
    return p;
}

// How many clusters of `ks` CTAs of this kernel the device holds at once
// (cudaOccupancyMaxActiveClusters; cached per kernel, device, size and shared
// memory). On B200 this is not SMs / ks: clusters are placed inside one GPC,
// and with one 512-thread CTA per SM it measured 148, 74, 45, 33, 26, 22, 15,
// 15 for ks = 1..8.
static int max_active_clusters(ef_ctx *ctx, const void *kern, int threads, size_t smem, int ks) {
    static std::mutex mu;
    static std::map<std::tuple<const void *, int, int, size_t>, int> cache;
    const auto key = std::make_tuple(kern, ctx->device, ks, smem);
    {
        std::lock_guard<std::mutex> g(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ks, 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    std::lock_guard<std::mutex> g(mu);
    cache[key] = n;
    return n;
}

// Warps per rowgroup: two (16-warp CTAs) where the kernel fits 128 registers
// per thread, else one.
template <int TYPE, int TQ, int NT, bool SWIGLU> constexpr int kh_of() {
    return !SWIGLU && (NT == 1 || TYPE == EF_Q8_0 || TYPE == EF_Q4_0) ? 2 : 1;
}

template <int TYPE, int TQ, int NT, bool SWIGLU, bool FUSED>
static int launch_kernel(ef_ctx *ctx, GemvArgs &a, int64_t rowblocks, bool fused) {
    constexpr int KH = kh_of<TYPE, TQ, NT, SWIGLU>();
    constexpr int threads = GV_WARPS * KH * 32;
    auto kern = ef_gemv_kernel<TYPE, TQ, NT, SWIGLU, FUSED, KH>;
    static std::atomic<unsigned long long> configured{0};   // per instantiation, one bit per device
    if (ctx->device < 64 && !(configured.load() & (1ull << ctx->device))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return check_cuda(ctx, e, "gemv smem attribute");
        configured.fetch_or(1ull << ctx->device);
    }
    // The widest k-split (at most 8 slices, a portable cluster) whose clusters
    // all fit on the device at once. Measured on B200 over 1024-12288 rows x
    // 2048-8192 columns: the time falls as the split widens until the grid no
    // longer fits in one wave, then rises by 40-70 %.
    GemvPlan p = {};
    size_t smem = 0;
    for (int ks = (int)std::min<int64_t>(8, a.nchunks); ks >= 1; ks--) {
        p = gemv_plan(rowblocks, a.nchunks, a.xb, fused, ks);
        smem = gemv_smem<TYPE, NT, SWIGLU, KH>(p.xs_bytes, ks);
        if (ks == 1 || (smem <= 227 * 1024 && rowblocks <= max_active_clusters(ctx, (const void *)kern, threads, smem, ks)))
            break;
    }
    a.kslices = p.kslices;
    a.phase_chunks = p.phase_chunks;
    a.whole = p.whole;
    a.xs_bytes = p.xs_bytes;
    a.xs_half = p.xs_half;
    const int64_t ctas = p.ctas;
    a.ctas = ctas;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    if (cfg.dynamicSmemBytes > 227 * 1024)
        return set_err(ctx, EF_ERR_RANGE, "gemv: %zu bytes of shared memory needed", cfg.dynamicSmemBytes);
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (ctx->pdl) {
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
    ctx->launches++;
    return check_cuda(ctx, cudaLaunchKernelEx(&cfg, kern, a), "gemv launch");
}

// Up to this many tokens each CTA stages its own activation data (one kernel
// per call); above it a prep kernel writes the data once into context scratch.
constexpr int FUSED_MAX_TOKENS = 2;

template <int TYPE> static int x_bytes_per_chunk(int M) {
    return Tr<TYPE>::I8 ? i8_xbytes<TYPE>(M) : f16_xbytes<TYPE>(M);
}

template <int TYPE, int TQ, int NT, bool SWIGLU>
static int launch_t(ef_ctx *ctx, GemvArgs &a, const ef_weight *const *ws, int n, const float *x) {
    a.xb = x_bytes_per_chunk<TYPE>(a.M);
    a.x = x;
    a.K = ws[0]->k;
    const bool fused = a.M <= FUSED_MAX_TOKENS;
    if (!fused) {
        // activation data for all chunks -> context scratch slot 0
        const size_t xbytes = (size_t)a.nchunks * a.xb;
        if (int rc = ensure_scratch(ctx, 0, xbytes)) return rc;
        a.xf = (const uint8_t *)ctx->scratch[0];
        const int64_t work = Tr<TYPE>::I8 ? a.nchunks * i8_tq(a.M) * i8_nt(a.M) * 32
                                          : a.nchunks * a.M * (Tr<TYPE>::CHUNK / 4);
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
        cfg.numAttrs = ctx->pdl ? 1 : 0;
        ctx->launches++;
        if (int rc = check_cuda(ctx, cudaLaunchKernelEx(&cfg, ef_gemv_xprep<TYPE>, x, a.M, a.K, a.nchunks, a.xb,
                                                        (uint8_t *)ctx->scratch[0]), "gemv xprep launch"))
            return rc;
    } else {
        a.xf = nullptr;
    }
    int rowblocks = 0;
    for (int i = 0; i < n; i++) {
        rowblocks += (int)((ws[i]->rowgroups + GV_WARPS - 1) / GV_WARPS);
        a.rb_end[i] = rowblocks;
    }
    // (1-2 tokens run TQ <= 2 for the 8-bit types and one 8-token tile for the others)
    if constexpr (NT == 1 && (!Tr<TYPE>::I8 || TQ <= 2))
        if (fused) return launch_kernel<TYPE, TQ, NT, SWIGLU, true>(ctx, a, rowblocks, fused);
    return launch_kernel<TYPE, TQ, NT, SWIGLU, false>(ctx, a, rowblocks, fused);
}

template <int TYPE, bool SWIGLU>
static int launch_type(ef_ctx *ctx, GemvArgs &a, const ef_weight *const *ws, int n, const float *x) {
    const int M = a.M;
    if constexpr (Tr<TYPE>::I8) {
        if (M <= 1) return launch_t<TYPE, 1, 1, SWIGLU>(ctx, a, ws, n, x);
        if (M <= 2) return launch_t<TYPE, 2, 1, SWIGLU>(ctx, a, ws, n, x);
        if (M <= 4) return launch_t<TYPE, 4, 1, SWIGLU>(ctx, a, ws, n, x);
    }
    if (M <= 8) return launch_t<TYPE, 8, 1, SWIGLU>(ctx, a, ws, n, x);
    return launch_t<TYPE, 8, 2, SWIGLU>(ctx, a, ws, n, x);
}

template <int TYPE>
static int launch_sw(ef_ctx *ctx, GemvArgs &a, bool sw, const ef_weight *const *ws, int n, const float *x) {
    return sw ? launch_type<TYPE, true>(ctx, a, ws, n, x) : launch_type<TYPE, false>(ctx, a, ws, n, x);
}

int launch_gemv(ef_ctx *ctx, const ef_weight *const *ws, int n, const ef_weight *w_up, const float *x, int M,
                float *const *ys, const GemvPush *push) {
    GemvArgs a = {};
    if (push) a.push = *push;
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
    int rc;
    switch (w0->type) {
    case EF_Q8_0: rc = launch_sw<EF_Q8_0>(ctx, a, sw, ws, n, x); break;
    case EF_Q4_0: rc = launch_sw<EF_Q4_0>(ctx, a, sw, ws, n, x); break;
    case EF_Q5_K: rc = launch_sw<EF_Q5_K>(ctx, a, sw, ws, n, x); break;
    case EF_Q2_K: rc = launch_sw<EF_Q2_K>(ctx, a, sw, ws, n, x); break;
    case EF_Q4_K: rc = launch_sw<EF_Q4_K>(ctx, a, sw, ws, n, x); break;
    case EF_Q6_K: rc = launch_sw<EF_Q6_K>(ctx, a, sw, ws, n, x); break;
    case EF_IQ2_XXS: rc = launch_sw<EF_IQ2_XXS>(ctx, a, sw, ws, n, x); break;
    case EF_IQ1_S: rc = launch_sw<EF_IQ1_S>(ctx, a, sw, ws, n, x); break;
    default: return set_err(ctx, EF_ERR_TYPE, "gemv: unsupported type %d", w0->type);
    }
    return rc;
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
    case EF_Q4_0: fb = (size_t)f16_xbytes<EF_Q4_0>(M); break;
    case EF_Q5_K: fb = (size_t)f16_xbytes<EF_Q5_K>(M); break;
    case EF_Q2_K: fb = (size_t)f16_xbytes<EF_Q2_K>(M); break;
    case EF_Q4_K: fb = (size_t)i8_xbytes<EF_Q4_K>(M); break;
    case EF_Q6_K: fb = (size_t)i8_xbytes<EF_Q6_K>(M); break;
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
    tmp.no_alloc = true;   // a size this file's check missed fails instead of allocating
    float *ys[1] = {y};
    const int rc = launch_gemv(&tmp, &w, 1, nullptr, x, M, ys);
    tmp.scratch[0] = nullptr;   // not the context's to free
    return rc;
}

#ifdef EF_GEMV_TRACE
// Sets the launch-phase trace buffer (cap records of 12 u64; null: off) and
// restarts its record count. Trace builds only; synchronizes the device.
extern "C" __attribute__((visibility("default"))) int ef_gemv_trace_set(void *buf, unsigned cap) {
    unsigned long long *p = (unsigned long long *)buf;
    const unsigned zero = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return EF_ERR_CUDA;
    if (cudaMemcpyToSymbol(ef::g_trace, &p, sizeof(p)) != cudaSuccess) return EF_ERR_CUDA;
    if (cudaMemcpyToSymbol(ef::g_trace_cap, &cap, sizeof(cap)) != cudaSuccess) return EF_ERR_CUDA;
    if (cudaMemcpyToSymbol(ef::g_trace_n, &zero, sizeof(zero)) != cudaSuccess) return EF_ERR_CUDA;
    return EF_OK;
}
#endif

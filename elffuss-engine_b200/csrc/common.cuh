// common.cuh -- tile layout of repacked GGUF weights, block decoders and PTX
// helpers shared by the repack, dequant, GEMV and GEMM kernels (sm_100a).
//
// TILE LAYOUT ("rowgroup tiles"). A weight tensor of `rows` x `k` is cut into
// rowgroups of 16 rows (rows padded to 16 with zero blocks) and, along k, into
// chunks of CHUNK_K weights (128 for Q8_0, one 256-weight superblock for the
// K-/i-quants; k padded to a whole chunk with zero blocks). Each (rowgroup,
// chunk) is one contiguous, 16-byte aligned tile of exactly 16 x the GGUF bytes
// of that piece -- the repack permutes bytes (and, for Q6_K, nibbles and 2-bit
// fields) but never adds any. Tiles of a rowgroup
// follow each other along k; rowgroups follow each other.
//
// Inside a tile the quant bytes are ordered for the tensor-core fragments: lane
// L = 4g + t of a warp owns rows g and g+8 of the rowgroup and, per row, the k
// positions of its A fragment (block t for Q8_0 / m16n8k16; positions 4t..4t+3
// and 16+4t..16+4t+3 of every 32 for Q4_K and Q6_K / m16n8k32 8-bit;
// 32-blocks 2t,2t+1 for the i-quants), and its bytes sit in 16-byte "parts":
// part p of lane L at tile + 512p + 16L, so one 128-bit load per part by the
// 32 lanes reads 512 contiguous bytes. Scales follow the parts. Per-type
// details are next to each scatter/gather below.
//
// The GGUF blocks themselves are restated from the reference decoders:
//   Q8_0 js/kernels.wgsl.js:154-169, Q4_K :227-250 (+scale_min_k4 :94-104),
//   Q6_K :269-330, IQ2_XXS :368-396, IQ1_S :805-822.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/elffuss_cuda.h"

namespace ef {

// Programmatic dependent launch. pdl_trigger: kernels queued after this one
// may be scheduled now; pdl_wait: block until the kernels this one depends on
// have finished and their writes are visible (a no-op without the launch
// attribute). Every kernel of a PDL chain executes pdl_wait in every CTA
// before its first read of an earlier kernel's output and before it exits, so
// completion stays transitive along the chain.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// sum over the CTA (blockDim.x a multiple of 32, <= 1024); `red` >= 32 floats
__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = lane < nw ? red[lane] : 0.f;
    return warp_sum(s);
}

// 16-byte asynchronous global -> shared copy (L2 only), its group commit and wait.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }


// ---------------------------------------------------------------- geometry --
struct TypeGeo {
    int block_elems;   // weights per GGUF block
    int block_bytes;   // bytes per GGUF block
    int chunk_k;       // weights per tile along k
    int tile_bytes;    // bytes per (16-row, chunk) tile = 16 * chunk_k / block_elems * block_bytes
};

__host__ __device__ inline bool geo_of(int type, TypeGeo &g) {
    switch (type) {
    case EF_Q8_0: g = {32, 34, 128, 2176}; return true;
    case EF_Q4_0: g = {32, 18, 128, 1152}; return true;
    case EF_Q4_K: g = {256, 144, 256, 2304}; return true;
    case EF_Q5_K: g = {256, 176, 256, 2816}; return true;
    case EF_Q2_K: g = {256, 84, 256, 1344}; return true;
    case EF_Q6_K: g = {256, 210, 256, 3360}; return true;
    case EF_IQ2_XXS: g = {256, 66, 256, 1056}; return true;
    case EF_IQ1_S: g = {256, 50, 256, 800}; return true;
    default: return false;
    }
}

constexpr int RG_ROWS = 16;   // rows per rowgroup tile

// ------------------------------------------------------------ byte helpers --
__host__ __device__ inline uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__host__ __device__ inline void wr32(uint8_t *p, uint32_t v) {
    p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
}

// Q6_K weight p of a GGUF block (kernels.wgsl.js:269-330): p = 128n + 32i + l,
// low 4 bits from ql[64n + 32(i&1) + l] (low nibble for i < 2, high for
// i >= 2), high 2 bits from qh[32n + l] >> 2i.
__host__ __device__ inline int q6_lo4(const uint8_t *blk, int p) {
    const int n = p >> 7, i = (p >> 5) & 3, l = p & 31;
    return (blk[64 * n + 32 * (i & 1) + l] >> (4 * (i >> 1))) & 15;
}
__host__ __device__ inline int q6_hi2(const uint8_t *blk, int p) {
    const int n = p >> 7, i = (p >> 5) & 3, l = p & 31;
    return (blk[128 + 32 * n + l] >> (2 * i)) & 3;
}

// Q4_0: bit position, inside a 32-bit tile word, of the word's weight m (0..7).
__host__ __device__ inline int q40_slot(int m) { return 16 * (m & 1) + 4 * (m >> 1); }

// --------------------------------------------- scatter (GGUF -> tile) -------
// Write GGUF block `blk` (row r of the rowgroup, block `bic` within the chunk)
// into tile `T`. Every output byte is written by exactly one block.
__host__ __device__ inline void scatter_block(int type, const uint8_t *blk, int r, int bic, uint8_t *T) {
    const int g = r & 7, hs = r >> 3;
    switch (type) {
    case EF_Q8_0: {
        // lane (g, t=bic) owns block bic of rows g and g+8. Parts 2hs, 2hs+1 hold
        // its 32 quants stored with the sign bit flipped (q ^ 0x80 = q + 128 as
        // an unsigned byte); the f16 scale goes to 2048 + 4*lane + 2*hs.
        const int lane = 4 * g + bic;
        for (int i = 0; i < 32; i++)
            T[(2 * hs + (i >> 4)) * 512 + lane * 16 + (i & 15)] = blk[2 + i] ^ 0x80;
        T[2048 + lane * 4 + hs * 2] = blk[0];
        T[2048 + lane * 4 + hs * 2 + 1] = blk[1];
    } break;
    case EF_Q4_K: {
        // lane (g,t) owns, in each 32-byte qs group j, the bytes [4t, 4t+4)
        // and [16+4t, 16+4t+4): their low nibbles are weights of sub-block 2j,
        // their high nibbles of sub-block 2j+1, at the k positions of the
        // lane's 8-bit MMA fragment. Group j of row g/g+8 is 8 bytes at part
        // 2hs + (j>>1), offset 8*(j&1). The 16-byte header (d, dmin, 12 scale
        // bytes) is kept verbatim at 2048 + 16r.
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int j = 0; j < 4; j++) {
                uint8_t *d = T + (2 * hs + (j >> 1)) * 512 + lane * 16 + (j & 1) * 8;
                for (int b = 0; b < 4; b++) {
                    d[b] = blk[16 + 32 * j + 4 * t + b];
                    d[4 + b] = blk[16 + 32 * j + 16 + 4 * t + b];
                }
            }
        }
        for (int i = 0; i < 16; i++) T[2048 + r * 16 + i] = blk[i];
    } break;
    case EF_Q6_K: {
        // 8-bit MMA layout. Weight position p = 32s + 16h + 4t + b (step s =
        // 0..7, half h, lane column t, byte b) of row g + 8hs: lane (g,t) holds
        // for each step one word of low nibbles (byte b: position 32s+4t+b in
        // bits 0-3, 32s+16+4t+b in bits 4-7) at part 2hs + (s>>2), offset
        // 4(s&3); and for each pair of steps one word of 2-bit high fields
        // (byte b: step 2sp half 0 | half 1 | step 2sp+1 half 0 | half 1, two
        // bits each) at part 4 + hs, offset 4sp. int8 scales verbatim at
        // 3072 + 16r, d at 3328 + 4g + 2hs.
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int st = 0; st < 8; st++)
                for (int b = 0; b < 4; b++) {
                    const int p0 = 32 * st + 4 * t + b, p1 = p0 + 16;
                    T[(2 * hs + (st >> 2)) * 512 + lane * 16 + 4 * (st & 3) + b] =
                        (uint8_t)(q6_lo4(blk, p0) | (q6_lo4(blk, p1) << 4));
                }
            for (int sp = 0; sp < 4; sp++)
                for (int b = 0; b < 4; b++) {
                    const int p0 = 64 * sp + 4 * t + b;
                    T[(4 + hs) * 512 + lane * 16 + 4 * sp + b] =
                        (uint8_t)(q6_hi2(blk, p0) | (q6_hi2(blk, p0 + 16) << 2) | (q6_hi2(blk, p0 + 32) << 4) |
                                  (q6_hi2(blk, p0 + 48) << 6));
                }
        }
        for (int i = 0; i < 16; i++) T[3072 + r * 16 + i] = blk[192 + i];
        T[3328 + 4 * g + 2 * hs] = blk[208];
        T[3328 + 4 * g + 2 * hs + 1] = blk[209];
    } break;
    case EF_IQ2_XXS: {
        // lane (g,t) owns 32-blocks 2t, 2t+1: GGUF bytes [2+16t, 2+16t+16) at
        // part hs. d at 1024 + 4g + 2hs.
        for (int t = 0; t < 4; t++)
            for (int i = 0; i < 16; i++) T[hs * 512 + (4 * g + t) * 16 + i] = blk[2 + 16 * t + i];
        T[1024 + 4 * g + 2 * hs] = blk[0];
        T[1024 + 4 * g + 2 * hs + 1] = blk[1];
    } break;
    case EF_IQ1_S: {
        // lane (g,t) owns 32-blocks 2t, 2t+1: qs bytes [8t, 8t+8) at
        // 16*lane + 8hs, qh halves [2t, 2t+2) at 512 + 8*lane + 4hs, d at
        // 768 + 4g + 2hs.
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int i = 0; i < 8; i++) T[lane * 16 + hs * 8 + i] = blk[2 + 8 * t + i];
            for (int i = 0; i < 4; i++) T[512 + lane * 8 + hs * 4 + i] = blk[34 + 4 * t + i];
        }
        T[768 + 4 * g + 2 * hs] = blk[0];
        T[768 + 4 * g + 2 * hs + 1] = blk[1];
    } break;
    case EF_Q4_0: {
        // lane (g, t=bic) owns block bic of rows g and g+8: part hs holds its 32
        // nibbles, word j the weights 8j..8j+7 at nibble slots (bits) 0, 16,
        // 4, 20, 8, 24, 12, 28 -- so (w >> 8u) & 0x000F000F gives weights
        // 8j+4u, 8j+4u+1 and (w >> 8u+4) & 0x000F000F the next two, each in the
        // low bits of a 16-bit half; the f16 d goes to 1024 + 4*lane + 2*hs.
        const int lane = 4 * g + bic;
        for (int j = 0; j < 4; j++) {
            uint32_t wd = 0;
            for (int m = 0; m < 8; m++) {
                const int i = 8 * j + m;
                const uint32_t q = i < 16 ? (blk[2 + i] & 15) : (blk[2 + i - 16] >> 4);
                wd |= q << q40_slot(m);
            }
            for (int b = 0; b < 4; b++) T[hs * 512 + lane * 16 + 4 * j + b] = (uint8_t)(wd >> (8 * b));
        }
        T[1024 + lane * 4 + hs * 2] = blk[0];
        T[1024 + lane * 4 + hs * 2 + 1] = blk[1];
    } break;
    case EF_Q5_K: {
        // lane (g,t) owns the 64-weight group t (sub-blocks 2t: low nibbles,
        // 2t+1: high nibbles) of rows g and g+8. Parts 2hs, 2hs+1: its 32 qs
        // bytes; part 4 at 8*hs: two words of fifth bits, bit l = qh[l] bit 2t
        // (low) / 2t+1 (high); the row's d, dmin, scales verbatim at 2560 + 16 r.
        // bic = 0: a whole superblock per chunk.
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int b = 0; b < 32; b++) T[(2 * hs + (b >> 4)) * 512 + lane * 16 + (b & 15)] = blk[48 + 32 * t + b];
            uint32_t lo = 0, hi = 0;
            for (int l = 0; l < 32; l++) {
                lo |= (uint32_t)((blk[16 + l] >> (2 * t)) & 1) << l;
                hi |= (uint32_t)((blk[16 + l] >> (2 * t + 1)) & 1) << l;
            }
            for (int b = 0; b < 4; b++) {
                T[4 * 512 + lane * 16 + 8 * hs + b] = (uint8_t)(lo >> (8 * b));
                T[4 * 512 + lane * 16 + 8 * hs + 4 + b] = (uint8_t)(hi >> (8 * b));
            }
        }
        for (int b = 0; b < 16; b++) T[2560 + 16 * r + b] = blk[b];
    } break;
    case EF_Q2_K: {
        // lane (g,t) owns weights 64t..64t+63 (sub-blocks 4t..4t+3 of 16) of
        // rows g and g+8. Part hs word w, byte c: bits 2s'..2s'+1 = the 2-bit q
        // of weight 64t + 4(4w + s') + c (kernels.wgsl.js:192-217: byte
        // qs[32n + r] >> 2j for weight 128n + 32j + r); the four scale bytes
        // of its sub-blocks at 1024 + 8*lane + 4*hs; d, dmin at 1280 + 4 r.
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int w = 0; w < 4; w++)
                for (int c = 0; c < 4; c++) {
                    uint32_t byte = 0;
                    for (int sp = 0; sp < 4; sp++) {
                        const int i = 64 * t + 4 * (4 * w + sp) + c;
                        const int n = i >> 7, jj = (i >> 5) & 3, rr = i & 31;
                        byte |= (uint32_t)((blk[16 + 32 * n + rr] >> (2 * jj)) & 3) << (2 * sp);
                    }
                    T[hs * 512 + lane * 16 + 4 * w + c] = (uint8_t)byte;
                }
            for (int k = 0; k < 4; k++) T[1024 + 8 * lane + 4 * hs + k] = blk[4 * t + k];
        }
        for (int b = 0; b < 4; b++) T[1280 + 4 * r + b] = blk[80 + b];
    } break;
    default:
        break;
    }
}

// --------------------------------------------- gather (tile -> GGUF) --------
// Exact inverse of scatter_block.
__host__ __device__ inline void gather_block(int type, const uint8_t *T, int r, int bic, uint8_t *blk) {
    const int g = r & 7, hs = r >> 3;
    switch (type) {
    case EF_Q8_0: {
        const int lane = 4 * g + bic;
        for (int i = 0; i < 32; i++)
            blk[2 + i] = T[(2 * hs + (i >> 4)) * 512 + lane * 16 + (i & 15)] ^ 0x80;
        blk[0] = T[2048 + lane * 4 + hs * 2];
        blk[1] = T[2048 + lane * 4 + hs * 2 + 1];
    } break;
    case EF_Q4_K: {
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int j = 0; j < 4; j++) {
                const uint8_t *d = T + (2 * hs + (j >> 1)) * 512 + lane * 16 + (j & 1) * 8;
                for (int b = 0; b < 4; b++) {
                    blk[16 + 32 * j + 4 * t + b] = d[b];
                    blk[16 + 32 * j + 16 + 4 * t + b] = d[4 + b];
                }
            }
        }
        for (int i = 0; i < 16; i++) blk[i] = T[2048 + r * 16 + i];
    } break;
    case EF_Q6_K: {
        for (int i = 0; i < 192; i++) blk[i] = 0;
        for (int p = 0; p < 256; p++) {
            const int st = p >> 5, h = (p >> 4) & 1, lane = 4 * g + ((p >> 2) & 3), b = p & 3;
            const uint8_t nb = T[(2 * hs + (st >> 2)) * 512 + lane * 16 + 4 * (st & 3) + b];
            const uint8_t hb = T[(4 + hs) * 512 + lane * 16 + 4 * (st >> 1) + b];
            const int lo = h ? nb >> 4 : nb & 15, hi = (hb >> (2 * (2 * (st & 1) + h))) & 3;
            const int n = p >> 7, qi = (p >> 5) & 3, l = p & 31;
            blk[64 * n + 32 * (qi & 1) + l] |= (uint8_t)(lo << (4 * (qi >> 1)));
            blk[128 + 32 * n + l] |= (uint8_t)(hi << (2 * qi));
        }
        for (int i = 0; i < 16; i++) blk[192 + i] = T[3072 + r * 16 + i];
        blk[208] = T[3328 + 4 * g + 2 * hs];
        blk[209] = T[3328 + 4 * g + 2 * hs + 1];
    } break;
    case EF_IQ2_XXS: {
        for (int t = 0; t < 4; t++)
            for (int i = 0; i < 16; i++) blk[2 + 16 * t + i] = T[hs * 512 + (4 * g + t) * 16 + i];
        blk[0] = T[1024 + 4 * g + 2 * hs];
        blk[1] = T[1024 + 4 * g + 2 * hs + 1];
    } break;
    case EF_IQ1_S: {
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int i = 0; i < 8; i++) blk[2 + 8 * t + i] = T[lane * 16 + hs * 8 + i];
            for (int i = 0; i < 4; i++) blk[34 + 4 * t + i] = T[512 + lane * 8 + hs * 4 + i];
        }
        blk[0] = T[768 + 4 * g + 2 * hs];
        blk[1] = T[768 + 4 * g + 2 * hs + 1];
    } break;
    case EF_Q4_0: {
        const int lane = 4 * g + bic;
        uint32_t wds[4];
        for (int j = 0; j < 4; j++) wds[j] = rd32(T + hs * 512 + lane * 16 + 4 * j);
        for (int i = 0; i < 16; i++) {
            const uint32_t lo = (wds[i >> 3] >> q40_slot(i & 7)) & 15;
            const uint32_t hi = (wds[(i + 16) >> 3] >> q40_slot((i + 16) & 7)) & 15;
            blk[2 + i] = (uint8_t)(lo | (hi << 4));
        }
        blk[0] = T[1024 + lane * 4 + hs * 2];
        blk[1] = T[1024 + lane * 4 + hs * 2 + 1];
    } break;
    case EF_Q5_K: {
        for (int b = 0; b < 16; b++) blk[b] = T[2560 + 16 * r + b];
        for (int l = 0; l < 32; l++) blk[16 + l] = 0;
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int b = 0; b < 32; b++) blk[48 + 32 * t + b] = T[(2 * hs + (b >> 4)) * 512 + lane * 16 + (b & 15)];
            const uint32_t lo = rd32(T + 4 * 512 + lane * 16 + 8 * hs), hi = rd32(T + 4 * 512 + lane * 16 + 8 * hs + 4);
            for (int l = 0; l < 32; l++)
                blk[16 + l] |= (uint8_t)((((lo >> l) & 1) << (2 * t)) | (((hi >> l) & 1) << (2 * t + 1)));
        }
    } break;
    case EF_Q2_K: {
        for (int b = 0; b < 64; b++) blk[16 + b] = 0;
        for (int t = 0; t < 4; t++) {
            const int lane = 4 * g + t;
            for (int w = 0; w < 4; w++)
                for (int c = 0; c < 4; c++) {
                    const uint32_t byte = T[hs * 512 + lane * 16 + 4 * w + c];
                    for (int sp = 0; sp < 4; sp++) {
                        const int i = 64 * t + 4 * (4 * w + sp) + c;
                        const int n = i >> 7, jj = (i >> 5) & 3, rr = i & 31;
                        blk[16 + 32 * n + rr] |= (uint8_t)(((byte >> (2 * sp)) & 3) << (2 * jj));
                    }
                }
            for (int k = 0; k < 4; k++) blk[4 * t + k] = T[1024 + 8 * lane + 4 * hs + k];
        }
        for (int b = 0; b < 4; b++) blk[80 + b] = T[1280 + 4 * r + b];
    } break;
    default:
        break;
    }
}

// ------------------------------------------------ reference decoders --------
// f16 bits -> f32, exact (WGSL unpack2x16float, kernels.wgsl.js:91-93).
__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)bits16));
}

__device__ __forceinline__ void scale_min_k4(const uint8_t *sb, int j, int &sc, int &mn) {
    // kernels.wgsl.js:94-104
    if (j < 4) { sc = sb[j] & 63; mn = sb[j + 4] & 63; }
    else { sc = (sb[j + 4] & 0xF) | ((sb[j - 4] >> 6) << 4); mn = (sb[j + 4] >> 4) | ((sb[j] >> 6) << 4); }
}

// One GGUF block to f32 with the reference's operation order (every product is
// exact; Q4_K rounds once in d1*q - m1). `grid` = int8 codebook (8 per entry).
__device__ inline void decode_block(int type, const uint8_t *blk, const int8_t *grid, float *out) {
    switch (type) {
    case EF_Q8_0: {
        const float d = h2f(blk[0] | (blk[1] << 8));
        for (int i = 0; i < 32; i++) out[i] = __fmul_rn((float)(int8_t)blk[2 + i], d);
    } break;
    case EF_Q4_0: {
        // kernels.wgsl.js:171-190: low nibble -> weight i, high -> i + 16; (q - 8) * d
        const float d = h2f(blk[0] | (blk[1] << 8));
        for (int i = 0; i < 16; i++) {
            out[i] = __fmul_rn((float)((int)(blk[2 + i] & 15) - 8), d);
            out[i + 16] = __fmul_rn((float)((int)(blk[2 + i] >> 4) - 8), d);
        }
    } break;
    case EF_Q5_K: {
        // kernels.wgsl.js:333-362
        const float d = h2f(blk[0] | (blk[1] << 8)), dmin = h2f(blk[2] | (blk[3] << 8));
        for (int j = 0; j < 4; j++) {
            int s1, m1i, s2, m2i;
            scale_min_k4(blk + 4, 2 * j, s1, m1i);
            scale_min_k4(blk + 4, 2 * j + 1, s2, m2i);
            const float d1 = __fmul_rn(d, (float)s1), m1 = __fmul_rn(dmin, (float)m1i);
            const float d2 = __fmul_rn(d, (float)s2), m2 = __fmul_rn(dmin, (float)m2i);
            for (int l = 0; l < 32; l++) {
                const int q = blk[48 + 32 * j + l], h = blk[16 + l];
                const int a = (q & 15) + (((h >> (2 * j)) & 1) ? 16 : 0);
                const int b = (q >> 4) + (((h >> (2 * j + 1)) & 1) ? 16 : 0);
                out[64 * j + l] = __fsub_rn(__fmul_rn(d1, (float)a), m1);
                out[64 * j + 32 + l] = __fsub_rn(__fmul_rn(d2, (float)b), m2);
            }
        }
    } break;
    case EF_Q2_K: {
        // kernels.wgsl.js:192-217
        const float d = h2f(blk[80] | (blk[81] << 8)), dmin = h2f(blk[82] | (blk[83] << 8));
        for (int n = 0; n < 2; n++)
            for (int j = 0; j < 4; j++) {
                const int sa = blk[8 * n + 2 * j], sb = blk[8 * n + 2 * j + 1];
                const float dl1 = __fmul_rn(d, (float)(sa & 15)), ml1 = __fmul_rn(dmin, (float)(sa >> 4));
                const float dl2 = __fmul_rn(d, (float)(sb & 15)), ml2 = __fmul_rn(dmin, (float)(sb >> 4));
                for (int l = 0; l < 16; l++) {
                    const int qa = (blk[16 + 32 * n + l] >> (2 * j)) & 3, qb = (blk[16 + 32 * n + 16 + l] >> (2 * j)) & 3;
                    out[128 * n + 32 * j + l] = __fsub_rn(__fmul_rn(dl1, (float)qa), ml1);
                    out[128 * n + 32 * j + 16 + l] = __fsub_rn(__fmul_rn(dl2, (float)qb), ml2);
                }
            }
    } break;
    case EF_Q4_K: {
        const float d = h2f(blk[0] | (blk[1] << 8)), dmin = h2f(blk[2] | (blk[3] << 8));
        for (int j = 0; j < 4; j++) {
            int s1, m1i, s2, m2i;
            scale_min_k4(blk + 4, 2 * j, s1, m1i);
            scale_min_k4(blk + 4, 2 * j + 1, s2, m2i);
            const float d1 = __fmul_rn(d, (float)s1), m1 = __fmul_rn(dmin, (float)m1i);
            const float d2 = __fmul_rn(d, (float)s2), m2 = __fmul_rn(dmin, (float)m2i);
            for (int l = 0; l < 32; l++) {
                const uint8_t q = blk[16 + 32 * j + l];
                out[64 * j + l] = __fsub_rn(__fmul_rn(d1, (float)(q & 0xF)), m1);
                out[64 * j + 32 + l] = __fsub_rn(__fmul_rn(d2, (float)(q >> 4)), m2);
            }
        }
    } break;
    case EF_Q6_K: {
        const float d = h2f(blk[208] | (blk[209] << 8));
        for (int n = 0; n < 2; n++) {
            const uint8_t *ql = blk + 64 * n, *qh = blk + 128 + 32 * n;
            const int8_t *sc = (const int8_t *)(blk + 192 + 8 * n);
            for (int l = 0; l < 32; l++) {
                const int is = l >> 4;
                const int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = ((ql[32 + l] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = ((ql[32 + l] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                out[128 * n + l] = __fmul_rn(__fmul_rn(d, (float)sc[is]), (float)q1);
                out[128 * n + 32 + l] = __fmul_rn(__fmul_rn(d, (float)sc[is + 2]), (float)q2);
                out[128 * n + 64 + l] = __fmul_rn(__fmul_rn(d, (float)sc[is + 4]), (float)q3);
                out[128 * n + 96 + l] = __fmul_rn(__fmul_rn(d, (float)sc[is + 6]), (float)q4);
            }
        }
    } break;
    case EF_IQ2_XXS: {
        const float d = h2f(blk[0] | (blk[1] << 8));
        for (int ib = 0; ib < 8; ib++) {
            const uint32_t a0 = rd32(blk + 2 + 8 * ib), a1 = rd32(blk + 6 + 8 * ib);
            const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(a1 >> 28))), 0.25f);
            for (int l = 0; l < 4; l++) {
                const uint32_t gi = (a0 >> (8 * l)) & 0xFF;
                const uint32_t bits = (a1 >> (7 * l)) & 127u;
                const uint32_t signs = bits | ((uint32_t)(__popc(bits) & 1) << 7);
                for (int j = 0; j < 8; j++) {
                    const float gv = (float)(uint8_t)grid[8 * gi + j];
                    const float sg = (signs & (1u << j)) ? -1.0f : 1.0f;
                    out[32 * ib + 8 * l + j] = __fmul_rn(__fmul_rn(db, gv), sg);
                }
            }
        }
    } break;
    case EF_IQ1_S: {
        const float d = h2f(blk[0] | (blk[1] << 8));
        for (int ib = 0; ib < 8; ib++) {
            const uint32_t qh = blk[34 + 2 * ib] | (blk[35 + 2 * ib] << 8);
            const float dl = __fmul_rn(d, (float)(2u * ((qh >> 12) & 7u) + 1u));
            const float delta = (qh & 0x8000u) ? -0.125f : 0.125f;
            for (int l = 0; l < 4; l++) {
                const uint32_t gi = blk[2 + 4 * ib + l] | (((qh >> (3 * l)) & 7u) << 8);
                for (int j = 0; j < 8; j++)
                    out[32 * ib + 8 * l + j] = __fmul_rn(dl, __fadd_rn((float)grid[8 * gi + j], delta));
            }
        }
    } break;
    default:
        break;
    }
}

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    // (a & b) | c
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}
// word i of v (i < 4, after unrolling a compile-time constant)
__device__ __forceinline__ uint32_t wsel(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
// two f16 weights from the bytes of qbytes that `sel` picks (prmt selector
// 0x5140: bytes 0,1; 0x7362: bytes 2,3): q as (1024 + q) - 1024 exactly, then
// one f16 fma with the sub-block's f16(d * sc) and -f16(dmin * m)
__device__ __forceinline__ uint32_t f16_pair_dm(uint32_t qbytes, uint32_t sel, uint32_t d2, uint32_t negm2) {
    uint32_t r;
    const uint32_t q = hsub2u(prmt(qbytes, 0x64646464u, sel), 0x64006400u);
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(q), "r"(d2), "r"(negm2));
    return r;
}
// f32 -> f16x2 (v, v), round to nearest even
__device__ __forceinline__ uint32_t f16x2_bcast(float v) {
    const uint32_t h = __half_as_ushort(__float2half_rn(v));
    return h | (h << 16);
}
// bit c of x (c < 4) to bit 8c
__device__ __forceinline__ uint32_t spread4(uint32_t x) { return (x * 0x00204081u) & 0x01010101u; }
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b),
                        *reinterpret_cast<__half2 *>(&c));
    return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t hadd2u(uint32_t a, uint32_t b) {
    __half2 r = __hadd2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// D (+)= A(16x16 f16, row) * B(16x8 f16, col), f32 accumulate.
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 128-bit load of weights: read-only path, not kept in L1.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// D (+)= A(16x32 u8, row) * B(32x8 s8, col), s32 accumulate (exact).
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------ mbarriers and bulk async copies --
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the async proxy (bulk copies).
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Bounded wait for phase `parity` of `bar`: false after `limit` polls (the
// caller records the failure and stops waiting; nothing here spins forever).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t limit) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < limit; i++) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok) : "r"(a), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}
// Contiguous global -> shared copy (TMA engine, no tensor map, this CTA only);
// completes `bytes` of transaction count on `bar`. Both addresses and the
// size must be multiples of 16 bytes.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace ef

/*
 * elffuss_oracle.c -- CPU restatement of the Elffuss quantized matrix-product
 * arithmetic. TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and
 * the CPU-baseline leg of bench.py call it as the checker. The product path
 * (the CUDA library) never links or calls it.
 *
 * Every function names the reference file:line it restates (paths relative to
 * the utopia-ia/elffuss-engine snapshot). The reference is JavaScript + WGSL
 * over WebGPU and cannot run here, so this is a restatement; the block decoders
 * are pinned against gguf-py 0.19.0 (gguf.quants.dequantize), the llama.cpp-
 * family decoder the reference says it validates against (README.md:150-156).
 *
 * Block formats (ggml type ids, js/gguf.js:48-64):
 *   Q8_0    (8)  32 w,  34 B: f16 d | int8 qs[32]                 kernels.wgsl.js:154-169
 *   Q4_K   (12) 256 w, 144 B: f16 d | f16 dmin | u8 sc[12] | qs[128]  kernels.wgsl.js:227-250
 *   Q6_K   (14) 256 w, 210 B: ql[128] | qh[64] | int8 sc[16] | f16 d   kernels.wgsl.js:269-330
 *   IQ2_XXS(16) 256 w,  66 B: f16 d | 8 x (u32 a0, u32 a1)            kernels.wgsl.js:368-396
 *   IQ1_S  (19) 256 w,  50 B: f16 d | qs[32] | u16 qh[8]              kernels.wgsl.js:805-822
 *   Q4_0    (2)  32 w,  18 B: f16 d | nibbles[16]                     kernels.wgsl.js:176-190
 *   Q5_K   (13) 256 w, 176 B: f16 d | f16 dmin | u8 sc[12] | qh[32] | qs[128]  kernels.wgsl.js:333-362
 *   Q2_K   (10) 256 w,  84 B: sc[16] | qs[64] | f16 d | f16 dmin          kernels.wgsl.js:192-217
 *
 * Each dequantised weight is an exact f32 product (f16 scale x small integer),
 * except Q4_K's single rounding in d1*q - m1; the restatement keeps the
 * reference's operation order so the f32 bits are the reference's bits.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <pthread.h>

enum { OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q8_0 = 8, OR_Q2_K = 10, OR_Q4_K = 12, OR_Q5_K = 13,
       OR_Q6_K = 14, OR_IQ2_XXS = 16, OR_IQ1_S = 19 };

/* f16 -> f32, exact. Restates js/cpu.js:39-44 (deF16) and WGSL unpack2x16float
 * used by load_scale (kernels.wgsl.js:91-93). */
float or_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) { bits = s; }
        else {                       /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; sh++; }
            m &= 0x3ff;
            bits = s | ((uint32_t)(127 - 15 - sh + 1) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* f32 -> f16, round to nearest even. Restates js/cpu.js:84-99 (aF16) and the
 * WGSL vec4<f16>(f32) conversion of kernels.drift.wgsl.js:92-105. */
uint16_t or_f32_to_f16(float v) {
    uint32_t x;
    memcpy(&x, &v, 4);
    uint32_t s = (x >> 16) & 0x8000u, e = (x >> 23) & 0xff, m = x & 0x7fffffu;
    if (e == 0xff) return (uint16_t)(s | 0x7c00u | (m ? 0x200u : 0u));
    int ee = (int)e - 127 + 15;
    if (ee >= 0x1f) return (uint16_t)(s | 0x7c00u);
    if (ee <= 0) {
        if (ee < -10) return (uint16_t)s;
        uint32_t mm = (m | 0x800000u) >> (1 - ee);
        return (uint16_t)(s | ((mm + 0x1000u + ((mm >> 13) & 1u) - 1u) >> 13));
    }
    uint32_t r = s | ((uint32_t)ee << 10) | (m >> 13);
    uint32_t rest = m & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (r & 1u))) r++;
    return (uint16_t)r;
}

void or_f32_to_f16_array(const float *src, uint16_t *dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = or_f32_to_f16(src[i]);
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

int or_block_info(int type, int *elems, int *bytes) {
    switch (type) {
    case OR_Q8_0: *elems = 32; *bytes = 34; return 0;
    case OR_Q4_0: *elems = 32; *bytes = 18; return 0;
    case OR_Q4_K: *elems = 256; *bytes = 144; return 0;
    case OR_Q5_K: *elems = 256; *bytes = 176; return 0;
    case OR_Q2_K: *elems = 256; *bytes = 84; return 0;
    case OR_Q6_K: *elems = 256; *bytes = 210; return 0;
    case OR_IQ2_XXS: *elems = 256; *bytes = 66; return 0;
    case OR_IQ1_S: *elems = 256; *bytes = 50; return 0;
    default: return -1;
    }
}

/* scale_min_k4, kernels.wgsl.js:94-104: 6-bit scale/min pair j of the 12
 * packed bytes. */
static void scale_min_k4(const uint8_t *sb, int j, int *sc, int *mn) {
    if (j < 4) {
        *sc = sb[j] & 63;
        *mn = sb[j + 4] & 63;
    } else {
        *sc = (sb[j + 4] & 0xF) | ((sb[j - 4] >> 6) << 4);
        *mn = (sb[j + 4] >> 4) | ((sb[j] >> 6) << 4);
    }
}

/* One block to f32. `grid` is the i-quant codebook as int8 entries of 8 bytes
 * (IQ2_XXS: 256 entries, IQ1_S: 2048), quant-tables.js:40,107. */
static void dequant_block(int type, const uint8_t *blk, const int8_t *grid, float *out) {
    switch (type) {
    case OR_Q8_0: { /* kernels.wgsl.js:161-169: f32(q) * d */
        float d = or_f16_to_f32(rd16(blk));
        for (int i = 0; i < 32; i++) out[i] = (float)(int8_t)blk[2 + i] * d;
    } break;
    case OR_Q4_0: { /* kernels.wgsl.js:180-190: low nibble -> i, high -> i+16 */
        float d = or_f16_to_f32(rd16(blk));
        for (int i = 0; i < 16; i++) {
            uint8_t by = blk[2 + i];
            out[i] = (float)((int)(by & 0xF) - 8) * d;
            out[i + 16] = (float)((int)(by >> 4) - 8) * d;
        }
    } break;
    case OR_Q4_K: { /* kernels.wgsl.js:231-250: d1*q - m1, low nibbles first */
        float d = or_f16_to_f32(rd16(blk)), dmin = or_f16_to_f32(rd16(blk + 2));
        const uint8_t *sb = blk + 4, *qs = blk + 16;
        for (int j = 0; j < 4; j++) {
            int sc1, m1i, sc2, m2i;
            scale_min_k4(sb, 2 * j, &sc1, &m1i);
            scale_min_k4(sb, 2 * j + 1, &sc2, &m2i);
            float d1 = d * (float)sc1, m1 = dmin * (float)m1i;
            float d2 = d * (float)sc2, m2 = dmin * (float)m2i;
            for (int l = 0; l < 32; l++) {
                uint8_t q = qs[32 * j + l];
                /* d1*q is exact, so the only rounding is the subtraction. */
                out[64 * j + l] = d1 * (float)(q & 0xF) - m1;
                out[64 * j + 32 + l] = d2 * (float)(q >> 4) - m2;
            }
        }
    } break;
    case OR_Q5_K: { /* kernels.wgsl.js:333-362: Q4_K plus the fifth bit, qh[l] bit 2j / 2j+1 */
        float d = or_f16_to_f32(rd16(blk)), dmin = or_f16_to_f32(rd16(blk + 2));
        const uint8_t *sb = blk + 4, *qh = blk + 16, *qs = blk + 48;
        for (int j = 0; j < 4; j++) {
            int sc1, m1i, sc2, m2i;
            scale_min_k4(sb, 2 * j, &sc1, &m1i);
            scale_min_k4(sb, 2 * j + 1, &sc2, &m2i);
            float d1 = d * (float)sc1, m1 = dmin * (float)m1i;
            float d2 = d * (float)sc2, m2 = dmin * (float)m2i;
            for (int l = 0; l < 32; l++) {
                uint8_t q = qs[32 * j + l];
                int a = (q & 0xF) + ((qh[l] >> (2 * j)) & 1 ? 16 : 0);
                int b = (q >> 4) + ((qh[l] >> (2 * j + 1)) & 1 ? 16 : 0);
                out[64 * j + l] = d1 * (float)a - m1;
                out[64 * j + 32 + l] = d2 * (float)b - m2;
            }
        }
    } break;
    case OR_Q2_K: { /* kernels.wgsl.js:192-217: 2-bit q, 4+4-bit (scale, min) per 16 weights */
        float d = or_f16_to_f32(rd16(blk + 80)), dmin = or_f16_to_f32(rd16(blk + 82));
        for (int n = 0; n < 2; n++) {
            const uint8_t *qs = blk + 16 + 32 * n;
            for (int j = 0; j < 4; j++) {
                uint8_t sca = blk[8 * n + 2 * j], scb = blk[8 * n + 2 * j + 1];
                float dl1 = d * (float)(sca & 0xF), ml1 = dmin * (float)(sca >> 4);
                float dl2 = d * (float)(scb & 0xF), ml2 = dmin * (float)(scb >> 4);
                float *o = out + 128 * n + 32 * j;
                for (int l = 0; l < 16; l++) {
                    o[l] = dl1 * (float)((qs[l] >> (2 * j)) & 3) - ml1;
                    o[16 + l] = dl2 * (float)((qs[16 + l] >> (2 * j)) & 3) - ml2;
                }
            }
        }
    } break;
    case OR_Q6_K: { /* kernels.wgsl.js:298-330 and cpu.js:63-76 */
        float d = or_f16_to_f32(rd16(blk + 208));
        for (int n = 0; n < 2; n++) {
            const uint8_t *ql = blk + 64 * n, *qh = blk + 128 + 32 * n;
            const int8_t *sc = (const int8_t *)(blk + 192 + 8 * n);
            float *o = out + 128 * n;
            for (int l = 0; l < 32; l++) {
                int is = l >> 4;
                int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = ((ql[32 + l] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[32 + l] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                o[l] = (d * (float)sc[is]) * (float)q1;
                o[32 + l] = (d * (float)sc[is + 2]) * (float)q2;
                o[64 + l] = (d * (float)sc[is + 4]) * (float)q3;
                o[96 + l] = (d * (float)sc[is + 6]) * (float)q4;
            }
        }
    } break;
    case OR_IQ2_XXS: { /* kernels.wgsl.js:373-396; signs = 7 bits + even parity */
        float d = or_f16_to_f32(rd16(blk));
        for (int ib = 0; ib < 8; ib++) {
            uint32_t a0 = rd32(blk + 2 + 8 * ib), a1 = rd32(blk + 6 + 8 * ib);
            float db = d * (0.5f + (float)(a1 >> 28)) * 0.25f;
            for (int l = 0; l < 4; l++) {
                uint32_t gi = (a0 >> (8 * l)) & 0xFF;
                uint32_t bits = (a1 >> (7 * l)) & 127u;
                uint32_t signs = bits | ((uint32_t)(__builtin_popcount(bits) & 1) << 7);
                const int8_t *g = grid + 8 * gi;
                for (int j = 0; j < 8; j++) {
                    float gv = (float)(uint8_t)g[j];
                    float sg = (signs & (1u << j)) ? -1.0f : 1.0f;
                    out[32 * ib + 8 * l + j] = db * gv * sg;
                }
            }
        }
    } break;
    case OR_IQ1_S: { /* kernels.wgsl.js:805-822: dl*(grid + delta) */
        float d = or_f16_to_f32(rd16(blk));
        for (int ib = 0; ib < 8; ib++) {
            uint32_t qh = rd16(blk + 34 + 2 * ib);
            float dl = d * (float)(2u * ((qh >> 12) & 7u) + 1u);
            float delta = (qh & 0x8000u) ? -0.125f : 0.125f;
            for (int l = 0; l < 4; l++) {
                uint32_t gi = blk[2 + 4 * ib + l] | (((qh >> (3 * l)) & 7u) << 8);
                const int8_t *g = grid + 8 * gi;
                for (int j = 0; j < 8; j++)
                    out[32 * ib + 8 * l + j] = dl * ((float)g[j] + delta);
            }
        }
    } break;
    default:
        break;
    }
}

/* Full tensor to f32, block by block: dequantShader, kernels.wgsl.js:903-922
 * (ops.js:813-823). Returns -1 for an unknown type. */
int or_dequant(int type, const uint8_t *w, int64_t nblocks, const int8_t *grid, float *out) {
    int be, bb;
    if (or_block_info(type, &be, &bb)) return -1;
    for (int64_t b = 0; b < nblocks; b++) dequant_block(type, w + b * bb, grid, out + b * be);
    return 0;
}

/* Row-range worker shared by the two matmul restatements below. */
typedef struct {
    int type, w16, f64;
    const uint8_t *w;
    int64_t rows, k, tokens, r0, r1;
    const int8_t *grid;
    const float *x;
    const uint16_t *xh;
    double *yd;
    float *yf;
} mm_job;

static void *mm_rows(void *arg) {
    mm_job *j = (mm_job *)arg;
    int be, bb;
    or_block_info(j->type, &be, &bb);
    int64_t bpr = j->k / be;
    float rowbuf[256];
    for (int64_t r = j->r0; r < j->r1; r++) {
        if (j->f64) {
            for (int64_t t = 0; t < j->tokens; t++) j->yd[t * j->rows + r] = 0.0;
            for (int64_t b = 0; b < bpr; b++) {
                dequant_block(j->type, j->w + (r * bpr + b) * bb, j->grid, rowbuf);
                if (j->w16)
                    for (int i = 0; i < be; i++) rowbuf[i] = or_f16_to_f32(or_f32_to_f16(rowbuf[i]));
                for (int64_t t = 0; t < j->tokens; t++) {
                    double s = 0.0;
                    int64_t k0 = t * j->k + b * be;
                    if (j->xh)
                        for (int i = 0; i < be; i++) s += (double)rowbuf[i] * (double)or_f16_to_f32(j->xh[k0 + i]);
                    else
                        for (int i = 0; i < be; i++) s += (double)rowbuf[i] * (double)j->x[k0 + i];
                    j->yd[t * j->rows + r] += s;
                }
            }
        } else {
            /* f32, natural k order, one accumulator per (row, token). */
            float acc[16];
            for (int64_t t0 = 0; t0 < j->tokens; t0 += 16) {
                int64_t nt = j->tokens - t0 < 16 ? j->tokens - t0 : 16;
                for (int64_t t = 0; t < nt; t++) acc[t] = 0.0f;
                for (int64_t b = 0; b < bpr; b++) {
                    dequant_block(j->type, j->w + (r * bpr + b) * bb, j->grid, rowbuf);
                    for (int64_t t = 0; t < nt; t++) {
                        const float *xr = j->x + (t0 + t) * j->k + b * be;
                        float s = acc[t];
                        for (int i = 0; i < be; i++) s += rowbuf[i] * xr[i];
                        acc[t] = s;
                    }
                }
                for (int64_t t = 0; t < nt; t++) j->yf[(t0 + t) * j->rows + r] = acc[t];
            }
        }
    }
    return NULL;
}

static int mm_run(mm_job proto, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads > proto.rows) nthreads = proto.rows > 0 ? (int)proto.rows : 1;
    pthread_t th[256];
    mm_job jobs[256];
    int joinable[256];
    int64_t per = (proto.rows + nthreads - 1) / nthreads;
    for (int i = 0; i < nthreads; i++) {
        jobs[i] = proto;
        jobs[i].r0 = i * per < proto.rows ? i * per : proto.rows;
        jobs[i].r1 = (i + 1) * per < proto.rows ? (i + 1) * per : proto.rows;
        joinable[i] = 0;
    }
    for (int i = 1; i < nthreads; i++) {
        if (jobs[i].r0 >= jobs[i].r1) continue;
        if (pthread_create(&th[i], NULL, mm_rows, &jobs[i]) == 0) joinable[i] = 1;
        else mm_rows(&jobs[i]);           /* no thread: do the range here */
    }
    mm_rows(&jobs[0]);                    /* range 0 runs on the caller */
    for (int i = 1; i < nthreads; i++)
        if (joinable[i]) pthread_join(th[i], NULL);
    return 0;
}

/* y[t][r] = sum_k dequant(W)[r][k] * x[t][k], in f64 -- the matmul contract of
 * createQuantOps().matmul, ops.js:827-1101 (output [tokens][rows], f32 x
 * token-major). `xh` (optional, may be NULL) replaces x by f16 activations:
 * the GEMM2 contract, kernels.gemm2.wgsl.js:12-23,174-240, where W is also
 * rounded to f16 (`w16` != 0) as the reference's shared-memory tile does. */
int or_matmul_f64(int type, const uint8_t *w, int64_t rows, int64_t k, const int8_t *grid,
                  const float *x, const uint16_t *xh, int64_t tokens, int w16, double *y,
                  int nthreads) {
    int be, bb;
    if (or_block_info(type, &be, &bb) || k % be) return -1;
    mm_job j = {type, w16, 1, w, rows, k, tokens, 0, rows, grid, x, xh, y, NULL};
    return mm_run(j, nthreads);
}

/* The same product accumulated in f32 in natural k order, one output row per
 * work item: the generic matmul scaffold, kernels.wgsl.js:949-1186, as a CPU
 * loop. This is the timed CPU baseline ("port" of the reference arithmetic). */
int or_matmul_f32(int type, const uint8_t *w, int64_t rows, int64_t k, const int8_t *grid,
                  const float *x, int64_t tokens, float *y, int nthreads) {
    int be, bb;
    if (or_block_info(type, &be, &bb) || k % be) return -1;
    mm_job j = {type, 0, 0, w, rows, k, tokens, 0, rows, grid, x, NULL, NULL, y};
    return mm_run(j, nthreads);
}

/* ||dequant(W)[r]||_2 per row, f64: the row-norm factor of the acceptance
 * bound max|err| <= 1e-3 * ||row||_2 * ||x||_2. */
int or_row_norms(int type, const uint8_t *w, int64_t rows, int64_t k, const int8_t *grid,
                 double *out) {
    int be, bb;
    if (or_block_info(type, &be, &bb) || k % be) return -1;
    int64_t bpr = k / be;
    float rowbuf[256];
    for (int64_t r = 0; r < rows; r++) {
        double s = 0.0;
        for (int64_t b = 0; b < bpr; b++) {
            dequant_block(type, w + (r * bpr + b) * bb, grid, rowbuf);
            for (int i = 0; i < be; i++) s += (double)rowbuf[i] * (double)rowbuf[i];
        }
        out[r] = sqrt(s);
    }
    return 0;
}

/* silu(g) * u with silu(v) = v / (1 + exp(-v)): the GEMV2 SwiGLU epilogue,
 * kernels.gemv.wgsl.js:434-437,512-513, in f64. */
void or_swiglu_f64(const double *g, const double *u, int64_t n, double *out) {
    for (int64_t i = 0; i < n; i++) out[i] = g[i] / (1.0 + exp(-g[i])) * u[i];
}

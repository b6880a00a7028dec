// model.cu -- the non-matmul operations of a decoder step (sm_100a), for the
// synthetic LFM3- and Llama-shaped decoders that drive the GEMV / GEMM hot
// path end to end.
//
// Each restates one operation of the reference's forward (js/model.js,
// js/kernels.nn.wgsl.js, js/kernels.model.wgsl.js, js/kernels.ssm.wgsl.js,
// js/kernels.topk.wgsl.js):
//   rmsnorm            y = x * rsqrt(mean(x^2) + eps) * w     (kernels.nn.wgsl.js:46-80)
//   norm_add_norm      x += rmsnorm(o) * w_post (or += o); n = rmsnorm(x) * w_next
//                      (post-norm + residual + next norm, model.js:635-664)
//   shortconv          B|C|x split, B*x, causal depthwise conv with state,
//                      C*y (model.js:758-794, kernels.model.wgsl.js:45-86,
//                      kernels.ssm.wgsl.js:64-92)
//   rope_cache         optional per-head RMSNorm of q and k, NEOX or NORM RoPE,
//                      k and v into the caches at each row's position
//                      (model.js:853-945, kernels.nn.wgsl.js:87-139)
//   attention          softmax(q.k / sqrt(D)) with causal + window mask, times
//                      v, times sigmoid(per-head gate) (kernels.nn.wgsl.js:
//                      141-200, kernels.model.wgsl.js:89-105): split over the
//                      keys for one new token per sequence; for a prompt,
//                      64-key tiles shared by 128 (head, token) rows with an
//                      online softmax (one CTA per query row for head
//                      groupings other than 1, 2, 4, 8)
//   argmax             greedy token, strict '>' so the lowest index wins ties
//                      (sample.js:95-99); advances the device-side position;
//                      per-shard pairs and their selection for a sharded head
//   topk               the sampler's candidates, exactly (kernels.topk.wgsl.js)
//   swiglu             g * sigmoid(g) * u for the prompt's FFN
// Positions and tokens live in device memory, so one decode step can be
// captured as a CUDA graph and replayed with no host round trip.
// The KV caches hold f32, or f16 (the reference's kvF16 option,
// kernels.attn.wgsl.js:51-55, model.js:906-946: k after its norm and RoPE and v
// rounded to f16 when stored, to nearest even; q, the scores and every sum
// stay f32). Half the cache bytes, which decode attention reads whole.
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace ef {

// cache element loads and stores (f32 or f16 caches)
__device__ __forceinline__ float kv_f(float x) { return x; }
__device__ __forceinline__ float kv_f(__half x) { return __half2float(x); }
__device__ __forceinline__ void kv_put(float *p, float v) { *p = v; }
__device__ __forceinline__ void kv_put(__half *p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ float4 kv_ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 kv_ld4(const __half *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float2 kv_ld2(const float *p) { return *reinterpret_cast<const float2 *>(p); }
__device__ __forceinline__ float2 kv_ld2(const __half *p) { return __half22float2(*reinterpret_cast<const __half2 *>(p)); }


// One CTA per row of T = min(256, n/4) threads; each thread keeps V float4 of
// the row in registers (all loads issued before the first reduction),
// n = 4 * T * V.
template <int V>
__global__ void __launch_bounds__(256) ef_rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                      int n, float eps, float *__restrict__ y) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const float4 *xr = reinterpret_cast<const float4 *>(x + (int64_t)blockIdx.x * n);
    const float4 *wr = reinterpret_cast<const float4 *>(w);
    float4 *yr = reinterpret_cast<float4 *>(y + (int64_t)blockIdx.x * n);
    float4 v[V], wv[V];
#pragma unroll
    for (int j = 0; j < V; j++) {
        v[j] = xr[threadIdx.x + blockDim.x * j];
        wv[j] = wr[threadIdx.x + blockDim.x * j];
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < V; j++) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    const float scale = rsqrtf(block_sum(ss, red) / (float)n + eps);
#pragma unroll
    for (int j = 0; j < V; j++)
        yr[threadIdx.x + blockDim.x * j] = make_float4(v[j].x * scale * wv[j].x, v[j].y * scale * wv[j].y,
                                                v[j].z * scale * wv[j].z, v[j].w * scale * wv[j].w);
}

// x += rmsnorm(o) * w_post (or += o without a post-norm); nrm = rmsnorm(x) * w_next.
// Same shape rules as ef_rmsnorm_kernel.
template <int V>
__global__ void __launch_bounds__(256) ef_norm_add_norm_kernel(const float *__restrict__ o,
                                                            const float *__restrict__ w_post, float *__restrict__ x,
                                                            const float *__restrict__ w_next, int n, float eps,
                                                            float *__restrict__ nrm) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const int64_t row = (int64_t)blockIdx.x * (n / 4);
    const float4 *o4 = reinterpret_cast<const float4 *>(o) + row;
    float4 *x4 = reinterpret_cast<float4 *>(x) + row;
    float4 *n4 = reinterpret_cast<float4 *>(nrm) + row;
    const float4 *wp = reinterpret_cast<const float4 *>(w_post), *wn = reinterpret_cast<const float4 *>(w_next);
    float4 ov[V], xv[V], wpv[V], wnv[V];
#pragma unroll
    for (int j = 0; j < V; j++) {
        const int i = threadIdx.x + blockDim.x * j;
        ov[j] = o4[i];
        xv[j] = x4[i];
        wpv[j] = w_post ? wp[i] : make_float4(1.f, 1.f, 1.f, 1.f);
        wnv[j] = wn[i];
    }
    float s1 = 1.f;
    if (w_post) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < V; j++)
            ss += ov[j].x * ov[j].x + ov[j].y * ov[j].y + ov[j].z * ov[j].z + ov[j].w * ov[j].w;
        s1 = rsqrtf(block_sum(ss, red) / (float)n + eps);
    }
    float ss2 = 0.f;
#pragma unroll
    for (int j = 0; j < V; j++) {
        xv[j].x += ov[j].x * s1 * wpv[j].x;
        xv[j].y += ov[j].y * s1 * wpv[j].y;
        xv[j].z += ov[j].z * s1 * wpv[j].z;
        xv[j].w += ov[j].w * s1 * wpv[j].w;
        ss2 += xv[j].x * xv[j].x + xv[j].y * xv[j].y + xv[j].z * xv[j].z + xv[j].w * xv[j].w;
        x4[threadIdx.x + blockDim.x * j] = xv[j];
    }
    const float s2 = rsqrtf(block_sum(ss2, red) / (float)n + eps);
#pragma unroll
    for (int j = 0; j < V; j++)
        n4[threadIdx.x + blockDim.x * j] = make_float4(xv[j].x * s2 * wnv[j].x, xv[j].y * s2 * wnv[j].y,
                                                xv[j].z * s2 * wnv[j].z, xv[j].w * s2 * wnv[j].w);
}

// One thread per channel; tokens in order. bcx [T][3C] = B | C | x;
// state [K-1][C] (oldest first); w [C][K] in temporal order (r = 0 oldest).
template <int K>
__global__ void ef_shortconv_kernel(const float *__restrict__ bcx, const float *__restrict__ w, float *__restrict__ state,
                                 int tokens, int C, float *__restrict__ y) {
    pdl_trigger();
    pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float win[K - 1], wc[K];
#pragma unroll
    for (int r = 0; r < K - 1; r++) win[r] = state[(int64_t)r * C + c];
#pragma unroll
    for (int r = 0; r < K; r++) wc[r] = w[(int64_t)c * K + r];
    for (int t = 0; t < tokens; t++) {
        const float *row = bcx + (int64_t)t * 3 * C;
        const float bx = row[c] * row[2 * C + c];
        float acc = 0.f;
#pragma unroll
        for (int r = 0; r < K - 1; r++) acc += win[r] * wc[r];
        acc += bx * wc[K - 1];
        y[(int64_t)t * C + c] = row[C + c] * acc;
#pragma unroll
        for (int r = 0; r < K - 2; r++) win[r] = win[r + 1];
        win[K - 2] = bx;
    }
#pragma unroll
    for (int r = 0; r < K - 1; r++) state[(int64_t)r * C + c] = win[r];
}

// One warp per (token row, head), q heads first, then k heads. Rows are
// seqs x tokens (row r = sequence r / tokens, token t = r % tokens at position
// pos[seq] + t); q [rows][H][D] is rotated in place, k and v [rows][KVH][D]
// go to the caches [seqs][max_pos][KVH][D]. Lane pairs p = lane + 32 j
// (j < D/64): NEOX pairs elements (p, p + D/2), NORM pairs (2p, 2p + 1);
// theta = position * base^(-2p/D) (kernels.nn.wgsl.js:87-139). With wq / wk,
// the per-head RMSNorm comes first (model.js:877-917).
template <int D, bool NEOX, typename KV>
__global__ void ef_rope_cache_kernel(float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                                  const float *__restrict__ wq, const float *__restrict__ wk,
                                  const int *__restrict__ pos, int seqs, int tokens, int max_pos, int H, int KVH,
                                  float theta_scale, float eps, KV *__restrict__ kcache,
                                  KV *__restrict__ vcache) {
    pdl_trigger();
    pdl_wait();
    constexpr int J = D / 64;
    const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31, per = H + KVH;
    if (wid >= (int64_t)seqs * tokens * per) return;
    const int r = (int)(wid / per), head = (int)(wid - (int64_t)r * per);
    const int sq = r / tokens, t = r - sq * tokens;
    const int p = pos[sq] + t;
    const bool isq = head < H;
    const int hh = isq ? head : head - H;
    float *qrow = q + ((int64_t)r * H + hh) * D;
    const float *src = isq ? qrow : k + ((int64_t)r * KVH + hh) * D;
    const float *wn = isq ? wq : wk;
    float a[J], b[J];
    int i0[J], i1[J];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < J; j++) {
        const int pp = lane + 32 * j;
        i0[j] = NEOX ? pp : 2 * pp;
        i1[j] = NEOX ? pp + D / 2 : 2 * pp + 1;
        a[j] = src[i0[j]];
        b[j] = src[i1[j]];
        ss += a[j] * a[j] + b[j] * b[j];
    }
    if (wn) {
        const float scale = rsqrtf(warp_sum(ss) / (float)D + eps);
#pragma unroll
        for (int j = 0; j < J; j++) {
            a[j] = a[j] * scale * wn[i0[j]];
            b[j] = b[j] * scale * wn[i1[j]];
        }
    }
    const bool store = !isq && p >= 0 && p < max_pos;   // (a position past the caches is not stored)
    KV *kc = kcache + (((int64_t)sq * max_pos + p) * KVH + hh) * D;
#pragma unroll
    for (int j = 0; j < J; j++) {
        const float theta = (float)p * powf(theta_scale, (float)(lane + 32 * j));
        float sn, cs;
        sincosf(theta, &sn, &cs);
        const float r0 = a[j] * cs - b[j] * sn, r1 = a[j] * sn + b[j] * cs;
        if (isq) {
            qrow[i0[j]] = r0;
            qrow[i1[j]] = r1;
        } else if (store) {
            kv_put(kc + i0[j], r0);
            kv_put(kc + i1[j], r1);
        }
    }
    if (store) {
        const float *vr = v + ((int64_t)r * KVH + hh) * D;
        KV *vc = vcache + (((int64_t)sq * max_pos + p) * KVH + hh) * D;
#pragma unroll
        for (int j = 0; j < D / 32; j++) kv_put(vc + lane + 32 * j, vr[lane + 32 * j]);
    }
}

// CTA per (head h = blockIdx.x, query row r = blockIdx.y); rows as in
// ef_rope_cache_kernel. The query at position qp sees keys 0..qp of its
// sequence's caches, those with qp - key < window (window 0 = all); scale
// 1/sqrt(D); grouped heads (H / KVH queries per cache head); times
// sigmoid(gate[r][h]) when gate is given (kernels.nn.wgsl.js:141-200,
// kernels.model.wgsl.js:89-105). Scores in shared memory; the weighted sum of
// v rows is split over blockDim / D groups of keys, then added in group order.
template <int D, typename KV>
__global__ void __launch_bounds__(256) ef_attention_kernel(const float *__restrict__ q, const KV *__restrict__ kcache,
                                                        const KV *__restrict__ vcache,
                                                        const float *__restrict__ gate, const int *__restrict__ pos,
                                                        int tokens, int max_pos, int window, int H, int KVH,
                                                        float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float sc[];
    __shared__ float red[32];
    __shared__ float qs[D];
    __shared__ float part[256];
    const int h = blockIdx.x, r = blockIdx.y, kvh = h / (H / KVH);
    const int sq = r / tokens, t = r - sq * tokens;
    const int nkv = min(pos[sq] + t + 1, max_pos), qpos = nkv - 1;   // never past the caches
    const int k0 = window > 0 && qpos - window + 1 > 0 ? qpos - window + 1 : 0;
    const KV *kb = kcache + (int64_t)sq * max_pos * KVH * D;
    const KV *vb = vcache + (int64_t)sq * max_pos * KVH * D;
    const float *qr = q + ((int64_t)r * H + h) * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) qs[i] = qr[i] * rsqrtf((float)D);
    __syncthreads();
    float mx = -1e30f;
    for (int kk = k0 + threadIdx.x; kk < nkv; kk += blockDim.x) {
        const KV *kr = kb + ((int64_t)kk * KVH + kvh) * D;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < D / 4; i++) {
            const float4 kv = kv_ld4(kr + 4 * i);
            s += qs[4 * i] * kv.x + qs[4 * i + 1] * kv.y + qs[4 * i + 2] * kv.z + qs[4 * i + 3] * kv.w;
        }
        sc[kk - k0] = s;
        mx = fmaxf(mx, s);
    }
    {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        __syncthreads();
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = lane < nw ? red[lane] : -1e30f;
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    float sum = 0.f;
    for (int kk = k0 + threadIdx.x; kk < nkv; kk += blockDim.x) {
        const float e = expf(sc[kk - k0] - mx);
        sc[kk - k0] = e;
        sum += e;
    }
    sum = block_sum(sum, red);   // (its barriers also order the exp writes before the reads below)
    const float inv = 1.f / sum;
    constexpr int G = 256 / D;   // key groups
    const int d = threadIdx.x % D, g = threadIdx.x / D;
    float acc = 0.f;
    for (int kk = k0 + g; kk < nkv; kk += G) acc += sc[kk - k0] * kv_f(vb[((int64_t)kk * KVH + kvh) * D + d]);
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < D) {
        float o = 0.f;
#pragma unroll
        for (int gg = 0; gg < G; gg++) o += part[gg * D + d];
        o *= inv;
        if (gate) o = o / (1.0f + expf(-gate[(int64_t)r * H + h]));
        out[((int64_t)r * H + h) * D + d] = o;
    }
}

// Prompt attention (several new tokens per sequence), tiled in the manner of
// flash attention: CTA = (block of BQ = 128 / G consecutive query tokens of one
// sequence, cache head kvh) for the G = H / KVH query heads that share the
// cache head, so R = 128 (head, token) rows per CTA. The key range the rows
// can see goes through shared memory in tiles of 64 keys (each K and V row
// read once per CTA); per tile: scores S = Q K^T (a thread owns 8 rows x 4
// keys), the causal / window mask, an online softmax per row (running max m,
// running sum l, old output rescaled by exp(m_old - m_new)), and O += P V (a
// thread owns 8 rows x 4 or 8 dimensions of O in registers). All f32; same
// masking, scale, positions and gate as ef_attention_kernel (kernels.nn.wgsl.js:
// 141-200, kernels.model.wgsl.js:89-105). Rows of shared-memory tiles are
// padded by 4 floats so that the 16-byte loads of different rows fall in
// different banks. Query blocks are taken last to first: the longest key
// ranges start first.
constexpr int FA_R = 128, FA_BK = 64, FA_T = 256;
template <int D> constexpr size_t fa_smem() {
    return (size_t)(FA_R * (D + 4) + 2 * FA_BK * (D + 4) + FA_R * (FA_BK + 4) + 3 * FA_R) * sizeof(float);
}

template <int D, int G, typename KV>
__global__ void __launch_bounds__(FA_T, 1) ef_attn_prompt_kernel(const float *__restrict__ q, const KV *__restrict__ kcache,
                                                          const KV *__restrict__ vcache,
                                                          const float *__restrict__ gate, const int *__restrict__ pos,
                                                          int tokens, int max_pos, int window, int H, int KVH,
                                                          float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    constexpr int BQ = FA_R / G, LD = D + 4, LP = FA_BK + 4, C4 = D / 4, DV = D / 64;
    extern __shared__ float4 fa_smem4[];
    float *Qs = reinterpret_cast<float *>(fa_smem4);   // [R][LD], pre-scaled by 1/sqrt(D)
    float *Ks = Qs + FA_R * LD;                          // [BK][LD]
    float *Vs = Ks + FA_BK * LD;                         // [BK][LD]
    float *Ps = Vs + FA_BK * LD;                         // [R][LP] scores, then probabilities
    float *rm = Ps + FA_R * LP, *rl = rm + FA_R, *ra = rl + FA_R;   // running max, sum, rescale
    const int tid = threadIdx.x;
    const int qb = gridDim.x - 1 - blockIdx.x, kvh = blockIdx.y, sq = blockIdx.z;
    const int t0 = qb * BQ, p0 = pos[sq];
    const float scale = rsqrtf((float)D);
    for (int e = tid; e < FA_R * C4; e += FA_T) {
        const int i = e / C4, c = e - i * C4, tq = t0 + i % BQ;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tq < tokens) {
            v = *reinterpret_cast<const float4 *>(q + (((int64_t)sq * tokens + tq) * H + kvh * G + i / BQ) * D + 4 * c);
            v.x *= scale;
            v.y *= scale;
            v.z *= scale;
            v.w *= scale;
        }
        *reinterpret_cast<float4 *>(Qs + i * LD + 4 * c) = v;
    }
    for (int i = tid; i < FA_R; i += FA_T) {
        rm[i] = -INFINITY;
        rl[i] = 0.f;
    }
    // the keys any row of the block can see
    const int tl = (t0 + BQ < tokens ? t0 + BQ : tokens) - 1;
    const int qlo = p0 + t0 < max_pos ? p0 + t0 : max_pos - 1, qhi = p0 + tl < max_pos ? p0 + tl : max_pos - 1;
    const int klo = window > 0 && qlo - window + 1 > 0 ? qlo - window + 1 : 0;
    const int rg = tid >> 4, kg = tid & 15;   // S: rows 8rg.., keys kg + 16j; PV: rows 8rg.., dims 4kg.. (+64)
    int qp[8];                                // each row's position, -1 past the prompt
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int tq = t0 + (8 * rg + i) % BQ, p = p0 + tq;
        qp[i] = tq < tokens ? (p < max_pos ? p : max_pos - 1) : -1;
    }
    float o[8][4 * DV];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int c = 0; c < 4 * DV; c++) o[i][c] = 0.f;
    for (int kt = (klo / FA_BK) * FA_BK; kt <= qhi; kt += FA_BK) {
        __syncthreads();   // the previous tile's K, V and P are no longer read
        for (int e = tid; e < FA_BK * C4; e += FA_T) {
            const int j = e / C4, c = e - j * C4, key = kt + j;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (key <= qhi) {   // qhi < max_pos: inside the caches
                const int64_t off = (((int64_t)sq * max_pos + key) * KVH + kvh) * D + 4 * c;
                kv = kv_ld4(kcache + off);
                vv = kv_ld4(vcache + off);
            }
            *reinterpret_cast<float4 *>(Ks + j * LD + 4 * c) = kv;
            *reinterpret_cast<float4 *>(Vs + j * LD + 4 * c) = vv;
        }
        __syncthreads();
        float sc[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sc[i][j] = 0.f;
#pragma unroll 4
        for (int c = 0; c < D; c += 4) {
            float4 kk[4];
#pragma unroll
            for (int j = 0; j < 4; j++) kk[j] = *reinterpret_cast<const float4 *>(Ks + (kg + 16 * j) * LD + c);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 qq = *reinterpret_cast<const float4 *>(Qs + (8 * rg + i) * LD + c);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    sc[i][j] = fmaf(qq.w, kk[j].w, fmaf(qq.z, kk[j].z, fmaf(qq.y, kk[j].y, fmaf(qq.x, kk[j].x, sc[i][j]))));
            }
        }
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int key = kt + kg + 16 * j;
                const bool vis = qp[i] >= 0 && key <= qp[i] && (window <= 0 || qp[i] - key < window);
                Ps[(8 * rg + i) * LP + kg + 16 * j] = vis ? sc[i][j] : -INFINITY;
            }
        __syncthreads();
        {   // online softmax: two threads per row, 32 keys each
            const int row = tid >> 1, half = tid & 1;
            float *pr = Ps + row * LP + 32 * half;
            float mx = -INFINITY;
#pragma unroll 8
            for (int c = 0; c < 32; c++) mx = fmaxf(mx, pr[c]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            const float mold = rm[row], mnew = fmaxf(mold, mx);
            float alpha = 1.f, sum = 0.f;
            if (mnew != -INFINITY) {
                alpha = expf(mold - mnew);   // 0 while nothing was visible before
#pragma unroll 8
                for (int c = 0; c < 32; c++) {
                    const float e = expf(pr[c] - mnew);   // masked keys: exp(-inf) = 0
                    pr[c] = e;
                    sum += e;
                }
            } else {   // nothing visible so far: adds nothing
#pragma unroll 8
                for (int c = 0; c < 32; c++) pr[c] = 0.f;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            if (half == 0) {
                rm[row] = mnew;
                rl[row] = rl[row] * alpha + sum;
                ra[row] = alpha;
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float a = ra[8 * rg + i];
#pragma unroll
            for (int c = 0; c < 4 * DV; c++) o[i][c] *= a;
        }
#pragma unroll 2
        for (int j = 0; j < FA_BK; j += 4) {
            float4 pp[8];
#pragma unroll
            for (int i = 0; i < 8; i++) pp[i] = *reinterpret_cast<const float4 *>(Ps + (8 * rg + i) * LP + j);
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                float4 v[DV];
#pragma unroll
                for (int u = 0; u < DV; u++) v[u] = *reinterpret_cast<const float4 *>(Vs + (j + jj) * LD + 64 * u + 4 * kg);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float pv = jj == 0 ? pp[i].x : jj == 1 ? pp[i].y : jj == 2 ? pp[i].z : pp[i].w;
#pragma unroll
                    for (int u = 0; u < DV; u++) {
                        o[i][4 * u] = fmaf(pv, v[u].x, o[i][4 * u]);
                        o[i][4 * u + 1] = fmaf(pv, v[u].y, o[i][4 * u + 1]);
                        o[i][4 * u + 2] = fmaf(pv, v[u].z, o[i][4 * u + 2]);
                        o[i][4 * u + 3] = fmaf(pv, v[u].w, o[i][4 * u + 3]);
                    }
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int row = 8 * rg + i, tq = t0 + row % BQ, h = kvh * G + row / BQ;
        if (tq >= tokens) continue;
        const float l = rl[row];
        float f = l > 0.f ? 1.f / l : 0.f;
        const int64_t r = (int64_t)sq * tokens + tq;
        if (gate) f = f / (1.0f + expf(-gate[r * H + h]));
#pragma unroll
        for (int u = 0; u < DV; u++) {
            const float4 w = make_float4(o[i][4 * u] * f, o[i][4 * u + 1] * f, o[i][4 * u + 2] * f, o[i][4 * u + 3] * f);
            *reinterpret_cast<float4 *>(out + (r * H + h) * D + 64 * u + 4 * kg) = w;
        }
    }
}

// Decode attention split over the keys (one new token per row), in the
// manner of flash decoding: CTA = (key range `split` of cpc * AK keys, cache
// head kvh, row r) for all G = H / KVH query heads that share the cache head,
// AW warps, each on its own groups of KG keys of the range (groups w, w + AW,
// ...) with no CTA barrier until the end. A warp streams its groups' k and v
// rows into its own NB shared-memory slots (asynchronous 16-byte copies, NB - 1
// groups in flight). Per group: each lane takes E = D / 32 dimensions of the
// KG keys x G heads dot products, the KG * G partial sums are reduced over the
// lanes by one transposing butterfly (after it lane L holds the score of key
// (L % V) / G, head L % G, V = KG * G); the warp's running max m and sum l of
// exp(s - m) per head (online softmax) and, each lane for its dimensions, the
// running unnormalised sum of exp(s - m) * v, rescaled by exp(m_old - m_new).
// At the end the AW warps' (sum, m, l) are merged in warp order and the
// range's go to `part`; ef_attn_combine_kernel merges the ranges. Same masking
// and scale as ef_attention_kernel.
constexpr int AK = 32;         // keys per range unit (a range is cpc units)
constexpr int AW = 4;          // warps per CTA
constexpr int AT = AW * 32;    // threads per CTA
constexpr int ANB = 3;         // shared-memory slots per warp (groups in flight + 1)
template <int G> constexpr int akg() { return G >= 4 ? 32 / G : 8; }   // keys per group

// v[i] summed over the 32 lanes; afterwards lane L holds, in v[0], the sum of
// index L % V (plain butterfly over the lane bits >= log2(V), then a
// transposing one over the lower bits).
template <int V>
__device__ __forceinline__ void xreduce(float (&v)[V], int lane) {
#pragma unroll
    for (int s = 16; s >= V; s >>= 1)
#pragma unroll
        for (int i = 0; i < V; i++) v[i] += __shfl_xor_sync(0xffffffffu, v[i], s);
#pragma unroll
    for (int s = V / 2; s >= 1; s >>= 1) {
        const bool up = lane & s;
#pragma unroll
        for (int i = 0; i < s; i++) {
            const float send = up ? v[i] : v[i + s], keep = up ? v[i + s] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
    }
}

template <int D, int G, typename KV>
__global__ void __launch_bounds__(AT) ef_attn_part_kernel(const float *__restrict__ q, const KV *__restrict__ kcache,
                                                       const KV *__restrict__ vcache, const int *__restrict__ pos,
                                                       int tokens, int max_pos, int window, int H, int KVH, int cpc,
                                                       float *__restrict__ part) {
    pdl_trigger();
    pdl_wait();
    constexpr int KG = akg<G>(), V = KG * G, E = D / 32;
    extern __shared__ __align__(16) uint8_t kv_raw[];   // per warp: k [ANB][KG][D], then v [ANB][KG][D]
    __shared__ float wm[AW][G], wl[AW][G];
    __shared__ __align__(16) float wacc[AW][G][D];
    const int split = blockIdx.x, kvh = blockIdx.y, r = blockIdx.z, nsplit = gridDim.x;
    const int sq = r / tokens, t = r - sq * tokens;
    const int nkv = min(pos[sq] + t + 1, max_pos), qpos = nkv - 1;
    const int k0 = window > 0 && qpos - window + 1 > 0 ? qpos - window + 1 : 0;
    const int a = k0 + split * cpc * AK, b = min(nkv, a + cpc * AK);
    float *pr = part + (((int64_t)r * H + kvh * G) * nsplit + split) * (D + 2);   // head g at + g * nsplit * (D+2)
    if (a >= b) {                    // an empty range: weight 0 in the merge
        for (int i = threadIdx.x; i < G * (D + 2); i += AT) {
            const int g = i / (D + 2), c = i - g * (D + 2);
            pr[(int64_t)g * nsplit * (D + 2) + c] = c == D ? -1e30f : 0.f;
        }
        return;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    KV *ks = reinterpret_cast<KV *>(kv_raw) + (size_t)warp * 2 * ANB * KG * D, *vs = ks + ANB * KG * D;
    const KV *kb = kcache + (((int64_t)sq * max_pos + a) * KVH + kvh) * D;
    const KV *vb = vcache + (((int64_t)sq * max_pos + a) * KVH + kvh) * D;
    const int ngroups = (b - a + KG - 1) / KG;
    const int mine = ngroups > warp ? (ngroups - warp + AW - 1) / AW : 0;   // this warp's groups
    auto issue = [&](int t) {        // this warp's t-th group -> slot t % ANB (an empty commit past the end)
        if (t < mine) {
            constexpr int EP = 16 / sizeof(KV), C = D / EP;   // elements per 16-byte piece, pieces per row
            const int j0 = (warp + AW * t) * KG, n = min(KG, b - a - j0);
            KV *kd = ks + (t % ANB) * KG * D, *vd = vs + (t % ANB) * KG * D;
            for (int i = lane; i < n * C; i += 32) {
                const int j = i / C, cc = i - j * C;
                cp_async16(kd + j * D + EP * cc, kb + (int64_t)(j0 + j) * KVH * D + EP * cc);
                cp_async16(vd + j * D + EP * cc, vb + (int64_t)(j0 + j) * KVH * D + EP * cc);
            }
        }
        cp_commit();
    };
#pragma unroll
    for (int t0 = 0; t0 < ANB - 1; t0++) issue(t0);
    float qv[G][E];
    const float qscale = rsqrtf((float)D);
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < E; e++) qv[g][e] = q[((int64_t)r * H + kvh * G + g) * D + lane * E + e] * qscale;
    const int mg = lane % G;         // the head whose running max / sum this lane keeps
    float m = -INFINITY, l = 0.f;
    float acc[G][E];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < E; e++) acc[g][e] = 0.f;
    for (int t = 0; t < mine; t++) {
        issue(t + ANB - 1);
        cp_wait<ANB - 1>();
        __syncwarp();
        const int n = min(KG, b - a - (warp + AW * t) * KG);
        const KV *kg = ks + (t % ANB) * KG * D, *vg = vs + (t % ANB) * KG * D;
        // partial scores of the KG keys x G heads over this lane's dimensions
        float sv[V];
#pragma unroll
        for (int j = 0; j < KG; j++) {
            float kr[E];
            if (j < n) {
                if constexpr (E == 4) {
                    const float4 v4 = kv_ld4(kg + j * D + lane * 4);
                    kr[0] = v4.x; kr[1] = v4.y; kr[2] = v4.z; kr[3] = v4.w;
                } else {
                    const float2 v2 = kv_ld2(kg + j * D + lane * 2);
                    kr[0] = v2.x; kr[1] = v2.y;
                }
            } else {
#pragma unroll
                for (int e = 0; e < E; e++) kr[e] = 0.f;
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
                float s = 0.f;
#pragma unroll
                for (int e = 0; e < E; e++) s += qv[g][e] * kr[e];
                sv[j * G + g] = s;
            }
        }
        xreduce<V>(sv, lane);
        const int ji = (lane % V) / G;                // this lane's key of the group
        const float sc = ji < n ? sv[0] : -INFINITY;
        // online softmax per head over the group's keys (lanes of one head differ in bits log2 G .. log2 V - 1)
        float gm = sc;
#pragma unroll
        for (int s = G; s < V; s <<= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, s));
        const float mnew = fmaxf(m, gm);
        const float p = ji < n ? expf(sc - mnew) : 0.f;
        float ps = p;
#pragma unroll
        for (int s = G; s < V; s <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, s);
        const float alpha = expf(m - mnew);           // 0 for the first group (m = -inf)
        m = mnew;
        l = l * alpha + ps;
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float ag = __shfl_sync(0xffffffffu, alpha, g);
#pragma unroll
            for (int e = 0; e < E; e++) acc[g][e] *= ag;
        }
#pragma unroll
        for (int j = 0; j < KG; j++) {
            if (j < n) {
                float vr[E];
                if constexpr (E == 4) {
                    const float4 v4 = kv_ld4(vg + j * D + lane * 4);
                    vr[0] = v4.x; vr[1] = v4.y; vr[2] = v4.z; vr[3] = v4.w;
                } else {
                    const float2 v2 = kv_ld2(vg + j * D + lane * 2);
                    vr[0] = v2.x; vr[1] = v2.y;
                }
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const float pg = __shfl_sync(0xffffffffu, p, j * G + g);
#pragma unroll
                    for (int e = 0; e < E; e++) acc[g][e] += pg * vr[e];
                }
            }
        }
        __syncwarp();                // the slot is reissued ANB - 1 groups later
    }
    cp_wait<0>();
    // merge the warps, in warp order
    if (lane < G) {
        wm[warp][lane] = m;          // (lane < G: mg == lane)
        wl[warp][lane] = l;
    }
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < E; e++) wacc[warp][g][lane * E + e] = acc[g][e];
    (void)mg;
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += AT) {
        const int g = i / D, d = i - g * D;
        float M = wm[0][g];
#pragma unroll
        for (int w = 1; w < AW; w++) M = fmaxf(M, wm[w][g]);
        float o = 0.f, L = 0.f;
#pragma unroll
        for (int w = 0; w < AW; w++) {
            const float f = expf(wm[w][g] - M);       // 0 for a warp without keys (m = -inf)
            o += f * wacc[w][g][d];
            L += f * wl[w][g];
        }
        float *op = pr + (int64_t)g * nsplit * (D + 2);
        op[d] = o;
        if (d == 0) {
            op[D] = M;
            op[D + 1] = L;
        }
    }
}

// The same split with f16 caches and up to 4 query heads per cache head, on
// the tensor cores (mma.sync m16n8k16, f16 operands, f32 accumulate). Each
// warp takes groups of 16 keys. Scores: S[key][col] = K[key][:] . Q'[:][col],
// K from shared memory by ldmatrix, Q' the G query heads (pre-scaled by
// 1/sqrt(D)) each split into two f16 columns, hi = f16(q) and lo = f16(q - hi),
// so that hi + lo carries q to about 22 bits and the f32 sum of the exact
// f16 x f16 products keeps f32 accuracy; score = S[.][2h] + S[.][2h+1].
// Online softmax per head as in the kernel above (lane (g, t) holds keys g
// and g + 8 of head t). Values: out^T[d][col] += V^T[d][key] . P'[key][col],
// V^T by ldmatrix.trans, P' the probabilities split the same way (gathered
// from their lanes by shuffles), out = out^T[.][2h] + out^T[.][2h+1]. K and V
// rows sit in shared memory with 16 bytes of padding per row (the 8 rows of
// an ldmatrix read fall in different banks).
constexpr int AHK = 16;        // keys per group (one MMA row tile)
constexpr int AHNB = 3;        // shared-memory slots per warp

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
// (hi, lo) f16 split of v, packed as the pair (first, second) of a b16x2 register half
__device__ __forceinline__ __half split_part(float v, int lo) {
    const __half h = __float2half_rn(v);
    return lo ? __float2half_rn(v - __half2float(h)) : h;
}
__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

template <int D, int G>
__global__ void __launch_bounds__(AT) ef_attn_part_h_kernel(const float *__restrict__ q,
                                                         const __half *__restrict__ kcache,
                                                         const __half *__restrict__ vcache,
                                                         const int *__restrict__ pos, int tokens, int max_pos,
                                                         int window, int H, int KVH, int cpc,
                                                         float *__restrict__ part) {
    static_assert(G <= 4, "two f16 columns per query head, 8 columns per MMA");
    pdl_trigger();
    pdl_wait();
    constexpr int LD = D + 8;        // padded row (halves)
    constexpr int KS = D / 16;       // MMA k-steps of the scores, m-tiles of the values
    extern __shared__ __align__(16) uint8_t kv_raw[];   // per warp: k [AHNB][AHK][LD], then v [AHNB][AHK][LD]
    __shared__ float wm[AW][G], wl[AW][G];
    __shared__ __align__(16) float wacc[AW][G][D];
    const int split = blockIdx.x, kvh = blockIdx.y, r = blockIdx.z, nsplit = gridDim.x;
    const int sq = r / tokens, t0k = r - sq * tokens;
    const int nkv = min(pos[sq] + t0k + 1, max_pos), qpos = nkv - 1;
    const int k0 = window > 0 && qpos - window + 1 > 0 ? qpos - window + 1 : 0;
    const int a = k0 + split * cpc * AK, b = min(nkv, a + cpc * AK);
    float *pr = part + (((int64_t)r * H + kvh * G) * nsplit + split) * (D + 2);
    if (a >= b) {
        for (int i = threadIdx.x; i < G * (D + 2); i += AT) {
            const int g = i / (D + 2), c = i - g * (D + 2);
            pr[(int64_t)g * nsplit * (D + 2) + c] = c == D ? -1e30f : 0.f;
        }
        return;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    __half *ks = reinterpret_cast<__half *>(kv_raw) + (size_t)warp * 2 * AHNB * AHK * LD, *vs = ks + AHNB * AHK * LD;
    const __half *kb = kcache + (((int64_t)sq * max_pos + a) * KVH + kvh) * D;
    const __half *vb = vcache + (((int64_t)sq * max_pos + a) * KVH + kvh) * D;
    const int ngroups = (b - a + AHK - 1) / AHK;
    const int mine = ngroups > warp ? (ngroups - warp + AW - 1) / AW : 0;
    auto issue = [&](int it) {
        if (it < mine) {
            constexpr int C = D / 8;     // 16-byte pieces per row
            const int j0 = (warp + AW * it) * AHK, n = min(AHK, b - a - j0);
            __half *kd = ks + (it % AHNB) * AHK * LD, *vd = vs + (it % AHNB) * AHK * LD;
            for (int i = lane; i < n * C; i += 32) {
                const int j = i / C, cc = i - j * C;
                cp_async16(kd + j * LD + 8 * cc, kb + (int64_t)(j0 + j) * KVH * D + 8 * cc);
                cp_async16(vd + j * LD + 8 * cc, vb + (int64_t)(j0 + j) * KVH * D + 8 * cc);
            }
        }
        cp_commit();
    };
#pragma unroll
    for (int i = 0; i < AHNB - 1; i++) issue(i);
    // B fragments of Q' for the KS k-steps: column g = head g / 2, part g % 2
    uint32_t qb[KS][2];
    {
        const int hg = g >> 1, lo = g & 1;
        const float qscale = rsqrtf((float)D);
        const float *qh = q + ((int64_t)r * H + kvh * G + (hg < G ? hg : 0)) * D;
#pragma unroll
        for (int s = 0; s < KS; s++) {
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (hg < G) {
                v[0] = qh[s * 16 + 2 * t] * qscale;
                v[1] = qh[s * 16 + 2 * t + 1] * qscale;
                v[2] = qh[s * 16 + 2 * t + 8] * qscale;
                v[3] = qh[s * 16 + 2 * t + 9] * qscale;
            }
            qb[s][0] = pack_h2(split_part(v[0], lo), split_part(v[1], lo));
            qb[s][1] = pack_h2(split_part(v[2], lo), split_part(v[3], lo));
        }
    }
    const bool head = t < G;         // this lane's softmax head is t
    float m = -INFINITY, l = 0.f;
    float acc[KS][4];
#pragma unroll
    for (int i = 0; i < KS; i++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[i][e] = 0.f;
    const int lr = (lane & 7) + ((lane >> 3) & 1) * 8, lc = (lane >> 4) * 8;   // ldmatrix A rows / cols
    const int vk = (lane & 7) + (lane >> 4) * 8, vd = ((lane >> 3) & 1) * 8;   // ldmatrix.trans: key / dim
    for (int it = 0; it < mine; it++) {
        issue(it + AHNB - 1);
        cp_wait<AHNB - 1>();
        __syncwarp();
        const int n = min(AHK, b - a - (warp + AW * it) * AHK);
        const __half *kg = ks + (it % AHNB) * AHK * LD, *vg = vs + (it % AHNB) * AHK * LD;
        // scores
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < KS; s++) {
            uint32_t af[4];
            ldsm_x4(af, kg + lr * LD + s * 16 + lc);
            mma_f16_16816(sc, af[0], af[1], af[2], af[3], qb[s][0], qb[s][1]);
        }
        // lane (g, t): keys g and g + 8 of head t (columns 2t, 2t + 1); keys past n masked
        // (their rows in shared memory are stale or unset: their scores are never used)
        const float s0 = head && g < n ? sc[0] + sc[1] : -INFINITY;
        const float s1 = head && g + 8 < n ? sc[2] + sc[3] : -INFINITY;
        float gm = fmaxf(s0, s1);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
        const float mnew = head ? fmaxf(m, gm) : 0.f;
        const float p0 = head && g < n ? expf(s0 - mnew) : 0.f;
        const float p1 = head && g + 8 < n ? expf(s1 - mnew) : 0.f;
        float ps = p0 + p1;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        const float alpha = head ? expf(m - mnew) : 1.f;   // 0 for the first group (m = -inf)
        if (head) {
            m = mnew;
            l = l * alpha + ps;
        }
        // P' B fragment: rows (keys) 2t, 2t+1, 2t+8, 2t+9 of column g (head g / 2, part g % 2)
        const int hg = g >> 1, lo = g & 1;
        const float q0 = __shfl_sync(0xffffffffu, p0, 8 * t + hg), q1 = __shfl_sync(0xffffffffu, p0, 8 * t + 4 + hg);
        const float q2 = __shfl_sync(0xffffffffu, p1, 8 * t + hg), q3 = __shfl_sync(0xffffffffu, p1, 8 * t + 4 + hg);
        const uint32_t pb0 = hg < G ? pack_h2(split_part(q0, lo), split_part(q1, lo)) : 0u;
        const uint32_t pb1 = hg < G ? pack_h2(split_part(q2, lo), split_part(q3, lo)) : 0u;
        // values: rescale, then add V^T P' (keys past n have p = 0; their V rows are
        // zero-filled below so that stale data cannot be Inf or NaN)
        if (n < AHK) {
            __half *vw = const_cast<__half *>(vg);
            for (int i = lane; i < (AHK - n) * (D / 2); i += 32) {
                const int j = n + i / (D / 2), c = i - (j - n) * (D / 2);
                reinterpret_cast<uint32_t *>(vw + j * LD)[c] = 0u;
            }
            __syncwarp();
        }
#pragma unroll
        for (int i = 0; i < KS; i++) {
            acc[i][0] *= alpha;
            acc[i][1] *= alpha;
            acc[i][2] *= alpha;
            acc[i][3] *= alpha;
            uint32_t af[4];
            ldsm_x4_t(af, vg + vk * LD + i * 16 + vd);
            mma_f16_16816(acc[i], af[0], af[1], af[2], af[3], pb0, pb1);
        }
        __syncwarp();                // the slot is reissued AHNB - 1 groups later
    }
    cp_wait<0>();
    // merge the warps, in warp order: lane (g, t) holds out[16 i + g] and out[16 i + g + 8] of head t
    if (head && g == 0) {
        wm[warp][t] = m;
        wl[warp][t] = l;
    }
    if (head)
#pragma unroll
        for (int i = 0; i < KS; i++) {
            wacc[warp][t][16 * i + g] = acc[i][0] + acc[i][1];
            wacc[warp][t][16 * i + g + 8] = acc[i][2] + acc[i][3];
        }
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += AT) {
        const int h = i / D, d = i - h * D;
        float M = wm[0][h];
#pragma unroll
        for (int w = 1; w < AW; w++) M = fmaxf(M, wm[w][h]);
        float o = 0.f, L = 0.f;
#pragma unroll
        for (int w = 0; w < AW; w++) {
            const float f = expf(wm[w][h] - M);
            o += f * wacc[w][h][d];
            L += f * wl[w][h];
        }
        float *op = pr + (int64_t)h * nsplit * (D + 2);
        op[d] = o;
        if (d == 0) {
            op[D] = M;
            op[D + 1] = L;
        }
    }
}

// out[r][h] = sum over ranges of exp(m_s - M) acc_s / sum of exp(m_s - M) l_s
// (M = the largest m_s); times sigmoid(gate[r][h]) when given. CTA (head,
// row) of CT threads = CT / D groups of ranges x D dimensions: the ranges'
// weights first, then each thread its dimension over its group's ranges
// (many loads in flight), then the groups added in order.
constexpr int CT = 512;

template <int D>
__global__ void __launch_bounds__(CT) ef_attn_combine_kernel(const float *__restrict__ part,
                                                          const float *__restrict__ gate, int H, int nsplit,
                                                          float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float wgt[];   // [nsplit]
    __shared__ float red[CT / 32];
    __shared__ float sums[CT / D][D + 1];
    constexpr int SG = CT / D;
    const int h = blockIdx.x, r = blockIdx.y;
    const float *pr = part + ((int64_t)r * H + h) * nsplit * (D + 2);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float M = -1e30f;
    for (int s = threadIdx.x; s < nsplit; s += CT) M = fmaxf(M, pr[(int64_t)s * (D + 2) + D]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (lane == 0) red[warp] = M;
    __syncthreads();
    M = red[0];
#pragma unroll
    for (int w = 1; w < CT / 32; w++) M = fmaxf(M, red[w]);
    for (int s = threadIdx.x; s < nsplit; s += CT) wgt[s] = expf(pr[(int64_t)s * (D + 2) + D] - M);
    __syncthreads();
    const int d = threadIdx.x % D, sg = threadIdx.x / D;
    float acc = 0.f, L = 0.f;
#pragma unroll 8
    for (int s = sg; s < nsplit; s += SG) {
        const float w = wgt[s];
        acc += w * pr[(int64_t)s * (D + 2) + d];
        L += w * pr[(int64_t)s * (D + 2) + D + 1];
    }
    sums[sg][d] = acc;
    if (d == 0) sums[sg][D] = L;
    __syncthreads();
    if (sg == 0) {
        float o = 0.f, ll = 0.f;
#pragma unroll
        for (int g = 0; g < SG; g++) {
            o += sums[g][d];
            ll += sums[g][D];
        }
        o /= ll;
        if (gate) o = o / (1.0f + expf(-gate[(int64_t)r * H + h]));
        out[((int64_t)r * H + h) * D + d] = o;
    }
}

// ---------------------------------------------------------------- top-k ---
// The m first logits of a row in the sampler's order -- larger value first,
// the lower index first among equal values (kernels.topk.wgsl.js:3-36,
// topk.js) -- exactly, as 64-bit keys (value key << 32 | ~index) sorted in
// shared memory: each CTA sorts one chunk of TK_CHUNK logits and keeps its m
// first (every element of the row's top m is in its chunk's top m), one CTA
// per row sorts the union. The value key orders f32 bits as numbers with -0
// equal to +0; NaN logits set flag 2 for the row (their order cannot be
// reproduced, kernels.topk.wgsl.js:18-36).
constexpr int TK_CHUNK = 4096;

__device__ __forceinline__ uint32_t order_key(uint32_t bits) {
    const uint32_t b = bits == 0x80000000u ? 0u : bits;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// descending bitonic sort of n (a power of two) keys in shared memory
__device__ void bitonic_desc(unsigned long long *a, int n) {
    for (int k = 2; k <= n; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const unsigned long long x = a[i], y = a[l];
                    const bool desc = (i & k) == 0;
                    if (desc ? x < y : x > y) {
                        a[i] = y;
                        a[l] = x;
                    }
                }
            }
        }
    __syncthreads();
}

__global__ void __launch_bounds__(512) ef_topk_chunk_kernel(const float *__restrict__ logits, int n, int m,
                                                         unsigned long long *__restrict__ cand,
                                                         int *__restrict__ flags) {
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long a[TK_CHUNK];
    __shared__ int nan_seen;
    const int chunk = blockIdx.x, row = blockIdx.y, nch = gridDim.x;
    const uint32_t *lr = reinterpret_cast<const uint32_t *>(logits + (int64_t)row * n);
    if (threadIdx.x == 0) nan_seen = 0;
    __syncthreads();
    bool nan = false;
    for (int i = threadIdx.x; i < TK_CHUNK; i += blockDim.x) {
        const int idx = chunk * TK_CHUNK + i;
        unsigned long long v = 0;                     // padding: below every logit
        if (idx < n) {
            const uint32_t bits = lr[idx];
            nan |= (bits & 0x7fffffffu) > 0x7f800000u;
            v = ((unsigned long long)order_key(bits) << 32) | (uint32_t)~(uint32_t)idx;
        }
        a[i] = v;
    }
    if (nan) atomicOr(&nan_seen, 1);
    bitonic_desc(a, TK_CHUNK);
    unsigned long long *out = cand + ((int64_t)row * nch + chunk) * m;
    for (int i = threadIdx.x; i < m; i += blockDim.x) out[i] = a[i];
    if (threadIdx.x == 0 && nan_seen) atomicOr(flags + row, 2);
}

__global__ void __launch_bounds__(1024) ef_topk_final_kernel(const float *__restrict__ logits, int n, int m, int nch,
                                                          int sort_n, const unsigned long long *__restrict__ cand,
                                                          int *__restrict__ ids, float *__restrict__ vals) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ unsigned long long u[];
    const int row = blockIdx.x;
    const unsigned long long *c = cand + (int64_t)row * nch * m;
    for (int i = threadIdx.x; i < sort_n; i += blockDim.x) u[i] = i < nch * m ? c[i] : 0ull;
    bitonic_desc(u, sort_n);
    const int cnt = m < n ? m : n;
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
        int id = -1;
        float v = 0.f;
        if (i < cnt) {
            id = (int)~(uint32_t)(u[i] & 0xffffffffull);
            v = logits[(int64_t)row * n + id];          // the logit's own bits
        }
        ids[(int64_t)row * m + i] = id;
        vals[(int64_t)row * m + i] = v;
    }
}

// out = g * sigmoid(g) * u, elementwise (kernels.nn.wgsl.js swiglu; the same
// expression as the fused SwiGLU GEMV's epilogue).
__global__ void ef_swiglu_kernel(const float *__restrict__ g, const float *__restrict__ u, int64_t n,
                              float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float a = g[i];
        out[i] = a / (1.0f + expf(-a)) * u[i];
    }
}

// The step's token: writes it, records it in out_tokens[*pos + 1 - out_base]
// when that index is in [0, out_cap), and advances *pos.
__device__ __forceinline__ void finish_step(int tok, int *token, int *pos, int *out_tokens, int out_base,
                                            int out_cap) {
    *token = tok;
    const int np = *pos + 1;
    const int slot = np - out_base;
    if (out_tokens && slot >= 0 && slot < out_cap) out_tokens[slot] = tok;
    *pos = np;
}

// Greedy argmax over the n logits of row blockIdx.x (strict '>': lowest index
// wins ties). PAIR = false: finish_step with the winner (token, pos and
// out_tokens of that row). PAIR = true (one vocabulary shard of a
// tensor-parallel head): the row's pair[0] = the best value's bits, pair[1] =
// its index + offset, for argmax_select over the shards.
template <bool PAIR>
__global__ void __launch_bounds__(1024) ef_argmax_kernel(const float *__restrict__ logits, int n,
                                                      int *__restrict__ token, int *__restrict__ pos,
                                                      int *__restrict__ out_tokens, int out_base, int out_cap,
                                                      int offset, int *__restrict__ pair) {
    pdl_trigger();
    pdl_wait();
    logits += (int64_t)blockIdx.x * n;
    if (PAIR) {
        pair += 2 * blockIdx.x;
    } else {
        token += blockIdx.x;
        pos += blockIdx.x;
        if (out_tokens) out_tokens += (int64_t)blockIdx.x * out_cap;
    }
    __shared__ float bv[32];
    __shared__ int bi[32];
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    // float4 of each thread in order, 8 loads in flight; then the scalar tail
    const int n4 = n / 4;
    const float4 *l4 = reinterpret_cast<const float4 *>(logits);
    for (int base = 0; base < n4; base += 8 * blockDim.x) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = base + u * blockDim.x + threadIdx.x;
            v[u] = i < n4 ? l4[i] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i4 = 4 * (base + u * blockDim.x + threadIdx.x);
            const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
            for (int c = 0; c < 4; c++)
                if (e[c] > best || (e[c] == best && i4 + c < bidx)) {
                    best = e[c];
                    bidx = i4 + c;
                }
        }
    }
    for (int i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) {
        const float v = logits[i];
        if (v > best || (v == best && i < bidx)) {
            best = v;
            bidx = i;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (ov > best || (ov == best && oi < bidx)) {
            best = ov;
            bidx = oi;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = bidx;
    }
    __syncthreads();
    if (warp == 0) {
        best = lane < nw ? bv[lane] : -INFINITY;
        bidx = lane < nw ? bi[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
            if (ov > best || (ov == best && oi < bidx)) {
                best = ov;
                bidx = oi;
            }
        }
        if (lane == 0) {
            if (PAIR) {
                pair[0] = __float_as_int(best);
                pair[1] = bidx + offset;
            } else {
                finish_step(bidx, token, pos, out_tokens, out_base, out_cap);
            }
        }
    }
}

// Row blockIdx.x: the winner over the shards' (value, index) pairs (pairs
// [nranks][rows][2]), in the same order as one argmax over the whole
// vocabulary: larger value, then lower index.
__global__ void ef_argmax_select_kernel(const int *__restrict__ pairs, int npairs, int *__restrict__ token,
                                     int *__restrict__ pos, int *__restrict__ out_tokens, int out_base,
                                     int out_cap) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x, rows = gridDim.x;
    token += row;
    pos += row;
    if (out_tokens) out_tokens += (int64_t)row * out_cap;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    for (int i = threadIdx.x; i < npairs; i += 32) {
        const float v = __int_as_float(pairs[2 * (i * rows + row)]);
        const int ix = pairs[2 * (i * rows + row) + 1];
        if (v > best || (v == best && ix < bidx)) {
            best = v;
            bidx = ix;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (ov > best || (ov == best && oi < bidx)) {
            best = ov;
            bidx = oi;
        }
    }
    if (threadIdx.x == 0) finish_step(bidx, token, pos, out_tokens, out_base, out_cap);
}

static int grid1d(int64_t n, int b) { return (int)((n + b - 1) / b); }

template <int D, int G>
static int part_h_launch(ef_ctx *ctx, dim3 grid, const float *q, const __half *kcache, const __half *vcache,
                         const int *pos, int tokens, int max_pos, int window, int heads, int kv_heads, int cpc,
                         float *part) {
    constexpr size_t smem = (size_t)AW * 2 * AHNB * AHK * (D + 8) * sizeof(__half);
    static std::atomic<unsigned long long> configured{0};   // per instantiation, one bit per device
    if (ctx->device < 64 && !(configured.load() & (1ull << ctx->device))) {
        if (int rc = check_cuda(ctx, cudaFuncSetAttribute(ef_attn_part_h_kernel<D, G>,
                                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                "attention smem attribute"))
            return rc;
        configured.fetch_or(1ull << ctx->device);
    }
    return launch_on(ctx, ef_attn_part_h_kernel<D, G>, grid, AT, smem, "attention launch", q, kcache, vcache, pos,
                     tokens, max_pos, window, heads, kv_heads, cpc, part);
}

template <int D, int G, typename KV>
static int part_launch(ef_ctx *ctx, dim3 grid, const float *q, const KV *kcache, const KV *vcache, const int *pos,
                       int tokens, int max_pos, int window, int heads, int kv_heads, int cpc, float *part) {
    if constexpr (std::is_same<KV, __half>::value && G <= 4)   // f16 caches: the tensor-core version
        return part_h_launch<D, G>(ctx, grid, q, kcache, vcache, pos, tokens, max_pos, window, heads, kv_heads, cpc,
                                   part);
    constexpr size_t smem = (size_t)AW * 2 * ANB * akg<G>() * D * sizeof(KV);
    static std::atomic<unsigned long long> configured{0};   // per instantiation, one bit per device
    if (ctx->device < 64 && !(configured.load() & (1ull << ctx->device))) {
        if (int rc = check_cuda(ctx, cudaFuncSetAttribute(ef_attn_part_kernel<D, G, KV>,
                                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                "attention smem attribute"))
            return rc;
        configured.fetch_or(1ull << ctx->device);
    }
    return launch_on(ctx, ef_attn_part_kernel<D, G, KV>, grid, AT, smem, "attention launch", q, kcache, vcache, pos,
                     tokens, max_pos, window, heads, kv_heads, cpc, part);
}

template <int D, int G, typename KV>
static int prompt_attn_launch(ef_ctx *ctx, int seqs, const float *q, const KV *kcache, const KV *vcache,
                              const float *gate, const int *pos, int tokens, int max_pos, int window, int heads,
                              int kv_heads, float *out) {
    constexpr size_t smem = fa_smem<D>();
    static std::atomic<unsigned long long> configured{0};   // per instantiation, one bit per device
    if (ctx->device < 64 && !(configured.load() & (1ull << ctx->device))) {
        if (int rc = check_cuda(ctx, cudaFuncSetAttribute(ef_attn_prompt_kernel<D, G, KV>,
                                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                "prompt attention smem attribute"))
            return rc;
        configured.fetch_or(1ull << ctx->device);
    }
    const dim3 grid((unsigned)((tokens + FA_R / G - 1) / (FA_R / G)), (unsigned)kv_heads, (unsigned)seqs);
    return launch_on(ctx, ef_attn_prompt_kernel<D, G, KV>, grid, FA_T, smem, "prompt attention launch", q, kcache,
                     vcache, gate, pos, tokens, max_pos, window, heads, kv_heads, out);
}

template <typename KV>
static int rope_launch(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                       const int *pos, int seqs, int tokens, int max_pos, int heads, int kv_heads, int head_dim,
                       int neox, float theta_base, float eps, KV *kcache, KV *vcache) {
    const float theta_scale = powf(theta_base, -2.0f / (float)head_dim);
    const int64_t warps = (int64_t)seqs * tokens * (heads + kv_heads);
    const int grid = (int)((warps + 7) / 8);
#define EF_ROPE(DD, NX)                                                                                          \
    return launch_on(ctx, ef_rope_cache_kernel<DD, NX, KV>, grid, 256, 0, "rope_cache launch", q, k, v, wq, wk, pos, \
                     seqs, tokens, max_pos, heads, kv_heads, theta_scale, eps, kcache, vcache)
    if (head_dim == 64) {
        if (neox) EF_ROPE(64, true);
        EF_ROPE(64, false);
    }
    if (neox) EF_ROPE(128, true);
    EF_ROPE(128, false);
#undef EF_ROPE
}

template <typename KV>
static int qk_norm_rope_cache(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                              const int *pos, int max_pos, int heads, int kv_heads, int head_dim, float theta_base,
                              float eps, KV *kcache, KV *vcache) {
    if (!ctx || !q || !k || !v || !wq || !wk || !pos || !kcache || !vcache || heads < 1 || kv_heads < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "qk_norm_rope_cache: bad arguments") : EF_ERR_INVALID;
    if (head_dim != 64) return set_err(ctx, EF_ERR_SHAPE, "qk_norm_rope_cache: head_dim %d (64 supported)", head_dim);
    return rope_launch(ctx, q, k, v, wq, wk, pos, 1, 1, max_pos, heads, kv_heads, 64, 1, theta_base, eps, kcache,
                       vcache);
}

template <typename KV>
static int rope_cache(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                      const int *pos, int seqs, int tokens, int max_pos, int heads, int kv_heads, int head_dim,
                      int rope_mode, float theta_base, float eps, KV *kcache, KV *vcache) {
    if (!ctx || !q || !k || !v || !pos || !kcache || !vcache || heads < 1 || kv_heads < 1 || seqs < 1 ||
        tokens < 1 || max_pos < 1 || (!wq) != (!wk))
        return ctx ? set_err(ctx, EF_ERR_INVALID, "rope_cache: bad arguments") : EF_ERR_INVALID;
    if (head_dim != 64 && head_dim != 128)
        return set_err(ctx, EF_ERR_SHAPE, "rope_cache: head_dim %d (64 or 128 supported)", head_dim);
    if (rope_mode != EF_ROPE_NORM && rope_mode != EF_ROPE_NEOX)
        return set_err(ctx, EF_ERR_INVALID, "rope_cache: unknown RoPE mode %d", rope_mode);
    if ((int64_t)seqs * tokens > 65535) return set_err(ctx, EF_ERR_RANGE, "rope_cache: more than 65535 rows");
    return rope_launch(ctx, q, k, v, wq, wk, pos, seqs, tokens, max_pos, heads, kv_heads, head_dim,
                       rope_mode == EF_ROPE_NEOX, theta_base, eps, kcache, vcache);
}

template <typename KV>
static int attention_launch(ef_ctx *ctx, const float *q, const KV *kcache, const KV *vcache,
                            const float *head_gate, const int *pos, int seqs, int tokens, int max_pos, int window,
                            int heads, int kv_heads, int head_dim, float *out) {
    const int span = window > 0 && window < max_pos ? window : max_pos;
    const int G = heads / kv_heads;
    if (tokens == 1 && (G == 1 || G == 2 || G == 4 || G == 8)) {
        // one new token per sequence: the keys split over CTAs (ranges of cpc
        // chunks, as few as keep about 8 CTAs per SM in the grid), then merged
        const int64_t rows = seqs;
        const int chunks = (span + AK - 1) / AK;
        const int64_t want = (8LL * ctx->sm_count + rows * kv_heads - 1) / (rows * kv_heads);
        const int cpc = (int)((chunks + std::min<int64_t>(chunks, want) - 1) / std::min<int64_t>(chunks, want));
        const int nsplit = (chunks + cpc - 1) / cpc;
        const size_t bytes = (size_t)rows * heads * nsplit * (head_dim + 2) * sizeof(float);
        if (int rc = ensure_scratch(ctx, 2, bytes)) return rc;
        float *part = (float *)ctx->scratch[2];
        const dim3 pg(nsplit, kv_heads, (unsigned)rows);
#define EF_PART(DD, GG)                                                                                          \
    rc = part_launch<DD, GG, KV>(ctx, pg, q, kcache, vcache, pos, tokens, max_pos, window, heads, kv_heads, cpc, part)
        int rc;
        if (head_dim == 64) {
            switch (G) {
            case 1: EF_PART(64, 1); break;
            case 2: EF_PART(64, 2); break;
            case 4: EF_PART(64, 4); break;
            default: EF_PART(64, 8); break;
            }
        } else {
            switch (G) {
            case 1: EF_PART(128, 1); break;
            case 2: EF_PART(128, 2); break;
            case 4: EF_PART(128, 4); break;
            default: EF_PART(128, 8); break;
            }
        }
#undef EF_PART
        if (rc) return rc;
        const dim3 cg(heads, (unsigned)rows);
        const size_t cs = (size_t)nsplit * sizeof(float);
        if (cs > 48 * 1024) return set_err(ctx, EF_ERR_RANGE, "attention: %d key ranges", nsplit);
        if (head_dim == 64)
            return launch_on(ctx, ef_attn_combine_kernel<64>, cg, CT, cs, "attention combine launch",
                             (const float *)part, head_gate, heads, nsplit, out);
        return launch_on(ctx, ef_attn_combine_kernel<128>, cg, CT, cs, "attention combine launch", (const float *)part,
                         head_gate, heads, nsplit, out);
    }
    if (G == 1 || G == 2 || G == 4 || G == 8) {
        // several new tokens per sequence: key tiles shared by a block of queries
        switch (head_dim * 16 + G) {
        case 64 * 16 + 1: return prompt_attn_launch<64, 1, KV>(ctx, seqs, q, kcache, vcache, head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
        case 64 * 16 + 2: return prompt_attn_launch<64, 2, KV>(ctx, seqs, q, kcache, vcache, head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
        case 64 * 16 + 4: return prompt_attn_launch<64, 4, KV>(ctx, seqs, q, kcache, vcache, head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
        case 64 * 16 + 8: return prompt_attn_launch<64, 8, KV>(ctx, seqs, q, kcache, vcache, head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
        case 128 * 16 + 1: return prompt_attn_launch<128, 1, KV>(ctx, seqs, q, kcache, vcache, head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
        case 128 * 16 + 2: return prompt_attn_launch<128, 2, KV>(ctx, seqs, q, kcache, vcache, head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
        case 128 * 16 + 4: return prompt_attn_launch<128, 4, KV>(ctx, seqs, q, kcache, vcache, head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
        default: return prompt_attn_launch<128, 8, KV>(ctx, seqs, q, kcache, vcache, head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
        }
    }
    // other head groupings: a CTA per (head, query row), scores of all keys in shared memory
    const size_t smem = (size_t)span * 4;
    if (smem > 200 * 1024) return set_err(ctx, EF_ERR_RANGE, "attention: %d keys exceed shared memory", span);
    static std::atomic<unsigned long long> configured[2] = {{0}, {0}};
    const int di = head_dim == 64 ? 0 : 1;
    if (ctx->device < 64 && !(configured[di].load() & (1ull << ctx->device))) {
        cudaError_t e = di == 0 ? cudaFuncSetAttribute(ef_attention_kernel<64, KV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       200 * 1024)
                                : cudaFuncSetAttribute(ef_attention_kernel<128, KV>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (int rc = check_cuda(ctx, e, "attention smem attribute")) return rc;
        configured[di].fetch_or(1ull << ctx->device);
    }
    const dim3 grid(heads, seqs * tokens);
    if (di == 0)
        return launch_on(ctx, ef_attention_kernel<64, KV>, grid, 256, smem, "attention launch", q, kcache, vcache,
                         head_gate, pos, tokens, max_pos, window, heads, kv_heads, out);
    return launch_on(ctx, ef_attention_kernel<128, KV>, grid, 256, smem, "attention launch", q, kcache, vcache, head_gate,
                     pos, tokens, max_pos, window, heads, kv_heads, out);
}

template <typename KV>
static int attn_decode(ef_ctx *ctx, const float *q, const KV *kcache, const KV *vcache, const float *head_gate,
                       const int *pos, int max_pos, int window, int heads, int kv_heads, int head_dim, float *out) {
    if (!ctx || !q || !kcache || !vcache || !pos || !out || heads < 1 || kv_heads < 1 || heads % kv_heads)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "attn_decode: bad arguments") : EF_ERR_INVALID;
    if (head_dim != 64) return set_err(ctx, EF_ERR_SHAPE, "attn_decode: head_dim %d (64 supported)", head_dim);
    return attention_launch(ctx, q, kcache, vcache, head_gate, pos, 1, 1, max_pos, window, heads, kv_heads, 64, out);
}

template <typename KV>
static int attention(ef_ctx *ctx, const float *q, const KV *kcache, const KV *vcache, const float *head_gate,
                     const int *pos, int seqs, int tokens, int max_pos, int window, int heads, int kv_heads,
                     int head_dim, float *out) {
    if (!ctx || !q || !kcache || !vcache || !pos || !out || heads < 1 || kv_heads < 1 || heads % kv_heads ||
        seqs < 1 || tokens < 1 || max_pos < 1 || window < 0)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "attention: bad arguments") : EF_ERR_INVALID;
    if (head_dim != 64 && head_dim != 128)
        return set_err(ctx, EF_ERR_SHAPE, "attention: head_dim %d (64 or 128 supported)", head_dim);
    if ((int64_t)seqs * tokens > 65535) return set_err(ctx, EF_ERR_RANGE, "attention: more than 65535 rows");
    return attention_launch(ctx, q, kcache, vcache, head_gate, pos, seqs, tokens, max_pos, window, heads, kv_heads,
                            head_dim, out);
}

}  // namespace ef

using namespace ef;

extern "C" {


int ef_rmsnorm(ef_ctx *ctx, const float *x, const float *w, int rows, int n, float eps, float *y) {
    if (!ctx || !x || !w || !y || rows < 1 || n < 1) return ctx ? set_err(ctx, EF_ERR_INVALID, "rmsnorm: bad arguments") : EF_ERR_INVALID;
    int th = 0;
    const int v = norm_v(n, th);
    if (!v) return set_err(ctx, EF_ERR_SHAPE, "rmsnorm: n=%d (a multiple of 128 up to 8192, power-of-2 blocks)", n);
    int rc = EF_OK;
    switch (v) {
    case 1: rc = launch_on(ctx, ef_rmsnorm_kernel<1>, rows, th, 0, "rmsnorm launch", x, w, n, eps, y); break;
    case 2: rc = launch_on(ctx, ef_rmsnorm_kernel<2>, rows, th, 0, "rmsnorm launch", x, w, n, eps, y); break;
    case 4: rc = launch_on(ctx, ef_rmsnorm_kernel<4>, rows, th, 0, "rmsnorm launch", x, w, n, eps, y); break;
    default: rc = launch_on(ctx, ef_rmsnorm_kernel<8>, rows, th, 0, "rmsnorm launch", x, w, n, eps, y); break;
    }
    return rc;
}

int ef_norm_add_norm(ef_ctx *ctx, const float *o, const float *w_post, float *x, const float *w_next, int rows, int n,
                     float eps, float *nrm) {
    if (!ctx || !o || !x || !w_next || !nrm || rows < 1 || n < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "norm_add_norm: bad arguments") : EF_ERR_INVALID;
    int th = 0;
    const int v = norm_v(n, th);
    if (!v) return set_err(ctx, EF_ERR_SHAPE, "norm_add_norm: n=%d (a multiple of 128 up to 8192, power-of-2 blocks)", n);
    int rc = EF_OK;
    switch (v) {
    case 1: rc = launch_on(ctx, ef_norm_add_norm_kernel<1>, rows, th, 0, "norm_add_norm launch", o, w_post, x, w_next, n, eps, nrm); break;
    case 2: rc = launch_on(ctx, ef_norm_add_norm_kernel<2>, rows, th, 0, "norm_add_norm launch", o, w_post, x, w_next, n, eps, nrm); break;
    case 4: rc = launch_on(ctx, ef_norm_add_norm_kernel<4>, rows, th, 0, "norm_add_norm launch", o, w_post, x, w_next, n, eps, nrm); break;
    default: rc = launch_on(ctx, ef_norm_add_norm_kernel<8>, rows, th, 0, "norm_add_norm launch", o, w_post, x, w_next, n, eps, nrm); break;
    }
    return rc;
}

int ef_shortconv(ef_ctx *ctx, const float *bcx, const float *conv_w, float *state, int tokens, int channels, int kernel,
                 float *y) {
    if (!ctx || !bcx || !conv_w || !state || !y || tokens < 1 || channels < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "shortconv: bad arguments") : EF_ERR_INVALID;
    if (kernel != 3) return set_err(ctx, EF_ERR_SHAPE, "shortconv: kernel %d (3 supported)", kernel);
    return launch_on(ctx, ef_shortconv_kernel<3>, grid1d(channels, 256), 256, 0, "shortconv launch", bcx, conv_w,
                     state, tokens, channels, y);
}

int ef_qk_norm_rope_cache(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                          const int *pos, int max_pos, int heads, int kv_heads, int head_dim, float theta_base,
                          float eps, float *kcache, float *vcache) {
    return qk_norm_rope_cache(ctx, q, k, v, wq, wk, pos, max_pos, heads, kv_heads, head_dim, theta_base, eps, kcache,
                              vcache);
}

int ef_qk_norm_rope_cache_f16(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                              const int *pos, int max_pos, int heads, int kv_heads, int head_dim, float theta_base,
                              float eps, uint16_t *kcache, uint16_t *vcache) {
    return qk_norm_rope_cache(ctx, q, k, v, wq, wk, pos, max_pos, heads, kv_heads, head_dim, theta_base, eps,
                              reinterpret_cast<__half *>(kcache), reinterpret_cast<__half *>(vcache));
}

int ef_rope_cache(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                  const int *pos, int seqs, int tokens, int max_pos, int heads, int kv_heads, int head_dim,
                  int rope_mode, float theta_base, float eps, float *kcache, float *vcache) {
    return rope_cache(ctx, q, k, v, wq, wk, pos, seqs, tokens, max_pos, heads, kv_heads, head_dim, rope_mode,
                      theta_base, eps, kcache, vcache);
}

int ef_rope_cache_f16(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                      const int *pos, int seqs, int tokens, int max_pos, int heads, int kv_heads, int head_dim,
                      int rope_mode, float theta_base, float eps, uint16_t *kcache, uint16_t *vcache) {
    return rope_cache(ctx, q, k, v, wq, wk, pos, seqs, tokens, max_pos, heads, kv_heads, head_dim, rope_mode,
                      theta_base, eps, reinterpret_cast<__half *>(kcache), reinterpret_cast<__half *>(vcache));
}

int ef_attn_decode(ef_ctx *ctx, const float *q, const float *kcache, const float *vcache, const float *head_gate,
                   const int *pos, int max_pos, int window, int heads, int kv_heads, int head_dim, float *out) {
    return attn_decode(ctx, q, kcache, vcache, head_gate, pos, max_pos, window, heads, kv_heads, head_dim, out);
}

int ef_attn_decode_f16(ef_ctx *ctx, const float *q, const uint16_t *kcache, const uint16_t *vcache,
                       const float *head_gate, const int *pos, int max_pos, int window, int heads, int kv_heads,
                       int head_dim, float *out) {
    return attn_decode(ctx, q, reinterpret_cast<const __half *>(kcache), reinterpret_cast<const __half *>(vcache),
                       head_gate, pos, max_pos, window, heads, kv_heads, head_dim, out);
}

int ef_attention(ef_ctx *ctx, const float *q, const float *kcache, const float *vcache, const float *head_gate,
                 const int *pos, int seqs, int tokens, int max_pos, int window, int heads, int kv_heads, int head_dim,
                 float *out) {
    return attention(ctx, q, kcache, vcache, head_gate, pos, seqs, tokens, max_pos, window, heads, kv_heads, head_dim,
                     out);
}

int ef_attention_f16(ef_ctx *ctx, const float *q, const uint16_t *kcache, const uint16_t *vcache,
                     const float *head_gate, const int *pos, int seqs, int tokens, int max_pos, int window, int heads,
                     int kv_heads, int head_dim, float *out) {
    return attention(ctx, q, reinterpret_cast<const __half *>(kcache), reinterpret_cast<const __half *>(vcache),
                     head_gate, pos, seqs, tokens, max_pos, window, heads, kv_heads, head_dim, out);
}

int ef_topk(ef_ctx *ctx, const float *logits, int rows, int n, int m, int *ids, float *vals, int *flags) {
    if (!ctx || !logits || !ids || !vals || !flags || rows < 1 || rows > 65535 || n < 1 || m < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "topk: bad arguments") : EF_ERR_INVALID;
    if (m > EF_TOPK_MAX_M || n > EF_TOPK_MAX_N)
        return set_err(ctx, EF_ERR_RANGE, "topk: m=%d n=%d (at most %d and %d)", m, n, EF_TOPK_MAX_M, EF_TOPK_MAX_N);
    const int nch = (n + TK_CHUNK - 1) / TK_CHUNK;
    int sort_n = 1;
    while (sort_n < nch * m) sort_n <<= 1;
    const size_t smem = (size_t)sort_n * 8;
    if (int rc = ensure_scratch(ctx, 3, (size_t)rows * nch * m * 8)) return rc;
    static std::atomic<unsigned long long> configured{0};
    if (ctx->device < 64 && !(configured.load() & (1ull << ctx->device))) {
        if (int rc = check_cuda(ctx, cudaFuncSetAttribute(ef_topk_final_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                          227 * 1024), "topk smem attribute"))
            return rc;
        configured.fetch_or(1ull << ctx->device);
    }
    if (int rc = check_cuda(ctx, cudaMemsetAsync(flags, 0, (size_t)rows * sizeof(int), ctx->stream), "topk flags"))
        return rc;
    unsigned long long *cand = (unsigned long long *)ctx->scratch[3];
    if (int rc = launch_on(ctx, ef_topk_chunk_kernel, dim3(nch, rows), 512, 0, "topk launch", logits, n, m, cand, flags))
        return rc;
    return launch_on(ctx, ef_topk_final_kernel, rows, 1024, smem, "topk launch", logits, n, m, nch, sort_n,
                     (const unsigned long long *)cand, ids, vals);
}

int ef_swiglu(ef_ctx *ctx, const float *gate, const float *up, int64_t n, float *out) {
    if (!ctx || !gate || !up || !out || n < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "swiglu: bad arguments") : EF_ERR_INVALID;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    return launch_on(ctx, ef_swiglu_kernel, (int)blocks, 256, 0, "swiglu launch", gate, up, n, out);
}

int ef_argmax_step(ef_ctx *ctx, const float *logits, int n, int *token, int *pos, int *out_tokens, int out_base,
                   int out_cap) {
    return ef_argmax_rows(ctx, logits, 1, n, token, pos, out_tokens, out_base, out_cap);
}

int ef_argmax_rows(ef_ctx *ctx, const float *logits, int rows, int n, int *tokens, int *pos, int *out_tokens,
                   int out_base, int out_cap) {
    if (!ctx || !logits || !tokens || !pos || n < 1 || rows < 1 || rows > 65535)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "argmax: bad arguments") : EF_ERR_INVALID;
    return launch_on(ctx, ef_argmax_kernel<false>, rows, 1024, 0, "argmax launch", logits, n, tokens, pos, out_tokens,
                     out_base, out_cap, 0, (int *)nullptr);
}

int ef_argmax_partial(ef_ctx *ctx, const float *logits, int rows, int n, int offset, int *pairs) {
    if (!ctx || !logits || !pairs || n < 1 || offset < 0 || rows < 1 || rows > 65535)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "argmax_partial: bad arguments") : EF_ERR_INVALID;
    return launch_on(ctx, ef_argmax_kernel<true>, rows, 1024, 0, "argmax_partial launch", logits, n, (int *)nullptr,
                     (int *)nullptr, (int *)nullptr, 0, 0, offset, pairs);
}

int ef_argmax_select(ef_ctx *ctx, const int *pairs, int nranks, int rows, int *tokens, int *pos, int *out_tokens,
                     int out_base, int out_cap) {
    if (!ctx || !pairs || !tokens || !pos || nranks < 1 || rows < 1 || rows > 65535)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "argmax_select: bad arguments") : EF_ERR_INVALID;
    return launch_on(ctx, ef_argmax_select_kernel, rows, 32, 0, "argmax_select launch", pairs, nranks, tokens, pos,
                     out_tokens, out_base, out_cap);
}

}  // extern "C"

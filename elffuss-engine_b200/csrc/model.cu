// model.cu -- the non-matmul operations of a decoder step (sm_100a), for the
// synthetic LFM3-shaped decoder that drives the GEMV hot path end to end.
//
// Each restates one operation of the reference's forward (js/model.js,
// js/kernels.nn.wgsl.js, js/kernels.model.wgsl.js, js/kernels.ssm.wgsl.js):
//   rmsnorm            y = x * rsqrt(mean(x^2) + eps) * w     (kernels.nn.wgsl.js:46-80)
//   norm_add_norm      x += rmsnorm(o) * w_post; n = rmsnorm(x) * w_next
//                      (post-norm + residual + next norm, model.js:635-664)
//   shortconv          B|C|x split, B*x, causal depthwise conv with state,
//                      C*y (model.js:758-794, kernels.model.wgsl.js:45-86,
//                      kernels.ssm.wgsl.js:64-92)
//   qk_norm_rope_cache per-head RMSNorm of q and k, NEOX RoPE, k and v into
//                      the cache at the current position (model.js:853-945,
//                      kernels.nn.wgsl.js:87-139)
//   attn_decode        softmax(q.k / sqrt(D)) with causal + window mask, times
//                      v, times sigmoid(per-head gate) (kernels.nn.wgsl.js:
//                      141-200, kernels.model.wgsl.js:89-105)
//   argmax_step        greedy token, strict '>' so the lowest index wins ties
//                      (sample.js:95-99); advances the device-side position
// Positions and tokens live in device memory, so one decode step can be
// captured as a CUDA graph and replayed with no host round trip.
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace ef {

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

// One CTA per row of T = min(256, n/4) threads; each thread keeps V float4 of
// the row in registers (all loads issued before the first reduction),
// n = 4 * T * V.
template <int V>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                      int n, float eps, float *__restrict__ y) {
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
// Same shape rules as rmsnorm_kernel.
template <int V>
__global__ void __launch_bounds__(256) norm_add_norm_kernel(const float *__restrict__ o,
                                                            const float *__restrict__ w_post, float *__restrict__ x,
                                                            const float *__restrict__ w_next, int n, float eps,
                                                            float *__restrict__ nrm) {
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
__global__ void shortconv_kernel(const float *__restrict__ bcx, const float *__restrict__ w, float *__restrict__ state,
                                 int tokens, int C, float *__restrict__ y) {
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

// One warp per head (q heads first, then k heads); head_dim 64 = 2 per lane.
// NEOX pairs (i, i + D/2); theta = pos * base^(-2i/D).
__global__ void qk_norm_rope_cache_kernel(float *__restrict__ q, const float *__restrict__ k,
                                          const float *__restrict__ v, const float *__restrict__ wq,
                                          const float *__restrict__ wk, const int *__restrict__ pos, int max_pos,
                                          int H, int KVH, float theta_scale, float eps,
                                          float *__restrict__ kcache, float *__restrict__ vcache) {
    constexpr int D = 64;
    const int head = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (head >= H + KVH) return;
    const int p = *pos;
    const bool isq = head < H;
    const int hh = isq ? head : head - H;
    const float *src = isq ? q + hh * D : k + hh * D;
    const float *wn = isq ? wq : wk;
    const float x0 = src[lane], x1 = src[lane + 32];
    const float scale = rsqrtf(warp_sum(x0 * x0 + x1 * x1) / (float)D + eps);
    const float n0 = x0 * scale * wn[lane], n1 = x1 * scale * wn[lane + 32];
    const float theta = (float)p * powf(theta_scale, (float)lane);
    float sn, cs;
    sincosf(theta, &sn, &cs);
    const float r0 = n0 * cs - n1 * sn, r1 = n0 * sn + n1 * cs;
    if (isq) {
        q[hh * D + lane] = r0;
        q[hh * D + lane + 32] = r1;
    } else if (p >= 0 && p < max_pos) {   // (a position past the caches is not stored)
        float *kc = kcache + ((int64_t)p * KVH + hh) * D;
        kc[lane] = r0;
        kc[lane + 32] = r1;
        float *vc = vcache + ((int64_t)p * KVH + hh) * D;
        vc[lane] = v[hh * D + lane];
        vc[lane + 32] = v[hh * D + lane + 32];
    }
}

// One CTA per query head; keys 0..pos, visible when pos - key < window
// (window 0 = all). Scores into shared memory, then out[d] = sum p * v.
__global__ void attn_decode_kernel(const float *__restrict__ q, const float *__restrict__ kcache,
                                   const float *__restrict__ vcache, const float *__restrict__ gate,
                                   const int *__restrict__ pos, int max_pos, int window, int H, int KVH,
                                   float *__restrict__ out) {
    constexpr int D = 64;
    extern __shared__ float sc[];
    __shared__ float red[32];
    __shared__ float qs[D];
    const int h = blockIdx.x, kvh = h / (H / KVH);
    const int nkv = min(*pos + 1, max_pos), qpos = nkv - 1;   // never past the caches
    const int k0 = window > 0 && qpos - window + 1 > 0 ? qpos - window + 1 : 0;
    if (threadIdx.x < D) qs[threadIdx.x] = q[h * D + threadIdx.x] * rsqrtf((float)D);
    __syncthreads();
    float mx = -1e30f;
    for (int kk = k0 + threadIdx.x; kk < nkv; kk += blockDim.x) {
        const float4 *kr = reinterpret_cast<const float4 *>(kcache + ((int64_t)kk * KVH + kvh) * D);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < D / 4; i++) {
            const float4 kv = kr[i];
            s += qs[4 * i] * kv.x + qs[4 * i + 1] * kv.y + qs[4 * i + 2] * kv.z + qs[4 * i + 3] * kv.w;
        }
        sc[kk - k0] = s;
        mx = fmaxf(mx, s);
    }
    // block max
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
    if (threadIdx.x < D) {
        const int d = threadIdx.x;
        float acc = 0.f;
        for (int kk = k0; kk < nkv; kk++) acc += sc[kk - k0] * vcache[((int64_t)kk * KVH + kvh) * D + d];
        float o = acc * inv;
        if (gate) o = o / (1.0f + expf(-gate[h]));
        out[h * D + d] = o;
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

// Greedy argmax over n logits (strict '>': lowest index wins ties). PAIR =
// false: finish_step with the winner. PAIR = true (one vocabulary shard of a
// tensor-parallel head): pair[0] = the best value's bits, pair[1] = its index
// + offset, for argmax_select over the shards.
template <bool PAIR>
__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ logits, int n,
                                                      int *__restrict__ token, int *__restrict__ pos,
                                                      int *__restrict__ out_tokens, int out_base, int out_cap,
                                                      int offset, int *__restrict__ pair) {
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

// The winner over the shards' (value, index) pairs, in the same order as one
// argmax over the whole vocabulary: larger value, then lower index.
__global__ void argmax_select_kernel(const int *__restrict__ pairs, int npairs, int *__restrict__ token,
                                     int *__restrict__ pos, int *__restrict__ out_tokens, int out_base,
                                     int out_cap) {
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    for (int i = threadIdx.x; i < npairs; i += 32) {
        const float v = __int_as_float(pairs[2 * i]);
        const int ix = pairs[2 * i + 1];
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

}  // namespace ef

using namespace ef;

extern "C" {

// Row of n: T = min(256, n/4) threads with V float4 each, n = 4 * T * V,
// V in {1, 2, 4, 8}; 0 when n has no such split (n a multiple of 128 up to 8192).
static int norm_v(int n, int &threads) {
    if (n < 128 || n % 128) return 0;
    threads = n / 4 < 256 ? n / 4 : 256;
    if (n % (4 * threads)) return 0;
    const int v = n / (4 * threads);
    return v == 1 || v == 2 || v == 4 || v == 8 ? v : 0;
}

int ef_rmsnorm(ef_ctx *ctx, const float *x, const float *w, int rows, int n, float eps, float *y) {
    if (!ctx || !x || !w || !y || rows < 1 || n < 1) return ctx ? set_err(ctx, EF_ERR_INVALID, "rmsnorm: bad arguments") : EF_ERR_INVALID;
    int th = 0;
    const int v = norm_v(n, th);
    if (!v) return set_err(ctx, EF_ERR_SHAPE, "rmsnorm: n=%d (a multiple of 128 up to 8192, power-of-2 blocks)", n);
    ctx->launches++;
    switch (v) {
    case 1: rmsnorm_kernel<1><<<rows, th, 0, ctx->stream>>>(x, w, n, eps, y); break;
    case 2: rmsnorm_kernel<2><<<rows, th, 0, ctx->stream>>>(x, w, n, eps, y); break;
    case 4: rmsnorm_kernel<4><<<rows, th, 0, ctx->stream>>>(x, w, n, eps, y); break;
    default: rmsnorm_kernel<8><<<rows, th, 0, ctx->stream>>>(x, w, n, eps, y); break;
    }
    return check_cuda(ctx, cudaGetLastError(), "rmsnorm launch");
}

int ef_norm_add_norm(ef_ctx *ctx, const float *o, const float *w_post, float *x, const float *w_next, int rows, int n,
                     float eps, float *nrm) {
    if (!ctx || !o || !x || !w_next || !nrm || rows < 1 || n < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "norm_add_norm: bad arguments") : EF_ERR_INVALID;
    int th = 0;
    const int v = norm_v(n, th);
    if (!v) return set_err(ctx, EF_ERR_SHAPE, "norm_add_norm: n=%d (a multiple of 128 up to 8192, power-of-2 blocks)", n);
    ctx->launches++;
    switch (v) {
    case 1: norm_add_norm_kernel<1><<<rows, th, 0, ctx->stream>>>(o, w_post, x, w_next, n, eps, nrm); break;
    case 2: norm_add_norm_kernel<2><<<rows, th, 0, ctx->stream>>>(o, w_post, x, w_next, n, eps, nrm); break;
    case 4: norm_add_norm_kernel<4><<<rows, th, 0, ctx->stream>>>(o, w_post, x, w_next, n, eps, nrm); break;
    default: norm_add_norm_kernel<8><<<rows, th, 0, ctx->stream>>>(o, w_post, x, w_next, n, eps, nrm); break;
    }
    return check_cuda(ctx, cudaGetLastError(), "norm_add_norm launch");
}

int ef_shortconv(ef_ctx *ctx, const float *bcx, const float *conv_w, float *state, int tokens, int channels, int kernel,
                 float *y) {
    if (!ctx || !bcx || !conv_w || !state || !y || tokens < 1 || channels < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "shortconv: bad arguments") : EF_ERR_INVALID;
    if (kernel != 3) return set_err(ctx, EF_ERR_SHAPE, "shortconv: kernel %d (3 supported)", kernel);
    ctx->launches++;
    shortconv_kernel<3><<<grid1d(channels, 256), 256, 0, ctx->stream>>>(bcx, conv_w, state, tokens, channels, y);
    return check_cuda(ctx, cudaGetLastError(), "shortconv launch");
}

int ef_qk_norm_rope_cache(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                          const int *pos, int max_pos, int heads, int kv_heads, int head_dim, float theta_base,
                          float eps, float *kcache, float *vcache) {
    if (!ctx || !q || !k || !v || !wq || !wk || !pos || !kcache || !vcache || heads < 1 || kv_heads < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "qk_norm_rope_cache: bad arguments") : EF_ERR_INVALID;
    if (head_dim != 64) return set_err(ctx, EF_ERR_SHAPE, "qk_norm_rope_cache: head_dim %d (64 supported)", head_dim);
    const float theta_scale = powf(theta_base, -2.0f / (float)head_dim);
    ctx->launches++;
    qk_norm_rope_cache_kernel<<<grid1d(heads + kv_heads, 8), 256, 0, ctx->stream>>>(
        q, k, v, wq, wk, pos, max_pos, heads, kv_heads, theta_scale, eps, kcache, vcache);
    return check_cuda(ctx, cudaGetLastError(), "qk_norm_rope_cache launch");
}

int ef_attn_decode(ef_ctx *ctx, const float *q, const float *kcache, const float *vcache, const float *head_gate,
                   const int *pos, int max_pos, int window, int heads, int kv_heads, int head_dim, float *out) {
    if (!ctx || !q || !kcache || !vcache || !pos || !out || heads < 1 || kv_heads < 1 || heads % kv_heads)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "attn_decode: bad arguments") : EF_ERR_INVALID;
    if (head_dim != 64) return set_err(ctx, EF_ERR_SHAPE, "attn_decode: head_dim %d (64 supported)", head_dim);
    const int span = window > 0 && window < max_pos ? window : max_pos;
    const size_t smem = (size_t)span * 4;
    if (smem > 200 * 1024) return set_err(ctx, EF_ERR_RANGE, "attn_decode: %d keys exceed shared memory", span);
    static unsigned long long configured = 0;
    if (ctx->device < 64 && !(configured & (1ull << ctx->device))) {
        if (int rc = check_cuda(ctx, cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                          200 * 1024), "attn smem attribute"))
            return rc;
        configured |= 1ull << ctx->device;
    }
    ctx->launches++;
    attn_decode_kernel<<<heads, 256, smem, ctx->stream>>>(q, kcache, vcache, head_gate, pos, max_pos, window, heads,
                                                          kv_heads, out);
    return check_cuda(ctx, cudaGetLastError(), "attn_decode launch");
}

int ef_argmax_step(ef_ctx *ctx, const float *logits, int n, int *token, int *pos, int *out_tokens, int out_base,
                   int out_cap) {
    if (!ctx || !logits || !token || !pos || n < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "argmax_step: bad arguments") : EF_ERR_INVALID;
    ctx->launches++;
    argmax_kernel<false><<<1, 1024, 0, ctx->stream>>>(logits, n, token, pos, out_tokens, out_base, out_cap, 0,
                                                       nullptr);
    return check_cuda(ctx, cudaGetLastError(), "argmax_step launch");
}

int ef_argmax_partial(ef_ctx *ctx, const float *logits, int n, int offset, int *pair) {
    if (!ctx || !logits || !pair || n < 1 || offset < 0)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "argmax_partial: bad arguments") : EF_ERR_INVALID;
    ctx->launches++;
    argmax_kernel<true><<<1, 1024, 0, ctx->stream>>>(logits, n, nullptr, nullptr, nullptr, 0, 0, offset, pair);
    return check_cuda(ctx, cudaGetLastError(), "argmax_partial launch");
}

int ef_argmax_select(ef_ctx *ctx, const int *pairs, int npairs, int *token, int *pos, int *out_tokens,
                     int out_base, int out_cap) {
    if (!ctx || !pairs || !token || !pos || npairs < 1)
        return ctx ? set_err(ctx, EF_ERR_INVALID, "argmax_select: bad arguments") : EF_ERR_INVALID;
    ctx->launches++;
    argmax_select_kernel<<<1, 32, 0, ctx->stream>>>(pairs, npairs, token, pos, out_tokens, out_base, out_cap);
    return check_cuda(ctx, cudaGetLastError(), "argmax_select launch");
}

}  // extern "C"

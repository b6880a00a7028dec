/*
 * elffuss_cuda.h -- C ABI of the B200 (sm_100a) quantized matrix-product path.
 *
 * This library replaces, for the GGUF block-quantized GEMV (decode) and GEMM
 * (prefill), the WebGPU objects and WGSL kernels behind the reference's
 * operator API `createQuantOps(device, {ctx, ...})` (js/ops.js:748-1142):
 *   device + context + buffer pool   js/device.js:66-165, js/ops.js:134-469
 *   load-time repack                 js/repack.js:153-306
 *   dequant / matmul / gemv / gemm2  js/ops.js:813-1101, js/ops.gemv.js:148-215,
 *                                    js/ops.gemm2.js:266-302
 * Plain pointers, sizes and opaque handles only; no C++ or torch types.
 *
 * Conventions
 *   - Every call returns an int status: EF_OK (0), EF_NOT_APPLICABLE (1, the
 *     reference's `null` return from gemv/gemm2: "this path does not apply,
 *     the caller falls back", js/ops.gemv.js:13-21, js/ops.gemm2.js:5-8), or a
 *     negative error (the reference's `throw new Error(...)`). The message of
 *     the last error is kept per context: ef_last_error().
 *   - All device work is asynchronous and ordered on the context's stream
 *     (the reference records into one command batch and syncs only at
 *     readback, js/ops.js:665-679, js/device.js:165). ef_stream_sync waits.
 *   - Activations are token-major f32 [tokens][k]; outputs f32 [tokens][rows]
 *     (js/ops.js:827-829, 1085-1100).
 *   - Device pointers passed in (x, y, dev_out) must be 16-byte aligned.
 */
#ifndef ELFFUSS_CUDA_H
#define ELFFUSS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EF_ABI_VERSION 1

#if defined(__GNUC__)
#define EF_API __attribute__((visibility("default")))
#else
#define EF_API
#endif

/* Status codes. */
enum {
    EF_OK = 0,
    EF_NOT_APPLICABLE = 1,   /* path does not apply; caller falls back (reference `null`) */
    EF_ERR_INVALID = -1,     /* null handle / pointer, negative or zero size */
    EF_ERR_TYPE = -2,        /* unsupported quant type (js/ops.js:769-770) */
    EF_ERR_SHAPE = -3,       /* k not a multiple of the block, bad rows/tokens (js/ops.js:850-852) */
    EF_ERR_CUDA = -4,        /* CUDA runtime failure; message in ef_last_error */
    EF_ERR_OOM = -5,         /* device allocation failed */
    EF_ERR_MISMATCH = -6,    /* weight handle does not match the call (js/repack.js:268-286) */
    EF_ERR_RANGE = -7,       /* offset/size outside a buffer, or a slice outside a tensor */
    EF_ERR_TIMEOUT = -8      /* a bounded device wait gave up (a tensor-parallel peer, a GEMM pipeline stage) */
};

/* GGUF tensor types (ggml ids, js/gguf.js:48-64). */
enum {
    EF_F32 = 0, EF_F16 = 1, EF_Q4_0 = 2, EF_Q8_0 = 8, EF_Q2_K = 10, EF_Q4_K = 12, EF_Q5_K = 13, EF_Q6_K = 14,
    EF_IQ2_XXS = 16, EF_IQ1_S = 19
};

typedef struct ef_ctx ef_ctx;        /* device + stream + buffer pool (js/ops.js:134 createContext) */
typedef struct ef_buf ef_buf;        /* device allocation (a GPUBuffer of the reference) */
typedef struct ef_weight ef_weight;  /* a weight tensor repacked on the device (creaBufferR) */
typedef struct ef_tp ef_tp;          /* tensor-parallel exchange buffers of one rank (no reference counterpart) */
typedef struct ef_gguf ef_gguf;      /* an opened GGUF file (js/gguf.js parseGGUF) */

/* ---- library / context ---------------------------------------------------- */

/* ABI version of the loaded library (EF_ABI_VERSION). */
EF_API int ef_version(void);

/* Block geometry of a type: elements and bytes per GGUF block (js/kernels.wgsl.js:886-892
 * QUANT_TYPES). EF_ERR_TYPE for a type without a decoder here. */
EF_API int ef_type_info(int type, int *block_elems, int *block_bytes);

/* Create a context on CUDA device `device` with its own stream.
 * Replaces requestDevice() + createContext() (js/device.js:66, js/ops.js:134). */
EF_API int ef_ctx_create(int device, ef_ctx **out);
EF_API int ef_ctx_destroy(ef_ctx *ctx);

/* Run subsequent work on a caller-owned cudaStream_t (e.g. torch's current
 * stream); NULL selects the CUDA default stream. Until the first call the
 * context uses a stream of its own. */
EF_API int ef_ctx_set_stream(ef_ctx *ctx, void *cuda_stream);

/* Programmatic dependent launch for this context's kernels (on != 0): each
 * kernel may be scheduled while the one before it on the stream finishes,
 * fetching what does not depend on it (the weights) early, and waits for
 * that kernel's results before reading them. On by default (the environment
 * variable EF_PDL=0 turns the default off). Weight loads synchronize the
 * stream, so weights are complete before any later kernel starts. No
 * counterpart in the reference. */
EF_API int ef_ctx_set_pdl(ef_ctx *ctx, int on);
EF_API void *ef_ctx_stream(const ef_ctx *ctx);

/* Wait for all work queued on the context's stream (the readback sync point,
 * js/device.js:165). */
EF_API int ef_stream_sync(ef_ctx *ctx);

/* Message of the last failing call on this context ("" if none). */
EF_API const char *ef_last_error(const ef_ctx *ctx);

/* Number of kernels this context has launched so far (host-side counter,
 * incremented at every launch; launches recorded into a CUDA graph count once,
 * at capture). Diagnostic only: no counterpart in the reference. */
EF_API uint64_t ef_ctx_launch_count(const ef_ctx *ctx);

/* ---- buffers (ctx.alloc / recycle / upload, js/ops.js:242-307,1129-1133) --- */

EF_API int ef_alloc(ef_ctx *ctx, size_t bytes, ef_buf **out);
EF_API int ef_free(ef_ctx *ctx, ef_buf *buf);
EF_API void *ef_buf_ptr(const ef_buf *buf);
EF_API size_t ef_buf_size(const ef_buf *buf);
/* Host <-> device copies, ordered on the context stream; ef_download waits. */
EF_API int ef_upload(ef_ctx *ctx, ef_buf *buf, size_t offset, const void *host, size_t n);
EF_API int ef_download(ef_ctx *ctx, const ef_buf *buf, size_t offset, void *host, size_t n);
/* Pool marks: every ef_alloc after `mark` that is not in `live` is freed by
 * ef_scratch_release (ctx.recycleDesde(mark, ...live), js/ops.js:295-307). */
EF_API int ef_scratch_mark(ef_ctx *ctx, uint64_t *mark);
EF_API int ef_scratch_release(ef_ctx *ctx, uint64_t mark, ef_buf *const *live, int nlive);

/* ---- weights (load-time repack, js/repack.js:153-306, js/model.js:312-329) --- */

/* Upload a row-major GGUF tensor (rows x k weights, raw block bytes) and repack
 * it on the device into the tile layout the kernels read. Replaces
 * reordena/creaBufferR/marcaBufferR (js/repack.js:187,241,293). */
EF_API int ef_weight_load(ef_ctx *ctx, int type, const void *host_gguf, int64_t rows, int64_t k,
                   ef_weight **out);
/* The same from GGUF bytes already in device memory (not modified). */
EF_API int ef_weight_load_device(ef_ctx *ctx, int type, const void *dev_gguf, int64_t rows,
                          int64_t k, ef_weight **out);
/* Load the sub-matrix rows [row0, row0+nrows) x columns [k0, k0+nk) of a host
 * GGUF tensor of rows x k: the shard of one tensor-parallel rank (column-
 * parallel: a row range; row-parallel: a k range, k0 and nk multiples of the
 * block). No reference counterpart: the reference is single-device. */
EF_API int ef_weight_load_slice(ef_ctx *ctx, int type, const void *host_gguf, int64_t rows, int64_t k,
                         int64_t row0, int64_t nrows, int64_t k0, int64_t nk, ef_weight **out);
/* The shard of tensor-parallel rank `rank` of `nranks` of a host GGUF tensor
 * of rows x k, as ef_weight_load_slice loads it: shard_axis 0 = column-
 * parallel (rows / nranks consecutive output rows), 1 = row-parallel
 * (k / nranks consecutive input columns, whole blocks). The split must be
 * even (EF_ERR_SHAPE otherwise). The drop-in boundary's TP weight loader; no
 * reference counterpart: the reference is single-device. */
EF_API int ef_weight_load_shard(ef_ctx *ctx, int type, const void *host_gguf, int64_t rows, int64_t k,
                                int shard_axis, int rank, int nranks, ef_weight **out);
EF_API int ef_weight_free(ef_ctx *ctx, ef_weight *w);
EF_API int ef_weight_info(const ef_weight *w, int *type, int64_t *rows, int64_t *k, size_t *dev_bytes);
/* Inverse repack: write the original GGUF bytes (rows * k/elems * bytes) to
 * `dev_gguf_out`. The round-trip hook of vuelveAlGGUF (js/repack.js:201-219). */
EF_API int ef_weight_unpack(ef_ctx *ctx, const ef_weight *w, void *dev_gguf_out);

/* ---- operators ------------------------------------------------------------- */

/* Rows [row0, row0+nrows) of dequant(W) to f32 [nrows][k], bit-exact with the
 * reference decoders. quant.dequant (js/ops.js:813-823, kernels.wgsl.js:903). */
EF_API int ef_dequant(ef_ctx *ctx, const ef_weight *w, int64_t row0, int64_t nrows, float *dev_out);

/* Rows of dequant(W) chosen by device-side ids: out[t][:] = dequant(W)[ids[t]]
 * for t < tokens (f32 [tokens][k]); an id outside [0, rows) gives zeros.
 * quant.gather (js/ops.js:1104-1118, gatherShader kernels.wgsl.js:1199), the
 * embedding lookup; the ids are read on the device, so the call can sit in a
 * captured CUDA graph. */
EF_API int ef_gather(ef_ctx *ctx, const ef_weight *w, const int *dev_ids, int tokens, float *dev_out);

/* ef_gather fused with the first layer's input norm (the reference's fusion
 * F2, js/ops.fusion.js:152-165): x[t] = the dequantized row ids[t] (the same
 * bits as ef_gather; zeros outside the rows) and nrm[t] = x[t] *
 * rsqrt(mean(x[t]^2) + eps) * w_norm. Rows of k <= 51200 floats. */
EF_API int ef_gather_rmsnorm(ef_ctx *ctx, const ef_weight *w, const int *dev_ids, int tokens, const float *w_norm,
                             float eps, float *x, float *nrm);

/* Decode GEMV, 1 <= M <= 16 tokens: y[M][rows] = x[M][k] . dequant(W)^T.
 * quant.gemv.matmul / quant.matmul for few tokens (js/ops.gemv.js:148-165,
 * js/ops.js:834-837). EF_NOT_APPLICABLE for M > 16. */
EF_API int ef_gemv(ef_ctx *ctx, const ef_weight *w, const float *x, int M, float *y);

/* Fused gate/up GEMV with the SwiGLU epilogue: y = silu(Wg.x) * (Wu.x),
 * silu(v) = v / (1 + exp(-v)). quant.gemv.gateUp (js/ops.gemv.js:166-190,
 * kernels.gemv.wgsl.js:434-437). Wg and Wu share type, rows and k. */
EF_API int ef_gemv_swiglu(ef_ctx *ctx, const ef_weight *wg, const ef_weight *wu, const float *x, int M,
                   float *y);

/* 1..4 matrices with the same x and k, each to its own output (Q/K/V/gate in
 * one launch). quant.gemv.secciones (js/ops.gemv.js:192-215). */
EF_API int ef_gemv_sections(ef_ctx *ctx, const ef_weight *const *ws, int n, const float *x, int M,
                     float *const *ys);

/* Prefill GEMM, M >= 1 tokens (tuned for M >= 128): y[M][rows] with x given as
 * f16 (x_type EF_F16, [M][k]) or f32 (EF_F32, converted to f16 with round to
 * nearest even first, js/ops.gemm2.js:175-196). W is dequantised to f16 and
 * multiplied on the tcgen05 tensor cores with f32 accumulation
 * (gemm2.matmul, js/ops.gemm2.js:266-289, kernels.gemm2.wgsl.js:174-240).
 * `flags` is reserved (0). */
EF_API int ef_gemm(ef_ctx *ctx, const ef_weight *w, const void *x, int x_type, int M, float *y,
            uint32_t flags);

/* Synchronizes the context's stream and reports whether a prefill GEMM gave up
 * on one of its bounded pipeline waits (about a second each) since the last
 * call: EF_ERR_TIMEOUT then (the flag is cleared; those GEMMs' outputs are
 * invalid), else EF_OK. The kernel never spins without a limit; it stops
 * issuing work, lets its own copies land and frees its tensor memory. No
 * reference counterpart (WebGPU has no device-side waits). */
EF_API int ef_gemm_status(ef_ctx *ctx);

/* Test hook for the bounded waits above: sets how many polls each pipeline
 * wait of later GEMMs on the context's device makes before it gives up
 * (negative restores the default, about a second; 0 makes every wait give up
 * without polling, so the next GEMM stops at once and ef_gemm_status reports
 * EF_ERR_TIMEOUT). The kernel still lets its own copies and tensor-core work
 * drain before it exits. Synchronizes the context's stream. No reference
 * counterpart. */
EF_API int ef_gemm_set_wait_limit(ef_ctx *ctx, int polls);

/* Decode GEMV that allocates nothing (no counterpart in the reference, which
 * is single-device and allocates through its own buffer pool). ef_gemv keeps
 * its per-call activation fragments in context scratch that it grows with
 * cudaMalloc on the first call of a larger shape; some callers cannot allow
 * that: hosts whose device memory is owned entirely by another allocator (a
 * framework's caching allocator or a fixed arena), and decode loops that
 * cannot take the implicit device synchronization of an allocation or a
 * free. This variant uses a file-scope device array of
 * 1 MiB instead, held by every GPU that loads the library until the process
 * exits; it supports k up to the point where the activation data exceeds
 * 1 MiB (k up to about 30,000 for 9-16 tokens and 61,000 for 3-8 tokens;
 * 1-2 tokens keep it in shared memory and have no limit) and returns
 * EF_ERR_RANGE beyond that. No context is needed: work is queued on
 * `cuda_stream` (NULL = default stream) of the current device, which must be
 * the device `w` was loaded on. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture. All calls share the one array: calls that overlap on the
 * GPU (other streams, other threads) race; each call overwrites the whole part
 * of the array it reads, so nothing needs clearing. Same arguments, result and
 * status codes as ef_gemv (no per-call error message). */
EF_API int ef_gemv_noalloc(const ef_weight *w, const float *x, int M, float *y, void *cuda_stream);

/* The dispatcher of quant.matmul (js/ops.js:827-1101): GEMV for tokens <= 16,
 * GEMM above, same contract and output. */
EF_API int ef_matmul(ef_ctx *ctx, const ef_weight *w, const float *x, int tokens, float *y);

/* ---- decoder-step operations ---------------------------------------------
 * The non-matmul steps of the reference's forward (js/model.js), used by the
 * synthetic LFM3-shaped decoder that measures the GEMV path end to end. All
 * pointers are device pointers, f32 unless stated; rows are contiguous.
 * Positions are int32 in device memory so that a decode step can be captured
 * as a CUDA graph. */

/* y = x * rsqrt(mean(x^2) + eps) * w per row of n (nn.rmsnorm,
 * kernels.nn.wgsl.js:46-80); n = 128 * 2^j up to 8192 (other multiples of
 * 512 up to 8192 where n / min(256, n/4) / 4 is 1, 2, 4 or 8), rows 16-byte
 * aligned. */
EF_API int ef_rmsnorm(ef_ctx *ctx, const float *x, const float *w, int rows, int n, float eps, float *y);

/* Per row: x += rmsnorm(o) * w_post (x += o when w_post is NULL), then
 * nrm = rmsnorm(x) * w_next -- post-norm, residual and the next block's norm
 * in one pass (js/model.js:635-664, fusion F1 js/ops.fusion.js:131-150).
 * Same n and alignment rules as ef_rmsnorm. */
EF_API int ef_norm_add_norm(ef_ctx *ctx, const float *o, const float *w_post, float *x, const float *w_next,
                            int rows, int n, float eps, float *nrm);

/* Gated short convolution (js/model.js:758-794): bcx [tokens][3C] = B | C | x,
 * y[t][c] = C[t][c] * sum_r win[c][t+r] * w[c][r] over the window of the
 * kernel-1 previous B*x values (state [kernel-1][C], oldest first, updated in
 * place) followed by the tokens' B*x; w [C][kernel] in temporal order.
 * kernel 3 only. */
EF_API int ef_shortconv(ef_ctx *ctx, const float *bcx, const float *conv_w, float *state, int tokens, int channels,
                        int kernel, float *y);

/* One decode token: per-head RMSNorm (weights wq, wk [head_dim]) of q [heads]
 * [head_dim] (in place) and k [kv_heads][head_dim], NEOX RoPE at position
 * *pos with theta = pos * theta_base^(-2i/head_dim), then k and v written to
 * the caches [max_pos][kv_heads][head_dim] at *pos (js/model.js:853-945); a
 * position at or past max_pos is not stored. head_dim 64 only. */
EF_API int ef_qk_norm_rope_cache(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq,
                                 const float *wk, const int *pos, int max_pos, int heads, int kv_heads,
                                 int head_dim, float theta_base, float eps, float *kcache, float *vcache);

/* One decode token of attention over cache positions 0..*pos (a key is
 * visible when *pos - key < window; window 0 = all), scale 1/sqrt(head_dim),
 * grouped heads (heads / kv_heads queries per cache head); when head_gate is
 * not NULL each head's output is multiplied by sigmoid(head_gate[h])
 * (kernels.nn.wgsl.js:141-200, kernels.model.wgsl.js:89-105). out
 * [heads][head_dim]; head_dim 64 only; max_pos = the caches' capacity. */
EF_API int ef_attn_decode(ef_ctx *ctx, const float *q, const float *kcache, const float *vcache,
                          const float *head_gate, const int *pos, int max_pos, int window, int heads, int kv_heads,
                          int head_dim, float *out);

/* The same three with f16 caches (the reference's kvF16 option,
 * js/kernels.attn.wgsl.js:51-55, js/model.js:906-946): k (after its norm and
 * RoPE) and v are rounded to f16, to nearest even, when stored; q, the scores
 * and every sum stay f32. Caches are f16 bit patterns, same layout. */
EF_API int ef_qk_norm_rope_cache_f16(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq,
                                     const float *wk, const int *pos, int max_pos, int heads, int kv_heads,
                                     int head_dim, float theta_base, float eps, uint16_t *kcache, uint16_t *vcache);
EF_API int ef_attn_decode_f16(ef_ctx *ctx, const float *q, const uint16_t *kcache, const uint16_t *vcache,
                              const float *head_gate, const int *pos, int max_pos, int window, int heads,
                              int kv_heads, int head_dim, float *out);

/* Greedy sampling (js/sample.js:95-99): *token = argmax of n logits (strict
 * '>', the lowest index wins ties); *pos += 1; when out_tokens is not NULL the
 * token is also stored at out_tokens[new *pos - out_base] if that index is in
 * [0, out_cap). */
EF_API int ef_argmax_step(ef_ctx *ctx, const float *logits, int n, int *token, int *pos, int *out_tokens,
                          int out_base, int out_cap);

/* Several rows at once (one per sequence of a batch): row r's argmax updates
 * tokens[r], pos[r] and out_tokens[r * out_cap + new pos[r] - out_base]
 * (when in [0, out_cap)); logits [rows][n]. */
EF_API int ef_argmax_rows(ef_ctx *ctx, const float *logits, int rows, int n, int *tokens, int *pos,
                          int *out_tokens, int out_base, int out_cap);

/* Tensor-parallel greedy head (the LM head split by vocabulary rows over the
 * ranks; the reference has one device and no counterpart, its single-device
 * argmax is js/sample.js:95-99). ef_argmax_partial: for each of `rows` rows of
 * this rank's n logits, pairs[2r] = the best value's f32 bits, pairs[2r+1] =
 * its index + offset (the shard's first vocabulary id). ef_argmax_select:
 * given the ranks' pairs gathered in rank order ([nranks][rows][2] ints), each
 * row's winner in the order of one argmax over the whole vocabulary (larger
 * value, then lower index), then the same update as ef_argmax_rows. */
EF_API int ef_argmax_partial(ef_ctx *ctx, const float *logits, int rows, int n, int offset, int *pairs);
EF_API int ef_argmax_select(ef_ctx *ctx, const int *pairs, int nranks, int rows, int *tokens, int *pos,
                            int *out_tokens, int out_base, int out_cap);

/* RoPE pairing (js/kernels.nn.wgsl.js:27, js/state.js:345-349): NORM rotates
 * adjacent elements (2i, 2i+1) -- llama --, NEOX elements (i, i + D/2) --
 * lfm3, qwen35. */
#define EF_ROPE_NORM 0
#define EF_ROPE_NEOX 2

/* Attention input for `seqs` sequences of `tokens` new tokens each (rows r =
 * seq * tokens + t, token t of sequence s at position pos[s] + t): optional
 * per-head RMSNorm (wq, wk [head_dim], both NULL for none: llama has no
 * QK-norm, js/model.js:905-917), RoPE in `rope_mode` with theta = position *
 * theta_base^(-2i/head_dim) on q [rows][heads][head_dim] (in place) and k
 * [rows][kv_heads][head_dim], then k and v into the caches
 * [seqs][max_pos][kv_heads][head_dim] (js/model.js:895-945); positions at or
 * past max_pos are not stored. head_dim 64 or 128; rows <= 65535. */
EF_API int ef_rope_cache(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                         const int *pos, int seqs, int tokens, int max_pos, int heads, int kv_heads, int head_dim,
                         int rope_mode, float theta_base, float eps, float *kcache, float *vcache);

/* Causal attention for the rows of ef_rope_cache: the query at position p of
 * sequence s attends to that sequence's cache positions 0..p (those with
 * p - key < window; window 0 = all), scale 1/sqrt(head_dim), heads / kv_heads
 * queries per cache head, times sigmoid(head_gate[r][h]) when head_gate is not
 * NULL (js/model.js:946-983, kernels.nn.wgsl.js:141-200). out
 * [rows][heads][head_dim]; head_dim 64 or 128. A prompt of T tokens is one
 * call with tokens = T after ef_rope_cache has stored all T. */
EF_API int ef_attention(ef_ctx *ctx, const float *q, const float *kcache, const float *vcache,
                        const float *head_gate, const int *pos, int seqs, int tokens, int max_pos, int window,
                        int heads, int kv_heads, int head_dim, float *out);

/* ef_rope_cache / ef_attention with f16 caches (f16 bit patterns, same
 * layout; rounding as ef_qk_norm_rope_cache_f16). */
EF_API int ef_rope_cache_f16(ef_ctx *ctx, float *q, const float *k, const float *v, const float *wq, const float *wk,
                             const int *pos, int seqs, int tokens, int max_pos, int heads, int kv_heads, int head_dim,
                             int rope_mode, float theta_base, float eps, uint16_t *kcache, uint16_t *vcache);
EF_API int ef_attention_f16(ef_ctx *ctx, const float *q, const uint16_t *kcache, const uint16_t *vcache,
                            const float *head_gate, const int *pos, int seqs, int tokens, int max_pos, int window,
                            int heads, int kv_heads, int head_dim, float *out);

/* Sampling candidates on the device (kernels.topk.wgsl.js, topk.js): for each
 * of `rows` rows of n logits, the m first in the sampler's order -- larger
 * value first, the lower index first among equal values, -0 equal to +0 --
 * exactly: ids[r][i] and vals[r][i] (the logit's own f32 bits) for i < m in
 * that order (ids -1 past n). flags[r] = 2 when the row holds a NaN (the
 * order is then not the sampler's; read the row instead). m <=
 * EF_TOPK_MAX_M, n <= EF_TOPK_MAX_N. */
#define EF_TOPK_MAX_M 256
#define EF_TOPK_MAX_N 262144
EF_API int ef_topk(ef_ctx *ctx, const float *logits, int rows, int n, int m, int *ids, float *vals, int *flags);

/* out[i] = gate[i] * sigmoid(gate[i]) * up[i] for the n elements (the
 * prompt-side SwiGLU after two separate GEMMs; js/model.js:651-655). */
EF_API int ef_swiglu(ef_ctx *ctx, const float *gate, const float *up, int64_t n, float *out);

/* ---- GGUF files (js/gguf.js parseGGUF :324-438 and the type table :48-76).
 * ef_gguf_open maps the file and checks its structure as the reference does
 * (magic, version 2-3, no big-endian files, unique non-empty keys, value
 * types, general.alignment a uint32 power of two, unique tensor names, <= 4
 * dimensions, a known non-retired type, ne0 a multiple of the block, each
 * tensor's offset the padded running sum, data inside the file); on failure
 * it returns a negative status and, when err is given, a message. Tensors:
 * index, name, ggml type, dimensions (ne0 = k first; missing ones = 1), file
 * offset and bytes; ef_gguf_tensor_data points into the mapping. Metadata:
 * key, value type (GGUF codes 0..12: u8 i8 u16 i16 u32 i32 f32 bool string
 * array u64 i64 f64), for arrays the element type and count, and a pointer
 * to the little-endian value (strings: the bytes, count = length; arrays of
 * strings: not decoded). ef_gguf_load_weight loads a tensor as a weight
 * (k = ne0, rows = ne1 * ne2 * ne3) through ef_weight_load. */
EF_API int ef_gguf_open(const char *path, ef_gguf **out, char *err, size_t errlen);
EF_API int ef_gguf_close(ef_gguf *g);
EF_API int ef_gguf_header(const ef_gguf *g, uint32_t *version, uint32_t *alignment, uint64_t *data_start,
                          int64_t *n_tensors, int64_t *n_meta);
EF_API int ef_gguf_tensor(const ef_gguf *g, int64_t i, const char **name, int *type, int *n_dims, int64_t *dims,
                          uint64_t *file_offset, uint64_t *bytes);
EF_API int64_t ef_gguf_find_tensor(const ef_gguf *g, const char *name);
EF_API const void *ef_gguf_tensor_data(const ef_gguf *g, int64_t i);
EF_API int64_t ef_gguf_find_key(const ef_gguf *g, const char *key);
EF_API int ef_gguf_meta(const ef_gguf *g, int64_t i, const char **key, int *type, int *elem_type, uint64_t *count,
                        const void **value);
EF_API int ef_gguf_load_weight(ef_ctx *ctx, const ef_gguf *g, const char *name, ef_weight **out);

/* ---- Tensor-parallel decode collectives (one process per GPU, one node).
 * The reference runs on one device and has none; these replace the
 * all-reduce after each row-parallel projection and the gather of the
 * sharded head's argmax pairs (the TP entry points the drop-in boundary
 * lists: ef_tp_init / ef_allreduce_sum / ef_allgather). Each rank creates
 * its exchange buffers, publishes their CUDA IPC handle (EF_TP_HANDLE_BYTES
 * bytes), and connects to the others' handles (nranks * EF_TP_HANDLE_BYTES
 * bytes in rank order; its own entry is ignored). A call is one kernel per
 * rank that stores its data into every rank's buffer over NVLink and waits
 * for the others' (release / acquire flags): every rank must make the same
 * calls in the same order. A wait longer than timeout_s records the error
 * and turns every later call into a no-op; ef_tp_status reports it
 * (EF_ERR_TIMEOUT). Calls are stream-ordered and may be captured in a CUDA
 * graph. max_bytes bounds one call's data per rank. */
#define EF_TP_MAX_RANKS 8
#define EF_TP_HANDLE_BYTES 64
EF_API int ef_tp_create(ef_ctx *ctx, int rank, int nranks, size_t max_bytes, double timeout_s, ef_tp **out);
EF_API int ef_tp_handle(ef_ctx *ctx, const ef_tp *tp, void *handle_out);
EF_API int ef_tp_connect(ef_ctx *ctx, ef_tp *tp, const void *handles);
/* buf[i] = sum over ranks r = 0, 1, ... (in that order) of rank r's buf[i];
 * the same bits on every rank. */
EF_API int ef_allreduce_sum(ef_ctx *ctx, ef_tp *tp, float *buf, int64_t n);
/* dst[r * bytes ...] = rank r's src (bytes a multiple of 4). */
EF_API int ef_allgather(ef_ctx *ctx, ef_tp *tp, const void *src, int64_t bytes, void *dst);
/* The row-parallel GEMV of a decoder layer with its all-reduce and the norms
 * after it, fused: y = W x (this rank's columns; M tokens, W's rows = the
 * hidden size n) is stored by the GEMV kernel straight into every rank's
 * exchange buffer over NVLink; then o = the sum over ranks (in rank order)
 * and, per token row, x_resid += rmsnorm(o) * w_post (or += o when w_post is
 * NULL) and nrm = rmsnorm(x_resid) * w_next -- the same as ef_gemv followed by
 * ef_allreduce_sum and ef_norm_add_norm, with one launch and one exchange
 * fewer (js/model.js:635-664 for the norms). n a multiple of 128 up to 8192,
 * M <= 16, M * n * 4 bytes within max_bytes. */
EF_API int ef_gemv_allreduce_norm(ef_ctx *ctx, ef_tp *tp, const ef_weight *w, const float *x, int M,
                                  const float *w_post, float *x_resid, const float *w_next, float eps, float *nrm);
/* A row-sharded GEMV with the all-gather of its output, fused: y = W x (this
 * rank's rows of the whole matrix, M tokens) is stored by the GEMV kernel
 * straight into every rank's exchange buffer over NVLink, then yall[r * n + i]
 * = rank r's y[i] (n = M x this rank's rows, the same on every rank) -- the
 * same as ef_gemv followed by ef_allgather, with one launch and one exchange
 * fewer. M <= 16, M * rows * 4 bytes within max_bytes. Shares the fused call
 * counter with ef_gemv_allreduce_norm (calls on one stream, in order). No
 * reference counterpart: the reference is single-device. */
EF_API int ef_gemv_allgather(ef_ctx *ctx, ef_tp *tp, const ef_weight *w, const float *x, int M, float *yall);
EF_API int ef_tp_status(ef_ctx *ctx, const ef_tp *tp);
EF_API int ef_tp_destroy(ef_ctx *ctx, ef_tp *tp);

#ifdef __cplusplus
}
#endif
#endif /* ELFFUSS_CUDA_H */

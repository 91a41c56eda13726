/*
 * tinygiant.h — C ABI of the B200 TinyGiant MoE expert-FFN library
 * (tinygiant_b200/libtinygiant.so).
 *
 * Plain pointers and sizes only.  Every entry point returns TG_OK (0) or a
 * negative TG_E* status; tg_last_error() gives the calling thread's last message.
 *
 * Two groups:
 *  - tg_*   the reference's entry points, same argument order and meaning,
 *           on host pointers; each call copies its inputs to the GPU, runs the
 *           kernels and copies the result back before returning.
 *  - tgx_*  device-resident API: a context owns the model in HBM and runs the
 *           routed MoE decode on caller streams (cudaStream_t passed as void*).
 *
 * Weight format: ggml Q4_0 (18-byte blocks: fp16 d, 16 bytes of nibbles) in the
 * reference's expert-contiguous relayout order gate | up | down
 * (reference tinygiant/relayout.py:142-157).  Activations are quantised to ggml
 * Q8_0 (34-byte blocks).  Row lengths (embed, inter, ncols) must be multiples of
 * 256, as the reference's QK_K-blocked kernels require.
 */
#ifndef TINYGIANT_H
#define TINYGIANT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TG_OK 0
#define TG_EINVAL (-1)        /* bad argument (null pointer, bad dims, index range) */
#define TG_ECUDA (-2)         /* a CUDA call failed; see tg_last_error() */
#define TG_ENOMEM (-3)        /* device or pinned host allocation failed */
#define TG_EUNSUPPORTED (-4)  /* format or configuration not implemented */
#define TG_ENODEV (-5)        /* no CUDA device */
#define TG_ETIMEOUT (-6)      /* a bounded device wait gave up */

/* down_format codes of tg_expert_forward_mixed (reference libtinygiant.c:599-643
 * uses 0 = Q4_K, 1 = f16, 2 = Q6_K; this library adds 3 = all-Q4_0 expert). */
#define TG_FMT_Q4_K 0
#define TG_FMT_F16 1
#define TG_FMT_Q6_K 2
#define TG_FMT_Q4_0 3

const char *tg_last_error(void);
int tg_version(void);
int tg_device_count(void);

/* ===================== reference-shaped entry points (host pointers) ===================== */

/* Q8_0-quantise x[n] (n a multiple of 32) into n/32 ggml blocks of 34 bytes.
 * Replaces the quantiser inside the reference library, csrc/libtinygiant.c:61-89. */
int tg_quantize_q8_0(const float *x, void *out, int n);

/* Q4_0-quantise x[n] into n/32 ggml blocks of 18 bytes (gguf Q4_0.quantize_blocks);
 * the weight format the reference's relayout stores (tinygiant/relayout.py:111-157). */
int tg_quantize_q4_0(const float *x, void *out, long long n);

/* Exact int32 dot of every Q4_0 block of W[nrows][ncols] with the matching Q8_0 block
 * of xq: out[r][b] = sum_j (q4 - 8) * q8.  The integer core of dot_q4k_q8,
 * csrc/libtinygiant.c:104-169 (vdotq_s32 part, lines 135-158). */
int tg_block_dots_q4_0(const uint8_t *W, const void *xq, int32_t *out, int nrows, int ncols);

/* out[r] = W[r] . Q8_0(in).  Q4_0 twin of tg_matmul_q4k, csrc/libtinygiant.c:187-190. */
int tg_matmul_q4_0(const uint8_t *q4_matrix, const float *input, float *output, int nrows, int ncols);

/* out += weight * down(silu(gate . x) * (up . x)), x and h Q8_0-quantised; q4_data is
 * one expert blob gate | up | down.  Q4_0 twin of tg_expert_forward, csrc/libtinygiant.c:555-595. */
int tg_expert_forward_q4_0(const uint8_t *q4_data, const float *input, float *output, float weight,
                           int embed_dim, int inter_dim);

/* csrc/libtinygiant.c:599-643 with separate gate/up/down pointers (the symbol the
 * reference engine calls, tinygiant/engine.py:249-257; bound at tinygiant/_lib.py:40-41).
 * down_format TG_FMT_Q4_K / TG_FMT_F16 / TG_FMT_Q6_K: Q4_K gate and up, down in that
 * format, the reference's formats and float order (see below); TG_FMT_Q4_0: all three
 * matrices Q4_0, this library's decode format.  Other codes return TG_EINVAL. */
int tg_expert_forward_mixed(const uint8_t *gate_q4, const uint8_t *up_q4, const void *down_data,
                            int down_format, const float *input, float *output, float weight,
                            int embed_dim, int inter_dim);

/* ---- the reference library's own formats (csrc/libtinygiant.c) ----
 * Q4_K: 144-byte super-blocks of 256 values (fp16 d, fp16 dmin, 12 bytes of 6-bit
 * sub-block scales and mins, 128 bytes of nibbles); Q6_K: 210-byte super-blocks (ql,
 * qh, int8 scales, fp16 d); activations of Q4_K / Q6_K products are quantised to
 * 256-wide Q8 blocks (scale = amax/127, round-half-even codes).  Float operations
 * follow the reference source in order, each rounded separately (no contraction);
 * results are bit-identical to oracle/tg_ref.c.  Row lengths: multiples of 256 for
 * Q4_K / Q6_K (<= 65536), of 8 for f16 / f32 (<= 32768). */

/* output[r] = row_r . Q8(input), csrc/libtinygiant.c:173-190 (_lib.py:42). */
int tg_matmul_q4k(const uint8_t *q4_matrix, const float *input, float *output, int nrows, int ncols);
/* Q6_K rows, csrc/libtinygiant.c:194-273 (_lib.py:43). */
int tg_matmul_q6k(const uint8_t *q6_matrix, const float *input, float *output, int nrows, int ncols);
/* f16 rows on the unquantised input, csrc/libtinygiant.c:262-296 (_lib.py:46): eight
 * running fused sums (columns v, v + 8, ...) folded (v, v + 4) then pairwise. */
int tg_f16_matvec(const uint16_t *A, const float *x, float *out, int nrows, int ncols);
/* f32 rows, csrc/libtinygiant.c:298-318 (_lib.py:45), same order as tg_f16_matvec. */
int tg_f32_matvec(const float *A, const float *x, float *out, int nrows, int ncols);
/* out = x * scale * weight, scale = 1/sqrtf(sum x^2 / dim + eps) with the sum as four
 * fused chains folded pairwise, csrc/libtinygiant.c:322-340 (_lib.py:44); dim % 4 == 0. */
int tg_rms_norm(const float *x, const float *weight, float *out, int dim, float eps);
/* GQA attention decode of one token, csrc/libtinygiant.c:364-456 (tg_attention_decode,
 * fp32 wq [n_heads*head_dim][embed], wk / wv [n_kv*head_dim][embed], wo
 * [embed][n_heads*head_dim]) and :460-551 (tg_attention_decode_q4: the same matrices
 * with Q4_K wq / wk / wo and f16 wv); called by engine.py:205-226.  q, k, v
 * projections; per-head RMSNorm (eps 1e-6) of q and k; RoPE with the rows of `pos` of
 * rope_cos / rope_sin [positions][head_dim/2]; k and v written to row kv_len of the
 * caches kv_k / kv_v [n_kv][kv_max][head_dim]; query head h attends over kv head
 * h / (n_heads/n_kv), rows 0 .. kv_len; output[embed] = wo . attention (written, not
 * added).  head_dim % 8 == 0 and <= 256; n_heads / n_kv_heads <= 32; Q4_K needs embed
 * and n_heads*head_dim to be multiples of 256. */
int tg_attention_decode(const float *wq, const float *wk, const float *wv, const float *wo,
                        const float *q_norm_w, const float *k_norm_w, float *kv_k, float *kv_v, int kv_len,
                        int kv_max, const float *rope_cos, const float *rope_sin, const float *input, float *output,
                        int embed_dim, int n_heads, int n_kv_heads, int head_dim, int pos);
int tg_attention_decode_q4(const uint8_t *wq_q4, const uint8_t *wk_q4, const uint16_t *wv_f16,
                           const uint8_t *wo_q4, const float *q_norm_w, const float *k_norm_w, float *kv_k,
                           float *kv_v, int kv_len, int kv_max, const float *rope_cos, const float *rope_sin,
                           const float *input, float *output, int embed_dim, int n_heads, int n_kv_heads,
                           int head_dim, int pos);
/* One whole decoder layer, csrc/libtinygiant.c:662-702 (registered by _lib.py:65-74):
 * RMSNorm of x (eps 1e-6) with attn_norm_w, tg_attention_decode (fp32 weights; row
 * kv_len of kv_k / kv_v is written), x += attention output; RMSNorm with ffn_norm_w,
 * then the n_active (<= 64) experts accumulated from zero in order with
 * tg_expert_forward_mixed (gate_ptrs[e], up_ptrs[e], down_ptrs[e], down format
 * down_is_f16[e]: 0 Q4_K, 1 f16, 2 Q6_K, 3 Q4_0, weight expert_weights[e]), x += that
 * sum.  x is updated in place.  The reference's routing stays with the caller, as in
 * the reference. */
int tg_transformer_layer(const float *wq, const float *wk, const float *wv, const float *wo,
                         const float *attn_norm_w, const float *q_norm_w, const float *k_norm_w,
                         const float *ffn_norm_w, float *kv_k, float *kv_v, int kv_len, int kv_max,
                         const float *rope_cos, const float *rope_sin, const uint8_t **gate_ptrs,
                         const uint8_t **up_ptrs, const void **down_ptrs, const int *down_is_f16,
                         const float *expert_weights, int n_active, float *x, int embed_dim, int inter_dim,
                         int n_heads, int n_kv_heads, int head_dim, int pos);
/* output += weight * expert(input) of one all-Q4_K blob gate | up | down,
 * csrc/libtinygiant.c:555-595 (_lib.py:39). */
int tg_expert_forward(const uint8_t *q4_data, const float *input, float *output, float weight,
                      int embed_dim, int inter_dim);
/* output = sum_e weights[e] * expert_e(input), from zero, experts in order (1..64 Q4_K
 * blobs), csrc/libtinygiant.c:647-655 (exported, not bound by the reference's Python). */
int tg_moe_forward(const uint8_t **expert_ptrs, const float *weights, int n_experts, const float *input,
                   float *output, int embed_dim, int inter_dim);

/* output = sum_e weights[e] * expert_e(input), accumulated in e order from zero.
 * Q4_0 twin of tg_moe_forward, csrc/libtinygiant.c:647-655. */
int tg_moe_forward_q4_0(const uint8_t **expert_ptrs, const float *weights, int n_experts,
                        const float *input, float *output, int embed_dim, int inter_dim);

/* Bytes of the fixed device scratch of tg_expert_forward_q4_0_noalloc (per device). */
#define TG_NOALLOC_SCRATCH_BYTES 4194304

/* tg_expert_forward_q4_0 on DEVICE pointers (q4_data 2-byte aligned, input/output
 * 4-byte aligned), enqueued on `stream` (cudaStream_t; NULL = default stream) and
 * returning without waiting for it.  No counterpart in the reference: it exists for
 * callers that cannot let a library allocate (a fully committed HBM budget, or a
 * latency-bound loop where cudaMalloc/cudaFree may stall).  It allocates nothing,
 * on the device or the host; its scratch is a fixed TG_NOALLOC_SCRATCH_BYTES array
 * per device, so an expert needing more (expert bytes rounded up to 256, + 40 * inter/32
 * + 256) is rejected with TG_EINVAL.  The first call on each device sets that scratch
 * up (symbol address, one synchronous copy): make it before any stream capture.
 * That set-up is kept for the life of the process: after a cudaDeviceReset of a device
 * the stored address and table are stale, so do not call this entry point on that
 * device again in the same process.
 * Calls overlapping in time on one device share the scratch and race; order them. */
int tg_expert_forward_q4_0_noalloc(const uint8_t *q4_data, const float *input, float *output, float weight,
                                   int embed_dim, int inter_dim, void *stream);

/* mlock the pages of [addr, addr+len); returns mlock's result (0 or -1), as
 * csrc/libtinygiant.c:761-766 does. */
int tg_mlock(const void *addr, size_t len);

/* posix_madvise(WILLNEED) of the pages of [addr, addr+len), csrc/libtinygiant.c:745-750;
 * returns posix_madvise's result (the reference's is void). */
int tg_prefetch(const void *addr, size_t len);
/* tg_prefetch over count ranges, csrc/libtinygiant.c:752-759; the first nonzero result. */
int tg_prefetch_batch(const void **addrs, const size_t *lens, int count);

/* ===================== device-resident API ===================== */

typedef struct tgx_ctx tgx_ctx;

typedef struct {
    int embed;      /* hidden size H (multiple of 256) */
    int inter;      /* expert intermediate size I (multiple of 256) */
    int n_experts;  /* routed experts per layer E (<= 1024) */
    int top_k;      /* experts per token k (<= 16) */
    int n_layers;   /* MoE layers L */
    float rms_eps;  /* FFN RMSNorm epsilon; <= 0 selects 1e-6 (tinygiant/_constants.py RMS_EPS) */
} tgx_shape;

/* Create a context on `device` holding L x E experts and L routers in HBM.
 * Model shape constants follow tinygiant/_constants.py. */
int tgx_ctx_create(int device, const tgx_shape *shape, tgx_ctx **out);
int tgx_ctx_destroy(tgx_ctx *ctx);

/* Bytes of one expert blob (gate | up | down, Q4_0) for this context's shape. */
size_t tgx_expert_bytes(const tgx_ctx *ctx);

/* Copy n experts (ggml blobs, expert-contiguous as in a layer_NNN.q4.bin file,
 * tinygiant/relayout.py:142-157) into layer `layer` starting at expert `first`.
 * src is host memory (pinned or pageable) unless src_on_device. */
int tgx_load_experts(tgx_ctx *ctx, int layer, int first, int n, const void *src, int src_on_device);

/* tgx_load_experts for blobs already in the row-split layout the kernels read (each
 * matrix row: its Q4_0 blocks' 16-byte nibble groups, then their fp16 scales; a
 * version-4 "rows" relayout stores experts so): a plain copy, no repack. */
int tgx_load_experts_rows(tgx_ctx *ctx, int layer, int first, int n, const void *src, int src_on_device);

/* Read n experts of a layer back as ggml blobs into host memory. */
int tgx_read_experts(tgx_ctx *ctx, int layer, int first, int n, void *dst_host);

/* out_dev += weight * expert(x_dev) for expert `expert` of layer `layer` held in the
 * context: tg_expert_forward_q4_0 (csrc/libtinygiant.c:555-595, the reference's
 * tg_expert_forward) on device memory: Q8_0 of x, gate and up rows, SwiGLU, Q8_0 of h,
 * down rows, enqueued on `stream`.  The first call allocates a pointer table and an h
 * buffer in the context. */
int tgx_expert_forward(tgx_ctx *ctx, int layer, int expert, const float *x_dev, float *out_dev, float weight,
                       void *stream);

/* Set layer `layer`'s router, R[E][embed] fp32 row-major (engine.py:231 `self.routers[i]`). */
int tgx_set_router(tgx_ctx *ctx, int layer, const float *R, int src_on_device);

/* Set layer `layer`'s FFN RMSNorm weight w[embed] (engine.py:229 `self.ffn_norms[i]`; default all 1). */
int tgx_set_ffn_norm(tgx_ctx *ctx, int layer, const float *w, int src_on_device);

/* Fill every expert with Q4_0(N(0, w_sigma)) weights and every router with
 * N(0, r_sigma), generated on the device from `seed` (synthetic benchmark model). */
int tgx_fill_synthetic(tgx_ctx *ctx, uint64_t seed, float w_sigma, float r_sigma);

/* One MoE block on x_dev[embed] in place, as the reference engine runs it
 * (tinygiant/engine.py:229-258, attention excluded): normed = RMSNorm(x) * ffn_norm,
 * idx, w = top-k / softmax of R_layer . normed, x += sum_j w_j * expert_{idx_j}(normed). */
int tgx_moe_layer(tgx_ctx *ctx, int layer, float *x_dev, void *stream);

/* One decode step: all L MoE blocks chained on x_dev[embed], x_{l+1} = x_l + moe_l(norm_l(x_l)).
 * By default one persistent kernel runs all layers (one CTA per SM, weights
 * staged by bulk copies, no grid-wide barriers).  flags: TGX_EAGER launches
 * directly; otherwise the step is replayed from a CUDA graph captured on first
 * use for this x_dev.  TGX_MULTI selects the three-kernels-per-layer path. */
#define TGX_EAGER 1
#define TGX_MULTI 2   /* three kernels per layer instead of the single fused kernel per step */
int tgx_decode_step(tgx_ctx *ctx, float *x_dev, void *stream, int flags);

/* The MoE block for T tokens at once (prefill, or T independent decode streams),
 * in place on x_dev[T][embed]: each token gets exactly what tgx_moe_layer gives it,
 * bit for bit (engine.py:229-258 per token).  Each expert's weights are read once per
 * layer for all the tokens routed to it.  1 <= T <= 65536/top_k.  Grows a scratch
 * buffer in the context on first use of a larger T (cudaMalloc; not during capture). */
int tgx_moe_batched(tgx_ctx *ctx, int layer, float *x_dev, int T, void *stream);

/* All L MoE blocks for T tokens, layer after layer (tgx_moe_batched for l = 0 .. L-1).
 * With the automatic kernel choice and T <= 8, each token runs the fused single-token
 * step instead (the same bits, faster for few tokens). */
int tgx_decode_batched(tgx_ctx *ctx, float *x_dev, int T, void *stream);
/* expert matmul kernels of tgx_moe_batched / tgx_decode_batched: 0 auto (tensor cores,
 * tcgen05, when experts average >= 16 pairs), 1 dp4a, 2 tensor cores; these give the same
 * bits.  3: tensor cores with the fast epilogue (one fma per Q4_0 block: the same exact
 * int32 block dots, another fp32 summation order), within the reference's
 * accumulation-order tolerance rather than bit-identical.  tgx_sync_status reports an
 * expired bounded wait of the tensor-core kernels. */
int tgx_set_batched_kernels(tgx_ctx *ctx, int kernels);

/* The MoE block of layer `layer` over a given list of experts (routing decided by the
 * caller, e.g. a host-tier cache): x += sum_j weights[j] * expert_j((x * scale) * ffn_norm),
 * scale the layer's RMSNorm scale of x.  experts: host array of n DEVICE pointers to
 * expert blobs in the library's row-split layout (tgx_repack_experts); weights: host
 * array of n floats; 1 <= n <= 16.  The expert-forward order of engine.py:238-258. */
int tgx_experts_forward(tgx_ctx *ctx, int layer, const void *const *experts, const float *weights, int n,
                        float *x_dev, void *stream);

/* Convert n ggml expert blobs (relayout order, device memory) into the row-split
 * layout the kernels read; raw_dev and dst_dev must not overlap. */
int tgx_repack_experts(tgx_ctx *ctx, const void *raw_dev, void *dst_dev, int n, void *stream);

/* Synchronise the context's device and report whether a bounded wait inside the
 * fused decode kernel expired since the last call (TG_ETIMEOUT; the kernel's
 * cross-block state is then reset).  TG_OK otherwise. */
int tgx_sync_status(tgx_ctx *ctx);

/* Limit of every bounded wait inside the fused decode kernel, in SM cycles (0: the
 * default, 2e9, about one second at the B200's clock; else >= 1000).  A wait that runs
 * out makes the kernel record the failure and return; tgx_sync_status then reports
 * TG_ETIMEOUT and resets the kernel's state, and the context stays usable.  Applies to
 * launches made after the call (the context's captured decode graph is dropped and
 * recaptured); graphs captured elsewhere keep the limit they were captured with. */
int tgx_set_wait_limit(tgx_ctx *ctx, long long cycles);

/* Failure injection for tests, on the host: the fused kernel's launches after this
 * call wait for n (0..16) router-sum contributions that no block sends, as if n blocks
 * never arrived, so its first routing wait runs out at the wait limit.  n = 0 restores
 * normal operation.  Nothing faults: see tgx_set_wait_limit. */
int tgx_fused_inject_missing(tgx_ctx *ctx, int n);

/* Diagnostics of the fused path: its control words (epoch, finished blocks, error
 * stage, error detail = (layer << 20) | (entry << 8) | observed count) and the first
 * n_acc words of its routing accumulators ([L][8 copies][E + 1] count-tagged words).
 * Synchronises the device. */
int tgx_fused_debug(tgx_ctx *ctx, uint32_t *ctl4, uint64_t *acc, size_t n_acc);

/* One eager fused decode step on x_dev that also records, per layer and CTA, phase
 * stamps into stamps_host[L][ctas][32]: slots 0..15 %globaltimer (ns), slots 16..31
 * the SM's clock64 at the same events.  Slots: 0 routing and x seen, 1 gate/up copies
 * issued, 2 input quantised, 3 gate/up published, 4 early h gathered, 5 down data
 * landed, 6 down rows done, 7 next-layer sums sent, 8 first gate/up unit landed,
 * 9 top-k done, 10 down copies issued, 11 late h gathered (0 where a CTA has no such
 * event). */
int tgx_fused_trace(tgx_ctx *ctx, float *x_dev, uint64_t *stamps_host, void *stream);

/* The fused path's launch geometry: CTAs (0 when the shape runs on the
 * multi-kernel path), dynamic shared memory per CTA, weight staging bytes per CTA. */
int tgx_fused_info(tgx_ctx *ctx, int *ctas, int *smem_bytes, int *arena_bytes);

/* Routing chosen by the last tgx_moe_layer / tgx_decode_step for `layer`
 * (idx[k] in ascending-logit order, w[k], logits[E]); any pointer may be NULL.
 * Synchronises the context's device. */
int tgx_last_routing(tgx_ctx *ctx, int layer, int32_t *idx, float *w, float *logits);

/* ===================== experts sharded over devices ===================== */

/* Expert parallelism: rank r of G holds experts [r*E/G, (r+1)*E/G) of every layer
 * (n_experts % G == 0); routers and FFN norms are replicated.  One MoE layer for T
 * tokens x_dev[T][embed] (tinygiant/engine.py:229-258 per token):
 *   tgx_ep_moe_partial(ep, layer, x, T, y, s)  every rank: the same routing, then
 *       y[(t, j)][embed] for the pairs (token t, slot j) it owns, 0 for the others
 *       (y: tgx_ep_y_floats(ep, T) floats, caller-owned);
 *   sum y over the ranks (an NCCL all-reduce, or any exact sum: each element has one
 *       nonzero contribution);
 *   tgx_ep_combine(ep, x, T, y, s)  x[t] += sum_j w[t][j] * y[(t, j)] in slot order.
 * The result equals tgx_moe_batched on one device with all experts, bit for bit.
 * n_shared = 1 adds a shared expert (DeepSeek-V3-like): slot k of every token with
 * weight 1, replicated on every rank and computed, per token, by the rank holding the
 * fewest of that token's routed experts (ties to rank (t + i) mod G, smallest i).
 * The first partial call for a larger T allocates scratch (make it before any graph
 * capture). */
typedef struct tgx_ep tgx_ep;
int tgx_ep_create(int device, const tgx_shape *shape, int n_shared, int ep_rank, int ep_size, tgx_ep **out);
int tgx_ep_destroy(tgx_ep *ep);
int tgx_ep_expert_range(const tgx_ep *ep, int *first, int *n);
/* experts [first, first + n) of a layer (global ids inside this rank's range), ggml blobs */
int tgx_ep_load_experts(tgx_ep *ep, int layer, int first, int n, const void *src, int src_on_device);
/* the shared expert of a layer (n_shared = 1), one ggml blob gate | up | down */
int tgx_ep_load_shared(tgx_ep *ep, int layer, const void *src, int src_on_device);
/* read expert e of a layer (a local routed id, or n_experts for the shared expert) back
 * as one ggml blob into host memory */
int tgx_ep_read_expert(tgx_ep *ep, int layer, int e, void *dst_host);
int tgx_ep_set_router(tgx_ep *ep, int layer, const float *R, int src_on_device);
int tgx_ep_set_ffn_norm(tgx_ep *ep, int layer, const float *w, int src_on_device);
/* the values tgx_fill_synthetic gives the same experts of a full model */
int tgx_ep_fill_synthetic(tgx_ep *ep, uint64_t seed, float w_sigma, float r_sigma);
size_t tgx_ep_y_floats(const tgx_ep *ep, int T);
int tgx_ep_moe_partial(tgx_ep *ep, int layer, const float *x_dev, int T, float *y_dev, void *stream);
int tgx_ep_combine(tgx_ep *ep, float *x_dev, int T, const float *y_dev, void *stream);
/* expert matmul kernels of the partial step: 0 auto (tensor cores when experts average
 * >= 16 pairs), 1 dp4a, 2 tensor cores (tcgen05); these give the same bits.  3: tensor
 * cores with the fast epilogue, as in tgx_set_batched_kernels. */
int tgx_ep_set_kernels(tgx_ep *ep, int kernels);
/* synchronise `stream`; TG_ETIMEOUT (and the flag cleared) if a tensor-core kernel's
 * bounded wait expired since the last call */
int tgx_ep_status(tgx_ep *ep, void *stream);

/* The exchange over NVLink instead of a collective.  Every rank: tgx_ep_p2p_init(ep,
 * T_max, handle) allocates its exchange region and returns its CUDA IPC handle
 * (tgx_ep_p2p_handle_bytes() bytes); the caller gathers all ranks' handles in rank order
 * (any host-side exchange) and passes them to tgx_ep_p2p_connect.  Then one call per
 * layer, tgx_ep_moe_layer_p2p(ep, layer, x, T, stream): the partial step writes this
 * rank's (token, slot) sums into its own region (layer parity double buffer), one kernel
 * copies each of those rows (contiguous) into every peer's region over NVLink and, in its
 * last CTA, publishes this rank's epoch to every rank's flags, and the combine waits
 * (bounded, ~1 s) for all ranks' flags before adding in slot order.  All
 * ranks must run the same layers in the same order; bit-identical to the all-reduce path.
 * No collective library is involved; capturable in a CUDA graph (after the first call for
 * the largest T).  tgx_ep_p2p_status reports an expired wait (TG_ETIMEOUT). */
size_t tgx_ep_p2p_handle_bytes(void);
int tgx_ep_p2p_init(tgx_ep *ep, int T_max, void *handle_out);
int tgx_ep_p2p_connect(tgx_ep *ep, const void *handles);
int tgx_ep_moe_layer_p2p(tgx_ep *ep, int layer, float *x_dev, int T, void *stream);
int tgx_ep_p2p_status(tgx_ep *ep, void *stream);
/* close this rank's mappings of the peers' regions (after its last layer), those of the
 * fused decode too.  A region may be freed (tgx_ep_destroy) only once every rank has
 * disconnected: put a barrier between the two. */
int tgx_ep_p2p_disconnect(tgx_ep *ep);

/* The whole decode step of one token in ONE persistent kernel per rank (the one-device
 * tgx_decode_step's kernel restricted to the local experts): every rank routes every
 * layer, computes the gate/up and down rows of the slots whose expert it holds, and
 * stores each output row's per-slot value into every rank's y buffer over NVLink as a
 * tagged 64-bit word; each rank then combines all k slots in slot order, so every rank
 * ends every layer with the same hidden state, bit-identical to tgx_decode_step
 * (tinygiant/engine.py:229-258 per layer, attention excluded).  No shared expert.
 *   tgx_ep_fused_init(ep, handle)     every rank: state, plan, y buffer; its CUDA IPC
 *                                     handle (tgx_ep_p2p_handle_bytes() bytes) out
 *   tgx_ep_fused_connect(ep, handles) all ranks' handles in rank order
 *   tgx_ep_decode_step(ep, x, stream) every rank, the same x (device f32[embed]), in place;
 *                                     all ranks take the same steps
 *   tgx_ep_fused_trace                the same with per-CTA phase stamps ([L][CTAs][32]
 *                                     u64: globaltimer ns at slots 0..15, clock64 at 16..31)
 * Every wait is bounded (tgx_ep_set_wait_limit, SM cycles; 0 = ~1 s); tgx_ep_fused_status
 * reports an expired one (TG_ETIMEOUT).  To recover, every rank calls
 * tgx_ep_fused_reset(ep, e) with the same e above every rank's tgx_ep_fused_epoch. */
int tgx_ep_fused_init(tgx_ep *ep, void *handle_out);
int tgx_ep_fused_connect(tgx_ep *ep, const void *handles);
int tgx_ep_decode_step(tgx_ep *ep, float *x_dev, void *stream);
int tgx_ep_fused_trace(tgx_ep *ep, float *x_dev, uint64_t *stamps_host, void *stream);
int tgx_ep_fused_info(tgx_ep *ep, int *ctas, int *smem_bytes);
int tgx_ep_set_wait_limit(tgx_ep *ep, long long cycles);
int tgx_ep_fused_last_routing(tgx_ep *ep, int layer, int32_t *idx, float *w);
int tgx_ep_fused_status(tgx_ep *ep, void *stream);
int tgx_ep_fused_epoch(tgx_ep *ep, unsigned *epoch);
int tgx_ep_fused_reset(tgx_ep *ep, unsigned epoch);

/* Token dispatch: every rank holds its OWN tokens (not a copy of all of them).  Per layer:
 *   tgx_ep_dispatch(ep, layer, x, T, send, counts, s)  route this rank's T tokens
 *       (x: device f32[T][embed]); one record of tgx_ep_record_bytes(ep) bytes per (token,
 *       slot) pair into send (device, T * (top_k + n_shared) records), grouped by
 *       destination rank in rank order: a routed slot goes to its expert's holder, the
 *       shared slot stays on this rank; counts (device int[ep_size]) = records per rank.
 *       A record is a 16-byte header (int32 expert id, int32 pair index t * slots + j at
 *       the sender, 0, 0) and the token's Q8_0 row in ggml form.
 *   (caller) exchange the counts, then the records (an all-to-all: rank q's group of
 *       this rank's send goes to rank q, received groups in source-rank order)
 *   tgx_ep_dispatch_experts(ep, layer, recv, n, y, s)  the n received records' expert
 *       FFNs, y: device f32[n][embed] in record order
 *   (caller) the reverse all-to-all of y, so each rank gets back one row per record it
 *       sent, in its send order
 *   tgx_ep_dispatch_combine(ep, x, T, y_back, s)  x[t] += sum_j w[t][j] * y[(t, j)] in
 *       slot order.
 * Bit-identical to the single-device batched path (tinygiant/engine.py:229-258 per
 * token).  tgx_ep_status reports an expired wait of the tensor-core expert kernels. */
size_t tgx_ep_record_bytes(const tgx_ep *ep);
/* The same dispatch device-side, with no host sync and capturable in a CUDA graph: every
 * rank tgx_ep_dispatch_p2p_init(ep, T_max, handle) (its region: records in, y rows back,
 * flags; CUDA IPC handle of tgx_ep_p2p_handle_bytes() bytes), the caller gathers all
 * handles in rank order, tgx_ep_dispatch_p2p_connect; then per layer
 * tgx_ep_moe_layer_dispatch_p2p(ep, layer, x, T, s) on every rank (1 <= T <= T_max, its
 * own tokens): records are stored into their destinations' regions over NVLink, counts
 * travel in the flags, y rows come back the same way, and the combine adds in slot order.
 * Bounded waits (~1 s; tgx_ep_dispatch_p2p_status reports TG_ETIMEOUT); after one the
 * ranks must set up again.  tgx_ep_dispatch_p2p_counts: records received and sent by the
 * last call.  tgx_ep_p2p_disconnect closes these mappings too. */
int tgx_ep_dispatch_p2p_init(tgx_ep *ep, int T_max, void *handle_out);
int tgx_ep_dispatch_p2p_connect(tgx_ep *ep, const void *handles);
int tgx_ep_moe_layer_dispatch_p2p(tgx_ep *ep, int layer, float *x_dev, int T, void *stream);
int tgx_ep_dispatch_p2p_counts(tgx_ep *ep, int *received, int *sent);
int tgx_ep_dispatch_p2p_status(tgx_ep *ep, void *stream);
int tgx_ep_dispatch(tgx_ep *ep, int layer, const float *x_dev, int T, void *send_dev, int *counts_dev, void *stream);
int tgx_ep_dispatch_experts(tgx_ep *ep, int layer, const void *recv_dev, int n_recv, float *y_dev, void *stream);
int tgx_ep_dispatch_combine(tgx_ep *ep, float *x_dev, int T, const float *y_back_dev, void *stream);

/* ===================== the reference's formats on device pointers ===================== */

/* Device bytes of a rows x cols matrix of format fmt (0 Q4_K, 1 f16, 2 Q6_K, 4 f32;
 * the same as the reference's byte size), or 0 for a shape the kernels do not take. */
size_t tgx_kq_matrix_bytes(int fmt, long long rows, int cols);
/* Convert a matrix in the reference's byte layout (src_dev) into the kernels' device
 * layout (dst_dev, same size, 16-byte aligned, not aliasing src): Q6_K blocks are
 * split into 208-byte bodies followed by the fp16 d of every block; the other formats
 * are copied unchanged. */
int tgx_kq_prepare(int fmt, const void *src_dev, void *dst_dev, long long rows, int cols, void *stream);
/* y_dev[rows] = W . x (tg_matmul_q4k / tg_matmul_q6k / tg_f16_matvec / tg_f32_matvec on
 * device memory; W in device layout, all pointers 16-byte aligned). */
int tgx_kq_matvec(int fmt, const void *W_dev, const float *x_dev, float *y_dev, int rows, int cols, void *stream);
/* tg_rms_norm on device memory (x, w, out 16-byte aligned; dim % 4 == 0), e.g. the
 * final norm before the output projection (engine.py:261-265). */
int tgx_rms_norm(const float *x_dev, const float *w_dev, float *out_dev, int dim, float eps, void *stream);
/* Scratch bytes of tgx_kq_experts_forward for n experts (0 for a bad shape). */
size_t tgx_kq_scratch_bytes(int n, int embed, int inter);

/* flags of tgx_kq_experts_forward: the kernel before this call on `stream` is a
 * tgx_kq_experts_forward that writes none of this call's weights or pointer arrays
 * (only x / out): this call's weight fetch then starts before that kernel ends. */
#define TGX_KQ_CHAINED 1

/* n experts at once (tg_moe_forward / tg_expert_forward_mixed on device memory):
 * out = (accumulate ? out : 0) + sum_e w[e] * down_e(silu(gate_e . x) * (up_e . x)),
 * experts in order; out may equal x.  gate_dev / up_dev / down_dev: DEVICE arrays of n
 * device pointers (Q4_K gate and up; down in down_format 0 / 1 / 2, device layout);
 * w_dev: n floats.  scratch: tgx_kq_scratch_bytes(n, embed, inter) bytes, 256-byte
 * aligned, zero-filled before its first use; every call leaves it ready for the next
 * (of any shape that fits it), and calls sharing it must be ordered on one stream.  Allocates nothing; two kernel
 * launches on `stream`, the second a programmatic dependent of the first. */
int tgx_kq_experts_forward(const void *const *gate_dev, const void *const *up_dev, const void *const *down_dev,
                           int down_format, int n, const float *w_dev, const float *x_dev, float *out_dev,
                           int embed, int inter, int accumulate, void *scratch, size_t scratch_bytes, int flags,
                           void *stream);

/* tg_attention_decode (q4 = 0) / tg_attention_decode_q4 (q4 = 1) on device memory:
 * every pointer is a device pointer (16-byte aligned), the caches [n_kv][kv_max][head_dim]
 * stay resident, `output` is written.  scratch: tgx_attention_scratch_bytes(n_heads,
 * n_kv_heads, head_dim, kv_max) bytes.  Seven kernel launches on `stream` (three
 * projections, norm + RoPE + append, scores, softmax + V, output projection); allocates
 * nothing.  kv_max <= 32768. */
size_t tgx_attention_scratch_bytes(int n_heads, int n_kv_heads, int head_dim, int kv_max);
int tgx_attention_decode(int q4, const void *wq, const void *wk, const void *wv, const void *wo,
                         const float *q_norm_w, const float *k_norm_w, float *kv_k, float *kv_v, int kv_len,
                         int kv_max, const float *rope_cos, const float *rope_sin, const float *input, float *output,
                         int embed_dim, int n_heads, int n_kv_heads, int head_dim, int pos, void *scratch,
                         size_t scratch_bytes, void *stream);

/* ===================== device-resident attention and the whole decode layer ===================== */

/* The attention half of a decode layer for an n_layers model (engine.py:199-226,
 * tinygiant/engine.py's _forward_c): per layer wq, wk, wv, wo (q4: Q4_K / f16 as in
 * tg_attention_decode_q4, else fp32), the q / k norm weights and the attention RMSNorm
 * weight; rope tables [kv_max][head_dim/2] (default: base 1e6, evaluated in double);
 * KV caches [n_layers][2][n_kv][kv_max][head_dim] fp32 (zero at creation); and a
 * device position word = rows already cached, 0 at creation. */
typedef struct tgx_attn tgx_attn;
int tgx_attn_create(int device, int q4, int n_layers, int embed_dim, int n_heads, int n_kv_heads, int head_dim,
                    int kv_max, float eps, tgx_attn **out);
int tgx_attn_destroy(tgx_attn *a);
/* Device bytes of one layer's four matrices (each in a 256-byte aligned slot). */
size_t tgx_attn_layer_bytes(const tgx_attn *a);
/* Copy one layer's weights in; any pointer may be NULL to keep that part. */
int tgx_attn_set_layer(tgx_attn *a, int layer, const void *wq, const void *wk, const void *wv, const void *wo,
                       const float *q_norm_w, const float *k_norm_w, const float *attn_norm_w, int src_on_device);
/* Replace the rope tables with the first kv_max rows of cos / sin [n_pos][head_dim/2]
 * (the reference's build_rope_cache). */
int tgx_attn_set_rope(tgx_attn *a, const float *rope_cos, const float *rope_sin, int n_pos, int src_on_device);
/* Set the position (rows cached; 0 starts a new sequence, engine.py:145-148).  Synchronises. */
int tgx_attn_set_pos(tgx_attn *a, int pos);
/* Synchronise, report the device position, and TG_EINVAL if a step ran at a position
 * outside the cache since the last call (such a step writes nothing). */
int tgx_attn_status(tgx_attn *a, int *pos);
/* Device pointers of layer `layer`'s caches [n_kv][kv_max][head_dim]. */
int tgx_attn_kv(tgx_attn *a, int layer, float **kv_k_dev, float **kv_v_dev);
/* Synchronise and copy layer `layer`'s caches [n_kv][kv_max][head_dim] to host memory
 * (either pointer may be NULL). */
int tgx_attn_read_kv(tgx_attn *a, int layer, float *kv_k_host, float *kv_v_host);
/* x_dev[embed] += attention(RMSNorm(x) * attn_norm) of layer `layer` at the device
 * position (engine.py:203-226): tg_rms_norm then the tg_attention_decode step with
 * kv_len = pos; the position does not move. */
int tgx_attn_layer(tgx_attn *a, int layer, float *x_dev, void *stream);
/* pos += 1 on the device (after the last layer of a token). */
int tgx_attn_advance(tgx_attn *a, void *stream);
/* One decode token through every layer: x += attention_l(x), then the MoE block of
 * layer l (tgx_moe_layer on `moe`; NULL: attention only), for l = 0 .. n_layers - 1,
 * then pos += 1.  Replayed from a CUDA graph captured on first use for this x_dev and
 * moe (flags TGX_EAGER: launched directly).  TG_EINVAL once the cache is full. */
int tgx_decode_token(tgx_attn *a, tgx_ctx *moe, float *x_dev, void *stream, int flags);

#ifdef __cplusplus
}
#endif

#endif /* TINYGIANT_H */

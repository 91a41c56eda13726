/*
 * tg_ref.h — CPU oracle for TinyGiant's MoE expert-FFN hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, always as the checker (or the timed CPU arm).
 *
 * Block formats (ggml, pinned by gguf.quants 0.19.0):
 *   Q4_0: 18 B per 32 weights = fp16 d | u8 qs[16]; element j   = (qs[j] & 15) - 8,
 *                                                  element j+16 = (qs[j] >> 4) - 8.
 *   Q8_0: 34 B per 32 values  = fp16 d | i8 qs[32].
 *
 * Arithmetic modes (argument `mode` below):
 *   TG_REF_ORDER (0)  the reference's order: block sums accumulated sequentially
 *                     (csrc/libtinygiant.c:104-169, 173-185), libm expf in SiLU
 *                     (libtinygiant.c:580-583) and in the router softmax.
 *   TG_MIRROR   (1)   the device kernels' fixed order: each row dot is split over
 *                     32 lanes (lane L sums blocks L, L+32, ...) and reduced with
 *                     an xor butterfly; SiLU/softmax use tg_expf (Cody-Waite + Taylor).
 *   TG_FAST_MMA (2)   as TG_MIRROR, except each row dot: the tensor-core kernels'
 *                     fast epilogue, one accumulator taking
 *                     acc = fmaf((float)sumi, d_w * d_x, acc) block after block, the
 *                     blocks in lane-class order (classes in 5-bit-reversed order
 *                     0, 16, 8, 24, ..., each class's blocks l, l + 32, ... ascending).
 * Routing arithmetic is the same in all modes except for exp: logits are exact
 * fixed-point sums of fp32 products (see ref_router_logits).
 */
#ifndef TG_REF_H
#define TG_REF_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { TG_REF_ORDER = 0, TG_MIRROR = 1, TG_FAST_MMA = 2 };
enum { REF_QK = 32, REF_Q4_0_BYTES = 18, REF_Q8_0_BYTES = 34 };

float    ref_f16_to_f32(uint16_t h);
uint16_t ref_f32_to_f16(float f);
float    ref_expf(float x);                 /* tg_expf, the shared exp definition */

void ref_quantize_q8_0(const float *x, uint8_t *out, int64_t n);
void ref_quantize_q4_0(const float *x, uint8_t *out, int64_t n);
void ref_dequantize_q8_0(const uint8_t *q, float *out, int64_t n);
void ref_dequantize_q4_0(const uint8_t *q, float *out, int64_t n);

int32_t ref_block_dot_q4_0_q8_0(const uint8_t *wblk, const uint8_t *xblk);
void    ref_block_dots(const uint8_t *W, const uint8_t *xq, int32_t *out,
                       int rows, int cols);
float   ref_row_dot(const uint8_t *wrow, const uint8_t *xq, int nblocks, int mode);
void    ref_matvec_q4_0(const uint8_t *W, const uint8_t *xq, float *y,
                        int rows, int cols, int mode);

float   ref_silu_mul(float g, float u, int mode);

/* out[i] += w * y[i], y = down(silu(gate.xq) * (up.xq)) with h requantised. */
void ref_expert_forward(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                        const float *x, float *out, float w,
                        int embed, int inter, int mode);

/* Same, also returning the stage outputs (for stage-wise tests). Any of the
 * stage pointers may be NULL. */
void ref_expert_forward_stages(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                               const float *x, float *out, float w,
                               int embed, int inter, int mode,
                               uint8_t *xq_out, float *g_out, float *u_out,
                               float *h_out, uint8_t *hq_out, float *y_out);

void ref_router_logits(const float *R, const float *x, int n_experts, int hidden,
                       float *logits);
void ref_topk_softmax(const float *logits, int n_experts, int k,
                      int32_t *idx, float *w, int mode);

/* One MoE block (engine.py:229-258 without the norms): route x, run the top-k
 * experts of `layer_blob` (experts contiguous, each gate|up|down Q4_0, stride
 * expert_bytes), and add the weighted sum to x in place.  idx/w/logits may be NULL. */
void ref_moe_layer(const uint8_t *layer_blob, size_t expert_bytes, const float *R,
                   float *x, int n_experts, int k, int embed, int inter, int mode,
                   int32_t *idx, float *w, float *logits);

/* FFN RMSNorm scale 1/sqrtf(ss/dim + eps) with ss summed exactly in fixed point. */
float ref_rms_scale(const float *x, int dim, float eps);

/* The engine's MoE block: normed = RMSNorm(x)*normw (normw NULL = ones), route
 * and run the experts on normed, x += weighted expert sum (engine.py:229-258). */
void ref_moe_block(const uint8_t *layer_blob, size_t expert_bytes, const float *R, const float *normw,
                   float eps, float *x, int n_experts, int k, int embed, int inter, int mode,
                   int32_t *idx, float *w, float *logits);

/* Decode step: n_layers chained MoE blocks, x_{l+1} = x_l + moe_l(norm_l(x_l)). */
void ref_decode_step(const uint8_t *const *layer_blobs, const float *const *routers,
                     const float *const *norms /* [n_layers] or NULL */, float eps,
                     int n_layers, float *x, int n_experts, int k, int embed, int inter,
                     int mode, int32_t *idx_out /* [n_layers*k] or NULL */);

/* Batched tokens: T independent tokens through one MoE block (x is [T][embed]). */
void ref_quantize_q8k(const float *x, uint8_t *out, int64_t n);
float ref_dot_q4k(const uint8_t *q4, const uint8_t *xq, int bpr);
float ref_dot_q6k(const uint8_t *q6, const uint8_t *xq, int bpr);
float ref_dot_f16(const uint16_t *row, const float *x, int ncols);
float ref_dot_f32(const float *row, const float *x, int ncols);
void ref_rms_norm_k(const float *x, const float *w, float *out, int dim, float eps);
void ref_matvec_k(const void *W, int fmt, const float *x, float *y, int rows, int cols);
void ref_expert_forward_k(const uint8_t *gate, const uint8_t *up, const void *down, int down_format,
                          const float *x, float *out, float w, int embed, int inter, int mode);
void ref_moe_block_batched_shared(const uint8_t *layer_blob, size_t expert_bytes, const float *R,
                                  const float *normw, float eps, float *x, int T, int n_experts, int k, int embed,
                                  int inter, int mode, int n_threads, const uint8_t *shared_blob);
void ref_moe_block_batched(const uint8_t *layer_blob, size_t expert_bytes, const float *R, const float *normw,
                           float eps, float *x, int T, int n_experts, int k, int embed, int inter, int mode,
                           int n_threads);
void ref_moe_layer_batched(const uint8_t *layer_blob, size_t expert_bytes, const float *R,
                           float *x, int T, int n_experts, int k, int embed, int inter,
                           int mode, int n_threads);

/* Multi-threaded decode step for the CPU baseline (OpenMP over rows). */
void ref_decode_step_mt(const uint8_t *const *layer_blobs, const float *const *routers,
                        const float *const *norms, float eps, int n_layers, float *x, int n_experts, int k,
                        int embed, int inter, int mode, int n_threads);

/* Attention decode of one token (csrc/libtinygiant.c:344-551): q4 = 0 all-fp32 weights
 * (tg_attention_decode), q4 = 1 Q4_K wq/wk/wo and f16 wv (tg_attention_decode_q4).
 * Appends k, v at row kv_len of the caches [n_kv][kv_max][head_dim]; writes output. */
void ref_rope(float *x, int n_heads, int head_dim, const float *cos_row, const float *sin_row);
void ref_attention_decode(int q4, const void *wq, const void *wk, const void *wv, const void *wo,
                          const float *q_norm_w, const float *k_norm_w, float *kv_k, float *kv_v, int kv_len,
                          int kv_max, const float *rope_cos, const float *rope_sin, const float *input,
                          float *output, int embed, int n_heads, int n_kv, int head_dim, int pos, int mode);

/* Seeded synthetic data: splitmix64 stream -> N(0, sigma) floats (Box-Muller). */
void ref_fill_normal(float *out, int64_t n, uint64_t seed, float sigma);

#ifdef __cplusplus
}
#endif
#endif

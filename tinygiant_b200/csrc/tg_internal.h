// tg_internal.h — launchers shared between the kernel and C-ABI translation units.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "tg_layout.h"

namespace tg {

// ggml Q4_0 rows -> row-split rows (same bytes, same size); src and dst may not alias.
cudaError_t launch_repack_rows(const uint8_t* src, uint8_t* dst, long long nrows, int nb,
                               cudaStream_t s);
// row-split rows -> ggml Q4_0 rows.
cudaError_t launch_unpack_rows(const uint8_t* src, uint8_t* dst, long long nrows, int nb,
                               cudaStream_t s);

// f32[n] -> activation form (and, if ggml != null, ggml Q8_0 blocks).
cudaError_t launch_quantize_act(const float* x, int n, ActView a, uint8_t* ggml, cudaStream_t s);
// ggml Q8_0 blocks -> activation form.
cudaError_t launch_q8_0_to_act(const uint8_t* ggml, int nb, ActView a, cudaStream_t s);
// f32[n] -> ggml Q4_0 blocks.
cudaError_t launch_quantize_q4_0(const float* x, long long n, uint8_t* out, cudaStream_t s);

// y[r] = row_r . x  (row-split weights, activation form input)
cudaError_t launch_matvec(const uint8_t* W, ActView x, float* y, int rows, int nb, cudaStream_t s);
// exact int32 block dots sumi[r][b]
cudaError_t launch_block_dots(const uint8_t* W, ActView x, int32_t* out, int rows, int nb,
                              cudaStream_t s);

// Router: logits, top-k, softmax weights and the chosen experts' base pointers.
// acc: int64[E] zeroed accumulators, counter: zeroed uint; both are left zeroed.
// Routing of the normed input: x * normw * scale, scale = RMSNorm scale of x (written
// to scale_out for the gate/up kernel).  acc: int64[E + 1] zeroed; left zeroed.
cudaError_t launch_router_topk(const float* R, const float* x, const float* normw, float eps, int E, int H,
                               int k, long long* acc, unsigned* counter, float* logits, int* idx,
                               float* w, float* scale_out, const uint8_t* layer_base, size_t expert_bytes,
                               const uint8_t** expert_ptrs, cudaStream_t s);

// Grouped gate/up + SwiGLU + Q8_0 requant of h for k experts.
// experts: device array of k expert bases (row-split layout).
// hq: k activation blocks of I/32 each, laid out expert after expert (act_bytes(nbI) each).
// h_dbg (optional): f32 [k][I].
// x is quantised as is, or as (x * *scale) * normw when scale is not null.
cudaError_t launch_gateup(const uint8_t* const* experts, int k, const float* x, const float* normw,
                          const float* scale, Geom g, uint8_t* hq, float* h_dbg, float* gu_dbg,
                          cudaStream_t s);

// Down projections of k experts + weighted combine, per output row r:
//   acc = accumulate ? out[r] : 0;  for j: acc = acc + w[j]*y_j[r]
//   out[r] = resid ? resid[r] + acc : acc
// w: device float[k] (or null: use w_host_scalar for k == 1).
cudaError_t launch_down_combine(const uint8_t* const* experts, int k, const uint8_t* hq,
                                const float* w, float w_scalar, Geom g, const float* resid,
                                float* out, int accumulate, float* y_dbg, cudaStream_t s);

// out[i] ~ N(0, sigma); value i depends only on (seed, base + i); base must be even.
cudaError_t launch_fill_normal(float* out, long long n, unsigned long long seed, unsigned long long base,
                               float sigma, cudaStream_t s);

// Synthetic Q4_0 experts N(0, sigma) written directly in row-split form (value index =
// base + position in the f32 expert tensors, so a weight does not depend on the launch split).
cudaError_t launch_fill_experts_q4_0(uint8_t* dst, int n_experts, Geom g, unsigned long long seed,
                                     unsigned long long base, float sigma, cudaStream_t s);

// out[c][r] = in[r][c] (fp32, rows x cols -> cols x rows).
cudaError_t launch_transpose(const float* in, float* out, int rows, int cols, cudaStream_t s);

// *scale = RMSNorm scale of x[H] (exact fixed-point sum of squares), one CTA.
cudaError_t launch_rms_scale(const float* x, int H, float eps, float* scale, cudaStream_t s);

// Raise dynamic shared-memory limits for the shapes a context uses (call before capture).
cudaError_t prepare_kernels(Geom g, int k);

// The MoE block for T tokens at once, in place on X[T][H] (tg_batched.cu).  layer:
// the layer's row-split experts; R: its router [E][H]; scratch of at
// least batched_scratch_bytes(g, E, k, T); idx_out / w_out / logits_out optional
// ([T][k], [T][k], [T][E]).  batched_smem_bytes: the largest dynamic shared memory
// a CTA of the path needs.
// kernels: which expert matmuls run — BATCHED_AUTO picks the tensor-core path
// (tg_tc.cu) when experts average >= 16 pairs, BATCHED_DP4A / BATCHED_MMA force one;
// those give the same bits.  BATCHED_MMA_FAST: the tensor cores with the one-fma
// epilogue, within the accumulation-order tolerance instead of bit-identical.
constexpr int BATCHED_AUTO = 0, BATCHED_DP4A = 1, BATCHED_MMA = 2, BATCHED_MMA_FAST = 3;
size_t batched_scratch_bytes(const Geom& g, int E, int k, int T);
size_t batched_smem_bytes(const Geom& g);
cudaError_t launch_moe_batched(const uint8_t* layer, Geom g, const float* R, const float* normw, float eps, int E,
                               int k, float* X, int T, void* scratch, size_t scratch_bytes, int* idx_out,
                               float* w_out, float* logits_out, int kernels, cudaStream_t s);
// Tensor-core expert matmuls (tg_tc.cu) over the grouped pairs: down = 0 gives the gate
// sums (out0) and up sums (out1) [pair][I] from the tokens' Q8_0 x (act = xq per token),
// down = 1 the down sums y [pair][H] from the pairs' Q8_0 h (act = hq per pair).  Rows of
// I and H must be multiples of 128.  err is set when a bounded wait expired.
// tile_pre[a] (a = 0 .. active count): prefix sums of the active experts' 32-token
// tiles (q4_mma_tile_tokens()).
bool q4_mma_supported(const Geom& g);
int q4_mma_tile_tokens();
cudaError_t launch_q4_mma(const uint8_t* layer, const uint8_t* shared, int E, int e_lo, Geom g, int down,
                          const int* off, const int* list, const int* active, const int* tile_pre, int n_act, int ks,
                          const uint8_t* act, float* out0, float* out1, unsigned* err, bool exact, cudaStream_t s);
// The two halves of launch_moe_batched, generalised to experts sharded over G devices
// and an optional shared expert.  Partial: routing of all T tokens (every device
// computes the same), then y[(t, j)][H] for the pairs this device owns (routed slot j < k:
// its expert lies in [e_lo, e_lo + e_n), e_lo = rank * e_n, e_n * G = E; the shared slot
// j = k when n_shared = 1: this device holds the fewest of token t's routed experts, ties
// to (t + i) mod G, smallest i), y = 0 for the others when G > 1.  layer points at
// expert e_lo, shared at the shared expert (weight 1, id E).  w_out receives the
// routing weights [T][k + n_shared].  Scratch of batched_partial_bytes, whose first word
// is an error flag (zero it when the scratch is allocated; a tensor-core launch whose
// bounded wait expired sets it).  Combine:
// X[t] += sum_j w[t][j] * y[(t, j)] in slot order (ks = k + n_shared slots).  With the y
// of every device summed in between (one nonzero term per element, so the sum is
// exact), the result is the single-device one bit for bit.  zero_y = false leaves the
// other devices' pairs of y untouched (an exchange that writes them itself); owned, when
// given ([1 + T * ks] ints), receives the count and list of the pairs this device computed.
size_t batched_partial_bytes(const Geom& g, int E, int n_shared, int k, int T);
cudaError_t launch_moe_batched_partial(const uint8_t* layer, const uint8_t* shared, int e_lo, int e_n, int rank,
                                       int G, Geom g, const float* R, const float* normw, float eps, int E,
                                       int n_shared, int k, const float* X, int T, void* scratch,
                                       size_t scratch_bytes, float* y, int* idx_out, float* w_out,
                                       float* logits_out, int kernels, cudaStream_t s, bool zero_y = true,
                                       int* owned = nullptr);
cudaError_t launch_moe_batched_combine(float* X, int T, int H, int ks, const float* wts, const float* y,
                                       cudaStream_t s);
// The partial step's halves.  Route: T tokens' fixed-point router sums (S, [T][E]),
// top-k + softmax (idx / wts [T][k + n_shared], the shared slot last: id E, weight 1)
// and the Q8_0 activation rows xq [T].  Experts: y[(t, j)][H] for the pairs (token t,
// slot j of ks) this device computes (ownership as in the partial step: rank of G, e_n
// experts each; rank 0 of G = 1 with e_n = E + n_shared takes every pair), from the
// tokens' activation rows xq; scratch of experts_scratch_bytes (error flag first);
// pairs_per_expert_div: the experts the pairs spread over, for the kernel choice;
// err_flag, when given, replaces the scratch's own error flag; n_pairs_dev, when given,
// holds the pair count on the device and n_tok * ks is only its upper bound (grids and
// scratch are sized for the bound).
size_t experts_scratch_bytes(const Geom& g, int E, int n_shared, size_t n_pairs);
cudaError_t launch_batched_route(Geom g, const float* R, const float* normw, float eps, int E, int n_shared, int k,
                                 const float* X, int T, unsigned long long* S, int* idx, float* wts, float* logits_out,
                                 uint8_t* xq, cudaStream_t s);
cudaError_t launch_batched_experts(const uint8_t* layer, const uint8_t* shared, int E, int e_lo, int e_n, int rank,
                                   int G, Geom g, int n_shared, int k, int ks, const int* idx, int n_tok,
                                   const uint8_t* xq, void* scratch, size_t scratch_bytes, float* y, int* owned,
                                   int kernels, int pairs_per_expert_div, cudaStream_t s,
                                   unsigned* err_flag = nullptr, const int* n_pairs_dev = nullptr);

// The reference library's own formats (tg_kquant.cu).  fmt: KQ_Q4K (ggml Q4_K
// blocks), KQ_F16, KQ_Q6K (split layout: 208-byte bodies of all blocks, then their
// fp16 d), KQ_F32.  Rows of the quantised formats hold a multiple of 256 values,
// float rows a multiple of 8; matrices and vectors 16-byte aligned.
constexpr int KQ_Q4K = 0, KQ_F16 = 1, KQ_Q6K = 2, KQ_F32 = 4;
bool kq_valid(int fmt, int rows, int cols);
size_t kq_matrix_bytes(int fmt, long long rows, int cols);   // ggml bytes (= device bytes)
size_t kq_smem_bytes(int fmt, int cols);
// Q6_K ggml blocks -> split layout; raw and dst must not alias.
cudaError_t launch_kq_split_q6k(const uint8_t* raw, uint8_t* dst, long long nblk, cudaStream_t s);
// y[rows] = W . x (Q4_K / Q6_K on the 256-wide Q8 blocks of x; f16 / f32 on x), or
// y[r] = y[r] + (W . x)[r] with accumulate.  pdl: start as a programmatic dependent of
// the previous kernel on s (the weight copies overlap it; x is read after it
// completes); it must not write W.
cudaError_t launch_kq_matvec(int fmt, const uint8_t* W, const float* x, float* y, int rows, int cols, cudaStream_t s,
                             bool pdl = false, bool accumulate = false);
// h[e][I] = silu(gate_e . x) * (up_e . x) for n Q4_K experts (device pointer arrays).
// pdl: start as a programmatic dependent of the previous kernel on s, which must not
// write the weights or the pointer arrays.
cudaError_t launch_kq_gateup(const uint8_t* const* gate, const uint8_t* const* up, int n, const float* x, int H,
                             int I, float* h, bool pdl, cudaStream_t s);
// out[H] = (accumulate ? out : 0) + sum_e w[e] * (down_e . h_e), experts in order;
// launched as a programmatic dependent (of the gate/up kernel that writes h).
// scratch: kq_down_scratch_bytes(n, H, I) bytes (H <= 16384), zero before the first
// launch; every launch leaves it ready for the next, whatever the shapes.
size_t kq_down_scratch_bytes(int n, int H, int I);
cudaError_t launch_kq_down(int fmt, const uint8_t* const* down, int n, const float* h, const float* w, int H, int I,
                           float* out, int accumulate, void* scratch, cudaStream_t s);
// tg_rms_norm in the reference's order (dim a multiple of 4).
cudaError_t launch_rms_norm_ref(const float* x, const float* w, float* out, int dim, float eps, cudaStream_t s);

// The reference's attention decode step (tg_attn.cu; csrc/libtinygiant.c:344-551).
// q4: Q4_K wq / wk / wo and f16 wv (tg_attention_decode_q4), else fp32 weights
// (tg_attention_decode).  Caches [n_kv][kv_max][head_dim] fp32; k and v of this token
// go to row kv_len; rope tables [positions][head_dim / 2], row pos used.  pos_dev:
// when set, kv_len = pos = *pos_dev, read on the device (for graph replay).
// scratch: attention_scratch_bytes(...) bytes.
constexpr int ATTN_MAX_ROWS = 32768;   // kv_max bound: a softmax weight per row + the V ring in shared memory
bool attention_valid(int q4, int embed, int n_heads, int n_kv, int head_dim, int kv_max);
size_t attention_scratch_bytes(int n_heads, int n_kv, int head_dim, int kv_max);
// pos_dev[1] is the error word of the device-position form: a position outside
// [0, kv_max) sets it to 1 and the step writes nothing.  accumulate: out += result.
cudaError_t launch_attention(int q4, const uint8_t* wq, const uint8_t* wk, const uint8_t* wv, const uint8_t* wo,
                             const float* q_norm, const float* k_norm, float* kv_k, float* kv_v, int kv_len,
                             int kv_max, const float* rope_cos, const float* rope_sin, const float* x, float* out,
                             int embed, int n_heads, int n_kv, int head_dim, int pos, int* pos_dev,
                             void* scratch, cudaStream_t s, bool accumulate = false);

// Record msg as the calling thread's tg_last_error() text; returns code.
int set_error(int code, const char* msg);

}  // namespace tg

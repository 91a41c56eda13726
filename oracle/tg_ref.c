/*
 * tg_ref.c — CPU oracle for TinyGiant's MoE expert-FFN hot path.
 *
 * TEST INFRASTRUCTURE ONLY: a portable C restatement of the reference's scalar
 * routines, used by tests/, __graft_entry__.smoke() and bench.py's CPU arm as
 * the checker.  The shipped library never links or calls it.
 *
 * What it follows (paths relative to the reference project):
 *   fp16 -> fp32 ............ csrc/libtinygiant.c:24-33
 *   Q8 quantiser structure .. csrc/libtinygiant.c:61-89  (block amax, scale = amax/127,
 *                             per-element round) with ggml Q8_0 semantics
 *                             (gguf/quants.py Q8_0.quantize_blocks, gguf 0.19.0)
 *   Q4_0 weights ............ gguf/quants.py Q4_0.quantize_blocks / dequantize_blocks
 *   block dot ............... csrc/libtinygiant.c:104-169 and csrc/test_libtinygiant.c:22-61
 *                             (integer block dot, then scale, then fp32 accumulation)
 *   matvec .................. csrc/libtinygiant.c:173-190 (quantise input once, one dot per row)
 *   expert forward .......... csrc/libtinygiant.c:555-595 / 599-643 (quantise x, gate rows,
 *                             up rows, g/(1+exp(-g))*u, requantise h, down rows, out += w*y)
 *   MoE combine ............. csrc/libtinygiant.c:647-655, tinygiant/engine.py:238-258
 *   router / top-k / softmax  tinygiant/engine.py:231-236
 *
 * Build with -ffp-contract=off: every float operation below is a separately
 * rounded IEEE operation unless written as fmaf().
 */
#include "tg_ref.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ fp16 */

/* csrc/libtinygiant.c:24-33: IEEE half -> float, subnormals normalised. */
float ref_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int ee = 1;
            while (!(m & 0x400u)) { m <<= 1; ee--; }
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(ee + 112) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112) << 23) | (m << 13);
    }
    float r;
    memcpy(&r, &bits, 4);
    return r;
}

/* float -> IEEE half, round to nearest even (numpy astype(float16), ggml FP32_TO_FP16). */
uint16_t ref_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    int e = (int)(ax >> 23) - 127;
    uint32_t m = ax & 0x7FFFFFu;
    if (e > 15) return (uint16_t)(sign | 0x7C00u);
    if (e >= -14) {
        uint32_t r = ((uint32_t)(e + 15) << 10) | (m >> 13);
        uint32_t rem = m & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    /* half subnormal: units of 2^-24 */
    if (ax < 0x00800000u) return (uint16_t)sign; /* float subnormal/zero -> 0 */
    uint32_t full = 0x800000u | m;          /* value = full * 2^(e-23) */
    int s = -(e + 1);                        /* shift to units of 2^-24 */
    if (s >= 32) return (uint16_t)sign;
    uint32_t q = full >> s;
    uint32_t rem = full & ((1u << s) - 1u);
    uint32_t half = 1u << (s - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/* ------------------------------------------------------------------ exp */

/*
 * tg_expf: exp(x) by Cody-Waite argument reduction (W. J. Cody and W. Waite,
 * "Software Manual for the Elementary Functions", 1980) and the degree-7 Taylor
 * polynomial of exp on |r| <= ln2/2 (truncation error < r^8/8! ~ 5.3e-9).
 *   k = rint(x * log2 e),  r = (x - k*ln2_hi) - k*ln2_lo,  exp(x) = 2^k * P(r)
 * ln2_hi carries 12 significant bits so k*ln2_hi is exact; the scale by 2^k is
 * split in two power-of-two multiplies so only a subnormal result rounds.
 * The device kernels evaluate the identical sequence of IEEE operations.
 */
float ref_expf(float x) {
    if (x != x) return x;
    if (x > 89.0f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const float log2e = 0x1.715476p+0f;
    const float ln2_hi = 0x1.62ep-1f;
    const float ln2_lo = 0x1.0bfbe8p-15f;
    float kf = rintf(x * log2e);
    float r = fmaf(-kf, ln2_hi, x);
    r = fmaf(-kf, ln2_lo, r);
    float p = 0x1.a01a02p-13f;          /* 1/7! */
    p = fmaf(p, r, 0x1.6c16c2p-10f);    /* 1/6! */
    p = fmaf(p, r, 0x1.111112p-7f);     /* 1/5! */
    p = fmaf(p, r, 0x1.555556p-5f);     /* 1/4! */
    p = fmaf(p, r, 0x1.555556p-3f);     /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int k = (int)kf;
    int k1 = k / 2, k2 = k - k1;
    uint32_t b1 = (uint32_t)(k1 + 127) << 23, b2 = (uint32_t)(k2 + 127) << 23;
    float s1, s2;
    memcpy(&s1, &b1, 4);
    memcpy(&s2, &b2, 4);
    return (p * s1) * s2;
}

/* ------------------------------------------------------------------ quantisers */

/* Q8_0 (gguf Q8_0.quantize_blocks; structure of libtinygiant.c:61-89 with
 * 32-wide blocks, fp16 scale, round half away from zero). */
void ref_quantize_q8_0(const float *x, uint8_t *out, int64_t n) {
    int64_t nb = n / REF_QK;
    for (int64_t b = 0; b < nb; b++) {
        const float *xb = x + b * REF_QK;
        uint8_t *ob = out + b * REF_Q8_0_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < REF_QK; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = ref_f32_to_f16(d);
        memcpy(ob, &dh, 2);
        for (int j = 0; j < REF_QK; j++) {
            float v = xb[j] * id;
            ob[2 + j] = (uint8_t)(int8_t)roundf(v);
        }
    }
}

/* Q4_0 (gguf Q4_0.quantize_blocks): d = (signed value of max |x|) / -8,
 * q = min(15, trunc(x/d + 8.5)), low nibbles = elements 0..15. */
void ref_quantize_q4_0(const float *x, uint8_t *out, int64_t n) {
    int64_t nb = n / REF_QK;
    #pragma omp parallel for schedule(static) if (nb > 65536)
    for (int64_t b = 0; b < nb; b++) {
        const float *xb = x + b * REF_QK;
        uint8_t *ob = out + b * REF_Q4_0_BYTES;
        /* first element of largest magnitude (numpy argmax of |x|) */
        float amax = fabsf(xb[0]), mx = xb[0];
        for (int j = 1; j < REF_QK; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) { amax = a; mx = xb[j]; }
        }
        float d = mx / -8.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = ref_f32_to_f16(d);
        memcpy(ob, &dh, 2);
        uint8_t q[REF_QK];
        for (int j = 0; j < REF_QK; j++) {
            float v = truncf(xb[j] * id + 8.5f);
            int qi = (int)v;
            q[j] = (uint8_t)(qi > 15 ? 15 : qi);
        }
        for (int j = 0; j < 16; j++) ob[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
    }
}

void ref_dequantize_q8_0(const uint8_t *q, float *out, int64_t n) {
    for (int64_t b = 0; b < n / REF_QK; b++) {
        const uint8_t *qb = q + b * REF_Q8_0_BYTES;
        uint16_t dh;
        memcpy(&dh, qb, 2);
        float d = ref_f16_to_f32(dh);
        for (int j = 0; j < REF_QK; j++) out[b * REF_QK + j] = (float)(int8_t)qb[2 + j] * d;
    }
}

void ref_dequantize_q4_0(const uint8_t *q, float *out, int64_t n) {
    for (int64_t b = 0; b < n / REF_QK; b++) {
        const uint8_t *qb = q + b * REF_Q4_0_BYTES;
        uint16_t dh;
        memcpy(&dh, qb, 2);
        float d = ref_f16_to_f32(dh);
        for (int j = 0; j < 16; j++) {
            out[b * REF_QK + j] = (float)((qb[2 + j] & 15) - 8) * d;
            out[b * REF_QK + j + 16] = (float)((qb[2 + j] >> 4) - 8) * d;
        }
    }
}

/* ------------------------------------------------------------------ dots */

/* Integer block dot of one Q4_0 block with one Q8_0 block
 * (the vdotq_s32 part of libtinygiant.c:135-158, written as in test_libtinygiant.c:41-53). */
int32_t ref_block_dot_q4_0_q8_0(const uint8_t *wblk, const uint8_t *xblk) {
    const uint8_t *qs = wblk + 2;
    const int8_t *xs = (const int8_t *)(xblk + 2);
    int32_t s = 0;
    for (int j = 0; j < 16; j++) {
        s += ((int32_t)(qs[j] & 15) - 8) * (int32_t)xs[j];
        s += ((int32_t)(qs[j] >> 4) - 8) * (int32_t)xs[j + 16];
    }
    return s;
}

void ref_block_dots(const uint8_t *W, const uint8_t *xq, int32_t *out, int rows, int cols) {
    int nb = cols / REF_QK;
    for (int r = 0; r < rows; r++)
        for (int b = 0; b < nb; b++)
            out[(size_t)r * nb + b] = ref_block_dot_q4_0_q8_0(
                W + ((size_t)r * nb + b) * REF_Q4_0_BYTES, xq + (size_t)b * REF_Q8_0_BYTES);
}

static inline float block_term(const uint8_t *wblk, const uint8_t *xblk) {
    uint16_t dw, dx;
    memcpy(&dw, wblk, 2);
    memcpy(&dx, xblk, 2);
    int32_t s = ref_block_dot_q4_0_q8_0(wblk, xblk);
    /* ggml: sumf += sumi * d_w * d_x, evaluated left to right */
    return ((float)s * ref_f16_to_f32(dw)) * ref_f16_to_f32(dx);
}

/* 32-lane xor butterfly, the device warp reduction order. */
static inline float butterfly32(float *p) {
    for (int off = 16; off >= 1; off >>= 1) {
        float q[32];
        for (int l = 0; l < 32; l++) q[l] = p[l] + p[l ^ off];
        memcpy(p, q, sizeof(q));
    }
    return p[0];
}

/* 5-bit reversal: the lane class visited at ordinal c */
static inline int rev5(int c) {
    return ((c & 1) << 4) | ((c & 2) << 2) | (c & 4) | ((c & 8) >> 2) | ((c & 16) >> 4);
}

float ref_row_dot(const uint8_t *wrow, const uint8_t *xq, int nb, int mode) {
    if (mode == TG_FAST_MMA) {
        float acc = 0.0f;
        for (int c = 0; c < 32; c++)
            for (int b = rev5(c); b < nb; b += 32) {
                const uint8_t *wblk = wrow + (size_t)b * REF_Q4_0_BYTES, *xblk = xq + (size_t)b * REF_Q8_0_BYTES;
                uint16_t dw, dx;
                memcpy(&dw, wblk, 2);
                memcpy(&dx, xblk, 2);
                const float d = ref_f16_to_f32(dw) * ref_f16_to_f32(dx);
                acc = fmaf((float)ref_block_dot_q4_0_q8_0(wblk, xblk), d, acc);
            }
        return acc;
    }
    if (mode == TG_REF_ORDER) {
        float total = 0.0f;
        for (int b = 0; b < nb; b++)
            total += block_term(wrow + (size_t)b * REF_Q4_0_BYTES, xq + (size_t)b * REF_Q8_0_BYTES);
        return total;
    }
    float p[32];
    for (int l = 0; l < 32; l++) {
        float acc = 0.0f;
        for (int b = l; b < nb; b += 32)
            acc = acc + block_term(wrow + (size_t)b * REF_Q4_0_BYTES, xq + (size_t)b * REF_Q8_0_BYTES);
        p[l] = acc;
    }
    return butterfly32(p);
}

void ref_matvec_q4_0(const uint8_t *W, const uint8_t *xq, float *y, int rows, int cols, int mode) {
    int nb = cols / REF_QK;
    for (int r = 0; r < rows; r++)
        y[r] = ref_row_dot(W + (size_t)r * nb * REF_Q4_0_BYTES, xq, nb, mode);
}

/* ------------------------------------------------------------------ expert */

float ref_silu_mul(float g, float u, int mode) {
    float e = mode == TG_REF_ORDER ? expf(-g) : ref_expf(-g);
    float silu = g / (1.0f + e);
    return silu * u;
}

void ref_expert_forward_stages(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                               const float *x, float *out, float w,
                               int embed, int inter, int mode,
                               uint8_t *xq_out, float *g_out, float *u_out,
                               float *h_out, uint8_t *hq_out, float *y_out) {
    int nbe = embed / REF_QK, nbi = inter / REF_QK;
    uint8_t *xq = malloc((size_t)nbe * REF_Q8_0_BYTES);
    uint8_t *hq = malloc((size_t)nbi * REF_Q8_0_BYTES);
    float *g = malloc(sizeof(float) * inter), *u = malloc(sizeof(float) * inter);
    float *h = malloc(sizeof(float) * inter), *y = malloc(sizeof(float) * embed);
    ref_quantize_q8_0(x, xq, embed);
    ref_matvec_q4_0(gate, xq, g, inter, embed, mode);
    ref_matvec_q4_0(up, xq, u, inter, embed, mode);
    for (int i = 0; i < inter; i++) h[i] = ref_silu_mul(g[i], u[i], mode);
    ref_quantize_q8_0(h, hq, inter);
    ref_matvec_q4_0(down, hq, y, embed, inter, mode);
    if (out)
        for (int i = 0; i < embed; i++) out[i] = out[i] + w * y[i];
    if (xq_out) memcpy(xq_out, xq, (size_t)nbe * REF_Q8_0_BYTES);
    if (hq_out) memcpy(hq_out, hq, (size_t)nbi * REF_Q8_0_BYTES);
    if (g_out) memcpy(g_out, g, sizeof(float) * inter);
    if (u_out) memcpy(u_out, u, sizeof(float) * inter);
    if (h_out) memcpy(h_out, h, sizeof(float) * inter);
    if (y_out) memcpy(y_out, y, sizeof(float) * embed);
    free(xq); free(hq); free(g); free(u); free(h); free(y);
}

void ref_expert_forward(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                        const float *x, float *out, float w, int embed, int inter, int mode) {
    ref_expert_forward_stages(gate, up, down, x, out, w, embed, inter, mode,
                              NULL, NULL, NULL, NULL, NULL, NULL);
}

/* ------------------------------------------------------------------ routing */

/*
 * Router logits (engine.py:231, logits = router @ normed).  Each product
 * R[e][r]*x[r] is rounded to fp32, clamped to +-256, converted to fixed point
 * with 2^-32 units (round to nearest even) and summed in int64, so the sum is
 * exact and independent of how the rows are split across threads or blocks
 * (|sum| <= 2^14 * 2^8 * 2^32 = 2^54 for up to 2^14 rows):
 *   logit_e = float(2^-32 * sum_r rint(clamp(fl(R[e][r]*x[r])) * 2^32))
 */
static inline int64_t router_fixed(float r, float x) {
    float p = r * x;
    p = fminf(fmaxf(p, -256.0f), 256.0f);
    return llrintf(p * 0x1p32f);
}
void ref_router_logits(const float *R, const float *x, int n_experts, int hidden, float *logits) {
    for (int e = 0; e < n_experts; e++) {
        int64_t s = 0;
        for (int r = 0; r < hidden; r++) s += router_fixed(R[(size_t)e * hidden + r], x[r]);
        logits[e] = (float)((double)s * 0x1p-32);
    }
}

/*
 * Top-k + renormalised softmax (engine.py:232-236): idx = argsort(logits)[-k:]
 * (ascending, so idx[k-1] is the largest; equal logits order by expert id),
 * w = exp(l - max) / sum(exp(l - max)).  The sum over k = 8 uses numpy's
 * pairwise order ((e0+e1)+(e2+e3))+((e4+e5)+(e6+e7)); other k sum sequentially.
 */
void ref_topk_softmax(const float *logits, int n_experts, int k, int32_t *idx, float *w, int mode) {
    for (int i = 0; i < n_experts; i++) {
        int rank = 0;
        for (int j = 0; j < n_experts; j++)
            if (logits[j] > logits[i] || (logits[j] == logits[i] && j > i)) rank++;
        if (rank < k) idx[k - 1 - rank] = i;
    }
    float m = logits[idx[k - 1]];
    float ex[64];
    for (int j = 0; j < k; j++) {
        float a = logits[idx[j]] - m;
        ex[j] = mode == TG_REF_ORDER ? expf(a) : ref_expf(a);
    }
    float s;
    if (k <= 8) {
        float t[8];
        for (int j = 0; j < 8; j++) t[j] = j < k ? ex[j] : 0.0f;
        s = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
    } else {
        s = 0.0f;
        for (int j = 0; j < k; j++) s = s + ex[j];
    }
    for (int j = 0; j < k; j++) w[j] = ex[j] / s;
}

/* ------------------------------------------------------------------ RMS norm */

/*
 * The FFN RMSNorm in front of each MoE block (engine.py:229-230, tg_rms_norm
 * csrc/libtinygiant.c:322-340: scale = 1/sqrtf(ss/dim + eps), out = (x*scale)*w).
 * ss is summed exactly in fixed point: each fl(x*x), clamped to [0, 2^22], in
 * units of 2^-16, so the sum does not depend on how rows are split.
 */
static inline int64_t ss_fixed(float x) {
    float p = x * x;
    p = fminf(p, 0x1p22f);
    return llrintf(p * 0x1p16f);
}

float ref_rms_scale(const float *x, int dim, float eps) {
    int64_t s = 0;
    for (int r = 0; r < dim; r++) s += ss_fixed(x[r]);
    float ss = (float)((double)s * 0x1p-16);
    return 1.0f / sqrtf(ss / (float)dim + eps);
}

/* Router logits of the normed input without forming it first:
 * logit_e = fl(scale * float(2^-32 * sum_r rint(clamp(fl(R[e][r] * fl(x_r * w_r))) * 2^32))),
 * i.e. R . normed with the scalar RMS scale applied after the exact sum. */
static void block_logits(const float *R, const float *x, const float *w, float scale,
                         int n_experts, int hidden, float *logits) {
    for (int e = 0; e < n_experts; e++) {
        int64_t s = 0;
        for (int r = 0; r < hidden; r++) s += router_fixed(R[(size_t)e * hidden + r], w ? x[r] * w[r] : x[r]);
        logits[e] = scale * (float)((double)s * 0x1p-32);
    }
}

/* ------------------------------------------------------------------ MoE block */

static void expert_ptrs(const uint8_t *blob, int embed, int inter,
                        const uint8_t **g, const uint8_t **u, const uint8_t **d) {
    size_t t = (size_t)inter * (embed / REF_QK) * REF_Q4_0_BYTES;
    *g = blob;
    *u = blob + t;
    *d = blob + 2 * t;
}

void ref_moe_layer(const uint8_t *layer_blob, size_t expert_bytes, const float *R,
                   float *x, int n_experts, int k, int embed, int inter, int mode,
                   int32_t *idx_out, float *w_out, float *logits_out) {
    float *logits = malloc(sizeof(float) * n_experts);
    int32_t idx[64];
    float w[64];
    ref_router_logits(R, x, n_experts, embed, logits);
    ref_topk_softmax(logits, n_experts, k, idx, w, mode);
    float *moe = calloc((size_t)embed, sizeof(float));
    for (int j = 0; j < k; j++) {
        const uint8_t *g, *u, *d;
        expert_ptrs(layer_blob + (size_t)idx[j] * expert_bytes, embed, inter, &g, &u, &d);
        ref_expert_forward(g, u, d, x, moe, w[j], embed, inter, mode);
    }
    for (int i = 0; i < embed; i++) x[i] = x[i] + moe[i];
    if (idx_out) memcpy(idx_out, idx, sizeof(int32_t) * k);
    if (w_out) memcpy(w_out, w, sizeof(float) * k);
    if (logits_out) memcpy(logits_out, logits, sizeof(float) * n_experts);
    free(moe);
    free(logits);
}

/* The engine's MoE block (engine.py:229-258 without attention): normed =
 * RMSNorm(x) * w, route on normed, run the top-k experts on normed, x += moe. */
/* The MoE block with an optional shared expert (DeepSeek-V3-like configs): after the k
 * routed experts, moe += 1 * shared(normed), then x += moe. */
static void moe_block_impl(const uint8_t *layer_blob, size_t expert_bytes, const float *R, const float *normw,
                           float eps, float *x, int n_experts, int k, int embed, int inter, int mode,
                           int32_t *idx_out, float *w_out, float *logits_out, const uint8_t *shared_blob);

void ref_moe_block(const uint8_t *layer_blob, size_t expert_bytes, const float *R, const float *normw,
                   float eps, float *x, int n_experts, int k, int embed, int inter, int mode,
                   int32_t *idx_out, float *w_out, float *logits_out) {
    moe_block_impl(layer_blob, expert_bytes, R, normw, eps, x, n_experts, k, embed, inter, mode, idx_out, w_out,
                   logits_out, NULL);
}

static void moe_block_impl(const uint8_t *layer_blob, size_t expert_bytes, const float *R, const float *normw,
                           float eps, float *x, int n_experts, int k, int embed, int inter, int mode,
                           int32_t *idx_out, float *w_out, float *logits_out, const uint8_t *shared_blob) {
    float *logits = malloc(sizeof(float) * n_experts);
    float *normed = malloc(sizeof(float) * embed);
    int32_t idx[64];
    float w[64];
    float scale = ref_rms_scale(x, embed, eps);
    block_logits(R, x, normw, scale, n_experts, embed, logits);
    ref_topk_softmax(logits, n_experts, k, idx, w, mode);
    for (int r = 0; r < embed; r++) normed[r] = normw ? (x[r] * scale) * normw[r] : x[r] * scale;
    float *moe = calloc((size_t)embed, sizeof(float));
    for (int j = 0; j < k; j++) {
        const uint8_t *g, *u, *d;
        expert_ptrs(layer_blob + (size_t)idx[j] * expert_bytes, embed, inter, &g, &u, &d);
        ref_expert_forward(g, u, d, normed, moe, w[j], embed, inter, mode);
    }
    if (shared_blob) {
        const uint8_t *g, *u, *d;
        expert_ptrs(shared_blob, embed, inter, &g, &u, &d);
        ref_expert_forward(g, u, d, normed, moe, 1.0f, embed, inter, mode);
    }
    for (int i = 0; i < embed; i++) x[i] = x[i] + moe[i];
    if (idx_out) memcpy(idx_out, idx, sizeof(int32_t) * k);
    if (w_out) memcpy(w_out, w, sizeof(float) * k);
    if (logits_out) memcpy(logits_out, logits, sizeof(float) * n_experts);
    free(moe);
    free(normed);
    free(logits);
}

void ref_decode_step(const uint8_t *const *layer_blobs, const float *const *routers,
                     const float *const *norms, float eps, int n_layers, float *x, int n_experts, int k,
                     int embed, int inter, int mode, int32_t *idx_out) {
    size_t eb = (size_t)3 * inter * (embed / REF_QK) * REF_Q4_0_BYTES;
    for (int l = 0; l < n_layers; l++)
        ref_moe_block(layer_blobs[l], eb, routers[l], norms ? norms[l] : NULL, eps, x, n_experts, k, embed,
                      inter, mode, idx_out ? idx_out + (size_t)l * k : NULL, NULL, NULL);
}

/* ------------------------------------------------------------------ threaded */

/* One MoE block with the per-row work spread over threads; same arithmetic as
 * ref_moe_layer (each row is still computed by one thread in the same order). */
static void moe_layer_mt(const uint8_t *layer_blob, size_t expert_bytes, const float *R, const float *normw,
                         float eps, float *x, int n_experts, int k, int embed, int inter, int mode,
                         uint8_t *xq, float *h, uint8_t *hq, float *logits, float *normed) {
    int nbe = embed / REF_QK, nbi = inter / REF_QK;
    int32_t idx[64];
    float w[64];
    float scale = ref_rms_scale(x, embed, eps);
    #pragma omp parallel for schedule(static)
    for (int e = 0; e < n_experts; e++) {
        int64_t s = 0;
        for (int r = 0; r < embed; r++)
            s += router_fixed(R[(size_t)e * embed + r], normw ? x[r] * normw[r] : x[r]);
        logits[e] = scale * (float)((double)s * 0x1p-32);
    }
    ref_topk_softmax(logits, n_experts, k, idx, w, mode);
    for (int r = 0; r < embed; r++) normed[r] = normw ? (x[r] * scale) * normw[r] : x[r] * scale;
    ref_quantize_q8_0(normed, xq, embed);
    size_t tb = (size_t)inter * nbe * REF_Q4_0_BYTES;
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < k * inter; t++) {
        int j = t / inter, i = t % inter;
        const uint8_t *blob = layer_blob + (size_t)idx[j] * expert_bytes;
        float g = ref_row_dot(blob + (size_t)i * nbe * REF_Q4_0_BYTES, xq, nbe, mode);
        float u = ref_row_dot(blob + tb + (size_t)i * nbe * REF_Q4_0_BYTES, xq, nbe, mode);
        h[t] = ref_silu_mul(g, u, mode);
    }
    for (int j = 0; j < k; j++)
        ref_quantize_q8_0(h + (size_t)j * inter, hq + (size_t)j * nbi * REF_Q8_0_BYTES, inter);
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < embed; r++) {
        float moe = 0.0f;
        for (int j = 0; j < k; j++) {
            const uint8_t *down = layer_blob + (size_t)idx[j] * expert_bytes + 2 * tb;
            float y = ref_row_dot(down + (size_t)r * nbi * REF_Q4_0_BYTES,
                                  hq + (size_t)j * nbi * REF_Q8_0_BYTES, nbi, mode);
            moe = moe + w[j] * y;
        }
        x[r] = x[r] + moe;
    }
}

void ref_decode_step_mt(const uint8_t *const *layer_blobs, const float *const *routers,
                        const float *const *norms, float eps, int n_layers, float *x, int n_experts, int k,
                        int embed, int inter, int mode, int n_threads) {
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#else
    (void)n_threads;
#endif
    size_t eb = (size_t)3 * inter * (embed / REF_QK) * REF_Q4_0_BYTES;
    uint8_t *xq = malloc((size_t)(embed / REF_QK) * REF_Q8_0_BYTES);
    float *h = malloc(sizeof(float) * (size_t)k * inter);
    uint8_t *hq = malloc((size_t)k * (inter / REF_QK) * REF_Q8_0_BYTES);
    float *logits = malloc(sizeof(float) * n_experts);
    float *normed = malloc(sizeof(float) * embed);
    for (int l = 0; l < n_layers; l++)
        moe_layer_mt(layer_blobs[l], eb, routers[l], norms ? norms[l] : NULL, eps, x, n_experts, k, embed,
                     inter, mode, xq, h, hq, logits, normed);
    free(xq); free(h); free(hq); free(logits); free(normed);
}

void ref_moe_layer_batched(const uint8_t *layer_blob, size_t expert_bytes, const float *R,
                           float *x, int T, int n_experts, int k, int embed, int inter,
                           int mode, int n_threads) {
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
    #pragma omp parallel for schedule(dynamic, 1)
#else
    (void)n_threads;
#endif
    for (int t = 0; t < T; t++)
        ref_moe_layer(layer_blob, expert_bytes, R, x + (size_t)t * embed, n_experts, k,
                      embed, inter, mode, NULL, NULL, NULL);
}

/* ------------------------------------------------------------------ the reference's K-quant path
 *
 * The shipped library's own formats (csrc/libtinygiant.c): Q4_K super-blocks of 256
 * values (144 B: fp16 d, fp16 dmin, 12 B of 6-bit sub-block scales/mins, 128 B of
 * nibbles), Q6_K (210 B), f16 rows, and 256-wide Q8 activation blocks {fp32 scale,
 * int32 sum, int8 qs[256]}.  Float work follows the reference's order statement by
 * statement (one block after another, C left-to-right, no contraction); integer dots
 * are exact. */

enum { REF_QKK = 256, REF_Q4K_BYTES = 144, REF_Q6K_BYTES = 210, REF_Q8K_BYTES = 264 };

/* libtinygiant.c:42-51 */
static void get_scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* libtinygiant.c:61-89: per 256 values amax, scale = amax/127, codes = round-half-even of
 * x * (127/amax) (vcvtnq_s32_f32), sum of codes.  Output: n/256 blocks of 264 bytes. */
void ref_quantize_q8k(const float *x, uint8_t *out, int64_t n) {
    for (int64_t b = 0; b < n / REF_QKK; b++) {
        const float *xb = x + b * REF_QKK;
        float amax = 0.0f;
        for (int i = 0; i < REF_QKK; i++) {
            float a = fabsf(xb[i]);
            if (a > amax) amax = a;
        }
        float sc = amax / 127.f;
        float inv = amax > 0 ? 127.f / amax : 0;
        uint8_t *o = out + b * REF_Q8K_BYTES;
        int32_t sum = 0;
        int8_t *qs = (int8_t *)(o + 8);
        for (int i = 0; i < REF_QKK; i++) {
            int32_t q = (int32_t)lrintf(xb[i] * inv);   /* round half to even */
            qs[i] = (int8_t)q;
            sum += q;
        }
        memcpy(o, &sc, 4);
        memcpy(o + 4, &sum, 4);
    }
}

/* Q4_K row dot, libtinygiant.c:104-169 */
float ref_dot_q4k(const uint8_t *q4, const uint8_t *xq, int bpr) {
    float total = 0;
    for (int b = 0; b < bpr; b++) {
        const uint8_t *bl = q4 + (size_t)b * REF_Q4K_BYTES;
        uint16_t dr, dmr;
        memcpy(&dr, bl, 2);
        memcpy(&dmr, bl + 2, 2);
        float d = ref_f16_to_f32(dr), dmin = ref_f16_to_f32(dmr);
        const uint8_t *scales = bl + 4, *qs = bl + 16;
        const uint8_t *xb = xq + (size_t)b * REF_Q8K_BYTES;
        float sx;
        memcpy(&sx, xb, 4);
        const int8_t *xqs = (const int8_t *)(xb + 8);
        float block_sum = 0;
        for (int g = 0; g < 4; g++) {
            uint8_t sc_lo, m_lo, sc_hi, m_hi;
            get_scale_min_k4(2 * g, scales, &sc_lo, &m_lo);
            get_scale_min_k4(2 * g + 1, scales, &sc_hi, &m_hi);
            int32_t dot_lo = 0, dot_hi = 0, sum_lo = 0, sum_hi = 0;
            for (int j = 0; j < 32; j++) {
                int lo = qs[g * 32 + j] & 0xF, hi = qs[g * 32 + j] >> 4;
                dot_lo += lo * xqs[g * 64 + j];
                dot_hi += hi * xqs[g * 64 + 32 + j];
                sum_lo += xqs[g * 64 + j];
                sum_hi += xqs[g * 64 + 32 + j];
            }
            block_sum += d * (float)sc_lo * (float)dot_lo - dmin * (float)m_lo * (float)sum_lo;
            block_sum += d * (float)sc_hi * (float)dot_hi - dmin * (float)m_hi * (float)sum_hi;
        }
        total += sx * block_sum;
    }
    return total;
}

/* Q6_K row dot, libtinygiant.c:194-243 */
float ref_dot_q6k(const uint8_t *q6, const uint8_t *xq, int bpr) {
    float total = 0;
    for (int b = 0; b < bpr; b++) {
        const uint8_t *bl = q6 + (size_t)b * REF_Q6K_BYTES;
        const uint8_t *ql = bl, *qh = bl + 128;
        const int8_t *sc = (const int8_t *)(bl + 192);
        uint16_t dr;
        memcpy(&dr, bl + 208, 2);
        float d = ref_f16_to_f32(dr);
        const uint8_t *xb = xq + (size_t)b * REF_Q8K_BYTES;
        float sx;
        memcpy(&sx, xb, 4);
        const int8_t *xqs = (const int8_t *)(xb + 8);
        float block_sum = 0;
        for (int half = 0; half < 2; half++) {
            const uint8_t *ql_h = ql + half * 64, *qh_h = qh + half * 32;
            const int8_t *sc_h = sc + half * 8, *xq_h = xqs + half * 128;
            for (int l = 0; l < 32; l += 16) {
                int is = l / 16;
                int32_t d1 = 0, d2 = 0, d3 = 0, d4 = 0;
                for (int kk = 0; kk < 16; kk++) {
                    int j = l + kk;
                    int v1 = (ql_h[j] & 0xF) | (((qh_h[j] >> 0) & 3) << 4);
                    int v2 = (ql_h[j + 32] & 0xF) | (((qh_h[j] >> 2) & 3) << 4);
                    int v3 = (ql_h[j] >> 4) | (((qh_h[j] >> 4) & 3) << 4);
                    int v4 = (ql_h[j + 32] >> 4) | (((qh_h[j] >> 6) & 3) << 4);
                    d1 += (v1 - 32) * xq_h[l + kk];
                    d2 += (v2 - 32) * xq_h[l + kk + 32];
                    d3 += (v3 - 32) * xq_h[l + kk + 64];
                    d4 += (v4 - 32) * xq_h[l + kk + 96];
                }
                block_sum += (float)sc_h[is + 0] * (float)d1;
                block_sum += (float)sc_h[is + 2] * (float)d2;
                block_sum += (float)sc_h[is + 4] * (float)d3;
                block_sum += (float)sc_h[is + 6] * (float)d4;
            }
        }
        total += d * sx * block_sum;
    }
    return total;
}

/* f16 row dot in the shape of libtinygiant.c:268-287: eight running fused sums, lane v
 * taking columns v, v + 8, ..., then (s0+s4 + s1+s5) + (s2+s6 + s3+s7) pairwise. */
float ref_dot_f16(const uint16_t *row, const float *x, int ncols) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i + 7 < ncols; i += 8)
        for (int v = 0; v < 8; v++) acc[v] = fmaf(ref_f16_to_f32(row[i + v]), x[i + v], acc[v]);
    float t0 = acc[0] + acc[4], t1 = acc[1] + acc[5], t2 = acc[2] + acc[6], t3 = acc[3] + acc[7];
    return (t0 + t1) + (t2 + t3);
}

/* f32 row dot, libtinygiant.c:300-318: the f16 order above on fp32 weights. */
float ref_dot_f32(const float *row, const float *x, int ncols) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i + 7 < ncols; i += 8)
        for (int v = 0; v < 8; v++) acc[v] = fmaf(row[i + v], x[i + v], acc[v]);
    float t0 = acc[0] + acc[4], t1 = acc[1] + acc[5], t2 = acc[2] + acc[6], t3 = acc[3] + acc[7];
    return (t0 + t1) + (t2 + t3);
}

/* tg_rms_norm, libtinygiant.c:322-340 (dim a multiple of 4): four running fused sums of
 * x^2 (lane v takes elements v, v + 4, ...), added pairwise, scale = 1 / sqrtf(ss/dim + eps),
 * out = (x * scale) * w. */
void ref_rms_norm_k(const float *x, const float *w, float *out, int dim, float eps) {
    float acc[4] = {0, 0, 0, 0};
    for (int i = 0; i + 3 < dim; i += 4)
        for (int v = 0; v < 4; v++) acc[v] = fmaf(x[i + v], x[i + v], acc[v]);
    float ss = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    float scale = 1.f / sqrtf(ss / dim + eps);
    for (int i = 0; i < dim; i++) out[i] = (x[i] * scale) * w[i];
}

/* fmt: 0 Q4_K, 1 f16, 2 Q6_K, 4 f32 (rows of the reference's own byte layout). */
void ref_matvec_k(const void *W, int fmt, const float *x, float *y, int rows, int cols) {
    int bpr = cols / REF_QKK;
    uint8_t *xq = malloc((size_t)bpr * REF_Q8K_BYTES);
    if (fmt == 0 || fmt == 2) ref_quantize_q8k(x, xq, cols);
    for (int r = 0; r < rows; r++) {
        if (fmt == 0) y[r] = ref_dot_q4k((const uint8_t *)W + (size_t)r * bpr * REF_Q4K_BYTES, xq, bpr);
        else if (fmt == 2) y[r] = ref_dot_q6k((const uint8_t *)W + (size_t)r * bpr * REF_Q6K_BYTES, xq, bpr);
        else if (fmt == 4) y[r] = ref_dot_f32((const float *)W + (size_t)r * cols, x, cols);
        else y[r] = ref_dot_f16((const uint16_t *)W + (size_t)r * cols, x, cols);
    }
    free(xq);
}

/* tg_expert_forward_mixed, libtinygiant.c:599-643 (down_format 0 = Q4_K also gives
 * tg_expert_forward, :555-595): Q4_K gate/up on Q8(256) of x, h = g / (1 + exp(-g)) * u,
 * down in its format (Q4_K and Q6_K on Q8(256) of h, f16 on h itself), out += w * y. */
void ref_expert_forward_k(const uint8_t *gate, const uint8_t *up, const void *down, int down_format,
                          const float *x, float *out, float w, int embed, int inter, int mode) {
    float *g = malloc(sizeof(float) * inter), *u = malloc(sizeof(float) * inter);
    float *h = malloc(sizeof(float) * inter), *y = malloc(sizeof(float) * embed);
    ref_matvec_k(gate, 0, x, g, inter, embed);
    ref_matvec_k(up, 0, x, u, inter, embed);
    for (int i = 0; i < inter; i++) h[i] = ref_silu_mul(g[i], u[i], mode);
    ref_matvec_k(down, down_format, h, y, embed, inter);
    for (int i = 0; i < embed; i++) out[i] += w * y[i];
    free(g); free(u); free(h); free(y);
}

/* The MoE block with its FFN RMSNorm for T independent tokens x[T][embed], in place:
 * ref_moe_block per token (engine.py:229-258 for each row of a batch); tokens run in
 * parallel across n_threads (0 = OpenMP default). */
void ref_moe_block_batched_shared(const uint8_t *layer_blob, size_t expert_bytes, const float *R,
                                  const float *normw, float eps, float *x, int T, int n_experts, int k, int embed,
                                  int inter, int mode, int n_threads, const uint8_t *shared_blob) {
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
    #pragma omp parallel for schedule(dynamic, 1)
#else
    (void)n_threads;
#endif
    for (int t = 0; t < T; t++)
        moe_block_impl(layer_blob, expert_bytes, R, normw, eps, x + (size_t)t * embed, n_experts, k, embed, inter,
                       mode, NULL, NULL, NULL, shared_blob);
}

void ref_moe_block_batched(const uint8_t *layer_blob, size_t expert_bytes, const float *R, const float *normw,
                           float eps, float *x, int T, int n_experts, int k, int embed, int inter, int mode,
                           int n_threads) {
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
    #pragma omp parallel for schedule(dynamic, 1)
#else
    (void)n_threads;
#endif
    for (int t = 0; t < T; t++)
        ref_moe_block(layer_blob, expert_bytes, R, normw, eps, x + (size_t)t * embed, n_experts, k, embed, inter,
                      mode, NULL, NULL, NULL);
}

/* ------------------------------------------------------------------ attention decode
 *
 * The reference's GQA attention step for one token (csrc/libtinygiant.c:344-551),
 * statement by statement, every float operation rounded on its own except the
 * source's fused multiply-adds (vfmaq_f32). */

/* apply_rope_inplace, libtinygiant.c:344-360: for each head and i < head_dim / 2, with
 * x1 = x[i], x2 = x[i + half], c = cos[i], s = sin[i] (the rows of position pos):
 *   x[i]        = x1*c - x2*s       (vmlsq_f32: multiply, multiply, subtract)
 *   x[i + half] = fma(x1, s, x2*c)  (vfmaq_f32 on vmulq_f32) */
void ref_rope(float *x, int n_heads, int head_dim, const float *c, const float *s) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        float *xh = x + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            float x1 = xh[i], x2 = xh[half + i];
            float a = x1 * c[i], b = x2 * s[i];
            xh[i] = a - b;
            xh[half + i] = fmaf(x1, s[i], x2 * c[i]);
        }
    }
}

/* One head's attention over seq cached rows (libtinygiant.c:406-453 / 498-547):
 * score_t = dot(q, k_t) * (1 / sqrtf(head_dim)), the dot as four fused chains (chain v
 * over d = v, v + 4, ...) added pairwise; softmax with the running max from -1e30, the
 * exps summed in t order; out[d] = fused sum over t of (e_t * inv_sum) * v_t[d]. */
static void attend_head(const float *q, const float *kc, const float *vc, int seq, int hd, float *out, float *sc,
                        int mode) {
    float inv_sqrt = 1.f / sqrtf((float)hd);
    float mx = -1e30f;
    for (int t = 0; t < seq; t++) {
        const float *kt = kc + (size_t)t * hd;
        float acc[4] = {0, 0, 0, 0};
        for (int d = 0; d + 3 < hd; d += 4)
            for (int v = 0; v < 4; v++) acc[v] = fmaf(q[d + v], kt[d + v], acc[v]);
        float dot = (acc[0] + acc[1]) + (acc[2] + acc[3]);
        sc[t] = dot * inv_sqrt;
        if (sc[t] > mx) mx = sc[t];
    }
    float sum = 0.f;
    for (int t = 0; t < seq; t++) {
        float a = sc[t] - mx;
        sc[t] = mode == TG_REF_ORDER ? expf(a) : ref_expf(a);
        sum += sc[t];
    }
    float inv = 1.f / sum;
    for (int d = 0; d < hd; d++) out[d] = 0.f;
    for (int t = 0; t < seq; t++) {
        float w = sc[t] * inv;
        const float *vt = vc + (size_t)t * hd;
        for (int d = 0; d < hd; d++) out[d] = fmaf(w, vt[d], out[d]);
    }
}

/* tg_attention_decode (libtinygiant.c:364-456, q4 = 0: wq, wk, wv, wo fp32) and
 * tg_attention_decode_q4 (:460-551, q4 = 1: wq, wk, wo Q4_K on Q8(256) of their input,
 * wv f16).  q = Wq.in, k = Wk.in, v = Wv.in; per-head RMSNorm (eps 1e-6) of q and k
 * with q_norm_w / k_norm_w; RoPE at pos; k and v appended to the caches
 * [n_kv][kv_max][head_dim] at row kv_len; GQA attention of query head h over kv head
 * h / (n_heads / n_kv) for rows 0..kv_len; output = Wo.attn (written, not added). */
void ref_attention_decode(int q4, const void *wq, const void *wk, const void *wv, const void *wo,
                          const float *q_norm_w, const float *k_norm_w, float *kv_k, float *kv_v, int kv_len,
                          int kv_max, const float *rope_cos, const float *rope_sin, const float *input,
                          float *output, int embed, int n_heads, int n_kv, int head_dim, int pos, int mode) {
    int qd = n_heads * head_dim, kvd = n_kv * head_dim, ratio = n_heads / n_kv, half = head_dim / 2;
    int seq = kv_len + 1;
    float *q = malloc(sizeof(float) * qd), *k = malloc(sizeof(float) * kvd), *v = malloc(sizeof(float) * kvd);
    float *qn = malloc(sizeof(float) * qd), *kn = malloc(sizeof(float) * kvd), *att = malloc(sizeof(float) * qd);
    float *sc = malloc(sizeof(float) * seq);
    ref_matvec_k(wq, q4 ? 0 : 4, input, q, qd, embed);
    ref_matvec_k(wk, q4 ? 0 : 4, input, k, kvd, embed);
    ref_matvec_k(wv, q4 ? 1 : 4, input, v, kvd, embed);
    for (int h = 0; h < n_heads; h++)
        ref_rms_norm_k(q + (size_t)h * head_dim, q_norm_w, qn + (size_t)h * head_dim, head_dim, 1e-6f);
    for (int h = 0; h < n_kv; h++)
        ref_rms_norm_k(k + (size_t)h * head_dim, k_norm_w, kn + (size_t)h * head_dim, head_dim, 1e-6f);
    ref_rope(qn, n_heads, head_dim, rope_cos + (size_t)pos * half, rope_sin + (size_t)pos * half);
    ref_rope(kn, n_kv, head_dim, rope_cos + (size_t)pos * half, rope_sin + (size_t)pos * half);
    for (int h = 0; h < n_kv; h++) {
        memcpy(kv_k + ((size_t)h * kv_max + kv_len) * head_dim, kn + (size_t)h * head_dim, sizeof(float) * head_dim);
        memcpy(kv_v + ((size_t)h * kv_max + kv_len) * head_dim, v + (size_t)h * head_dim, sizeof(float) * head_dim);
    }
    for (int h = 0; h < n_heads; h++) {
        int kvh = h / ratio;
        attend_head(qn + (size_t)h * head_dim, kv_k + (size_t)kvh * kv_max * head_dim,
                    kv_v + (size_t)kvh * kv_max * head_dim, seq, head_dim, att + (size_t)h * head_dim, sc, mode);
    }
    ref_matvec_k(wo, q4 ? 0 : 4, att, output, embed, qd);
    free(q); free(k); free(v); free(qn); free(kn); free(att); free(sc);
}

/* ------------------------------------------------------------------ data */

static inline uint64_t splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void ref_fill_normal(float *out, int64_t n, uint64_t seed, float sigma) {
    #pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < (n + 4095) / 4096; c++) {
        uint64_t s = seed ^ (0xD1B54A32D192ED03ull * (uint64_t)(c + 1));
        int64_t lo = c * 4096, hi = lo + 4096 < n ? lo + 4096 : n;
        for (int64_t i = lo; i < hi; i += 2) {
            double u1 = ((splitmix64(&s) >> 11) + 1.0) * 0x1p-53;
            double u2 = (splitmix64(&s) >> 11) * 0x1p-53;
            double rr = sqrt(-2.0 * log(u1));
            out[i] = (float)(sigma * rr * cos(6.283185307179586 * u2));
            if (i + 1 < hi) out[i + 1] = (float)(sigma * rr * sin(6.283185307179586 * u2));
        }
    }
}

// tg_device.cuh — device arithmetic shared by every TinyGiant B200 kernel.
//
// Every float operation that feeds a result is written with an explicit
// round-to-nearest intrinsic (__fmul_rn, __fadd_rn, __fmaf_rn, __fdiv_rn) so the
// compiler cannot contract or reorder it; the CPU oracle evaluates the same
// sequence of IEEE operations, which is what makes GPU and CPU bit-identical.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "tg_layout.h"

namespace tg {

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

// exp(x): Cody-Waite reduction + degree-7 Taylor polynomial (Horner, fused
// multiply-add), scaled by 2^k in two exact power-of-two steps.  Within 1 ulp of
// the correctly rounded result over the whole float range.
__device__ __forceinline__ float tg_expf(float x) {
    if (x != x) return x;
    if (x > 89.0f) return __int_as_float(0x7f800000);
    if (x < -104.0f) return 0.0f;
    float kf = rintf(__fmul_rn(x, 0x1.715476p+0f));
    float r = __fmaf_rn(-kf, 0x1.62ep-1f, x);
    r = __fmaf_rn(-kf, 0x1.0bfbe8p-15f, r);
    float p = 0x1.a01a02p-13f;
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int k = (int)kf;
    int k1 = k / 2, k2 = k - k1;
    return __fmul_rn(__fmul_rn(p, __int_as_float((k1 + 127) << 23)), __int_as_float((k2 + 127) << 23));
}

// SwiGLU element, csrc/libtinygiant.c:580-583: g / (1 + exp(-g)) * u.
__device__ __forceinline__ float silu_mul(float g, float u) {
    float e = tg_expf(-g);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u);
}

// A lane's share of a block's abs-max: |v|, or 0 for NaN, so the block amax is
// max(0, max over non-NaN |v|) (the CPU loop `if (|v| > amax) amax = |v|` from 0).
__device__ __forceinline__ float absmax_lane(float v) {
    float a = fabsf(v);
    return a > 0.0f ? a : 0.0f;
}

// Q8_0 scale of a block from its abs-max (ggml: d = amax/127, id = 1/d or 0).
struct Q8Scale { float id; uint16_t dh; };
__device__ __forceinline__ Q8Scale q8_scale(float amax) {
    float d = __fdiv_rn(amax, 127.0f);
    Q8Scale s;
    s.id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    s.dh = f32_to_f16_bits(d);
    return s;
}
__device__ __forceinline__ int q8_round(float x, float id) {
    return (int)roundf(__fmul_rn(x, id));     // round half away from zero
}

// Q4_0 element code (gguf Q4_0.quantize_blocks): min(15, trunc(x*id + 8.5)).
__device__ __forceinline__ int q4_code(float x, float id) {
    int q = (int)truncf(__fadd_rn(__fmul_rn(x, id), 8.5f));
    return q > 15 ? 15 : q;
}

// a (unsigned bytes) . b (signed bytes) + c
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Activation block held by one lane: 32 int8 codes, the fp32 value of the
// stored fp16 scale, and 8 * sum(codes) (folds the Q4_0 "-8" offset).
struct XBlk {
    int4 lo, hi;   // codes 0..15, 16..31
    float d;
    int s8;
};

// Exact int32 dot of one Q4_0 block (16 nibble bytes, ggml order) with an
// activation block: sum_j (q_j - 8) * x_j.  High nibbles are used in place
// (16*q) with an unsigned x signed dp4a and shifted back, which is exact.
__device__ __forceinline__ int block_sumi(uint4 w, const XBlk& x) {
    int lo = 0, hi = 0;
    lo = __dp4a((int)(w.x & 0x0F0F0F0Fu), x.lo.x, lo);
    lo = __dp4a((int)(w.y & 0x0F0F0F0Fu), x.lo.y, lo);
    lo = __dp4a((int)(w.z & 0x0F0F0F0Fu), x.lo.z, lo);
    lo = __dp4a((int)(w.w & 0x0F0F0F0Fu), x.lo.w, lo);
    hi = dp4a_us(w.x & 0xF0F0F0F0u, x.hi.x, hi);
    hi = dp4a_us(w.y & 0xF0F0F0F0u, x.hi.y, hi);
    hi = dp4a_us(w.z & 0xF0F0F0F0u, x.hi.z, hi);
    hi = dp4a_us(w.w & 0xF0F0F0F0u, x.hi.w, hi);
    return lo + (hi >> 4) - x.s8;
}

// One block's contribution, ggml order: (float)sumi * d_w * d_x.
__device__ __forceinline__ float block_term(int sumi, float dw, float dx) {
    return __fmul_rn(__fmul_rn(__int2float_rn(sumi), dw), dx);
}

// Warp-collective helpers reconverge the warp first: a full-mask shuffle that
// follows lane-divergent code otherwise waits a long time for the stragglers.
__device__ __forceinline__ float warp_sum_butterfly(float v) {
    __syncwarp();
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

__device__ __forceinline__ long long warp_sum_i64(long long v) {
    __syncwarp();
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Router product in fixed point: rint(clamp(fl(r*x), +-256) * 2^32).  The clamp
// bounds any sum over <= 2^14 rows by 2^54, so sums are exact, independent of
// how rows are split, and stay clear of the count tag kept from bit 56 up.
__device__ __forceinline__ long long router_fixed(float r, float x) {
    float p = __fmul_rn(r, x);
    p = fminf(fmaxf(p, -256.0f), 256.0f);
    return __float2ll_rn(__fmul_rn(p, 0x1p32f));
}
__device__ __forceinline__ float router_logit(long long s) {
    return __double2float_rn(__dmul_rn(__ll2double_rn(s), 0x1p-32));
}

// FFN RMSNorm (csrc/libtinygiant.c:322-340): ss = sum x^2 exactly, as fixed-point
// sums of fl(x*x) clamped to [0, 2^22] in units of 2^-16 (< 2^52 for <= 2^14 rows);
// scale = 1/sqrtf(ss/dim + eps).
__device__ __forceinline__ long long ss_fixed(float x) {
    float p = fminf(__fmul_rn(x, x), 0x1p22f);
    return __float2ll_rn(__fmul_rn(p, 0x1p16f));
}
__device__ __forceinline__ float rms_scale_from(long long s, int dim, float eps) {
    float ss = __double2float_rn(__dmul_rn(__ll2double_rn(s), 0x1p-16));
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
}

// Activation block b of an activation view (shared or global memory).
__device__ __forceinline__ XBlk load_xblk(const ActView& a, int b) {
    XBlk x;
    const int4* q = reinterpret_cast<const int4*>(a.qs + (size_t)b * 32);
    x.lo = q[0];
    x.hi = q[1];
    x.d = a.d[b];
    x.s8 = a.s8[b];
    return x;
}

// Quantise one 32-value block held one value per lane (lane = position).
// Returns the code; lane 0 also gets the fp16 scale bits and 8*sum.
struct Q8Lane { int q; uint16_t dh; int s8; };
__device__ __forceinline__ Q8Lane quantize_lane(float v) {
    __syncwarp();
    float am = absmax_lane(v);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    Q8Scale sc = q8_scale(am);
    Q8Lane r;
    r.q = q8_round(v, sc.id);
    int s = r.q;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    r.dh = sc.dh;
    r.s8 = 8 * s;
    return r;
}


constexpr int MAX_TOPK = 16;

// Top-k by rank: element i is selected when fewer than k elements beat it
// (larger logit, or equal logit and larger id); its ascending position is k-1-rank.
__device__ __forceinline__ void topk_softmax_block(const float* sl, int E, int k, int* sidx, float* sw) {
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        float li = sl[i];
        int rank = 0;
        for (int j = 0; j < E; j++) {
            float lj = sl[j];
            rank += (lj > li) || (lj == li && j > i);
        }
        if (rank < k) sidx[k - 1 - rank] = i;
    }
    __syncwarp();
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = sl[sidx[k - 1]];
        float ex[MAX_TOPK];
        for (int j = 0; j < k; j++) ex[j] = tg_expf(__fsub_rn(sl[sidx[j]], m));
        float s;
        if (k <= 8) {
            float t[8];
            for (int j = 0; j < 8; j++) t[j] = j < k ? ex[j] : 0.0f;
            s = __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3])),
                          __fadd_rn(__fadd_rn(t[4], t[5]), __fadd_rn(t[6], t[7])));
        } else {
            s = 0.0f;
            for (int j = 0; j < k; j++) s = __fadd_rn(s, ex[j]);
        }
        for (int j = 0; j < k; j++) sw[j] = __fdiv_rn(ex[j], s);
    }
    __syncwarp();
    __syncthreads();
}


}  // namespace tg

// tg_kquant.cu — the reference library's own weight formats on the GPU
// (csrc/libtinygiant.c): Q4_K and Q6_K super-blocks of 256 values against 256-wide
// Q8 activation blocks, f16 and f32 rows, and the RMSNorm, in the reference's float
// order.
//
// Float work follows the reference source statement by statement with every
// operation rounded on its own (the C text without contraction): within a block the
// sub-block terms in source order, then the row total over blocks in order.  Integer
// dots are exact (dp4a), so how they are split across lanes does not matter.
//
// A lane computes one (row, block) unit; a warp owns whole rows (32 / blocks-per-row
// of them, or one row when a row has more than 32 blocks), so the chain of a row's
// block terms runs in one lane and no step crosses warps.  A warp stages its units'
// bytes into shared memory with coalesced 16-byte cp.async copies, issued before the
// kernel waits for its inputs: every launch is a programmatic dependent launch, so a
// kernel's weight fetch overlaps the tail of the kernel before it, and only the reads
// of x / h wait (griddepcontrol.wait) for that kernel to complete.
//
// The expert down kernel runs one CTA per (row block, expert); each writes its rows'
// y_e to scratch, and the last CTA of a row block to arrive (a counter per row block,
// reset by that CTA) adds the experts' terms in expert order, so the combine keeps
// the reference's sequential order without any CTA waiting on another.
//
// Device layouts: Q4_K as ggml blocks (144 B, so every block is 16-byte aligned);
// Q6_K "split": the 208-byte bodies (ql | qh | scales) of all blocks of the matrix,
// then the fp16 d of all blocks (the 210-byte ggml block is only 2-byte aligned);
// f16 / f32 as row-major values.
#include <cuda_runtime.h>

#include "tg_device.cuh"
#include "tg_internal.h"

namespace tg {

namespace {

constexpr int KW = 4;                 // warps per CTA
constexpr int KT = KW * 32;
constexpr int Q4K_B = 144, Q6K_BODY = 208, Q6K_B = 210;
constexpr int XC = 272;               // stride of a block's 256 codes in shared memory (bank spread)
constexpr int FROWS = 4;              // rows per warp of the f16 / f32 matvec (8 lanes per row)
constexpr int FCH = 256;              // columns staged per step
constexpr int FDEPTH = 4;             // f16 / f32: column chunks of a warp's rows in flight
// FMT values: KQ_Q4K 0, KQ_F16 1, KQ_Q6K 2, KQ_F32 4 (tg_internal.h)

// Shared-memory activation of one vector of bpr blocks (quantised formats).
struct KAct {
    int8_t* codes;  // [bpr][XC]
    float* sx;      // [bpr] block scales
    int* s32;       // [bpr][8] code sums of the 32-value sub-blocks
    int* s16;       // [bpr][16] code sums of the 16-value groups
};

__host__ __device__ inline size_t r16(size_t n) { return (n + 15) & ~(size_t)15; }

__host__ __device__ inline size_t act_region(int fmt, int cols) {
    int bpr = cols / 256;
    if (fmt == KQ_F16 || fmt == KQ_F32) return (size_t)cols * 4;
    return r16((size_t)bpr * XC) + r16((size_t)bpr * 4) + (size_t)bpr * 32 + (size_t)bpr * 64;
}
__host__ __device__ inline int terms_per_warp(int cols) {
    int bpr = cols / 256;
    return bpr > 32 ? bpr : 32;
}
// Staging bytes of one warp: 32 units of the format's block (Q4_K 144 B, Q6_K body
// 208 B), or a ring of FDEPTH slots of four padded rows of 256 values (f16 / f32).
__host__ __device__ constexpr int fx_slot_bytes(int fmt) { return FROWS * (FCH * (fmt == KQ_F16 ? 2 : 4) + 16); }
__host__ __device__ constexpr int stage_bytes(int fmt) {
    return fmt == KQ_Q4K ? 32 * Q4K_B : fmt == KQ_Q6K ? 32 * Q6K_BODY : FDEPTH * fx_slot_bytes(fmt);
}
// stages per warp: gate and up (MODE 1), else one
__host__ __device__ inline size_t warp_bytes(int fmt, int mode, int cols) {
    return (size_t)(mode == 1 ? 2 : 1) * stage_bytes(fmt) + r16((size_t)terms_per_warp(cols) * 4);
}
__host__ __device__ inline size_t kq_smem(int fmt, int mode, int cols) {
    return act_region(fmt, cols) + (size_t)KW * warp_bytes(fmt, mode, cols);
}
__host__ __device__ inline int rows_per_warp(int fmt, int cols) {
    int bpr = cols / 256;
    return (fmt == KQ_F16 || fmt == KQ_F32) ? FROWS : (bpr >= 32 ? 1 : 32 / bpr);
}

__device__ inline KAct act_at(uint8_t* base, int bpr) {
    KAct a;
    a.codes = (int8_t*)base;
    a.sx = (float*)(base + r16((size_t)bpr * XC));
    a.s32 = (int*)((uint8_t*)a.sx + r16((size_t)bpr * 4));
    a.s16 = a.s32 + bpr * 8;
    return a;
}

// quantize_q8, csrc/libtinygiant.c:61-89, for one vector x[bpr * 256]: one warp per
// block, 8 values per lane.  scale = amax / 127, codes = round-half-even(x * (127 /
// amax)), or 0 when amax is 0.  Also the exact code sums of 32- and 16-value groups.
__device__ void quantize_q8k(const float* __restrict__ x, int bpr, KAct a, int warp, int lane) {
    for (int b = warp; b < bpr; b += KW) {
        const float4* src = reinterpret_cast<const float4*>(x + (size_t)b * 256 + lane * 8);
        float4 v0 = src[0], v1 = src[1];
        float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        float am = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
        float sc = __fdiv_rn(am, 127.0f);
        float inv = am > 0.0f ? __fdiv_rn(127.0f, am) : 0.0f;
        int q[8], s = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            q[i] = __float2int_rn(__fmul_rn(v[i], inv));
            s += q[i];
        }
        uint2 packed;
        packed.x = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((unsigned)(q[3] & 0xFF) << 24);
        packed.y = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((unsigned)(q[7] & 0xFF) << 24);
        *reinterpret_cast<uint2*>(a.codes + (size_t)b * XC + lane * 8) = packed;
        int s16 = s + __shfl_xor_sync(0xffffffffu, s, 1);
        int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
        if ((lane & 1) == 0) a.s16[b * 16 + (lane >> 1)] = s16;
        if ((lane & 3) == 0) a.s32[b * 8 + (lane >> 2)] = s32;
        if (lane == 0) a.sx[b] = sc;
    }
}

__device__ __forceinline__ unsigned byte_of(uint4 v, int i) {
    unsigned w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
    return (w >> (8 * (i & 3))) & 0xFFu;
}

// get_scale_min_k4, csrc/libtinygiant.c:42-51 (q = the block's 12 scale bytes,
// held as bytes 4..15 of its first 16-byte word).
__device__ __forceinline__ void scale_min_k4(int j, uint4 h, float& sc, float& m) {
#define QB(i) byte_of(h, 4 + (i))
    unsigned s, mm;
    if (j < 4) {
        s = QB(j) & 63;
        mm = QB(j + 4) & 63;
    } else {
        s = (QB(j + 4) & 0xF) | ((QB(j - 4) >> 6) << 4);
        mm = (QB(j + 4) >> 4) | ((QB(j) >> 6) << 4);
    }
#undef QB
    sc = (float)s;
    m = (float)mm;
}

__device__ __forceinline__ unsigned word_of(uint4 v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// One Q4_K block against activation block b: sx * block_sum, dot_q4k_q8
// (csrc/libtinygiant.c:104-169): block_sum += d*sc*dot - dmin*m*sum per sub-block.
__device__ __forceinline__ float q4k_term(const uint8_t* blk, const KAct& a, int b) {
    const uint4* w4 = reinterpret_cast<const uint4*>(blk);
    const uint4 hd = w4[0];
    const float d = f16_bits_to_f32((uint16_t)(hd.x & 0xFFFF));
    const float dmin = f16_bits_to_f32((uint16_t)(hd.x >> 16));
    const uint4* xc = reinterpret_cast<const uint4*>(a.codes + (size_t)b * XC);
    const int* s32 = a.s32 + b * 8;
    float bs = 0.0f;
#pragma unroll
    for (int g = 0; g < 4; g++) {
        int dl = 0, dh = 0;
#pragma unroll
        for (int hq = 0; hq < 2; hq++) {
            const uint4 q = w4[1 + 2 * g + hq];
            const uint4 xl = xc[4 * g + hq], xh = xc[4 * g + 2 + hq];
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const unsigned w = word_of(q, t);
                dl = dp4a_us(w & 0x0F0F0F0Fu, (int)word_of(xl, t), dl);
                dh = dp4a_us((w >> 4) & 0x0F0F0F0Fu, (int)word_of(xh, t), dh);
            }
        }
        float sc_lo, m_lo, sc_hi, m_hi;
        scale_min_k4(2 * g, hd, sc_lo, m_lo);
        scale_min_k4(2 * g + 1, hd, sc_hi, m_hi);
        float tl = __fsub_rn(__fmul_rn(__fmul_rn(d, sc_lo), __int2float_rn(dl)),
                             __fmul_rn(__fmul_rn(dmin, m_lo), __int2float_rn(s32[2 * g])));
        bs = __fadd_rn(bs, tl);
        float th = __fsub_rn(__fmul_rn(__fmul_rn(d, sc_hi), __int2float_rn(dh)),
                             __fmul_rn(__fmul_rn(dmin, m_hi), __int2float_rn(s32[2 * g + 1])));
        bs = __fadd_rn(bs, th);
    }
    return __fmul_rn(a.sx[b], bs);
}

// One Q6_K block (208-byte body + its d) against activation block b: d * sx *
// block_sum, dot_q6k_q8 (csrc/libtinygiant.c:194-243).  Values are the 6-bit codes
// minus 32; sum (v - 32) * x = dp4a(v, x) - 32 * sum(x), exactly.
__device__ __forceinline__ float q6k_term(const uint8_t* body, float d, const KAct& a, int b) {
    const uint4* ql4 = reinterpret_cast<const uint4*>(body);
    const uint4* qh4 = reinterpret_cast<const uint4*>(body + 128);
    const uint4 scw = *reinterpret_cast<const uint4*>(body + 192);
    const uint4* xc = reinterpret_cast<const uint4*>(a.codes + (size_t)b * XC);
    const int* s16 = a.s16 + b * 16;
    float bs = 0.0f;
#pragma unroll
    for (int half = 0; half < 2; half++) {
#pragma unroll
        for (int is = 0; is < 2; is++) {
            const uint4 A = ql4[4 * half + is], B = ql4[4 * half + 2 + is], Qh = qh4[2 * half + is];
            const uint4 X0 = xc[8 * half + is], X1 = xc[8 * half + is + 2], X2 = xc[8 * half + is + 4],
                        X3 = xc[8 * half + is + 6];
            int d1 = 0, d2 = 0, d3 = 0, d4 = 0;
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const unsigned a0 = word_of(A, t), b0 = word_of(B, t), h = word_of(Qh, t);
                const unsigned v1 = (a0 & 0x0F0F0F0Fu) | ((h & 0x03030303u) << 4);
                const unsigned v2 = (b0 & 0x0F0F0F0Fu) | (((h >> 2) & 0x03030303u) << 4);
                const unsigned v3 = ((a0 >> 4) & 0x0F0F0F0Fu) | (((h >> 4) & 0x03030303u) << 4);
                const unsigned v4 = ((b0 >> 4) & 0x0F0F0F0Fu) | (((h >> 6) & 0x03030303u) << 4);
                d1 = dp4a_us(v1, (int)word_of(X0, t), d1);
                d2 = dp4a_us(v2, (int)word_of(X1, t), d2);
                d3 = dp4a_us(v3, (int)word_of(X2, t), d3);
                d4 = dp4a_us(v4, (int)word_of(X3, t), d4);
            }
            const int g = 8 * half + is;   // scale index sc_h[is + 2q] and the matching 16-code group
            d1 -= 32 * s16[g];
            d2 -= 32 * s16[g + 2];
            d3 -= 32 * s16[g + 4];
            d4 -= 32 * s16[g + 6];
            bs = __fadd_rn(bs, __fmul_rn((float)(int8_t)byte_of(scw, g), __int2float_rn(d1)));
            bs = __fadd_rn(bs, __fmul_rn((float)(int8_t)byte_of(scw, g + 2), __int2float_rn(d2)));
            bs = __fadd_rn(bs, __fmul_rn((float)(int8_t)byte_of(scw, g + 4), __int2float_rn(d3)));
            bs = __fadd_rn(bs, __fmul_rn((float)(int8_t)byte_of(scw, g + 6), __int2float_rn(d4)));
        }
    }
    return __fmul_rn(__fmul_rn(d, a.sx[b]), bs);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_n() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Programmatic dependent launch: let the next kernel in the stream start, and wait
// for the previous one to complete (both return at once outside such launches).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Asynchronous coalesced copy of `bytes` (a multiple of 16, both ends 16-byte
// aligned) into a warp's staging area; one commit group per call.
__device__ __forceinline__ void stage_issue(uint8_t* dst, const uint8_t* __restrict__ src, int bytes, int lane) {
    const int n = bytes >> 4;
    for (int i = lane; i < n; i += 32) cp_async16(dst + 16 * i, src + 16 * i);
    cp_async_commit();
}

// Quantised rows [r0, r0 + nr) of matrix M: issue the copy of their units when they
// fit one chunk (32 units); returns whether it did.
template <int FMT>
__device__ __forceinline__ bool kq_issue(const uint8_t* __restrict__ M, int bpr, int r0, int nr, uint8_t* stage,
                                         int lane) {
    constexpr int BB = FMT == KQ_Q4K ? Q4K_B : Q6K_BODY;
    const int units = nr * bpr;
    if (units == 0 || units > 32) return false;
    stage_issue(stage, M + (size_t)r0 * bpr * BB, units * BB, lane);
    return true;
}

// Rows [r0, r0 + nr) of a quantised matrix against activation a: returns the row
// total of row r0 + lane in lanes < nr (0 elsewhere).  `issued`: the first chunk is
// already in flight (kq_issue).
template <int FMT>
__device__ float kq_rows_warp(const uint8_t* __restrict__ M, long long nblk, int bpr, int r0, int nr,
                              const KAct& a, uint8_t* stage, float* terms, int lane, bool issued) {
    constexpr int BB = FMT == KQ_Q4K ? Q4K_B : Q6K_BODY;
    const long long ubase = (long long)r0 * bpr;
    const int units = nr * bpr;
    const uint16_t* d6 = reinterpret_cast<const uint16_t*>(M + (size_t)nblk * Q6K_BODY);
    for (int c = 0; c < units; c += 32) {
        const int cnt = min(32, units - c);
        if (!(issued && c == 0)) {
            __syncwarp();
            stage_issue(stage, M + (size_t)(ubase + c) * BB, cnt * BB, lane);
        }
        cp_async_wait_all();
        __syncwarp();
        if (lane < cnt) {
            const int b = (c + lane) % bpr;
            float t;
            if constexpr (FMT == KQ_Q4K)
                t = q4k_term(stage + lane * BB, a, b);
            else
                t = q6k_term(stage + lane * BB, f16_bits_to_f32(__ldg(d6 + ubase + c + lane)), a, b);
            terms[c + lane] = t;
        }
        __syncwarp();
    }
    float tot = 0.0f;
    if (lane < nr)
        for (int j = 0; j < bpr; j++) tot = __fadd_rn(tot, terms[lane * bpr + j]);
    __syncwarp();
    return tot;
}

// Column chunk c (FCH values) of rows [r0, r0 + nr) of an f16 / f32 matrix into ring
// slot c % FDEPTH of a warp's staging area; one commit group per call (empty past the
// last chunk).
template <int FMT>
__device__ __forceinline__ void fx_issue(const uint8_t* __restrict__ M, int cols, int r0, int nr, uint8_t* stage,
                                         int c, int lane) {
    constexpr int ES = FMT == KQ_F16 ? 2 : 4;
    constexpr int RS = FCH * ES + 16;   // padded staged row stride
    if (c * FCH < cols) {
        const int c0 = c * FCH, cw = min(FCH, cols - c0), per_row = cw * ES / 16;
        uint8_t* slot = stage + (c % FDEPTH) * fx_slot_bytes(FMT);
        for (int i = lane; i < nr * per_row; i += 32) {
            const int r = i / per_row, k = i - r * per_row;
            cp_async16(slot + r * RS + k * 16, M + ((size_t)(r0 + r) * cols + c0) * ES + 16 * k);
        }
    }
    cp_async_commit();
}

// Rows [r0, r0 + nr) (nr <= 4) of an f16 / f32 matrix against fp32 x in shared
// memory, csrc/libtinygiant.c:262-318: lane (row i, chain v) runs the fused sum of
// columns v, v + 8, ...; the eight chains fold as (v, v + 4) then pairwise.  Returns
// the total in lane 8 * i.  FDEPTH column chunks stay in flight (`issued`: the
// first FDEPTH are already, fx_issue).
template <int FMT>
__device__ float fx_rows_warp(const uint8_t* __restrict__ M, int cols, int r0, int nr, const float* xs,
                              uint8_t* stage, int lane, bool issued) {
    constexpr int ES = FMT == KQ_F16 ? 2 : 4;
    constexpr int RS = FCH * ES + 16;
    const int ri = lane >> 3, v = lane & 7;
    if (!issued)
        for (int c = 0; c < FDEPTH; c++) fx_issue<FMT>(M, cols, r0, nr, stage, c, lane);
    const int nch = (cols + FCH - 1) / FCH;
    float acc = 0.0f;
    for (int c = 0; c < nch; c++) {
        cp_async_wait_n<FDEPTH - 1>();   // groups complete in order: chunk c has landed
        __syncwarp();
        const int c0 = c * FCH, cw = min(FCH, cols - c0);
        if (ri < nr) {
            const uint8_t* row = stage + (c % FDEPTH) * fx_slot_bytes(FMT) + ri * RS;
#pragma unroll 8
            for (int s = 0; s < cw / 8; s++) {
                const int col = 8 * s + v;
                float w = FMT == KQ_F16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t*>(row)[col])
                                        : reinterpret_cast<const float*>(row)[col];
                acc = __fmaf_rn(w, xs[c0 + col], acc);
            }
        }
        __syncwarp();
        fx_issue<FMT>(M, cols, r0, nr, stage, c + FDEPTH, lane);
    }
    cp_async_wait_n<0>();
    __syncwarp();
    const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));   // chains v and v + 4
    const float p = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 1));      // (t0 + t1), (t2 + t3)
    return __fadd_rn(p, __shfl_down_sync(0xffffffffu, p, 2));                // in lane 8i
}

struct KQParams {
    const uint8_t* mat;           // MODE 0: the matrix
    const uint8_t* const* A;      // MODE 1: gate matrices [n]; MODE 2: down matrices [n]
    const uint8_t* const* B;      // MODE 1: up matrices [n]
    const float* x;               // MODE 0 / 1: input [cols]; MODE 2: h [n][cols]
    const float* w;               // MODE 2: combine weights [n]
    float* out;                   // MODE 0: y [rows]; MODE 1: h [n][rows]; MODE 2: out [rows]
    float* ys;                    // MODE 2: per-expert rows y [n][rows]
    unsigned* cnt;                // MODE 2: arrivals per row block (zero between launches)
    int rows, cols, n, accumulate;
};

// MODE 0: y = M . x.  MODE 1 (grid.y = expert e): h_e = silu(gate_e . x) * (up_e . x),
// gate / up Q4_K.  MODE 2 (grid.y = expert e): y_e = down_e . h_e into ys; the last
// CTA of each row block then writes out = (accumulate ? out : 0) + sum_e w_e * y_e,
// experts added in order.
template <int FMT, int MODE>
__global__ void __launch_bounds__(KT) k_kq(KQParams p) {
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr bool FLOAT_FMT = FMT == KQ_F16 || FMT == KQ_F32;
    constexpr int SB = stage_bytes(FMT);
    const int cols = p.cols, bpr = cols / 256;
    uint8_t* act = sm;
    uint8_t* stage = sm + act_region(FMT, cols) + (size_t)warp * warp_bytes(FMT, MODE, cols);
    float* terms = reinterpret_cast<float*>(stage + (MODE == 1 ? 2 : 1) * SB);
    const KAct a = act_at(act, bpr);
    float* xs = reinterpret_cast<float*>(act);
    const int rpw = rows_per_warp(FMT, cols);
    const int r0 = (blockIdx.x * KW + warp) * rpw;
    const int nr = r0 < p.rows ? min(rpw, p.rows - r0) : 0;
    const long long nblk = (long long)p.rows * bpr;
    const bool has = FLOAT_FMT ? ((lane & 7) == 0 && (lane >> 3) < nr) : lane < nr;
    const int row = r0 + (FLOAT_FMT ? (lane >> 3) : lane);
    const int e = blockIdx.y;
    const uint8_t* M0 = MODE == 0 ? p.mat : p.A[e];

    pdl_trigger();
    // weights do not depend on the previous kernel: start their copies first
    bool issued0 = false, issued1 = false;
    if constexpr (!FLOAT_FMT) {
        issued0 = kq_issue<FMT>(M0, bpr, r0, nr, stage, lane);
        if constexpr (MODE == 1) issued1 = kq_issue<FMT>(p.B[e], bpr, r0, nr, stage + SB, lane);
    } else if (nr > 0) {
        for (int c = 0; c < FDEPTH; c++) fx_issue<FMT>(M0, cols, r0, nr, stage, c, lane);
        issued0 = true;
    }
    pdl_wait();
    const float* xin = MODE == 2 ? p.x + (size_t)e * cols : p.x;
    if constexpr (FLOAT_FMT) {
        for (int i = threadIdx.x; i < cols / 4; i += KT)
            reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(xin)[i];
    } else {
        quantize_q8k(xin, bpr, a, warp, lane);
    }
    __syncthreads();

    auto rows_dot = [&](const uint8_t* M, uint8_t* st, bool issued) -> float {
        if (nr == 0) return 0.0f;
        if constexpr (FLOAT_FMT)
            return fx_rows_warp<FMT>(M, cols, r0, nr, xs, st, lane, issued);
        else
            return kq_rows_warp<FMT>(M, nblk, bpr, r0, nr, a, st, terms, lane, issued);
    };

    if constexpr (MODE == 0) {
        float y = rows_dot(M0, stage, issued0);
        if (has) p.out[row] = p.accumulate ? __fadd_rn(p.out[row], y) : y;
    } else if constexpr (MODE == 1) {
        float g = rows_dot(M0, stage, issued0);
        float u = rows_dot(p.B[e], stage + SB, issued1);
        if (has) p.out[(size_t)e * p.rows + row] = silu_mul(g, u);
    } else {
        float y = rows_dot(M0, stage, issued0);
        if (has) p.ys[(size_t)e * p.rows + row] = y;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = atomicAdd(p.cnt + blockIdx.x, 1u) == (unsigned)(p.n - 1);
        __syncthreads();
        if (s_last) {
            __threadfence();
            const int rb = rpw * KW;
            const int lo = blockIdx.x * rb, hi = min(p.rows, lo + rb);
            for (int r = lo + threadIdx.x; r < hi; r += KT) {
                float acc = p.accumulate ? p.out[r] : 0.0f;
                for (int j = 0; j < p.n; j++)
                    acc = __fadd_rn(acc, __fmul_rn(__ldg(p.w + j), __ldcg(p.ys + (size_t)j * p.rows + r)));
                p.out[r] = acc;
            }
            if (threadIdx.x == 0) p.cnt[blockIdx.x] = 0u;
        }
    }
}

// Q6_K ggml blocks -> split layout (bodies, then d), one 2-byte word per thread.
__global__ void k_split_q6k(const uint16_t* __restrict__ src, uint8_t* __restrict__ dst, long long nblk) {
    const long long n = nblk * (Q6K_B / 2);
    uint16_t* body = reinterpret_cast<uint16_t*>(dst);
    uint16_t* dd = reinterpret_cast<uint16_t*>(dst + (size_t)nblk * Q6K_BODY);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long u = i / (Q6K_B / 2);
        const int k = (int)(i - u * (Q6K_B / 2));
        const uint16_t v = src[i];
        if (k < Q6K_BODY / 2)
            body[u * (Q6K_BODY / 2) + k] = v;
        else
            dd[u] = v;
    }
}

// tg_rms_norm, csrc/libtinygiant.c:322-340, one CTA: four fused sums of x^2 (chain v
// over elements v, v + 4, ...), folded pairwise; scale = 1 / sqrtf(ss / dim + eps);
// out = (x * scale) * w.
// x is staged in shared memory first (up to RMS_STAGE floats from a 16-byte aligned
// x; otherwise read from global memory), so the four chains run at the fused
// multiply-add latency.
constexpr int RMS_STAGE = 8192;
__global__ void k_rms_norm_ref(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out,
                               int dim, float eps) {
    __shared__ float s_scale;
    __shared__ __align__(16) float xs[RMS_STAGE];
    const bool staged = dim <= RMS_STAGE && ((uintptr_t)x & 15) == 0;
    if (staged) {
        for (int i = threadIdx.x; i < dim / 4; i += blockDim.x)
            reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(x)[i];
        __syncthreads();
    }
    const float* xv = staged ? xs : x;
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        float acc = 0.0f;
        if (lane < 4) {
#pragma unroll 16
            for (int i = lane; i < dim; i += 4) acc = __fmaf_rn(xv[i], xv[i], acc);
        }
        const float p = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));   // (s0 + s1), (s2 + s3)
        const float ss = __fadd_rn(p, __shfl_down_sync(0xffffffffu, p, 2));
        if (lane == 0) s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
    }
    __syncthreads();
    const float sc = s_scale;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(xv[i], sc), w[i]);
}

int row_blocks(int fmt, int rows, int cols) {
    const int rb = rows_per_warp(fmt, cols) * KW;
    return (rows + rb - 1) / rb;
}

// pdl: launch as a programmatic dependent of the previous kernel on the stream (its
// weight copies start before that kernel completes).  Only for a previous kernel that
// does not write this launch's weights or pointer arrays.
template <int FMT, int MODE>
cudaError_t launch_kq_t(const KQParams& p, int grid_y, bool pdl, cudaStream_t s) {
    const size_t smem = kq_smem(FMT, MODE, p.cols);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_kq<FMT, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(row_blocks(FMT, p.rows, p.cols), grid_y);
    cfg.blockDim = dim3(KT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_kq<FMT, MODE>, p);
}

template <int MODE>
cudaError_t launch_kq_fmt(int fmt, const KQParams& p, int grid_y, bool pdl, cudaStream_t s) {
    switch (fmt) {
        case KQ_Q4K: return launch_kq_t<KQ_Q4K, MODE>(p, grid_y, pdl, s);
        case KQ_Q6K: return launch_kq_t<KQ_Q6K, MODE>(p, grid_y, pdl, s);
        case KQ_F16: return launch_kq_t<KQ_F16, MODE>(p, grid_y, pdl, s);
        case KQ_F32: return launch_kq_t<KQ_F32, MODE>(p, grid_y, pdl, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool kq_valid(int fmt, int rows, int cols) {
    if (rows <= 0 || cols <= 0) return false;
    if (fmt == KQ_Q4K || fmt == KQ_Q6K) return cols % 256 == 0 && cols <= 65536;
    if (fmt == KQ_F16 || fmt == KQ_F32) return cols % 8 == 0 && cols <= 32768;   // x staged as fp32
    return false;
}

size_t kq_matrix_bytes(int fmt, long long rows, int cols) {
    switch (fmt) {
        case KQ_Q4K: return (size_t)rows * (cols / 256) * Q4K_B;
        case KQ_Q6K: return (size_t)rows * (cols / 256) * Q6K_B;
        case KQ_F16: return (size_t)rows * cols * 2;
        case KQ_F32: return (size_t)rows * cols * 4;
        default: return 0;
    }
}

size_t kq_smem_bytes(int fmt, int cols) {
    size_t a = kq_smem(fmt, 0, cols), b = kq_smem(fmt, 2, cols);
    return a > b ? a : b;
}

// Down scratch: the row-block arrival counters first, in a fixed region large enough
// for any shape (at least 4 rows per CTA, H <= 16384), so counters left at zero by
// one shape are zero for every other; then y [n][H].
constexpr size_t KQ_CNT_BYTES = 16384 / 4 * 4;

size_t kq_down_scratch_bytes(int n, int H, int I) {
    (void)I;
    return KQ_CNT_BYTES + r16((size_t)n * H * 4);
}

cudaError_t launch_kq_split_q6k(const uint8_t* raw, uint8_t* dst, long long nblk, cudaStream_t s) {
    if (nblk <= 0) return cudaSuccess;
    long long words = nblk * (Q6K_B / 2);
    int grid = (int)((words + 255) / 256);
    if (grid > 148 * 16) grid = 148 * 16;
    k_split_q6k<<<grid, 256, 0, s>>>(reinterpret_cast<const uint16_t*>(raw), dst, nblk);
    return cudaGetLastError();
}

cudaError_t launch_kq_matvec(int fmt, const uint8_t* W, const float* x, float* y, int rows, int cols, cudaStream_t s,
                             bool pdl, bool accumulate) {
    KQParams p{};
    p.mat = W;
    p.x = x;
    p.out = y;
    p.rows = rows;
    p.cols = cols;
    p.n = 1;
    p.accumulate = accumulate ? 1 : 0;
    return launch_kq_fmt<0>(fmt, p, 1, pdl, s);
}

cudaError_t launch_kq_gateup(const uint8_t* const* gate, const uint8_t* const* up, int n, const float* x, int H,
                             int I, float* h, bool pdl, cudaStream_t s) {
    KQParams p{};
    p.A = gate;
    p.B = up;
    p.x = x;
    p.out = h;
    p.rows = I;
    p.cols = H;
    p.n = n;
    return launch_kq_t<KQ_Q4K, 1>(p, n, pdl, s);
}

cudaError_t launch_kq_down(int fmt, const uint8_t* const* down, int n, const float* h, const float* w, int H, int I,
                           float* out, int accumulate, void* scratch, cudaStream_t s) {
    KQParams p{};
    p.A = down;
    p.x = h;
    p.w = w;
    p.out = out;
    p.cnt = (unsigned*)scratch;
    p.ys = (float*)((uint8_t*)scratch + KQ_CNT_BYTES);
    p.rows = H;
    p.cols = I;
    p.n = n;
    p.accumulate = accumulate;
    return launch_kq_fmt<2>(fmt, p, n, true, s);
}

cudaError_t launch_rms_norm_ref(const float* x, const float* w, float* out, int dim, float eps, cudaStream_t s) {
    k_rms_norm_ref<<<1, 1024, 0, s>>>(x, w, out, dim, eps);
    return cudaGetLastError();
}

}  // namespace tg

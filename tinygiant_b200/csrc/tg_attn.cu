// tg_attn.cu — the reference's GQA attention decode step for one token on the GPU
// (csrc/libtinygiant.c:344-551: tg_attention_decode with fp32 weights,
// tg_attention_decode_q4 with Q4_K wq / wk / wo and f16 wv).
//
//   q, k, v = Wq.x, Wk.x, Wv.x            k_kq matvecs (tg_kquant.cu), the reference's order
//   per-head RMSNorm of q and k, RoPE       k_attn_qk; k and v appended at row kv_len
//   scores, softmax, weighted sum of V     k_attn_scores, k_attn_softmax_v
//   out = Wo.attn                          k_kq matvec
//
// Float work follows the reference source operation by operation, each rounded on
// its own except the source's fused multiply-adds (vfmaq_f32):
//   * RMSNorm: four fused chains of x^2 (chain v over elements v, v + 4, ...) added
//     pairwise, scale = 1 / sqrtf(ss / dim + 1e-6), out = (x * scale) * w;
//   * RoPE (vmlsq_f32 / vfmaq_f32): x1' = x1*c - x2*s, x2' = fma(x1, s, x2*c);
//   * score_t = ((a0 + a1) + (a2 + a3)) * (1 / sqrtf(head_dim)), a_v the fused chain of
//     q[d] * k_t[d] over d = v, v + 4, ...;
//   * softmax: the max of -1e30 and the scores, e_t = exp(score_t - max), the e_t
//     summed in t order from 0, w_t = e_t * (1 / sum);
//   * out[d] = the fused chain of w_t * v_t[d] over t = 0 .. kv_len.
// exp is tg_expf (tg_device.cuh), as in every other kernel of this library.  So the
// results equal the oracle's bit for bit, and the reference's within its expf.
//
// The sum of the e_t and each output element are single chains over the cached rows,
// as in the reference; every other step runs in parallel over rows and heads.  The
// cache layout is the reference's, [n_kv][kv_max][head_dim] fp32 per layer.
//
// Every kernel is a programmatic dependent launch: it starts while its predecessor
// finishes and waits (griddepcontrol.wait) before reading that predecessor's output,
// so the projection kernels' weight copies overlap the kernels before them.  The
// position can come from a device word (pos_dev) so that a captured CUDA graph
// replays steps at successive positions; grids are then sized for kv_max and the
// blocks beyond the current rows return at once.
#include <cuda_runtime.h>

#include <cmath>
#include <string>
#include <vector>

#include "../../include/tinygiant.h"
#include "tg_device.cuh"
#include "tg_internal.h"

namespace tg {

namespace {

constexpr int ROWS = 32;   // cached rows per scores CTA: one per lane

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

struct AttnArgs {
    const float* qkv;        // projections: q [NH*HD] | k [NKV*HD] | v [NKV*HD]
    const float* q_norm;     // [HD]
    const float* k_norm;     // [HD]
    const float* rope_cos;   // [positions][HD/2]
    const float* rope_sin;
    float* qf;               // normalised, rotated q [NH*HD]
    float* kv_k;             // [NKV][kv_max][HD]
    float* kv_v;
    float* S;                // scores [NH][s_stride]
    float* att;              // attention output [NH*HD]
    int* pos_dev;            // when set: kv_len = pos = pos_dev[0]; pos_dev[1] the error word
    int NH, NKV, HD, kv_max, kv_len, pos;
    int s_stride;            // floats per score row: kv_max rounded up to 4 (16-byte rows)
};

__device__ __forceinline__ int kv_len_of(const AttnArgs& a) { return a.pos_dev ? *a.pos_dev : a.kv_len; }
__device__ __forceinline__ int pos_of(const AttnArgs& a) { return a.pos_dev ? *a.pos_dev : a.pos; }
// A device position outside the cache: the step writes no cache row (the host checks
// the immediate form before launching).
__device__ __forceinline__ bool bad_row(const AttnArgs& a, int kv_len) { return kv_len < 0 || kv_len >= a.kv_max; }

// Grid NH + NKV, one warp each, shared memory 4 * HD floats.  CTA b < NH: query head
// b -> qf.  CTA NH + j: kv head j -> k at row kv_len of kv_k, and v copied to row
// kv_len of kv_v (engine.py's cache append, libtinygiant.c:395-400).  The head's
// values, its norm weight and the rope rows are fetched together first.
__global__ void __launch_bounds__(32) k_attn_qk(AttnArgs a) {
    extern __shared__ __align__(16) float sv[];
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x, lane = threadIdx.x, HD = a.HD, half = HD / 2;
    const int kv_len = kv_len_of(a), pos = pos_of(a);
    if (bad_row(a, kv_len)) {
        if (b == 0 && lane == 0) a.pos_dev[1] = 1;
        return;
    }
    const bool is_q = b < a.NH;
    const int head = is_q ? b : b - a.NH;
    const float* src = a.qkv + (is_q ? (size_t)head * HD : (size_t)(a.NH + head) * HD);
    const float* w = is_q ? a.q_norm : a.k_norm;
    const float* c = a.rope_cos + (size_t)pos * half;
    const float* s = a.rope_sin + (size_t)pos * half;
    float* raw = sv;            // [HD]
    float* nrm = sv + HD;       // [HD]
    float* wn = sv + 2 * HD;    // [HD]
    float* cs = sv + 3 * HD;    // cos [half] | sin [half]
    for (int i = lane; i < HD; i += 32) {
        raw[i] = src[i];
        wn[i] = w[i];
    }
    for (int i = lane; i < half; i += 32) {
        cs[i] = c[i];
        cs[half + i] = s[i];
    }
    __syncwarp();
    float acc = 0.0f;
    if (lane < 4) {
#pragma unroll 8
        for (int i = lane; i < HD; i += 4) acc = __fmaf_rn(raw[i], raw[i], acc);
    }
    const float p = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));   // (s0 + s1), (s2 + s3)
    const float ss = __shfl_sync(0xffffffffu, __fadd_rn(p, __shfl_down_sync(0xffffffffu, p, 2)), 0);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), 1e-6f)));
    for (int i = lane; i < HD; i += 32) nrm[i] = __fmul_rn(__fmul_rn(raw[i], scale), wn[i]);
    __syncwarp();
    float* dst = is_q ? a.qf + (size_t)head * HD : a.kv_k + ((size_t)head * a.kv_max + kv_len) * HD;
    for (int i = lane; i < half; i += 32) {
        const float x1 = nrm[i], x2 = nrm[i + half], ci = cs[i], si = cs[half + i];
        dst[i] = __fsub_rn(__fmul_rn(x1, ci), __fmul_rn(x2, si));
        dst[i + half] = __fmaf_rn(x1, si, __fmul_rn(x2, ci));
    }
    if (!is_q) {
        const float* v = a.qkv + (size_t)(a.NH + a.NKV + head) * HD;
        float* vd = a.kv_v + ((size_t)head * a.kv_max + kv_len) * HD;
        for (int i = lane; i < HD; i += 32) vd[i] = v[i];
    }
}

// Grid (row chunks, NKV), block 32 * R threads (R = NH / NKV query heads of a kv
// head).  CTA (c, j) scores cached rows 32c .. 32c + 31 of kv head j against its R
// query heads: warp = query head, lane = row.  Rows are staged in shared memory with
// a stride of HD + 4 floats, which keeps the lanes' 16-byte reads on distinct banks.
__global__ void __launch_bounds__(1024) k_attn_scores(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    pdl_trigger();
    pdl_wait();
    const int HD = a.HD, R = a.NH / a.NKV, KS = HD + 4, q4 = HD / 4;
    const int kv_len = kv_len_of(a);
    const int seq = kv_len + 1;
    const int t0 = blockIdx.x * ROWS, j = blockIdx.y;
    if (bad_row(a, kv_len) || t0 >= seq) return;
    const int nt = min(ROWS, seq - t0);
    float* ks = sm;               // [32][KS]
    float* qs = sm + ROWS * KS;   // [R][HD]
    const float4* ksrc = reinterpret_cast<const float4*>(a.kv_k + ((size_t)j * a.kv_max + t0) * HD);
    for (int i = threadIdx.x; i < nt * q4; i += blockDim.x) {
        const int r = i / q4, c = i - r * q4;
        *reinterpret_cast<float4*>(ks + r * KS + 4 * c) = ksrc[i];
    }
    const float4* qsrc = reinterpret_cast<const float4*>(a.qf + (size_t)j * R * HD);
    for (int i = threadIdx.x; i < R * q4; i += blockDim.x) reinterpret_cast<float4*>(qs)[i] = qsrc[i];
    __syncthreads();
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane >= nt) return;
    const float* kr = ks + lane * KS;
    const float* qh = qs + w * HD;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 4
    for (int c = 0; c < q4; c++) {
        const float4 kv = *reinterpret_cast<const float4*>(kr + 4 * c);
        const float4 qv = *reinterpret_cast<const float4*>(qh + 4 * c);
        a0 = __fmaf_rn(qv.x, kv.x, a0);
        a1 = __fmaf_rn(qv.y, kv.y, a1);
        a2 = __fmaf_rn(qv.z, kv.z, a2);
        a3 = __fmaf_rn(qv.w, kv.w, a3);
    }
    const float dot = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    const float inv_sqrt = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
    a.S[(size_t)(j * R + w) * a.s_stride + t0 + lane] = __fmul_rn(dot, inv_sqrt);
}

constexpr int VST = 3;           // V ring stages
constexpr int VSTAGE = 32768;    // bytes per stage: whole cached rows
constexpr size_t SV_SMEM_MAX = 227 * 1024 - 64;   // dynamic shared memory of the softmax / V CTA

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int EPAD = 16;   // zero floats after each head's softmax weights (the sum reads 8 ahead)

// Floats per head of softmax weights: the rows, the padding, rounded to 16 bytes.
__host__ __device__ inline int e_stride(int cap) { return (cap + EPAD + 3) & ~3; }

// Query heads per softmax / V CTA: up to 4 of one kv head (dividing NH / NKV) while
// the ring and their softmax weights fit the shared memory.
__host__ __device__ inline int heads_per_cta(int R, int cap, size_t smem_max) {
    for (int hpc = 4; hpc > 1; hpc >>= 1)
        if (R % hpc == 0 && (size_t)VST * VSTAGE + (size_t)hpc * e_stride(cap) * 4 <= smem_max) return hpc;
    return 1;
}

// Grid NH / hpc, block hpc * wph * 32 threads (wph = warps per head, each thread four
// output columns).  Shared memory: a ring of VST stages of whole cached V rows (a
// stage is VSTAGE / (4 HD) rows, contiguous in the cache), then per head one softmax
// weight per cached row (+ EPAD).  The CTA's heads share one kv head, so each V row
// is staged once for all of them.
//   1. every thread starts the copies of the first VST stages;
//   2. the first warp of each head: max of -1e30 and its scores, e_t = exp(s_t - max),
//      lane 0 adds the e_t in row order, w_t = e_t * (1 / sum);
//   3. thread i of a head runs the chains of columns 4i .. 4i + 3 over the rows,
//      reading the ring; each stage is refilled as the chains leave it.
__global__ void __launch_bounds__(256) k_attn_softmax_v(AttnArgs a, int hpc, int cap) {
    extern __shared__ __align__(16) float sm[];
    pdl_trigger();
    pdl_wait();
    const int HD = a.HD, tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int wph = (HD / 4 + 31) / 32;
    const int hs = warp / wph, ht = tid - hs * wph * 32;   // head slot, thread within the head
    const int h = blockIdx.x * hpc + hs, j = h / (a.NH / a.NKV);
    const bool cols = 4 * ht < HD;
    const int kv_len = kv_len_of(a);
    if (bad_row(a, kv_len)) {   // attention output 0: the output projection then adds nothing
        if (cols) *reinterpret_cast<float4*>(a.att + (size_t)h * HD + 4 * ht) = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    // rows per stage: a multiple of 8, so each 8-row block's weights are two 16-byte reads
    const int seq = kv_len + 1, vr = (VSTAGE / (HD * 4)) & ~7, nch = (seq + vr - 1) / vr, gpr = HD / 4;
    float* ring = sm;                                           // [VST][VSTAGE / 4]
    float* e = sm + VST * (VSTAGE / 4) + (size_t)hs * e_stride(cap);   // this head's weights
    const float* vbase = a.kv_v + (size_t)j * a.kv_max * HD;
    auto issue = [&](int ch) {   // one commit group per call, empty past the last chunk
        if (ch < nch) {
            const int r0 = ch * vr, nr = min(vr, seq - r0);
            const float* src = vbase + (size_t)r0 * HD;
            float* dst = ring + (ch % VST) * (VSTAGE / 4);
            for (int i = tid; i < nr * gpr; i += nt) cp_async16(dst + 4 * i, src + 4 * i);
        }
        cp_async_commit();
    };
    if (ht < 32) {   // the head's first warp: its score row into e, ahead of the V copies
        const float* srow = a.S + (size_t)h * a.s_stride;
        for (int i = lane; i < (seq + 3) / 4; i += 32) cp_async16(e + 4 * i, srow + 4 * i);
    }
    cp_async_commit();
#pragma unroll
    for (int i = 0; i < VST; i++) issue(i);
    if (ht < 32) {   // the head's first warp: the softmax
        cp_async_wait<VST>();   // the score row has landed
        __syncwarp();
        float m = -1e30f;   // a NaN score never becomes the max, as with `>`
#pragma unroll 4
        for (int t = lane; t < seq; t += 32) m = fmaxf(m, e[t]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
#pragma unroll 4
        for (int t = lane; t < seq; t += 32) e[t] = tg_expf(__fsub_rn(e[t], m));
        for (int t = seq + lane; t < seq + EPAD; t += 32) e[t] = 0.0f;
        __syncwarp();
        float inv = 0.0f;
        if (lane == 0) {   // row order; 16-byte reads, the next two loaded before the adds
            const float4* e4 = reinterpret_cast<const float4*>(e);
            const int n8 = seq & ~7;
            float sum = 0.0f;
            float4 a0 = e4[0], a1 = e4[1];
#pragma unroll 2
            for (int t = 0; t < n8; t += 8) {
                const float4 b0 = e4[t / 4 + 2], b1 = e4[t / 4 + 3];
                sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, a0.x), a0.y), a0.z), a0.w);
                sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, a1.x), a1.y), a1.z), a1.w);
                a0 = b0;
                a1 = b1;
            }
            for (int t = n8; t < seq; t++) sum = __fadd_rn(sum, e[t]);
            inv = __fdiv_rn(1.0f, sum);
        }
        inv = __shfl_sync(0xffffffffu, inv, 0);
        for (int t = lane; t < seq; t += 32) e[t] = __fmul_rn(e[t], inv);
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int ch = 0; ch < nch; ch++) {
        cp_async_wait<VST - 1>();   // groups complete in order: chunk ch has landed
        __syncthreads();            // every thread's copies, and the weights
        const float* buf = ring + (ch % VST) * (VSTAGE / 4) + 4 * ht;
        const float* w = e + ch * vr;
        const int nr = min(vr, seq - ch * vr);
        if (cols) {   // blocks of 8 rows: their weights and V values loaded, then 32 fused steps row by row
            const int n8 = nr & ~7;
#pragma unroll 2
            for (int r = 0; r < n8; r += 8) {
                const float4 w0 = *reinterpret_cast<const float4*>(w + r);
                const float4 w1 = *reinterpret_cast<const float4*>(w + r + 4);
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; u++) v[u] = *reinterpret_cast<const float4*>(buf + (r + u) * HD);
                const float wr[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    acc.x = __fmaf_rn(wr[u], v[u].x, acc.x);
                    acc.y = __fmaf_rn(wr[u], v[u].y, acc.y);
                    acc.z = __fmaf_rn(wr[u], v[u].z, acc.z);
                    acc.w = __fmaf_rn(wr[u], v[u].w, acc.w);
                }
            }
            for (int r = n8; r < nr; r++) {
                const float4 v = *reinterpret_cast<const float4*>(buf + r * HD);
                const float wr = w[r];
                acc.x = __fmaf_rn(wr, v.x, acc.x);
                acc.y = __fmaf_rn(wr, v.y, acc.y);
                acc.z = __fmaf_rn(wr, v.z, acc.z);
                acc.w = __fmaf_rn(wr, v.w, acc.w);
            }
        }
        __syncthreads();            // the stage is free again
        issue(ch + VST);
    }
    cp_async_wait<0>();
    if (cols) *reinterpret_cast<float4*>(a.att + (size_t)h * HD + 4 * ht) = acc;
}

template <typename K, typename... Args>
cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

size_t r16f(size_t n) { return (n + 3) & ~(size_t)3; }   // floats, rounded to 16 bytes

}  // namespace

bool attention_valid(int q4, int embed, int n_heads, int n_kv, int head_dim, int kv_max) {
    if (embed <= 0 || n_heads <= 0 || n_kv <= 0 || head_dim < 8 || head_dim > 256 || head_dim % 8) return false;
    if (n_heads % n_kv || n_heads / n_kv > 32 || kv_max <= 0 || kv_max > ATTN_MAX_ROWS) return false;
    const int qd = n_heads * head_dim, kvd = n_kv * head_dim;
    const int fq = q4 ? KQ_Q4K : KQ_F32, fv = q4 ? KQ_F16 : KQ_F32;
    return kq_valid(fq, qd, embed) && kq_valid(fq, kvd, embed) && kq_valid(fv, kvd, embed) &&
           kq_valid(fq, embed, qd);
}

size_t attention_scratch_bytes(int n_heads, int n_kv, int head_dim, int kv_max) {
    const size_t qd = (size_t)n_heads * head_dim, kvd = (size_t)n_kv * head_dim;
    return 4 * (r16f(qd + 2 * kvd) + r16f(qd) + (size_t)n_heads * r16f(kv_max) + r16f(qd));
}

cudaError_t launch_attention(int q4, const uint8_t* wq, const uint8_t* wk, const uint8_t* wv, const uint8_t* wo,
                             const float* q_norm, const float* k_norm, float* kv_k, float* kv_v, int kv_len,
                             int kv_max, const float* rope_cos, const float* rope_sin, const float* x, float* out,
                             int embed, int n_heads, int n_kv, int head_dim, int pos, int* pos_dev,
                             void* scratch, cudaStream_t s, bool accumulate) {
    const int qd = n_heads * head_dim, kvd = n_kv * head_dim;
    float* base = static_cast<float*>(scratch);
    AttnArgs a{};
    a.qkv = base;
    a.qf = base + r16f((size_t)qd + 2 * kvd);
    a.S = a.qf + r16f(qd);
    a.s_stride = (int)r16f(kv_max);
    a.att = a.S + (size_t)n_heads * a.s_stride;
    a.q_norm = q_norm;
    a.k_norm = k_norm;
    a.rope_cos = rope_cos;
    a.rope_sin = rope_sin;
    a.kv_k = kv_k;
    a.kv_v = kv_v;
    a.pos_dev = pos_dev;
    a.NH = n_heads;
    a.NKV = n_kv;
    a.HD = head_dim;
    a.kv_max = kv_max;
    a.kv_len = kv_len;
    a.pos = pos;
    const int fq = q4 ? KQ_Q4K : KQ_F32, fv = q4 ? KQ_F16 : KQ_F32;
    float* qkv = base;
    cudaError_t e;
    if (wk == wq + kq_matrix_bytes(fq, qd, embed)) {   // wq | wk contiguous (the context's layout): one launch
        if ((e = launch_kq_matvec(fq, wq, x, qkv, qd + kvd, embed, s, true)) != cudaSuccess) return e;
    } else {
        if ((e = launch_kq_matvec(fq, wq, x, qkv, qd, embed, s, true)) != cudaSuccess) return e;
        if ((e = launch_kq_matvec(fq, wk, x, qkv + qd, kvd, embed, s, true)) != cudaSuccess) return e;
    }
    if ((e = launch_kq_matvec(fv, wv, x, qkv + qd + kvd, kvd, embed, s, true)) != cudaSuccess) return e;
    if ((e = launch_pdl(k_attn_qk, dim3(n_heads + n_kv), dim3(32), 4 * head_dim * sizeof(float), s, a)) != cudaSuccess)
        return e;
    // rows in play: all kv_max when the position comes from the device, else kv_len + 1
    const int cap = pos_dev ? kv_max : kv_len + 1;
    const int R = n_heads / n_kv;
    const size_t sc_smem = ((size_t)ROWS * (head_dim + 4) + (size_t)R * head_dim) * sizeof(float);
    if ((e = launch_pdl(k_attn_scores, dim3((cap + ROWS - 1) / ROWS, n_kv), dim3(32 * R), sc_smem, s, a)) != cudaSuccess)
        return e;
    const int hpc = heads_per_cta(R, cap, SV_SMEM_MAX);
    const size_t sv_smem = (size_t)VST * VSTAGE + (size_t)hpc * e_stride(cap) * sizeof(float);
    const int nt = hpc * ((head_dim / 4 + 31) / 32) * 32;
    if ((e = launch_pdl(k_attn_softmax_v, dim3(n_heads / hpc), dim3(nt), sv_smem, s, a, hpc, cap)) != cudaSuccess)
        return e;
    return launch_kq_matvec(fq, wo, a.att, out, embed, qd, s, true, accumulate);
}

}  // namespace tg

// ============================================================ C ABI (device pointers)

extern "C" size_t tgx_attention_scratch_bytes(int n_heads, int n_kv_heads, int head_dim, int kv_max) {
    if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || kv_max <= 0) return 0;
    return tg::attention_scratch_bytes(n_heads, n_kv_heads, head_dim, kv_max);
}

extern "C" int tgx_attention_decode(int q4, const void* wq, const void* wk, const void* wv, const void* wo,
                                    const float* q_norm_w, const float* k_norm_w, float* kv_k, float* kv_v,
                                    int kv_len, int kv_max, const float* rope_cos, const float* rope_sin,
                                    const float* input, float* output, int embed_dim, int n_heads, int n_kv_heads,
                                    int head_dim, int pos, void* scratch, size_t scratch_bytes, void* stream) {
    if (!wq || !wk || !wv || !wo || !q_norm_w || !k_norm_w || !kv_k || !kv_v || !rope_cos || !rope_sin || !input ||
        !output || !scratch)
        return tg::set_error(TG_EINVAL, "tgx_attention_decode: null pointer");
    if (!tg::attention_valid(q4, embed_dim, n_heads, n_kv_heads, head_dim, kv_max))
        return tg::set_error(TG_EINVAL,
                             "tgx_attention_decode: bad shape (head_dim a multiple of 8 in [8, 256]; n_heads a "
                             "multiple of n_kv_heads, at most 32 per kv head; Q4_K matrices need embed and "
                             "n_heads*head_dim multiples of 256; kv_max <= 32768)");
    if (kv_len < 0 || kv_len >= kv_max || pos < 0)
        return tg::set_error(TG_EINVAL, "tgx_attention_decode: need 0 <= kv_len < kv_max and pos >= 0");
    if (scratch_bytes < tg::attention_scratch_bytes(n_heads, n_kv_heads, head_dim, kv_max))
        return tg::set_error(TG_EINVAL, "tgx_attention_decode: scratch smaller than tgx_attention_scratch_bytes");
    cudaError_t e = tg::launch_attention(q4, (const uint8_t*)wq, (const uint8_t*)wk, (const uint8_t*)wv,
                                         (const uint8_t*)wo, q_norm_w, k_norm_w, kv_k, kv_v, kv_len, kv_max, rope_cos,
                                         rope_sin, input, output, embed_dim, n_heads, n_kv_heads, head_dim, pos,
                                         nullptr, scratch, (cudaStream_t)stream);
    if (e != cudaSuccess) return tg::set_error(TG_ECUDA, cudaGetErrorString(e));
    return TG_OK;
}

// ============================================================ device-resident attention state

namespace {

__global__ void k_pos_advance(int* pos) { pos[0] += 1; }

size_t r256(size_t n) { return (n + 255) & ~(size_t)255; }

}  // namespace

struct tgx_attn {
    int device = 0, q4 = 1, L = 0, E = 0, NH = 0, NKV = 0, HD = 0, kv_max = 0;
    float eps = 1e-6f;
    size_t bq = 0, bk = 0, bv = 0, bo = 0, layer_bytes = 0;   // matrix bytes, 256-byte aligned slots
    uint8_t* weights = nullptr;   // [L] wq | wk | wv | wo
    float* qk_norms = nullptr;    // [L][2][HD]
    float* attn_norms = nullptr;  // [L][E]
    float* rope = nullptr;        // cos [kv_max][HD/2] | sin [kv_max][HD/2]
    float* kv = nullptr;          // [L][2][NKV][kv_max][HD]
    int* pos = nullptr;           // [0] position = rows cached, [1] error word
    int host_pos = 0;             // the position the host expects the device word to hold
    float* normed = nullptr;      // [E]
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    cudaStream_t s = nullptr;
    cudaGraphExec_t gexec = nullptr;
    const float* gx = nullptr;
    tgx_ctx* gmoe = nullptr;

    float* kv_k(int l) { return kv + (size_t)l * 2 * NKV * kv_max * HD; }
    float* kv_v(int l) { return kv_k(l) + (size_t)NKV * kv_max * HD; }
    uint8_t* wq(int l) { return weights + (size_t)l * layer_bytes; }
};

namespace {

int attn_fail(int code, const std::string& msg) { return tg::set_error(code, msg.c_str()); }

#define ATT_CUDA(expr)                                                            \
    do {                                                                          \
        cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess) return attn_fail(TG_ECUDA, cudaGetErrorString(e_)); \
    } while (0)

struct AttnDevice {   // set and restore the current device around a call
    int prev = -1;
    explicit AttnDevice(int d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != d) cudaSetDevice(d);
    }
    ~AttnDevice() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Default rope tables: cos / sin of p * base^(-2i / head_dim), base 1e6 (the reference's
// ROPE_BASE), evaluated in double and rounded; tgx_attn_set_rope replaces them.
void default_rope(std::vector<float>& tab, int kv_max, int HD) {
    const int half = HD / 2;
    tab.assign((size_t)2 * kv_max * half, 0.0f);
    for (int p = 0; p < kv_max; p++)
        for (int i = 0; i < half; i++) {
            const double f = (double)p * std::pow(1.0e6, -2.0 * i / HD);
            tab[(size_t)p * half + i] = (float)std::cos(f);
            tab[(size_t)kv_max * half + (size_t)p * half + i] = (float)std::sin(f);
        }
}

int attn_layer_launch(tgx_attn* a, int layer, float* x, cudaStream_t s) {
    const uint8_t* w = a->wq(layer);
    ATT_CUDA(tg::launch_rms_norm_ref(x, a->attn_norms + (size_t)layer * a->E, a->normed, a->E, a->eps, s));
    const float* qn = a->qk_norms + (size_t)layer * 2 * a->HD;
    ATT_CUDA(tg::launch_attention(a->q4, w, w + a->bq, w + a->bq + a->bk, w + a->bq + a->bk + a->bv, qn, qn + a->HD,
                                  a->kv_k(layer), a->kv_v(layer), 0, a->kv_max, a->rope,
                                  a->rope + (size_t)a->kv_max * (a->HD / 2), a->normed, x, a->E, a->NH, a->NKV, a->HD,
                                  0, a->pos, a->scratch, s, true));
    return TG_OK;
}

int token_launch(tgx_attn* a, tgx_ctx* moe, float* x, cudaStream_t s) {
    for (int l = 0; l < a->L; l++) {
        int rc = attn_layer_launch(a, l, x, s);
        if (rc != TG_OK) return rc;
        if (moe && (rc = tgx_moe_layer(moe, l, x, s)) != TG_OK) return rc;
    }
    k_pos_advance<<<1, 1, 0, s>>>(a->pos);
    ATT_CUDA(cudaGetLastError());
    return TG_OK;
}

}  // namespace

extern "C" int tgx_attn_create(int device, int q4, int n_layers, int embed_dim, int n_heads, int n_kv_heads,
                               int head_dim, int kv_max, float eps, tgx_attn** out) {
    if (!out) return attn_fail(TG_EINVAL, "tgx_attn_create: null output");
    *out = nullptr;
    if (n_layers <= 0 || !tg::attention_valid(q4 ? 1 : 0, embed_dim, n_heads, n_kv_heads, head_dim, kv_max))
        return attn_fail(TG_EINVAL, "tgx_attn_create: bad shape (see tgx_attention_decode)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return attn_fail(TG_ENODEV, "no CUDA device");
    }
    if (device < 0 || device >= ndev) return attn_fail(TG_EINVAL, "tgx_attn_create: no such device");
    AttnDevice dg(device);
    tgx_attn* a = new tgx_attn();
    a->device = device;
    a->q4 = q4 ? 1 : 0;
    a->L = n_layers;
    a->E = embed_dim;
    a->NH = n_heads;
    a->NKV = n_kv_heads;
    a->HD = head_dim;
    a->kv_max = kv_max;
    a->eps = eps;
    const int qd = n_heads * head_dim, kvd = n_kv_heads * head_dim;
    const int fq = a->q4 ? tg::KQ_Q4K : tg::KQ_F32, fv = a->q4 ? tg::KQ_F16 : tg::KQ_F32;
    a->bq = r256(tg::kq_matrix_bytes(fq, qd, embed_dim));
    a->bk = r256(tg::kq_matrix_bytes(fq, kvd, embed_dim));
    a->bv = r256(tg::kq_matrix_bytes(fv, kvd, embed_dim));
    a->bo = r256(tg::kq_matrix_bytes(fq, embed_dim, qd));
    a->layer_bytes = a->bq + a->bk + a->bv + a->bo;
    a->scratch_bytes = tg::attention_scratch_bytes(n_heads, n_kv_heads, head_dim, kv_max);
    const size_t kv_bytes = (size_t)n_layers * 2 * kvd * kv_max * sizeof(float);
    bool ok = cudaMalloc((void**)&a->weights, a->layer_bytes * n_layers) == cudaSuccess &&
              cudaMalloc((void**)&a->qk_norms, sizeof(float) * n_layers * 2 * head_dim) == cudaSuccess &&
              cudaMalloc((void**)&a->attn_norms, sizeof(float) * n_layers * embed_dim) == cudaSuccess &&
              cudaMalloc((void**)&a->rope, sizeof(float) * kv_max * head_dim) == cudaSuccess &&
              cudaMalloc((void**)&a->kv, kv_bytes) == cudaSuccess &&
              cudaMalloc((void**)&a->pos, 2 * sizeof(int)) == cudaSuccess &&
              cudaMalloc((void**)&a->normed, sizeof(float) * embed_dim) == cudaSuccess &&
              cudaMalloc(&a->scratch, a->scratch_bytes) == cudaSuccess &&
              cudaStreamCreateWithFlags(&a->s, cudaStreamNonBlocking) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        tgx_attn_destroy(a);
        return attn_fail(TG_ENOMEM, "tgx_attn_create: device allocation failed");
    }
    std::vector<float> ones((size_t)n_layers * (2 * head_dim > embed_dim ? 2 * head_dim : embed_dim), 1.0f), tab;
    default_rope(tab, kv_max, head_dim);
    cudaError_t e = cudaMemsetAsync(a->weights, 0, a->layer_bytes * n_layers, a->s);
    if (e == cudaSuccess) e = cudaMemsetAsync(a->kv, 0, kv_bytes, a->s);
    if (e == cudaSuccess) e = cudaMemsetAsync(a->pos, 0, 2 * sizeof(int), a->s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(a->qk_norms, ones.data(), sizeof(float) * n_layers * 2 * head_dim, cudaMemcpyHostToDevice, a->s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(a->attn_norms, ones.data(), sizeof(float) * n_layers * embed_dim, cudaMemcpyHostToDevice, a->s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(a->rope, tab.data(), sizeof(float) * tab.size(), cudaMemcpyHostToDevice, a->s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(a->s);
    if (e != cudaSuccess) {
        tgx_attn_destroy(a);
        return attn_fail(TG_ECUDA, cudaGetErrorString(e));
    }
    *out = a;
    return TG_OK;
}

extern "C" int tgx_attn_destroy(tgx_attn* a) {
    if (!a) return TG_OK;
    AttnDevice dg(a->device);
    if (a->s) cudaStreamSynchronize(a->s);
    if (a->gexec) cudaGraphExecDestroy(a->gexec);
    for (void* p : {(void*)a->weights, (void*)a->qk_norms, (void*)a->attn_norms, (void*)a->rope, (void*)a->kv,
                    (void*)a->pos, (void*)a->normed, a->scratch})
        if (p) cudaFree(p);
    if (a->s) cudaStreamDestroy(a->s);
    delete a;
    return TG_OK;
}

extern "C" size_t tgx_attn_layer_bytes(const tgx_attn* a) { return a ? a->layer_bytes : 0; }

extern "C" int tgx_attn_set_layer(tgx_attn* a, int layer, const void* wq, const void* wk, const void* wv,
                                  const void* wo, const float* q_norm_w, const float* k_norm_w,
                                  const float* attn_norm_w, int src_on_device) {
    if (!a || layer < 0 || layer >= a->L) return attn_fail(TG_EINVAL, "tgx_attn_set_layer: bad context or layer");
    AttnDevice dg(a->device);
    const int qd = a->NH * a->HD, kvd = a->NKV * a->HD;
    const int fq = a->q4 ? tg::KQ_Q4K : tg::KQ_F32, fv = a->q4 ? tg::KQ_F16 : tg::KQ_F32;
    const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    uint8_t* w = a->wq(layer);
    struct Part { const void* src; uint8_t* dst; size_t n; } parts[4] = {
        {wq, w, tg::kq_matrix_bytes(fq, qd, a->E)},
        {wk, w + a->bq, tg::kq_matrix_bytes(fq, kvd, a->E)},
        {wv, w + a->bq + a->bk, tg::kq_matrix_bytes(fv, kvd, a->E)},
        {wo, w + a->bq + a->bk + a->bv, tg::kq_matrix_bytes(fq, a->E, qd)}};
    for (const Part& p : parts)
        if (p.src) ATT_CUDA(cudaMemcpyAsync(p.dst, p.src, p.n, kind, a->s));
    float* qn = a->qk_norms + (size_t)layer * 2 * a->HD;
    if (q_norm_w) ATT_CUDA(cudaMemcpyAsync(qn, q_norm_w, sizeof(float) * a->HD, kind, a->s));
    if (k_norm_w) ATT_CUDA(cudaMemcpyAsync(qn + a->HD, k_norm_w, sizeof(float) * a->HD, kind, a->s));
    if (attn_norm_w)
        ATT_CUDA(cudaMemcpyAsync(a->attn_norms + (size_t)layer * a->E, attn_norm_w, sizeof(float) * a->E, kind, a->s));
    ATT_CUDA(cudaStreamSynchronize(a->s));
    return TG_OK;
}

extern "C" int tgx_attn_set_rope(tgx_attn* a, const float* rope_cos, const float* rope_sin, int n_pos,
                                 int src_on_device) {
    if (!a || !rope_cos || !rope_sin || n_pos < a->kv_max)
        return attn_fail(TG_EINVAL, "tgx_attn_set_rope: null pointer or fewer rows than kv_max");
    AttnDevice dg(a->device);
    const size_t n = (size_t)a->kv_max * (a->HD / 2) * sizeof(float);
    const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    ATT_CUDA(cudaMemcpyAsync(a->rope, rope_cos, n, kind, a->s));
    ATT_CUDA(cudaMemcpyAsync((uint8_t*)a->rope + n, rope_sin, n, kind, a->s));
    ATT_CUDA(cudaStreamSynchronize(a->s));
    return TG_OK;
}

extern "C" int tgx_attn_set_pos(tgx_attn* a, int pos) {
    if (!a || pos < 0 || pos >= a->kv_max) return attn_fail(TG_EINVAL, "tgx_attn_set_pos: need 0 <= pos < kv_max");
    AttnDevice dg(a->device);
    ATT_CUDA(cudaDeviceSynchronize());
    int w[2] = {pos, 0};
    ATT_CUDA(cudaMemcpy(a->pos, w, sizeof(w), cudaMemcpyHostToDevice));
    a->host_pos = pos;
    return TG_OK;
}

extern "C" int tgx_attn_status(tgx_attn* a, int* pos) {
    if (!a) return attn_fail(TG_EINVAL, "tgx_attn_status: null context");
    AttnDevice dg(a->device);
    ATT_CUDA(cudaDeviceSynchronize());
    int w[2] = {0, 0};
    ATT_CUDA(cudaMemcpy(w, a->pos, sizeof(w), cudaMemcpyDeviceToHost));
    if (pos) *pos = w[0];
    if (w[1]) {
        int z = 0;
        ATT_CUDA(cudaMemcpy(a->pos + 1, &z, sizeof(int), cudaMemcpyHostToDevice));
        return attn_fail(TG_EINVAL, "attention: a step ran at a position outside the cache (nothing was written)");
    }
    return TG_OK;
}

extern "C" int tgx_attn_kv(tgx_attn* a, int layer, float** kv_k_dev, float** kv_v_dev) {
    if (!a || layer < 0 || layer >= a->L) return attn_fail(TG_EINVAL, "tgx_attn_kv: bad context or layer");
    if (kv_k_dev) *kv_k_dev = a->kv_k(layer);
    if (kv_v_dev) *kv_v_dev = a->kv_v(layer);
    return TG_OK;
}

extern "C" int tgx_attn_read_kv(tgx_attn* a, int layer, float* kv_k_host, float* kv_v_host) {
    if (!a || layer < 0 || layer >= a->L) return attn_fail(TG_EINVAL, "tgx_attn_read_kv: bad context or layer");
    AttnDevice dg(a->device);
    ATT_CUDA(cudaDeviceSynchronize());
    const size_t n = (size_t)a->NKV * a->kv_max * a->HD * sizeof(float);
    if (kv_k_host) ATT_CUDA(cudaMemcpy(kv_k_host, a->kv_k(layer), n, cudaMemcpyDeviceToHost));
    if (kv_v_host) ATT_CUDA(cudaMemcpy(kv_v_host, a->kv_v(layer), n, cudaMemcpyDeviceToHost));
    return TG_OK;
}

extern "C" int tgx_attn_layer(tgx_attn* a, int layer, float* x_dev, void* stream) {
    if (!a || !x_dev || layer < 0 || layer >= a->L) return attn_fail(TG_EINVAL, "tgx_attn_layer: bad arguments");
    if (a->host_pos >= a->kv_max) return attn_fail(TG_EINVAL, "tgx_attn_layer: the cache is full (pos == kv_max)");
    AttnDevice dg(a->device);
    return attn_layer_launch(a, layer, x_dev, (cudaStream_t)stream);
}

extern "C" int tgx_attn_advance(tgx_attn* a, void* stream) {
    if (!a) return attn_fail(TG_EINVAL, "tgx_attn_advance: null context");
    AttnDevice dg(a->device);
    k_pos_advance<<<1, 1, 0, (cudaStream_t)stream>>>(a->pos);
    ATT_CUDA(cudaGetLastError());
    a->host_pos++;
    return TG_OK;
}

extern "C" int tgx_decode_token(tgx_attn* a, tgx_ctx* moe, float* x_dev, void* stream, int flags) {
    if (!a || !x_dev) return attn_fail(TG_EINVAL, "tgx_decode_token: null argument");
    if (a->host_pos >= a->kv_max) return attn_fail(TG_EINVAL, "tgx_decode_token: the cache is full (pos == kv_max)");
    AttnDevice dg(a->device);
    cudaStream_t s = (cudaStream_t)stream;
    if (flags & TGX_EAGER) {
        int rc = token_launch(a, moe, x_dev, s);
        if (rc == TG_OK) a->host_pos++;
        return rc;
    }
    if (!a->gexec || a->gx != x_dev || a->gmoe != moe) {
        if (a->gexec) cudaGraphExecDestroy(a->gexec);
        a->gexec = nullptr;
        a->gx = nullptr;
        cudaGraph_t graph = nullptr;
        ATT_CUDA(cudaStreamBeginCapture(a->s, cudaStreamCaptureModeThreadLocal));
        int rc = token_launch(a, moe, x_dev, a->s);
        cudaError_t e = cudaStreamEndCapture(a->s, &graph);
        if (rc != TG_OK) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        ATT_CUDA(e);
        e = cudaGraphInstantiate(&a->gexec, graph, 0);
        cudaGraphDestroy(graph);
        ATT_CUDA(e);
        a->gx = x_dev;
        a->gmoe = moe;
    }
    ATT_CUDA(cudaGraphLaunch(a->gexec, s));
    a->host_pos++;
    return TG_OK;
}

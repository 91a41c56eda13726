// tg_kernels.cu — Q4_0 x Q8_0 kernels for the MoE expert-FFN path (sm_100a).
//
// Kernels (each mirrors a routine of the reference, cited at the kernel):
//   k_repack_rows / k_unpack_rows  ggml rows <-> row-split rows (layout in tg_layout.h)
//   k_quantize_act                 Q8_0 activation quantiser (libtinygiant.c:61-89)
//   k_quantize_q4_0                Q4_0 weight quantiser (gguf Q4_0.quantize_blocks)
//   k_matvec / k_block_dots        Q4_0 matvec (libtinygiant.c:173-185), exact block dots
//   k_router_topk                  router + top-k + softmax (engine.py:231-236)
//   k_gateup                       grouped gate/up + SwiGLU + Q8_0 requant (libtinygiant.c:566-586)
//   k_down_combine                 grouped down + weighted combine (libtinygiant.c:588-594,
//                                  647-655; engine.py:240-258)
// Row dots: one warp per row, lane L takes blocks L, L+32, ... and the 32
// partial sums are reduced with an xor butterfly (the oracle's mirror order).
#include <cuda_runtime.h>

#include <mutex>

#include "tg_device.cuh"
#include "tg_internal.h"

namespace tg {

namespace {

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_nc_u16(const void* p) {
    unsigned short v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Quantise f32 x[0 .. 32*nb) into an activation view, one warp per block.  With
// a norm (scale != null) the quantised values are (x * scale) * normw.
__device__ __forceinline__ void quantize_to_act(const float* __restrict__ x, int nb, ActView a,
                                                int warp, int nwarps, int lane,
                                                const float* __restrict__ normw = nullptr,
                                                const float* __restrict__ scale = nullptr) {
    const float sc = scale ? *scale : 1.0f;
    for (int b = warp; b < nb; b += nwarps) {
        float v = x[(size_t)b * 32 + lane];
        if (scale) v = __fmul_rn(__fmul_rn(v, sc), normw[(size_t)b * 32 + lane]);
        Q8Lane q = quantize_lane(v);
        a.qs[(size_t)b * 32 + lane] = (int8_t)q.q;
        if (lane == 0) {
            a.d[b] = f16_bits_to_f32(q.dh);
            a.s8[b] = q.s8;
        }
    }
}

// Store one Q4_0 block held one code per lane (lane = element) as nine aligned
// 16-bit words: scale, then nibble bytes (element j low, element j+16 high).
__device__ __forceinline__ void store_q4_0_block(uint8_t* o, uint16_t dh, int q, int lane) {
    __syncwarp();
    int qh = __shfl_down_sync(0xffffffffu, q, 16);
    unsigned byte = (unsigned)(q | (qh << 4)) & 0xffu;         // valid in lanes 0..15
    unsigned b0 = __shfl_sync(0xffffffffu, byte, (2 * lane) & 31);
    unsigned b1 = __shfl_sync(0xffffffffu, byte, (2 * lane + 1) & 31);
    uint16_t* o16 = reinterpret_cast<uint16_t*>(o);
    if (lane == 0) o16[0] = dh;
    if (lane < 8) o16[1 + lane] = (uint16_t)(b0 | (b1 << 8));
}

}  // namespace

// ------------------------------------------------------------------ layout

__global__ void k_repack_rows(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                              long long nblocks, int nb) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nblocks) return;
    long long row = t / nb;
    int b = (int)(t - row * nb);
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src + t * 18);
    uint8_t* rb = dst + row * (long long)nb * 18;
    uint4 v;
    v.x = (uint32_t)s[1] | ((uint32_t)s[2] << 16);
    v.y = (uint32_t)s[3] | ((uint32_t)s[4] << 16);
    v.z = (uint32_t)s[5] | ((uint32_t)s[6] << 16);
    v.w = (uint32_t)s[7] | ((uint32_t)s[8] << 16);
    *reinterpret_cast<uint4*>(rb + 16 * b) = v;
    *reinterpret_cast<uint16_t*>(rb + 16 * (long long)nb + 2 * b) = s[0];
}

__global__ void k_unpack_rows(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                              long long nblocks, int nb) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nblocks) return;
    long long row = t / nb;
    int b = (int)(t - row * nb);
    const uint8_t* rb = src + row * (long long)nb * 18;
    uint4 v = *reinterpret_cast<const uint4*>(rb + 16 * b);
    uint16_t* d = reinterpret_cast<uint16_t*>(dst + t * 18);
    d[0] = *reinterpret_cast<const uint16_t*>(rb + 16 * (long long)nb + 2 * b);
    d[1] = (uint16_t)v.x; d[2] = (uint16_t)(v.x >> 16);
    d[3] = (uint16_t)v.y; d[4] = (uint16_t)(v.y >> 16);
    d[5] = (uint16_t)v.z; d[6] = (uint16_t)(v.z >> 16);
    d[7] = (uint16_t)v.w; d[8] = (uint16_t)(v.w >> 16);
}

cudaError_t launch_repack_rows(const uint8_t* src, uint8_t* dst, long long nrows, int nb, cudaStream_t s) {
    long long n = nrows * nb;
    if (n <= 0) return cudaSuccess;
    k_repack_rows<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, dst, n, nb);
    return cudaGetLastError();
}

cudaError_t launch_unpack_rows(const uint8_t* src, uint8_t* dst, long long nrows, int nb, cudaStream_t s) {
    long long n = nrows * nb;
    if (n <= 0) return cudaSuccess;
    k_unpack_rows<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, dst, n, nb);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ quantisers

__global__ void k_quantize_act(const float* __restrict__ x, int nb, ActView a, uint8_t* __restrict__ ggml) {
    int warp = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5);
    int lane = threadIdx.x & 31;
    if (warp >= nb) return;
    float v = x[(size_t)warp * 32 + lane];
    Q8Lane q = quantize_lane(v);
    a.qs[(size_t)warp * 32 + lane] = (int8_t)q.q;
    if (lane == 0) {
        a.d[warp] = f16_bits_to_f32(q.dh);
        a.s8[warp] = q.s8;
    }
    if (ggml) {
        uint8_t* o = ggml + (size_t)warp * Q8_0_BYTES;
        o[2 + lane] = (uint8_t)(int8_t)q.q;
        if (lane == 0) {
            o[0] = (uint8_t)(q.dh & 0xff);
            o[1] = (uint8_t)(q.dh >> 8);
        }
    }
}

__global__ void k_q8_0_to_act(const uint8_t* __restrict__ ggml, int nb, ActView a) {
    int warp = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5);
    int lane = threadIdx.x & 31;
    if (warp >= nb) return;
    const uint8_t* o = ggml + (size_t)warp * Q8_0_BYTES;
    int q = (int)(int8_t)o[2 + lane];
    a.qs[(size_t)warp * 32 + lane] = (int8_t)q;
    int s = q;
    __syncwarp();
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
        a.d[warp] = f16_bits_to_f32((uint16_t)(o[0] | (o[1] << 8)));
        a.s8[warp] = 8 * s;
    }
}

// gguf Q4_0.quantize_blocks: d = x[argmax |x|] / -8 (first maximum),
// code = min(15, trunc(x/d + 8.5)), low nibble = element j, high = j + 16.
__global__ void k_quantize_q4_0(const float* __restrict__ x, long long nblocks, uint8_t* __restrict__ out) {
    long long blk = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (blk >= nblocks) return;
    float v = x[blk * 32 + lane];
    float am = fabsf(v);
    int ai = lane;
    __syncwarp();
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        float oa = __shfl_xor_sync(0xffffffffu, am, off);
        int oi = __shfl_xor_sync(0xffffffffu, ai, off);
        if (oa > am || (oa == am && oi < ai)) { am = oa; ai = oi; }
    }
    float mx = __shfl_sync(0xffffffffu, v, ai);
    float d = __fdiv_rn(mx, -8.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q = q4_code(v, id);
    store_q4_0_block(out + blk * Q4_0_BYTES, f32_to_f16_bits(d), q, lane);
}

cudaError_t launch_quantize_act(const float* x, int n, ActView a, uint8_t* ggml, cudaStream_t s) {
    int nb = n / 32;
    if (nb <= 0) return cudaSuccess;
    k_quantize_act<<<(nb + 7) / 8, 256, 0, s>>>(x, nb, a, ggml);
    return cudaGetLastError();
}

cudaError_t launch_q8_0_to_act(const uint8_t* ggml, int nb, ActView a, cudaStream_t s) {
    if (nb <= 0) return cudaSuccess;
    k_q8_0_to_act<<<(nb + 7) / 8, 256, 0, s>>>(ggml, nb, a);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q4_0(const float* x, long long n, uint8_t* out, cudaStream_t s) {
    long long nb = n / 32;
    if (nb <= 0) return cudaSuccess;
    k_quantize_q4_0<<<(unsigned)((nb + 7) / 8), 256, 0, s>>>(x, nb, out);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ matvec

__device__ __forceinline__ void act_to_smem(const ActView& g, ActView& sm, int nb, uint8_t* smem) {
    sm = act_view(smem, nb);
    const int4* src = reinterpret_cast<const int4*>(g.qs);
    int4* dst = reinterpret_cast<int4*>(sm.qs);
    for (int i = threadIdx.x; i < nb * 2; i += blockDim.x) dst[i] = src[i];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
        sm.d[i] = g.d[i];
        sm.s8[i] = g.s8[i];
    }
}

__global__ void __launch_bounds__(256) k_matvec(const uint8_t* __restrict__ W, ActView xa,
                                                float* __restrict__ y, int rows, int nb) {
    extern __shared__ __align__(16) uint8_t smem[];
    ActView xs;
    act_to_smem(xa, xs, nb, smem);
    __syncwarp();
    __syncthreads();
    int lane = threadIdx.x & 31;
    int warp = threadIdx.x >> 5;
    int nwarps = blockDim.x >> 5;
    size_t rb = (size_t)nb * 18;
    for (int r = blockIdx.x * nwarps + warp; r < rows; r += gridDim.x * nwarps) {
        const uint8_t* row = W + (size_t)r * rb;
        float acc = 0.0f;
        for (int b = lane; b < nb; b += 32) {
            uint4 w = ldg_nc_v4(row + 16 * b);
            float dw = f16_bits_to_f32(ldg_nc_u16(row + 16 * (size_t)nb + 2 * b));
            XBlk xb = load_xblk(xs, b);
            acc = __fadd_rn(acc, block_term(block_sumi(w, xb), dw, xb.d));
        }
        acc = warp_sum_butterfly(acc);
        if (lane == 0) y[r] = acc;
    }
}

__global__ void __launch_bounds__(256) k_block_dots(const uint8_t* __restrict__ W, ActView xa,
                                                    int32_t* __restrict__ out, int rows, int nb) {
    extern __shared__ __align__(16) uint8_t smem[];
    ActView xs;
    act_to_smem(xa, xs, nb, smem);
    __syncwarp();
    __syncthreads();
    int lane = threadIdx.x & 31;
    int warp = threadIdx.x >> 5;
    int nwarps = blockDim.x >> 5;
    size_t rb = (size_t)nb * 18;
    for (int r = blockIdx.x * nwarps + warp; r < rows; r += gridDim.x * nwarps) {
        const uint8_t* row = W + (size_t)r * rb;
        for (int b = lane; b < nb; b += 32) {
            uint4 w = ldg_nc_v4(row + 16 * b);
            out[(size_t)r * nb + b] = block_sumi(w, load_xblk(xs, b));
        }
    }
}

static int grid_for_rows(int rows, int warps_per_block) {
    int g = (rows + warps_per_block - 1) / warps_per_block;
    return g < 1 ? 1 : (g > 148 * 16 ? 148 * 16 : g);
}

cudaError_t launch_matvec(const uint8_t* W, ActView x, float* y, int rows, int nb, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    size_t sm = act_bytes(nb);
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_matvec, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
    }
    k_matvec<<<grid_for_rows(rows, 8), 256, sm, s>>>(W, x, y, rows, nb);
    return cudaGetLastError();
}

cudaError_t launch_block_dots(const uint8_t* W, ActView x, int32_t* out, int rows, int nb, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    size_t sm = act_bytes(nb);
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_block_dots, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
    }
    k_block_dots<<<grid_for_rows(rows, 8), 256, sm, s>>>(W, x, out, rows, nb);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ router

constexpr int ROUTER_HCHUNK = 256;
constexpr int MAX_EXPERTS = 1024;

// Routing of the normed hidden state (engine.py:229-236): warps 0..E-1 add
// fixed-point partial sums of R[e] . (x * normw) over a 256-column chunk into
// acc[e]; warp E adds the chunk's sum of x^2 into acc[E].  The last block to
// finish turns them into scale = 1/sqrt(ss/H + eps), logits = scale * sum, the
// top-k and softmax weights, and leaves acc zeroed.
__global__ void __launch_bounds__(256) k_router_topk(
    const float* __restrict__ R, const float* __restrict__ x, const float* __restrict__ normw, float eps,
    int E, int H, int k, unsigned long long* acc, unsigned* counter, float* logits, int* idx, float* w,
    float* scale_out, const uint8_t* layer_base, size_t expert_bytes, const uint8_t** expert_ptrs) {
    int lane = threadIdx.x & 31;
    int warp = threadIdx.x >> 5;
    int e = blockIdx.x * 8 + warp;
    int c0 = blockIdx.y * ROUTER_HCHUNK;
    if (e < E) {
        const float* rr = R + (size_t)e * H;
        long long s = 0;
        for (int c = c0 + 4 * lane; c < c0 + ROUTER_HCHUNK; c += 128) {
            float4 rv = __ldg(reinterpret_cast<const float4*>(rr + c));
            float4 xv = __ldg(reinterpret_cast<const float4*>(x + c));
            float4 nv = __ldg(reinterpret_cast<const float4*>(normw + c));
            s += router_fixed(rv.x, __fmul_rn(xv.x, nv.x)) + router_fixed(rv.y, __fmul_rn(xv.y, nv.y)) +
                 router_fixed(rv.z, __fmul_rn(xv.z, nv.z)) + router_fixed(rv.w, __fmul_rn(xv.w, nv.w));
        }
        s = warp_sum_i64(s);
        if (lane == 0) atomicAdd(acc + e, (unsigned long long)s);
    } else if (e == E) {
        long long s = 0;
        for (int c = c0 + 4 * lane; c < c0 + ROUTER_HCHUNK; c += 128) {
            float4 xv = __ldg(reinterpret_cast<const float4*>(x + c));
            s += ss_fixed(xv.x) + ss_fixed(xv.y) + ss_fixed(xv.z) + ss_fixed(xv.w);
        }
        s = warp_sum_i64(s);
        if (lane == 0) atomicAdd(acc + E, (unsigned long long)s);
    }
    __threadfence();
    __syncwarp();
    __syncthreads();
    __shared__ unsigned ticket;
    if (threadIdx.x == 0) ticket = atomicAdd(counter, 1u);
    __syncwarp();
    __syncthreads();
    if (ticket != gridDim.x * gridDim.y - 1) return;
    __threadfence();
    __shared__ float sl[MAX_EXPERTS];
    __shared__ int sidx[MAX_TOPK];
    __shared__ float sw[MAX_TOPK];
    __shared__ float sscale;
    __syncwarp();
    __syncthreads();
    if (threadIdx.x == 0) {
        long long ss = (long long)atomicExch(acc + E, 0ull);
        sscale = rms_scale_from(ss, H, eps);
        if (scale_out) *scale_out = sscale;
    }
    __syncwarp();
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        long long v = (long long)atomicExch(acc + i, 0ull);
        float l = __fmul_rn(sscale, router_logit(v));
        sl[i] = l;
        if (logits) logits[i] = l;
    }
    __syncwarp();
    __syncthreads();
    topk_softmax_block(sl, E, k, sidx, sw);
    if (threadIdx.x < k) {
        int j = threadIdx.x;
        idx[j] = sidx[j];
        w[j] = sw[j];
        if (expert_ptrs) expert_ptrs[j] = layer_base + (size_t)sidx[j] * expert_bytes;
    }
    if (threadIdx.x == 0) *counter = 0u;
}

cudaError_t launch_router_topk(const float* R, const float* x, const float* normw, float eps, int E, int H, int k,
                               long long* acc, unsigned* counter, float* logits, int* idx, float* w,
                               float* scale_out, const uint8_t* layer_base, size_t expert_bytes,
                               const uint8_t** expert_ptrs, cudaStream_t s) {
    if (E <= 0 || E > MAX_EXPERTS || k <= 0 || k > MAX_TOPK || k > E || H % ROUTER_HCHUNK != 0)
        return cudaErrorInvalidValue;
    dim3 grid((E + 1 + 7) / 8, H / ROUTER_HCHUNK);
    k_router_topk<<<grid, 256, 0, s>>>(R, x, normw, eps, E, H, k, reinterpret_cast<unsigned long long*>(acc),
                                       counter, logits, idx, w, scale_out, layer_base, expert_bytes, expert_ptrs);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ expert FFN

// grid (I/32, k), 256 threads.  CTA (c, j) computes gate and up rows
// 32c .. 32c+31 of expert j, h = silu(g)*u, and quantises that h block.
__global__ void __launch_bounds__(256) k_gateup(const uint8_t* const* __restrict__ experts,
                                                const float* __restrict__ x, const float* __restrict__ normw,
                                                const float* __restrict__ scale, Geom g,
                                                uint8_t* __restrict__ hq, float* __restrict__ h_dbg,
                                                float* __restrict__ gu_dbg) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float sh[32];
    int lane = threadIdx.x & 31;
    int warp = threadIdx.x >> 5;
    ActView xs = act_view(smem, g.nbH);
    quantize_to_act(x, g.nbH, xs, warp, 8, lane, normw, scale);
    __syncwarp();
    __syncthreads();

    const int j = blockIdx.y;
    const int i0 = blockIdx.x * 32 + warp * 4;
    const uint8_t* gate = experts[j];
    const uint8_t* up = gate + g.t_gu;
    const int nb = g.nbH;
    float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
    for (int b = lane; b < nb; b += 32) {
        uint4 wg[4], wu[4];
        uint16_t dg[4], du[4];
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint8_t* rg = gate + (size_t)(i0 + t) * g.row_gu;
            const uint8_t* ru = up + (size_t)(i0 + t) * g.row_gu;
            wg[t] = ldg_nc_v4(rg + 16 * b);
            wu[t] = ldg_nc_v4(ru + 16 * b);
            dg[t] = ldg_nc_u16(rg + 16 * (size_t)nb + 2 * b);
            du[t] = ldg_nc_u16(ru + 16 * (size_t)nb + 2 * b);
        }
        XBlk xb = load_xblk(xs, b);
#pragma unroll
        for (int t = 0; t < 4; t++) {
            ag[t] = __fadd_rn(ag[t], block_term(block_sumi(wg[t], xb), f16_bits_to_f32(dg[t]), xb.d));
            au[t] = __fadd_rn(au[t], block_term(block_sumi(wu[t], xb), f16_bits_to_f32(du[t]), xb.d));
        }
    }
#pragma unroll
    for (int t = 0; t < 4; t++) {
        float gv = warp_sum_butterfly(ag[t]);
        float uv = warp_sum_butterfly(au[t]);
        if (lane == t) {
            sh[warp * 4 + t] = silu_mul(gv, uv);
            if (gu_dbg) {
                gu_dbg[(size_t)j * 2 * g.I + i0 + t] = gv;
                gu_dbg[(size_t)j * 2 * g.I + g.I + i0 + t] = uv;
            }
        }
    }
    __syncwarp();
    __syncthreads();
    if (warp == 0) {
        float hv = sh[lane];
        Q8Lane q = quantize_lane(hv);
        ActView ha = act_view(hq + (size_t)j * act_bytes(g.nbI), g.nbI);
        int blk = blockIdx.x;
        ha.qs[(size_t)blk * 32 + lane] = (int8_t)q.q;
        if (lane == 0) {
            ha.d[blk] = f16_bits_to_f32(q.dh);
            ha.s8[blk] = q.s8;
        }
        if (h_dbg) h_dbg[(size_t)j * g.I + blk * 32 + lane] = hv;
    }
}

cudaError_t launch_gateup(const uint8_t* const* experts, int k, const float* x, const float* normw,
                          const float* scale, Geom g, uint8_t* hq, float* h_dbg, float* gu_dbg, cudaStream_t s) {
    if (k <= 0) return cudaSuccess;
    size_t sm = act_bytes(g.nbH);
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
    }
    dim3 grid(g.I / 32, k);
    k_gateup<<<grid, 256, sm, s>>>(experts, x, normw, scale, g, hq, h_dbg, gu_dbg);
    return cudaGetLastError();
}

constexpr int DOWN_ROWS_PER_CTA = 16;

// grid ceil(H/16), 256 threads: warp w computes output rows 16c + 2w, 16c + 2w + 1
// for all k experts and combines them in expert-slot order.
__global__ void __launch_bounds__(256) k_down_combine(const uint8_t* const* __restrict__ experts, int k,
                                                      const uint8_t* __restrict__ hq,
                                                      const float* __restrict__ wts, float w_scalar, Geom g,
                                                      const float* resid, float* out, int accumulate,
                                                      float* __restrict__ y_dbg) {
    extern __shared__ __align__(16) uint8_t smem[];
    int lane = threadIdx.x & 31;
    int warp = threadIdx.x >> 5;
    const int nb = g.nbI;
    const size_t ab = act_bytes(nb);
    {
        const int4* src = reinterpret_cast<const int4*>(hq);
        int4* dst = reinterpret_cast<int4*>(smem);
        int n16 = (int)(ab * k / 16);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
    }
    __syncwarp();
    __syncthreads();
    for (int rr = 0; rr < 2; rr++) {
        int r = blockIdx.x * DOWN_ROWS_PER_CTA + warp * 2 + rr;
        if (r >= g.H) break;
        float y[MAX_TOPK];
#pragma unroll
        for (int j = 0; j < MAX_TOPK; j++) y[j] = 0.0f;
        float acc[MAX_TOPK];
#pragma unroll
        for (int j = 0; j < MAX_TOPK; j++) acc[j] = 0.0f;
        for (int b0 = 0; b0 < nb; b0 += 32) {
            int b = b0 + lane;
            if (b < nb) {
                uint4 wv[MAX_TOPK];
                uint16_t dv[MAX_TOPK];
#pragma unroll
                for (int j = 0; j < MAX_TOPK; j++) {
                    if (j < k) {
                        const uint8_t* row = experts[j] + 2 * g.t_gu + (size_t)r * g.row_d;
                        wv[j] = ldg_nc_v4(row + 16 * b);
                        dv[j] = ldg_nc_u16(row + 16 * (size_t)nb + 2 * b);
                    }
                }
#pragma unroll
                for (int j = 0; j < MAX_TOPK; j++) {
                    if (j < k) {
                        ActView ha = act_view(smem + (size_t)j * ab, nb);
                        XBlk xb = load_xblk(ha, b);
                        acc[j] = __fadd_rn(acc[j], block_term(block_sumi(wv[j], xb), f16_bits_to_f32(dv[j]), xb.d));
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < MAX_TOPK; j++)
            if (j < k) y[j] = warp_sum_butterfly(acc[j]);
        if (lane == 0) {
            float a = accumulate ? out[r] : 0.0f;
#pragma unroll
            for (int j = 0; j < MAX_TOPK; j++) {
                if (j < k) {
                    float wj = wts ? wts[j] : w_scalar;
                    a = __fadd_rn(a, __fmul_rn(wj, y[j]));
                    if (y_dbg) y_dbg[(size_t)j * g.H + r] = y[j];
                }
            }
            out[r] = resid ? __fadd_rn(resid[r], a) : a;
        }
    }
}

cudaError_t launch_down_combine(const uint8_t* const* experts, int k, const uint8_t* hq, const float* w,
                                float w_scalar, Geom g, const float* resid, float* out, int accumulate,
                                float* y_dbg, cudaStream_t s) {
    if (k <= 0 || k > MAX_TOPK) return cudaErrorInvalidValue;
    size_t sm = act_bytes(g.nbI) * k;
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_down_combine, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
    }
    int grid = (g.H + DOWN_ROWS_PER_CTA - 1) / DOWN_ROWS_PER_CTA;
    k_down_combine<<<grid, 256, sm, s>>>(experts, k, hq, w, w_scalar, g, resid, out, accumulate, y_dbg);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ RMSNorm scale

// one CTA of 256 threads: *scale = 1/sqrt(sum x^2 / H + eps) with the exact
// fixed-point sum of the routing kernel (csrc/libtinygiant.c:322-340)
__global__ void __launch_bounds__(256) k_rms_scale(const float* __restrict__ x, int H, float eps,
                                                   float* __restrict__ scale) {
    __shared__ long long ws[8];
    long long s = 0;
    for (int r = threadIdx.x; r < H; r += blockDim.x) s += ss_fixed(x[r]);
    s = warp_sum_i64(s);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long t = 0;
        for (int w = 0; w < 8; w++) t += ws[w];
        *scale = rms_scale_from(t, H, eps);
    }
}

cudaError_t launch_rms_scale(const float* x, int H, float eps, float* scale, cudaStream_t s) {
    k_rms_scale<<<1, 256, 0, s>>>(x, H, eps, scale);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ synthetic data

__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// out[i] ~ N(0, sigma) for i in [0, n): value i depends only on (seed, base + i).
__global__ void k_fill_normal(float* __restrict__ out, long long n, unsigned long long seed,
                              unsigned long long base, float sigma) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long i = 2 * t;
    if (i >= n) return;
    unsigned long long z = mix64(seed + 0x9E3779B97F4A7C15ull * (unsigned long long)((base + i) / 2 + 1));
    float u1 = ((float)(z >> 40) + 1.0f) * 0x1p-24f;
    float u2 = (float)((z >> 16) & 0xFFFFFFull) * 0x1p-24f;
    float r = sqrtf(-2.0f * logf(u1)) * sigma;
    float sv, cv;
    sincospif(2.0f * u2, &sv, &cv);
    out[i] = r * cv;
    if (i + 1 < n) out[i + 1] = r * sv;
}

cudaError_t launch_fill_normal(float* out, long long n, unsigned long long seed, unsigned long long base,
                               float sigma, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    long long pairs = (n + 1) / 2;
    k_fill_normal<<<(unsigned)((pairs + 255) / 256), 256, 0, s>>>(out, n, seed, base, sigma);
    return cudaGetLastError();
}

// Synthetic experts straight into HBM: each warp owns one Q4_0 block, each lane
// draws its weight (value index = base + flat position in the expert blob's
// row-major f32 tensors), then the warp quantises the block as k_quantize_q4_0
// does and stores it in row-split form.
__global__ void k_fill_experts_q4_0(uint8_t* __restrict__ dst, int n_experts, Geom g, unsigned long long seed,
                                    unsigned long long base, float sigma) {
    long long blk = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    const long long per_expert_blocks = 3LL * g.I * g.nbH;  // = 3*H*I/32
    if (blk >= per_expert_blocks * n_experts) return;
    long long e = blk / per_expert_blocks;
    long long rem = blk - e * per_expert_blocks;
    // position inside the expert: gate rows, up rows (nbH blocks each), then down rows (nbI blocks)
    long long gu_blocks = 2LL * g.I * g.nbH;
    long long row;
    int b, nb;
    size_t row_bytes, tensor_off;
    if (rem < gu_blocks) {
        row = rem / g.nbH;
        b = (int)(rem - row * g.nbH);
        nb = g.nbH;
        row_bytes = g.row_gu;
        tensor_off = 0;
    } else {
        long long r2 = rem - gu_blocks;
        row = r2 / g.nbI;
        b = (int)(r2 - row * g.nbI);
        nb = g.nbI;
        row_bytes = g.row_d;
        tensor_off = 2 * g.t_gu;
    }
    unsigned long long vi = base + (unsigned long long)blk * 32 + lane;
    unsigned long long z = mix64(seed + 0x9E3779B97F4A7C15ull * (vi / 2 + 1));
    float u1 = ((float)(z >> 40) + 1.0f) * 0x1p-24f;
    float u2 = (float)((z >> 16) & 0xFFFFFFull) * 0x1p-24f;
    float sv, cv;
    sincospif(2.0f * u2, &sv, &cv);
    float v = sqrtf(-2.0f * logf(u1)) * sigma * ((vi & 1) ? sv : cv);
    float am = fabsf(v);
    int ai = lane;
    __syncwarp();
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        float oa = __shfl_xor_sync(0xffffffffu, am, off);
        int oi = __shfl_xor_sync(0xffffffffu, ai, off);
        if (oa > am || (oa == am && oi < ai)) { am = oa; ai = oi; }
    }
    float mx = __shfl_sync(0xffffffffu, v, ai);
    float d = __fdiv_rn(mx, -8.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q = q4_code(v, id);
    __syncwarp();
    int qh = __shfl_down_sync(0xffffffffu, q, 16);
    unsigned byte = (unsigned)(q | (qh << 4)) & 0xffu;        // valid in lanes 0..15
    unsigned b0 = __shfl_sync(0xffffffffu, byte, (2 * lane) & 31);
    unsigned b1 = __shfl_sync(0xffffffffu, byte, (2 * lane + 1) & 31);
    uint8_t* rowp = dst + e * g.expert_bytes + tensor_off + row * row_bytes;
    if (lane < 8) reinterpret_cast<uint16_t*>(rowp + 16 * b)[lane] = (uint16_t)(b0 | (b1 << 8));
    if (lane == 0) *reinterpret_cast<uint16_t*>(rowp + 16 * (size_t)nb + 2 * b) = f32_to_f16_bits(d);
}

cudaError_t launch_fill_experts_q4_0(uint8_t* dst, int n_experts, Geom g, unsigned long long seed,
                                     unsigned long long base, float sigma, cudaStream_t s) {
    long long nblk = 3LL * g.I * g.nbH * n_experts;
    if (nblk <= 0) return cudaSuccess;
    k_fill_experts_q4_0<<<(unsigned)((nblk + 7) / 8), 256, 0, s>>>(dst, n_experts, g, seed, base, sigma);
    return cudaGetLastError();
}

// out[c][r] = in[r][c] for a rows x cols fp32 matrix (32x32 tiles through shared memory).
__global__ void k_transpose(const float* __restrict__ in, float* __restrict__ out, int rows, int cols) {
    __shared__ float tile[32][33];
    int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = in[(size_t)r * cols + c];
    }
    __syncwarp();
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        int c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[(size_t)c * rows + r] = tile[threadIdx.x][i];
    }
}

cudaError_t launch_transpose(const float* in, float* out, int rows, int cols, cudaStream_t s) {
    dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
    k_transpose<<<grid, block, 0, s>>>(in, out, rows, cols);
    return cudaGetLastError();
}

// The dynamic shared-memory limit of a kernel is one process-wide attribute per
// device, and contexts and host-pointer calls of different shapes share it: it is only
// ever raised (per device, behind a mutex), so a smaller shape never lowers it under a
// larger one that another thread is about to launch.
cudaError_t prepare_kernels(Geom g, int k) {
    static std::mutex mu;
    static int raised[3][64] = {};   // [kernel][device]: the largest limit set so far
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const int sm_gu = (int)act_bytes(g.nbH);
    const int sm_d = (int)(act_bytes(g.nbI) * k);
    const void* fns[3] = {(const void*)k_gateup, (const void*)k_down_combine, (const void*)k_matvec};
    const int want[3] = {sm_gu, sm_d, sm_gu};
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < 3; i++) {
        if (want[i] <= 48 * 1024 || want[i] <= raised[i][dev]) continue;
        if ((e = cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize, want[i])) != cudaSuccess)
            return e;
        raised[i][dev] = want[i];
    }
    return cudaSuccess;
}

}  // namespace tg

// tg_batched.cu — the MoE block for T tokens at once (prefill / batched decode).
//
// Per layer (tinygiant/engine.py:229-258 applied to every token, attention excluded):
//   k_router_sums_batched   exact fixed-point router sums S[t][e] = sum_r R[e][r] * fl(x[t][r] * w[r]),
//                           split over 256-column chunks (int64 atomics: exact, split-independent)
//   k_topk_quant_batched    per token: sum x^2 -> RMSNorm scale, logits, top-k + softmax
//                           (engine.py:229-236), Q8_0 of (x * scale) * w (libtinygiant.c:61-89)
//   k_group_pairs           (token, slot) pairs grouped by expert (counting sort)
//   k_gateup_batched        per (expert, 16-row unit): the unit's gate and up rows are staged in
//                           shared memory once, then h = silu(g) * u for every token routed to
//                           the expert (libtinygiant.c:566-586)
//   k_quant_h               the Q8_0 blocks of h, one warp per (pair, block)
//   k_down_batched          per (expert, 16 output rows): the rows are staged once, then
//                           y[pair][r] for every token routed to the expert (:588-594)
//   k_combine_batched       x[t] += sum_j w[t][j] * y[(t, j)] in slot order (engine.py:240-258)
// Each token's values use the same reduction order as the single-token kernels (lane-strided
// block partials, xor butterfly), so a batch gives bit-identical results to T single-token
// calls and to the CPU oracle's mirror mode.
//
// An optional shared expert (DeepSeek-V3-like models) is slot k of every token, weight 1,
// expert id E; with experts sharded over G devices, a pair (token t, slot j) is computed by
// the device holding its routed expert, and a token's shared-expert pair by the device that
// holds the fewest of that token's routed experts (ties to (t + i) mod G, smallest i), a
// rule every device evaluates the same way.
#include <cuda_runtime.h>

#include "tg_device.cuh"
#include "tg_internal.h"

namespace tg {

namespace {

constexpr int RT_TOK = 4;         // tokens per router CTA
constexpr int DOWN_ROWS = 16;     // output rows per down CTA (2 per warp)
// tokens per pass of the batched dp4a kernels: wide tiles (gate/up 8 or 16, down 16) when
// experts average >= 8 pairs, narrow ones (2 or 4, 4) below, which keep more CTAs per SM
constexpr int WIDE_MIN_PAIRS = 8;

// Sum each of N (8, 16 or 32) per-lane values over the warp with the same pairing tree
// as N separate xor butterflies (so the same bits): at offsets 16, 8, ... each lane hands
// half of its remaining values to its partner and keeps the other half (the upper half
// when the lane has that offset's bit) until one value is left, then plain butterflies.
// Value j ends in lanes j * (32 / N) .. j * (32 / N) + 32 / N - 1.
template <int N>
__device__ __forceinline__ float warp_sum_transposed(float (&v)[N], int lane) {
    __syncwarp();
#pragma unroll
    for (int lvl = 0; lvl < 5; lvl++) {
        const int o = 16 >> lvl;          // offset of this level
        const int h = (N >> lvl) / 2;     // values handed over (0: one value left)
        if (h > 0) {
            const bool up = lane & o;
#pragma unroll
            for (int i = 0; i < h; i++) {
                const float send = up ? v[i] : v[i + h];
                const float keep = up ? v[i + h] : v[i];
                v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
            }
        } else {
            v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], o));
        }
    }
    return v[0];
}

// grid (ceil(T / RT_TOK), ceil(E / 8), H / 256), 256 threads: warp w adds expert
// 8 * blockIdx.y + w's fixed-point partial sums over a 256-column chunk for RT_TOK tokens
// into S[t][e] (exact int64, so the split does not change the sums; S starts at zero).
__global__ void __launch_bounds__(256) k_router_sums_batched(const float* __restrict__ X, int T,
                                                             const float* __restrict__ R,
                                                             const float* __restrict__ normw, int E, int H,
                                                             unsigned long long* __restrict__ S) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.y * 8 + warp;
    const int t0 = blockIdx.x * RT_TOK;
    const int nt = min(RT_TOK, T - t0);
    const int c0 = blockIdx.z * 256;
    if (e >= E) return;
    long long s[RT_TOK];
#pragma unroll
    for (int t = 0; t < RT_TOK; t++) s[t] = 0;
    const float* rr = R + (size_t)e * H;
    for (int c = c0 + 4 * lane; c < c0 + 256; c += 128) {
        const float4 rv = __ldg(reinterpret_cast<const float4*>(rr + c));
        const float4 nv = __ldg(reinterpret_cast<const float4*>(normw + c));
#pragma unroll
        for (int t = 0; t < RT_TOK; t++) {
            if (t < nt) {
                const float4 xv = __ldg(reinterpret_cast<const float4*>(X + (size_t)(t0 + t) * H + c));
                s[t] += router_fixed(rv.x, __fmul_rn(xv.x, nv.x)) + router_fixed(rv.y, __fmul_rn(xv.y, nv.y)) +
                        router_fixed(rv.z, __fmul_rn(xv.z, nv.z)) + router_fixed(rv.w, __fmul_rn(xv.w, nv.w));
            }
        }
    }
#pragma unroll
    for (int t = 0; t < RT_TOK; t++) {
        const long long v = warp_sum_i64(s[t]);
        if (lane == 0 && t < nt) atomicAdd(S + (size_t)(t0 + t) * E + e, (unsigned long long)v);
    }
}

// grid T, 256 threads: token t's RMSNorm scale, logits, top-k and softmax weights, and
// the Q8_0 activation form of (x * scale) * w.
__global__ void __launch_bounds__(256) k_topk_quant_batched(const float* __restrict__ X, const float* __restrict__ normw,
                                                            float eps, int E, int H, int k, int ks,
                                                            const unsigned long long* __restrict__ S, int* __restrict__ idx,
                                                            float* __restrict__ wts, float* __restrict__ logits,
                                                            uint8_t* __restrict__ xq) {
    __shared__ float sl[1024];
    __shared__ int sidx[MAX_TOPK];
    __shared__ float sw[MAX_TOPK];
    __shared__ long long wsum[8];
    __shared__ float sscale;
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float* x = X + (size_t)t * H;
    long long ss = 0;
    for (int r = threadIdx.x; r < H; r += blockDim.x) ss += ss_fixed(x[r]);
    ss = warp_sum_i64(ss);
    if (lane == 0) wsum[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long tot = 0;
        for (int w = 0; w < 8; w++) tot += wsum[w];
        sscale = rms_scale_from(tot, H, eps);
    }
    __syncthreads();
    const float scale = sscale;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const float l = __fmul_rn(scale, router_logit((long long)S[(size_t)t * E + e]));
        sl[e] = l;
        if (logits) logits[(size_t)t * E + e] = l;
    }
    __syncthreads();
    topk_softmax_block(sl, E, k, sidx, sw);
    if (threadIdx.x < k) {
        idx[(size_t)t * ks + threadIdx.x] = sidx[threadIdx.x];
        wts[(size_t)t * ks + threadIdx.x] = sw[threadIdx.x];
    } else if (threadIdx.x < ks) {   // the shared expert: id E, weight 1
        idx[(size_t)t * ks + threadIdx.x] = E;
        wts[(size_t)t * ks + threadIdx.x] = 1.0f;
    }
    // Q8_0 of the normed input, one warp per block (the single-token quantiser's order)
    const int nb = H / 32;
    ActView a = act_view(xq + (size_t)t * act_bytes(nb), nb);
    for (int b = warp; b < nb; b += 8) {
        const float v = __fmul_rn(__fmul_rn(x[(size_t)b * 32 + lane], scale), normw[(size_t)b * 32 + lane]);
        const Q8Lane q = quantize_lane(v);
        a.qs[(size_t)b * 32 + lane] = (int8_t)q.q;
        if (lane == 0) {
            a.d[b] = f16_bits_to_f32(q.dh);
            a.s8[b] = q.s8;
        }
    }
}

// one CTA of 256 threads: pairs p = t * k + j grouped by expert idx[p]; off[E + 1],
// list[T * k] (the order inside a group does not affect any result) and the active experts
// among those this device holds, [e_lo, e_lo + e_n)
// Whether this device (rank of G, holding routed experts [rank*e_n, (rank+1)*e_n))
// computes pair p = t * ks + j: a routed slot by its expert's holder, the shared slot
// (j >= k) by the holder of the fewest of token t's routed experts.
__device__ __forceinline__ bool pair_owned(const int* __restrict__ idx, int p, int ks, int k, int e_n, int rank,
                                           int G) {
    const int t = p / ks, j = p - t * ks;
    if (j < k) return idx[p] / e_n == rank;
    int best = 0, best_n = 1 << 30;
    for (int i = 0; i < G; i++) {
        const int r = (t + i) % G;
        int n = 0;
        for (int q = 0; q < k; q++) n += idx[(size_t)t * ks + q] / e_n == r;
        if (n < best_n) {
            best_n = n;
            best = r;
        }
    }
    return best == rank;
}

// one CTA of 256 threads: the pairs this device computes, grouped by expert id (routed
// experts 0..E-1, the shared expert E): off[E_tot + 1], list (the order inside a group
// does not affect any result) and active[0] = count, active[1..] = the experts, ascending
__global__ void __launch_bounds__(256) k_group_pairs(const int* __restrict__ idx, int n_pairs, int ks, int k,
                                                     int E_tot, int e_n, int rank, int G, int* __restrict__ off,
                                                     int* __restrict__ list, int* __restrict__ active,
                                                     int* __restrict__ owned, int* __restrict__ tile_pre, int tile,
                                                     const int* __restrict__ n_dev = nullptr) {
    __shared__ int cnt[1025];
    if (n_dev) n_pairs = *n_dev;   // the pair count on the device (n_pairs was an upper bound)
    __shared__ int pos[1025];
    for (int e = threadIdx.x; e < E_tot; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < n_pairs; p += blockDim.x)
        if (pair_owned(idx, p, ks, k, e_n, rank, G)) atomicAdd(&cnt[idx[p]], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0, na = 0, tiles = 0;
        for (int e = 0; e < E_tot; e++) {
            off[e] = acc;
            pos[e] = acc;
            acc += cnt[e];
            if (cnt[e]) {
                tile_pre[na] = tiles;          // token tiles of the active experts before this one
                tiles += (cnt[e] + tile - 1) / tile;
                active[1 + na++] = e;
            }
        }
        tile_pre[na] = tiles;
        off[E_tot] = acc;
        active[0] = na;
        if (owned) owned[0] = acc;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < n_pairs; p += blockDim.x)
        if (pair_owned(idx, p, ks, k, e_n, rank, G)) {
            const int slot = atomicAdd(&pos[idx[p]], 1);
            list[slot] = p;
            if (owned) owned[1 + slot] = p;
        }
}

// expert e's blob: a local routed expert, or the shared expert (e == E)
__device__ __forceinline__ const uint8_t* expert_base(const uint8_t* layer, const uint8_t* shared, int e, int E,
                                                      int e_lo, size_t expert_bytes) {
    return e == E ? shared : layer + (size_t)(e - e_lo) * expert_bytes;
}

// gate/up rows per CTA unit: 16, with the Q8_0 of h in a separate pass (k_quant_h).  Against
// 32-row units quantising h in place, the smaller units fit twice the CTAs per SM, so more
// weight loads are in flight: at the Qwen3 shape T = 64 -4%, T = 256 -12% per layer.
constexpr int GU_ROWS = 16;

// grid (I / 16, active experts), 256 threads.  CTA (c, a) takes the a-th active expert e and
// stages rows 16c .. 16c+15 of its gate and up in shared memory, then takes the pairs
// routed to e in tiles of P tokens: each warp owns 2 rows, each lane runs the lane-strided
// block chains of those rows for every token of the tile (a staged weight block is read
// once per tile), and two transposed reductions leave lane l with the gate and up sums of
// (row l / P, token l % P); h = silu(g) * u goes to hf[p] for k_quant_h.  Per (row, token)
// the arithmetic is exactly the single-token one.
template <int P>
__global__ void __launch_bounds__(256) k_gateup_batched(const uint8_t* __restrict__ layer,
                                                        const uint8_t* __restrict__ shared, int E, int e_lo, Geom g,
                                                        const int* __restrict__ off, const int* __restrict__ list,
                                                        const int* __restrict__ active, int ks,
                                                        const uint8_t* __restrict__ xq, float* __restrict__ hf) {
    constexpr int R = GU_ROWS;
    constexpr int RW = R / 8;        // rows per warp
    constexpr int NV = RW * P;       // sums per lane and matrix: 8 or 32
    constexpr int LPV = 32 / NV;     // lanes holding each reduced sum
    extern __shared__ __align__(16) uint8_t smem[];   // gate rows | up rows
    __shared__ int sp[P];            // the tile's pairs
    if ((int)blockIdx.y >= active[0]) return;
    const int e = active[1 + blockIdx.y], c = blockIdx.x;
    const int p0 = off[e], n = off[e + 1] - p0;
    if (n == 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint8_t* eb = expert_base(layer, shared, e, E, e_lo, g.expert_bytes);
    const size_t unit = (size_t)R * g.row_gu;
    {
        const int4* sg = reinterpret_cast<const int4*>(eb + (size_t)c * unit);
        const int4* su = reinterpret_cast<const int4*>(eb + g.t_gu + (size_t)c * unit);
        int4* d = reinterpret_cast<int4*>(smem);
        const int n16 = (int)(unit / 16);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) {
            d[i] = __ldg(sg + i);
            d[n16 + i] = __ldg(su + i);
        }
    }
    const uint8_t* gate = smem;
    const uint8_t* up = smem + unit;
    const int nb = g.nbH, i0 = warp * RW;
    const size_t abx = act_bytes(nb);
    for (int q0 = 0; q0 < n; q0 += P) {
        const int nt = min(P, n - q0);
        __syncthreads();   // the previous tile's sp is consumed (and, first time, the weights staged)
        if (threadIdx.x < P) sp[threadIdx.x] = threadIdx.x < nt ? list[p0 + q0 + threadIdx.x] : -1;
        __syncthreads();
        float ag[NV], au[NV];   // [row r][token t] at r * P + t
#pragma unroll
        for (int i = 0; i < NV; i++) ag[i] = au[i] = 0.0f;
        for (int b = lane; b < nb; b += 32) {
            uint4 wg[RW], wu[RW];
            float dg[RW], du[RW];
#pragma unroll
            for (int r = 0; r < RW; r++) {
                const uint8_t* rg = gate + (size_t)(i0 + r) * g.row_gu;
                const uint8_t* ru = up + (size_t)(i0 + r) * g.row_gu;
                wg[r] = *reinterpret_cast<const uint4*>(rg + 16 * b);
                wu[r] = *reinterpret_cast<const uint4*>(ru + 16 * b);
                dg[r] = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rg + 16 * (size_t)nb + 2 * b));
                du[r] = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ru + 16 * (size_t)nb + 2 * b));
            }
#pragma unroll
            for (int t = 0; t < P; t++) {
                if (t < nt) {
                    const ActView xa = act_view(xq + (size_t)(sp[t] / ks) * abx, nb);
                    const XBlk xb = load_xblk(xa, b);
#pragma unroll
                    for (int r = 0; r < RW; r++) {
                        ag[r * P + t] = __fadd_rn(ag[r * P + t], block_term(block_sumi(wg[r], xb), dg[r], xb.d));
                        au[r * P + t] = __fadd_rn(au[r * P + t], block_term(block_sumi(wu[r], xb), du[r], xb.d));
                    }
                }
            }
        }
        const float gv = warp_sum_transposed<NV>(ag, lane);
        const float uv = warp_sum_transposed<NV>(au, lane);
        const int j = lane / LPV, r = j / P, t = j % P;
        if (lane % LPV == 0 && t < nt) hf[(size_t)sp[t] * g.I + (size_t)c * R + i0 + r] = silu_mul(gv, uv);
    }
}

// one warp per (pair, block) of h: the Q8_0 activation form of hf[p] into hq[p]
// (the single-token quantiser, block by block, so the same bytes as the fused units);
// with uf, h = silu(hf) * uf first (hf, uf: the gate and up sums).  n_dev, when given,
// holds the pair count (the grid covers n_pairs, an upper bound).
__global__ void __launch_bounds__(256) k_quant_h(const float* __restrict__ hf, const float* __restrict__ uf,
                                                 int n_pairs, Geom g, uint8_t* __restrict__ hq,
                                                 const int* __restrict__ n_dev = nullptr) {
    const int lane = threadIdx.x & 31;
    const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (n_dev) n_pairs = *n_dev;
    if (wid >= (long long)n_pairs * g.nbI) return;
    const int p = (int)(wid / g.nbI), b = (int)(wid - (long long)p * g.nbI);
    const size_t i = (size_t)p * g.I + (size_t)b * 32 + lane;
    const Q8Lane qz = quantize_lane(uf ? silu_mul(hf[i], uf[i]) : hf[i]);
    ActView ha = act_view(hq + (size_t)p * act_bytes(g.nbI), g.nbI);
    ha.qs[(size_t)b * 32 + lane] = (int8_t)qz.q;
    if (lane == 0) {
        ha.d[b] = f16_bits_to_f32(qz.dh);
        ha.s8[b] = qz.s8;
    }
}

// grid (H / 16, active experts), 256 threads.  CTA (rb, a) takes the a-th active expert e,
// stages its down rows 16rb .. 16rb+15 (2 per warp), then takes the pairs routed to e in
// tiles of 16 tokens: each lane runs the lane-strided block chains of its warp's 2 rows
// for every token of the tile, and one transposed reduction leaves lane l with the sum of
// (row l / 16, token l % 16): y[p][r] = row . hq[p], exactly the single-token arithmetic.
template <int DT>
__global__ void __launch_bounds__(256) k_down_batched(const uint8_t* __restrict__ layer,
                                                      const uint8_t* __restrict__ shared, int E, int e_lo, Geom g,
                                                      const int* __restrict__ off, const int* __restrict__ list,
                                                      const int* __restrict__ active, const uint8_t* __restrict__ hq,
                                                      float* __restrict__ y) {
    constexpr int NV = 2 * DT;       // sums per lane: 2 rows x DT tokens
    constexpr int LPV = 32 / NV;
    extern __shared__ __align__(16) uint8_t smem[];   // DOWN_ROWS rows
    __shared__ int sp[DT];
    if ((int)blockIdx.y >= active[0]) return;
    const int e = active[1 + blockIdx.y], rb = blockIdx.x;
    const int p0 = off[e], n = off[e + 1] - p0;
    if (n == 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = rb * DOWN_ROWS;
    const int nrows = min(DOWN_ROWS, g.H - r0);
    {
        const int4* src = reinterpret_cast<const int4*>(expert_base(layer, shared, e, E, e_lo, g.expert_bytes) + 2 * g.t_gu +
                                                        (size_t)r0 * g.row_d);
        int4* d = reinterpret_cast<int4*>(smem);
        const int n16 = (int)((size_t)nrows * g.row_d / 16);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) d[i] = __ldg(src + i);
    }
    const int nb = g.nbI;
    const size_t abh = act_bytes(nb);
    const int lr0 = warp * 2;
    for (int q0 = 0; q0 < n; q0 += DT) {
        const int nt = min(DT, n - q0);
        __syncthreads();
        if (threadIdx.x < DT) sp[threadIdx.x] = threadIdx.x < nt ? list[p0 + q0 + threadIdx.x] : -1;
        __syncthreads();
        if (lr0 >= nrows) continue;
        float acc[NV];   // [row r][token t] at r * DT + t
#pragma unroll
        for (int i = 0; i < NV; i++) acc[i] = 0.0f;
        for (int b = lane; b < nb; b += 32) {
            uint4 wv[2];
            float dw[2];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const uint8_t* row = smem + (size_t)min(lr0 + r, nrows - 1) * g.row_d;
                wv[r] = *reinterpret_cast<const uint4*>(row + 16 * b);
                dw[r] = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(row + 16 * (size_t)nb + 2 * b));
            }
#pragma unroll
            for (int t = 0; t < DT; t++) {
                if (t < nt) {
                    const XBlk xb = load_xblk(act_view(hq + (size_t)sp[t] * abh, nb), b);
#pragma unroll
                    for (int r = 0; r < 2; r++)
                        acc[r * DT + t] = __fadd_rn(acc[r * DT + t], block_term(block_sumi(wv[r], xb), dw[r], xb.d));
                }
            }
        }
        const float yv = warp_sum_transposed<NV>(acc, lane);
        const int j = lane / LPV, r = j / DT, t = j % DT;
        if (lane % LPV == 0 && t < nt && lr0 + r < nrows) y[(size_t)sp[t] * g.H + r0 + lr0 + r] = yv;
    }
}

// grid (T, H / 256), 256 threads: x[t][r] = x[t][r] + (sum over slots j in order of
// w[t][j] * y[t*k+j][r]), one row per thread
__global__ void __launch_bounds__(256) k_combine_batched(float* __restrict__ X, int H, int k,
                                                         const float* __restrict__ wts, const float* __restrict__ y) {
    const int t = blockIdx.x;
    for (int r = blockIdx.y * blockDim.x + threadIdx.x; r < H; r += gridDim.y * blockDim.x) {
        float a = 0.0f;
        for (int j = 0; j < k; j++) a = __fadd_rn(a, __fmul_rn(wts[(size_t)t * k + j], y[((size_t)t * k + j) * H + r]));
        X[(size_t)t * H + r] = __fadd_rn(X[(size_t)t * H + r], a);
    }
}

}  // namespace

size_t batched_smem_bytes(const Geom& g) {
    size_t m = (size_t)2 * 16 * g.row_gu;
    m = m > (size_t)DOWN_ROWS * g.row_d ? m : (size_t)DOWN_ROWS * g.row_d;
    return m + 256;
}

static size_t r256(size_t n) { return (n + 255) & ~(size_t)255; }

size_t experts_scratch_bytes(const Geom& g, int E, int n_shared, size_t n_pairs) {
    const size_t E_tot = (size_t)E + n_shared;
    return r256(4) + r256((E_tot + 1) * 4) + r256((E_tot + 1) * 4) + r256(n_pairs * 4) + r256((E_tot + 2) * 4) +
           r256(n_pairs * act_bytes(g.nbI)) + r256(n_pairs * g.I * 4) + r256(n_pairs * g.I * 4);
}

size_t batched_partial_bytes(const Geom& g, int E, int n_shared, int k, int T) {
    const size_t ks = (size_t)k + n_shared, n_pairs = (size_t)T * ks;
    return experts_scratch_bytes(g, E, n_shared, n_pairs) + r256((size_t)T * E * 8) +
           r256((size_t)T * act_bytes(g.nbH)) + r256(n_pairs * 4) + r256(n_pairs * 4);
}

// the tensor-core expert matmuls pay off once experts average this many (token, slot)
// pairs; below it the dp4a kernels run
constexpr int MMA_MIN_PAIRS_PER_EXPERT = 16;

size_t batched_scratch_bytes(const Geom& g, int E, int k, int T) {
    const size_t n_pairs = (size_t)T * k;
    return batched_partial_bytes(g, E, 0, k, T) + r256(n_pairs * 4) + n_pairs * g.H * 4;
}

cudaError_t launch_batched_experts(const uint8_t* layer, const uint8_t* shared, int E, int e_lo, int e_n, int rank,
                                   int G, Geom g, int n_shared, int k, int ks, const int* idx, int n_tok,
                                   const uint8_t* xq, void* scratch, size_t scratch_bytes, float* y, int* owned,
                                   int kernels, int pairs_per_expert_div, cudaStream_t s, unsigned* err_flag,
                                   const int* n_pairs_dev) {
    const size_t n_pairs = (size_t)n_tok * ks;
    const int E_tot = E + n_shared;
    if (n_tok <= 0) return cudaSuccess;
    if (experts_scratch_bytes(g, E, n_shared, n_pairs) > scratch_bytes) return cudaErrorInvalidValue;
    uint8_t* p = static_cast<uint8_t*>(scratch);
    auto take = [&](size_t n) {
        uint8_t* r = p;
        p += r256(n);
        return r;
    };
    unsigned* err = reinterpret_cast<unsigned*>(take(4));   // first: at the scratch's start
    if (err_flag) err = err_flag;
    int* active = reinterpret_cast<int*>(take((size_t)(E_tot + 1) * 4));
    int* off = reinterpret_cast<int*>(take((size_t)(E_tot + 1) * 4));
    int* list = reinterpret_cast<int*>(take(n_pairs * 4));
    int* tile_pre = reinterpret_cast<int*>(take((size_t)(E_tot + 2) * 4));
    uint8_t* hq = take(n_pairs * act_bytes(g.nbI));
    float* hf = reinterpret_cast<float*>(take(n_pairs * g.I * 4));
    float* uf = reinterpret_cast<float*>(take(n_pairs * g.I * 4));

    int dev = 0, optin = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
    if (batched_smem_bytes(g) > (size_t)optin) return cudaErrorInvalidValue;
    k_group_pairs<<<1, 256, 0, s>>>(idx, (int)n_pairs, ks, k, E_tot, e_n, rank, G, off, list, active, owned,
                                    tile_pre, q4_mma_tile_tokens(), n_pairs_dev);
    const size_t max_act = (size_t)e_n + n_shared;
    const int n_act = (int)(n_pairs < max_act ? n_pairs : max_act);
    const bool mma = q4_mma_supported(g) &&
                     (kernels == BATCHED_MMA || kernels == BATCHED_MMA_FAST ||
                      (kernels == BATCHED_AUTO && n_pairs >= (size_t)MMA_MIN_PAIRS_PER_EXPERT * pairs_per_expert_div));
    const bool exact = kernels != BATCHED_MMA_FAST;
    if (mma) {
        if ((e = launch_q4_mma(layer, shared, E, e_lo, g, 0, off, list, active, tile_pre, n_act, ks, xq, hf, uf, err,
                               exact, s)) != cudaSuccess)
            return e;
        const long long warps = (long long)n_pairs * g.nbI;
        k_quant_h<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(hf, uf, (int)n_pairs, g, hq, n_pairs_dev);
        return launch_q4_mma(layer, shared, E, e_lo, g, 1, off, list, active, tile_pre, n_act, ks, hq, y, nullptr, err,
                             exact, s);
    }
    const int R_gu = GU_ROWS;
    const bool wide = n_pairs >= (size_t)WIDE_MIN_PAIRS * pairs_per_expert_div;
    const size_t sm_gu = (size_t)2 * R_gu * g.row_gu;
    auto gateup = [&](auto kern, int rows_per_cta) -> cudaError_t {
        cudaError_t r;
        if (sm_gu > 48 * 1024 &&
            (r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_gu)) != cudaSuccess)
            return r;
        kern<<<dim3(g.I / rows_per_cta, n_act), 256, sm_gu, s>>>(layer, shared, E, e_lo, g, off, list, active, ks, xq,
                                                                 hf);
        return cudaGetLastError();
    };
    e = wide ? gateup(k_gateup_batched<16>, GU_ROWS) : gateup(k_gateup_batched<4>, GU_ROWS);
    if (e != cudaSuccess) return e;
    {
        const long long warps = (long long)n_pairs * g.nbI;
        k_quant_h<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(hf, nullptr, (int)n_pairs, g, hq, n_pairs_dev);
    }
    const size_t sm_d = (size_t)DOWN_ROWS * g.row_d;
    auto down = [&](auto kern) -> cudaError_t {
        cudaError_t r;
        if (sm_d > 48 * 1024 &&
            (r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_d)) != cudaSuccess)
            return r;
        kern<<<dim3((g.H + DOWN_ROWS - 1) / DOWN_ROWS, n_act), 256, sm_d, s>>>(layer, shared, E, e_lo, g, off, list,
                                                                              active, hq, y);
        return cudaGetLastError();
    };
    return wide ? down(k_down_batched<16>) : down(k_down_batched<4>);
}

cudaError_t launch_batched_route(Geom g, const float* R, const float* normw, float eps, int E, int n_shared, int k,
                                 const float* X, int T, unsigned long long* S, int* idx, float* wts, float* logits_out,
                                 uint8_t* xq, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const int ks = k + n_shared;
    cudaError_t e;
    if ((e = cudaMemsetAsync(S, 0, (size_t)T * E * 8, s)) != cudaSuccess) return e;
    k_router_sums_batched<<<dim3((T + RT_TOK - 1) / RT_TOK, (E + 7) / 8, g.H / 256), 256, 0, s>>>(X, T, R, normw, E,
                                                                                                g.H, S);
    k_topk_quant_batched<<<T, 256, 0, s>>>(X, normw, eps, E, g.H, k, ks, S, idx, wts, logits_out, xq);
    return cudaGetLastError();
}

cudaError_t launch_moe_batched_partial(const uint8_t* layer, const uint8_t* shared, int e_lo, int e_n, int rank,
                                       int G, Geom g, const float* R, const float* normw, float eps, int E,
                                       int n_shared, int k, const float* X, int T, void* scratch,
                                       size_t scratch_bytes, float* y, int* idx_out, float* w_out,
                                       float* logits_out, int kernels, cudaStream_t s, bool zero_y,
                                       int* owned) {
    if (T <= 0) return cudaSuccess;
    if (E <= 0 || E > 1024 || k <= 0 || k > MAX_TOPK || k > E || n_shared < 0 || n_shared > 1 ||
        (n_shared && !shared) || k + n_shared > MAX_TOPK + 1 || G < 1 || rank < 0 || rank >= G || e_n * G != E ||
        e_lo != rank * e_n || batched_partial_bytes(g, E, n_shared, k, T) > scratch_bytes)
        return cudaErrorInvalidValue;
    const int ks = k + n_shared;
    const size_t n_pairs = (size_t)T * ks;
    // the expert step's scratch (error flag first, so at the scratch's start), then the
    // routing buffers
    const size_t xs = experts_scratch_bytes(g, E, n_shared, n_pairs);
    uint8_t* p = static_cast<uint8_t*>(scratch) + xs;
    auto take = [&](size_t n) {
        uint8_t* r = p;
        p += r256(n);
        return r;
    };
    unsigned long long* S = reinterpret_cast<unsigned long long*>(take((size_t)T * E * 8));
    uint8_t* xq = take((size_t)T * act_bytes(g.nbH));
    int* idx_s = reinterpret_cast<int*>(take(n_pairs * 4));
    float* wts_s = reinterpret_cast<float*>(take(n_pairs * 4));
    int* idx = idx_out ? idx_out : idx_s;
    float* wts = w_out ? w_out : wts_s;
    cudaError_t e;
    // pairs computed on other devices keep y = 0 (their owner adds theirs)
    if (G > 1 && zero_y && (e = cudaMemsetAsync(y, 0, n_pairs * g.H * 4, s)) != cudaSuccess) return e;
    if ((e = launch_batched_route(g, R, normw, eps, E, n_shared, k, X, T, S, idx, wts, logits_out, xq, s)) !=
        cudaSuccess)
        return e;
    return launch_batched_experts(layer, shared, E, e_lo, e_n, rank, G, g, n_shared, k, ks, idx, T, xq, scratch, xs, y,
                                  owned, kernels, E + n_shared, s);
}

cudaError_t launch_moe_batched_combine(float* X, int T, int H, int ks, const float* wts, const float* y,
                                       cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    k_combine_batched<<<dim3(T, (H + 255) / 256), 256, 0, s>>>(X, H, ks, wts, y);
    return cudaGetLastError();
}

cudaError_t launch_moe_batched(const uint8_t* layer, Geom g, const float* R, const float* normw, float eps, int E,
                               int k, float* X, int T, void* scratch, size_t scratch_bytes, int* idx_out,
                               float* w_out, float* logits_out, int kernels, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    if (E <= 0 || E > 1024 || k <= 0 || k > MAX_TOPK || k > E || batched_scratch_bytes(g, E, k, T) > scratch_bytes)
        return cudaErrorInvalidValue;
    // the partial step's buffers, then w (unless given) and y at the end of the scratch
    const size_t n_pairs = (size_t)T * k;
    uint8_t* base = static_cast<uint8_t*>(scratch);
    const size_t part = batched_partial_bytes(g, E, 0, k, T);
    float* wts = w_out ? w_out : reinterpret_cast<float*>(base + part);
    float* y = reinterpret_cast<float*>(base + part + r256(n_pairs * 4));
    cudaError_t e = launch_moe_batched_partial(layer, nullptr, 0, E, 0, 1, g, R, normw, eps, E, 0, k, X, T, scratch,
                                               part, y, idx_out, wts, logits_out, kernels, s);
    if (e != cudaSuccess) return e;
    return launch_moe_batched_combine(X, T, g.H, k, wts, y, s);
}

}  // namespace tg

// tg_decode.cu — the fused decode step: every MoE layer of one token in ONE
// persistent cooperative kernel (one CTA per SM: 16 compute warps + 1 producer warp).
//
// Per layer l (tinygiant/engine.py:229-258, attention excluded):
//   A  routing: wait until all CTAs' partial sums for layer l have landed in
//      acc[l] (count-tagged fixed point: R . (x * ffn_norm) per expert and sum x^2),
//      form the RMSNorm scale and the logits, top-k + softmax (engine.py:229-236);
//      every CTA computes the same result.
//   B  issue: the producer warp bulk-copies (cp.async.bulk, TMA) all of this CTA's
//      weight bytes for the layer into shared memory: its gate/up units (32 rows
//      of gate + up of one chosen expert), then its contiguous range of down rows
//      for all k chosen experts, the next layer's router columns for those rows
//      and the next layer's norm weights.  Meanwhile the compute warps quantise
//      RMSNorm(x_l) to Q8_0 (libtinygiant.c:322-340, 61-89).
//   C  gate/up: per unit, 32 gate and 32 up row dots, h = silu(g)*u, Q8_0 of the
//      32 h values (libtinygiant.c:566-586); the block is published as six
//      epoch-tagged 64-bit words (no separate flag round trip).
//   D  down: wait for all k*I/32 h blocks (polling their tags), then the CTA's
//      output rows for all k experts, combined in expert-slot order and added to
//      x (libtinygiant.c:588-594, engine.py:240-258); the rows' products with the
//      next router and their squares (fixed point, so partition-free and exact)
//      are added into acc[l+1] together with a count tag.
// Arithmetic is identical to the multi-kernel path and to the oracle's mirror
// order, so results are bit-identical.
//
// Every wait (mbarrier, tag poll) has a wall-clock limit; on expiry the kernel
// records an error in ctl[2..3], drains its own outstanding copies and returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "tg_decode.h"
#include "tg_device.cuh"

namespace tg {

namespace {

constexpr int NT = FUSED_THREADS;             // threads per CTA
constexpr int CW = FUSED_COMPUTE_WARPS;       // compute warps
constexpr int CT = CW * 32;                   // compute threads
constexpr int PT = CT;                        // the producer thread (lane 0 of the last warp)
constexpr unsigned long long CNT_UNIT = 1ull << 56;   // count tag unit in acc words (<= 255 CTAs)
// Wait limit in SM cycles (~1 s at the B200's 1.9-2 GHz; longer if clocks drop).
// clock64 is a per-SM counter and cheap to read, unlike %globaltimer.
constexpr long long WAIT_CYCLES = 2000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_add_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// CTA barriers.  __syncthreads is an aligned barrier: every warp must reach it
// converged.  Single-lane sections (the producer's copy issue, thread 0's
// bookkeeping) and per-thread spin exits leave warps diverged, so each barrier
// first reconverges its warp.
__device__ __forceinline__ void cta_sync() {
    __syncwarp();
    __syncthreads();
}
__device__ __forceinline__ int cta_sync_and(int pred) {
    __syncwarp();
    return __syncthreads_and(pred);
}

// Error path (kept out of line): first failure wins ctl[2] and its detail word.
__device__ __noinline__ void record_failure(unsigned* ctl, int* flags, unsigned code) {
    if (atomicCAS(ctl + 2, 0u, code) == 0u) ctl[3] = (unsigned)flags[1];
    flags[0] = 1;
}

// One Q8_0 block held one value per lane (lane = position): code, 8 * sum of
// codes, fp16 scale bits.  Kept out of line: it is called from several phases
// and the per-layer loop must stay small enough for the instruction cache.
struct Q8Res {
    int q;
    int s8;
    unsigned dh;
};
__device__ __noinline__ Q8Res q8_block_lane(float v) {
    __syncwarp();
    float am = absmax_lane(v);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    Q8Scale sc = q8_scale(am);
    Q8Res r;
    r.q = q8_round(v, sc.id);
    int s = r.q;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    r.s8 = 8 * s;
    r.dh = sc.dh;
    return r;
}

__device__ __noinline__ float silu_mul_out(float g, float u) { return silu_mul(g, u); }

// Sum each of 8 per-lane values over the warp with the same pairing tree as 8
// separate xor butterflies (so the same bits), in 9 shuffles: at offsets 16, 8, 4
// each lane hands half of its values to its partner and keeps the other half.
// Value j ends in lanes 4j .. 4j+3.
__device__ __forceinline__ float warp_sum8_transposed(const float (&v)[8], int lane) {
    __syncwarp();
    float a[4], b[2];
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float send = h16 ? v[i] : v[i + 4];
        float keep = h16 ? v[i + 4] : v[i];
        a[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 16));
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
        float send = h8 ? a[i] : a[i + 2];
        float keep = h8 ? a[i + 2] : a[i];
        b[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 8));
    }
    float send = h4 ? b[0] : b[1];
    float keep = h4 ? b[1] : b[0];
    float y = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
    y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 2));
    y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 1));
    return y;
}

// The same for 4 values (6 shuffles); value j ends in lanes 8j .. 8j+7.
__device__ __forceinline__ float warp_sum4_transposed(float v0, float v1, float v2, float v3, int lane) {
    __syncwarp();
    const bool h16 = lane & 16, h8 = lane & 8;
    float a0 = __fadd_rn(h16 ? v2 : v0, __shfl_xor_sync(0xffffffffu, h16 ? v0 : v2, 16));
    float a1 = __fadd_rn(h16 ? v3 : v1, __shfl_xor_sync(0xffffffffu, h16 ? v1 : v3, 16));
    float y = __fadd_rn(h8 ? a1 : a0, __shfl_xor_sync(0xffffffffu, h8 ? a0 : a1, 8));
    y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 4));
    y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 2));
    y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 1));
    return y;
}

__device__ __forceinline__ XBlk load_xblk_s(const ActView& a, int b) {
    XBlk x;
    const int4* q = reinterpret_cast<const int4*>(a.qs + (size_t)b * 32);
    x.lo = q[0];
    x.hi = q[1];
    x.d = a.d[b];
    x.s8 = a.s8[b];
    return x;
}

}  // namespace

template <bool TRACE>
__global__ void __launch_bounds__(NT, 1) k_decode_fused(FusedParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const FusedSmem S = fused_smem_layout(P);
    uint64_t* mbar_gu = reinterpret_cast<uint64_t*>(smem + S.mbar);     // [FUSED_MAX_GU]
    uint64_t* mbar_d = mbar_gu + FUSED_MAX_GU;                             // down rows + next router / norm
    uint64_t* mbar_rt0 = mbar_gu + FUSED_MAX_GU + 1;                       // first router columns + norm
    uint16_t* plan = reinterpret_cast<uint16_t*>(smem + S.plan);
    long long* slog_fx = reinterpret_cast<long long*>(smem + S.slogfx);
    float* slog = reinterpret_cast<float*>(smem + S.slog);
    int* sidx = reinterpret_cast<int*>(smem + S.sidx);
    float* sw = reinterpret_cast<float*>(smem + S.sw);
    int* flags = reinterpret_cast<int*>(smem + S.flags);   // [0] error seen, [1] error detail
    float* sscale = reinterpret_cast<float*>(flags + 2);   // RMSNorm scale of the current layer
    float* xs = reinterpret_cast<float*>(smem + S.xs);
    ActView xq = act_view(smem + S.xq, P.g.nbH);
    uint8_t* hq_base = smem + S.hq;
    uint8_t* rec = smem + S.rec;
    float* sh = reinterpret_cast<float*>(smem + S.sh);      // [2][32]
    uint8_t* hrec = smem + S.hrec;                           // [2][64]
    float* xnext = reinterpret_cast<float*>(smem + S.xnext);  // x of the next layer, this CTA's rows
    float* xw = reinterpret_cast<float*>(smem + S.xw);        // the same rows times the next norm weight
    float* rt = reinterpret_cast<float*>(smem + S.rt);        // router columns of this CTA's rows [rows][E]
    float* snorm = reinterpret_cast<float*>(smem + S.snorm);  // [2][H]
    uint8_t* arena = smem + S.arena;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, cta = blockIdx.x;
    const Geom g = P.g;
    const int E = P.E, k = P.k, nbH = g.nbH, nbI = g.nbI;
    const size_t ab_i = act_bytes(nbI);
    const uint32_t gu_unit_bytes = (uint32_t)(32 * g.row_gu);  // one of gate / up
    const uint32_t norm_bytes = (uint32_t)(4 * g.H);           // one layer's FFN norm weights

    if (tid < FUSED_PLAN) plan[tid] = P.plan[(size_t)cta * FUSED_PLAN + tid];
    if (tid == PT) {
        for (int i = 0; i < FUSED_MAX_GU + 2; i++) mbar_init(mbar_gu + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid == 0) {
        flags[0] = 0;
        flags[1] = 0;
    }
    cta_sync();
    const int n_gu = plan[0], d_lo = plan[1], d_n = plan[2];
    const uint16_t* gu_units = plan + 3;
    const uint32_t d_chunk = (uint32_t)d_n * (uint32_t)g.row_d;   // this CTA's rows of one expert's down
    const uint32_t rt_bytes = (uint32_t)d_n * (uint32_t)E * 4u;  // their router columns
    const unsigned epoch = ld_relaxed_u32(P.ctl);
    const unsigned long long tag = (unsigned long long)(epoch % 65535u + 1u);
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();

    // Producer-thread bookkeeping of armed, not yet waited mbarriers (for the error
    // path).  Every mbarrier completes at most once per layer, so the parity to
    // wait for in layer l is l & 1 (0 for the one-off first router copy).
    unsigned pending = 0;  // bits 0..3: gate/up units, bit 4: down group, bit 5: first router copy
    int cur_l = 0;

    auto fail = [&](unsigned code) { record_failure(P.ctl, flags, code); };
    auto error_seen = [&]() -> bool { return ld_relaxed_u32(P.ctl + 2) != 0; };
    // trace stamp: %globaltimer (ns) for cross-SM alignment and clock64 taken after
    // it, so cycle intervals exclude the timer read; slot 31 keeps the read's cost
    auto stamp = [&](int l, int slot) {
        if (TRACE) {
            const long long c0 = clock64();
            const unsigned long long t = gtime();
            const long long c1 = clock64();
            unsigned long long* row = P.trace + ((size_t)l * G + cta) * FUSED_TRACE;
            row[slot] = t;
            if (slot < 15) row[16 + slot] = (unsigned long long)c1;
            if (slot == 3) row[31] = (unsigned long long)(c1 - c0);
        }
    };
    // all threads: bounded wait on an mbarrier phase (records an error on timeout)
    auto wait_bar = [&](uint64_t* bar, unsigned parity, unsigned code) {
        const long long t0 = clock64();
        int spins = 0;
        while (!mbar_try_wait(bar, parity)) {
            if ((++spins & 255) == 0 && clock64() - t0 > WAIT_CYCLES) {
                if (lane == 0) fail(code);
                return;
            }
        }
    };

    // ---------------------------------------------------------------- first routing partials
    if (tid == PT) {
        mbar_arrive_expect_tx(mbar_rt0, rt_bytes + norm_bytes);
        if (d_n > 0) bulk_g2s(rt, P.RT + ((size_t)P.L0 * g.H + d_lo) * E, rt_bytes, mbar_rt0, pol_keep);
        bulk_g2s(snorm, P.normw + (size_t)P.L0 * g.H, norm_bytes, mbar_rt0, pol_keep);
        pending |= 1u << 5;
    }
    #pragma unroll 1
    for (int q = tid; q < d_n; q += NT) xnext[q] = P.x_in[d_lo + q];
    wait_bar(mbar_rt0, 0, 1);
    cta_sync();
    if (flags[0]) goto drain;
    if (tid == PT) pending &= ~(1u << 5);
    #pragma unroll 1
    for (int q = tid; q < d_n; q += NT) xw[q] = __fmul_rn(xnext[q], snorm[d_lo + q]);
    cta_sync();
    for (int e = tid; e <= E; e += NT) {
        long long s = 0;
        if (e < E)
#pragma unroll 1
            for (int q = 0; q < d_n; q++) s += router_fixed(rt[(size_t)q * E + e], xw[q]);
        else
#pragma unroll 1
            for (int q = 0; q < d_n; q++) s += ss_fixed(xnext[q]);
        atomicAdd(P.acc + e, CNT_UNIT + (unsigned long long)s);   // x_in is complete before the launch
    }

    for (int l = 0; l < P.nL; l++) {
        const int layer = P.L0 + l;
        cur_l = l;
        unsigned long long* accl = P.acc + (size_t)l * (E + 1);
        // ------------------------------------------------------------ A: routing
        {
            const long long t0 = clock64();
            int spins = 0;
            while (true) {
                int ok = 1;
                for (int e = tid; e <= E; e += NT) {
                    unsigned long long v = ld_relaxed_u64(accl + e);
                    unsigned long long cnt = (v + (1ull << 55)) >> 56;
                    if (cnt != (unsigned long long)G) {
                        ok = 0;
                        flags[1] = (l << 20) | ((e & 0xfff) << 8) | (int)(cnt & 0xff);
                    } else {
                        slog_fx[e] = (long long)(v - (unsigned long long)G * CNT_UNIT);
                    }
                }
                if (cta_sync_and(ok)) break;
                if (tid == 0 && ((++spins & 63) == 0) && (clock64() - t0 > WAIT_CYCLES || error_seen())) fail(2);
                cta_sync();
                if (flags[0]) goto drain;
            }
        }
        // thread 0 read acc[l][0] after every CTA's release: its acquire fence orders
        // this CTA's later reads of x_l (after the next barrier) behind all producers
        if (tid == 0) {
            fence_acq_rel_gpu();
            *sscale = rms_scale_from(slog_fx[E], g.H, P.eps);
        }
        cta_sync();
        if (tid == 0) stamp(l, 0);
        // logits of the normed input: scale * (R . (x * w)), scale = 1/sqrt(ss/H + eps);
        // once every CTA has contributed to acc[l], acc[l-1] is read by no one and is recycled
        {
            const float scale = *sscale;
#pragma unroll 1
            for (int e = tid; e < E; e += NT) slog[e] = __fmul_rn(scale, router_logit(slog_fx[e]));
            if (cta == 0 && l >= 1)
                for (int e = tid; e <= E; e += NT) accl[e - (E + 1)] = 0ull;
        }
        cta_sync();
        // top-k by rank: 4 threads per expert share the scan; the element beaten by
        // fewer than k others (larger logit, or equal logit and larger id) is kept
        for (int base = 0; base < E; base += NT / 4) {
            int e = base + (tid >> 2), part = tid & 3;
            int rank = 0;
            if (e < E) {
                float le = slog[e];
                int chunk = (E + 3) / 4;
                int j0 = part * chunk, j1 = min(E, j0 + chunk);
#pragma unroll 4
                for (int j = j0; j < j1; j++) {
                    float lj = slog[j];
                    rank += (lj > le) || (lj == le && j > e);
                }
            }
            __syncwarp();
            rank += __shfl_xor_sync(0xffffffffu, rank, 1);
            rank += __shfl_xor_sync(0xffffffffu, rank, 2);
            if (e < E && part == 0 && rank < k) sidx[k - 1 - rank] = e;
        }
        cta_sync();
        if (tid == 0) stamp(l, 9);
        // softmax over the k chosen logits (engine.py:233-236): lane j holds exp(l_j - max);
        // the sum for k <= 8 is ((e0+e1)+(e2+e3))+((e4+e5)+(e6+e7)), three xor steps
        if (warp == 0) {
            const float m = slog[sidx[k - 1]];
            float ex = lane < k ? tg_expf(__fsub_rn(slog[sidx[lane]], m)) : 0.0f;
            __syncwarp();
            float s;
            if (k <= 8) {
                float v = ex;
                v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
                v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
                v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
                s = __shfl_sync(0xffffffffu, v, 0);
            } else {
                s = 0.0f;
                for (int j = 0; j < k; j++) s = __fadd_rn(s, __shfl_sync(0xffffffffu, ex, j));
            }
            if (lane < k) sw[lane] = __fdiv_rn(ex, s);
        }
        cta_sync();
        if (tid == 0) stamp(l, 10);
        if (cta == 0) {
            if (tid < k) {
                P.idx_out[(size_t)layer * k + tid] = sidx[tid];
                P.w_out[(size_t)layer * k + tid] = sw[tid];
            }
            for (int e = tid; e < E; e += NT) P.logits_out[(size_t)layer * E + e] = slog[e];
        }

        // ------------------------------------------------------------ B: the producer issues all copies
        const uint8_t* lbase = P.weights + (size_t)layer * P.layer_bytes;
        const bool next = l + 1 < P.nL;
        const bool d_armed = d_n > 0 || next;   // mbar_d also carries the next layer's norm weights
        if (tid == PT) {
            stamp(l, 11);
            // the regions below were read by this CTA's threads in the previous layer
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            stamp(l, 12);
            for (int u = 0; u < n_gu; u++) {
                int unit = gu_units[u];
                int j = unit / nbI, c = unit - j * nbI;
                const uint8_t* eb = lbase + (size_t)sidx[j] * g.expert_bytes;
                uint8_t* dst = arena + (size_t)u * 2 * gu_unit_bytes;
                mbar_arrive_expect_tx(mbar_gu + u, 2 * gu_unit_bytes);
                bulk_g2s(dst, eb + (size_t)c * gu_unit_bytes, gu_unit_bytes, mbar_gu + u, pol_stream);
                bulk_g2s(dst + gu_unit_bytes, eb + g.t_gu + (size_t)c * gu_unit_bytes, gu_unit_bytes, mbar_gu + u,
                         pol_stream);
                pending |= 1u << u;
            }
            stamp(l, 13);
            if (d_armed) {
                mbar_arrive_expect_tx(mbar_d, (uint32_t)k * d_chunk + (next ? rt_bytes + norm_bytes : 0u));
                uint8_t* dbase = arena + (size_t)n_gu * 2 * gu_unit_bytes;
                if (d_n > 0)
#pragma unroll 1
                    for (int j = 0; j < k; j++)
                        bulk_g2s(dbase + (size_t)j * d_chunk,
                                 lbase + (size_t)sidx[j] * g.expert_bytes + 2 * g.t_gu + (size_t)d_lo * g.row_d,
                                 d_chunk, mbar_d, pol_stream);
                if (next) {
                    if (d_n > 0)
                        bulk_g2s(rt, P.RT + ((size_t)(layer + 1) * g.H + d_lo) * E, rt_bytes, mbar_d, pol_keep);
                    bulk_g2s(snorm + (size_t)((l + 1) & 1) * g.H, P.normw + (size_t)(layer + 1) * g.H, norm_bytes,
                             mbar_d, pol_keep);
                }
                pending |= 1u << 4;
            }
            stamp(l, 1);
        }
        // x_l -> shared (f32) and the Q8_0 activation form of RMSNorm(x_l), while the copies fly
        if (warp < CW) {
            const float* xsrc = l == 0 ? P.x_in : P.xbuf + (size_t)l * g.H;
#pragma unroll 1
            for (int i = tid; i < g.H; i += CT) xs[i] = __ldcg(xsrc + i);
        }
        cta_sync();
        if (tid == 0) stamp(l, 14);
        if (warp < CW) {
            const float scale = *sscale;
            const float* nw = snorm + (size_t)(l & 1) * g.H;
            for (int b = warp; b < nbH; b += CW) {
                // expert input = RMSNorm(x) * w = (x * scale) * w  (libtinygiant.c:336-339)
                const float v = __fmul_rn(__fmul_rn(xs[(size_t)b * 32 + lane], scale), nw[(size_t)b * 32 + lane]);
                const Q8Res r = q8_block_lane(v);
                xq.qs[(size_t)b * 32 + lane] = (int8_t)r.q;
                if (lane == 0) {
                    xq.d[b] = f16_bits_to_f32((uint16_t)r.dh);
                    xq.s8[b] = r.s8;
                }
            }
        }
        cta_sync();
        if (tid == 0) stamp(l, 2);

        // ------------------------------------------------------------ C: gate/up units
        for (int u = 0; u < n_gu; u++) {
            wait_bar(mbar_gu + u, (unsigned)l & 1u, 3);
            cta_sync();
            if (flags[0]) goto drain;
            if (u == 0 && tid == 0) stamp(l, 8);
            if (tid == PT) pending &= ~(1u << u);
            const int unit = gu_units[u];
            const int j = unit / nbI, c = unit - j * nbI;
            float* shu = sh + (u & 1) * 32;
            uint8_t* hr = hrec + (u & 1) * 64;
            if (warp < CW) {
                const uint8_t* gate = arena + (size_t)u * 2 * gu_unit_bytes;
                const uint8_t* up = gate + gu_unit_bytes;
                const int r0 = warp * 2;   // two h rows per compute warp (CW * 2 == 32)
                float ag0 = 0.f, ag1 = 0.f, au0 = 0.f, au1 = 0.f;
#pragma unroll 1
                for (int b = lane; b < nbH; b += 32) {
                    XBlk xb = load_xblk_s(xq, b);
                    const uint8_t* rg0 = gate + (size_t)r0 * g.row_gu;
                    const uint8_t* rg1 = rg0 + g.row_gu;
                    const uint8_t* ru0 = up + (size_t)r0 * g.row_gu;
                    const uint8_t* ru1 = ru0 + g.row_gu;
                    uint4 wg0 = *reinterpret_cast<const uint4*>(rg0 + 16 * b);
                    uint4 wg1 = *reinterpret_cast<const uint4*>(rg1 + 16 * b);
                    uint4 wu0 = *reinterpret_cast<const uint4*>(ru0 + 16 * b);
                    uint4 wu1 = *reinterpret_cast<const uint4*>(ru1 + 16 * b);
                    float dg0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rg0 + 16 * nbH + 2 * b));
                    float dg1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rg1 + 16 * nbH + 2 * b));
                    float du0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ru0 + 16 * nbH + 2 * b));
                    float du1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ru1 + 16 * nbH + 2 * b));
                    ag0 = __fadd_rn(ag0, block_term(block_sumi(wg0, xb), dg0, xb.d));
                    ag1 = __fadd_rn(ag1, block_term(block_sumi(wg1, xb), dg1, xb.d));
                    au0 = __fadd_rn(au0, block_term(block_sumi(wu0, xb), du0, xb.d));
                    au1 = __fadd_rn(au1, block_term(block_sumi(wu1, xb), du1, xb.d));
                }
                // gate0 ends in lanes 0-7, gate1 in 8-15, up0 in 16-23, up1 in 24-31
                const float y = warp_sum4_transposed(ag0, ag1, au0, au1, lane);
                const float hg = __shfl_sync(0xffffffffu, y, lane & 8);        // gate of this lane's row
                const float hu = __shfl_sync(0xffffffffu, y, 16 + (lane & 8));  // its up
                if ((lane & 23) == 0) shu[r0 + (lane >> 3)] = silu_mul_out(hg, hu);   // lanes 0 and 8
            }
            cta_sync();
            if (warp == 0) {
                const Q8Res r = q8_block_lane(shu[lane]);
                const int s = r.s8 >> 3;   // sum of the codes (|s| <= 32 * 127)
                hr[lane] = (uint8_t)(int8_t)r.q;
                if (lane == 0) {
                    hr[32] = (uint8_t)(r.dh & 0xff);
                    hr[33] = (uint8_t)(r.dh >> 8);
                    hr[34] = (uint8_t)(s & 0xff);
                    hr[35] = (uint8_t)((s >> 8) & 0xff);
                }
                __syncwarp();
                if (lane < 6) {
                    unsigned long long wv = tag << 48;
#pragma unroll
                    for (int t = 0; t < 6; t++) wv |= (unsigned long long)hr[lane * 6 + t] << (8 * t);
                    st_relaxed_u64(P.hqt + (((size_t)l * k + j) * nbI + c) * 6 + lane, wv);
                }
            }
            // the next unit writes the other sh / hrec buffer; the one after it is
            // ordered behind warp 0's publish by the next unit's barriers
        }
        if (tid == 0) stamp(l, 3);

        // ------------------------------------------------------------ D: down rows + combine + next routing
        if (d_n > 0) {
            // gather all k * nbI h blocks (tagged words) into shared memory
            const int nwords = k * nbI * 6;
            {
                const long long t0 = clock64();
                int spins = 0;
                while (true) {
                    int ok = 1;
#pragma unroll 1
                    for (int w = tid; w < nwords; w += NT) {
                        unsigned long long v = ld_relaxed_u64(P.hqt + (size_t)l * nwords + w);
                        if ((v >> 48) != tag) {
                            ok = 0;
                            flags[1] = (l << 20) | ((w / 6) & 0xfff) << 8 | (int)((v >> 48) & 0xff);
                        } else {
                            uint8_t* r = rec + (size_t)(w / 6) * 36 + (w % 6) * 6;
#pragma unroll
                            for (int t = 0; t < 6; t++) r[t] = (uint8_t)(v >> (8 * t));
                        }
                    }
                    if (cta_sync_and(ok)) break;
                    if (tid == 0 && ((++spins & 63) == 0) && (clock64() - t0 > WAIT_CYCLES || error_seen())) fail(4);
                    cta_sync();
                    if (flags[0]) goto drain;
                }
            }
            if (tid == 0) stamp(l, 4);
            // records -> activation form: codes, fp32 scale, 8*sum
#pragma unroll 1
            for (int i = tid; i < k * nbI; i += NT) {
                const uint8_t* r = rec + (size_t)i * 36;
                int j = i / nbI, b = i - j * nbI;
                ActView ha = act_view(hq_base + (size_t)j * ab_i, nbI);
                int4* dq = reinterpret_cast<int4*>(ha.qs + (size_t)b * 32);
                uint32_t wv[8];
#pragma unroll
                for (int t = 0; t < 8; t++)
                    wv[t] = (uint32_t)r[4 * t] | ((uint32_t)r[4 * t + 1] << 8) | ((uint32_t)r[4 * t + 2] << 16) |
                            ((uint32_t)r[4 * t + 3] << 24);
                dq[0] = make_int4((int)wv[0], (int)wv[1], (int)wv[2], (int)wv[3]);
                dq[1] = make_int4((int)wv[4], (int)wv[5], (int)wv[6], (int)wv[7]);
                ha.d[b] = f16_bits_to_f32((uint16_t)(r[32] | (r[33] << 8)));
                ha.s8[b] = 8 * (int)(int16_t)(uint16_t)(r[34] | (r[35] << 8));
            }
            cta_sync();
            if (tid == 0) stamp(l, 15);
        }
        if (d_armed) wait_bar(mbar_d, (unsigned)l & 1u, 5);
        cta_sync();
        if (flags[0]) goto drain;
        if (tid == PT) pending &= ~(1u << 4);
        if (tid == 0) stamp(l, 5);
        if (d_n > 0 && warp < CW) {
            const uint8_t* dbase = arena + (size_t)n_gu * 2 * gu_unit_bytes;
            float* xout = next ? P.xbuf + (size_t)(l + 1) * g.H : P.x_out;
            const float* nw1 = snorm + (size_t)((l + 1) & 1) * g.H;
            for (int q = warp; q < d_n; q += CW) {
                const int r = d_lo + q;
                float a = 0.0f;
                for (int j0 = 0; j0 < k; j0 += 8) {
                    // lane partials of up to 8 experts, then one transposed reduction
                    float acc[8];
#pragma unroll
                    for (int jj = 0; jj < 8; jj++) acc[jj] = 0.0f;
#pragma unroll 1
                    for (int b = lane; b < nbI; b += 32) {
#pragma unroll
                        for (int jj = 0; jj < 8; jj++) {
                            const int j = j0 + jj;
                            if (j < k) {
                                const uint8_t* row = dbase + (size_t)j * d_chunk + (size_t)q * g.row_d;
                                const ActView ha = act_view(hq_base + (size_t)j * ab_i, nbI);
                                const uint4 wv = *reinterpret_cast<const uint4*>(row + 16 * b);
                                const float dw =
                                    f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(row + 16 * nbI + 2 * b));
                                const XBlk xb = load_xblk_s(ha, b);
                                acc[jj] = __fadd_rn(acc[jj], block_term(block_sumi(wv, xb), dw, xb.d));
                            }
                        }
                    }
                    const float y = warp_sum8_transposed(acc, lane);   // expert j0+jj in lanes 4jj..4jj+3
                    for (int jj = 0; jj < 8 && j0 + jj < k; jj++)
                        a = __fadd_rn(a, __fmul_rn(sw[j0 + jj], __shfl_sync(0xffffffffu, y, 4 * jj)));
                }
                if (lane == 0) {
                    float xn = __fadd_rn(xs[r], a);
                    xout[r] = xn;
                    xnext[q] = xn;
                    if (next) xw[q] = __fmul_rn(xn, nw1[r]);
                }
            }
        }
        cta_sync();
        if (tid == 0) stamp(l, 6);
        if (next) {
            // release: the barrier orders every thread's x stores before thread 0's
            // fence, and the next barrier orders the fence before the adds
            if (tid == 0) fence_acq_rel_gpu();
            cta_sync();
            unsigned long long* accn = P.acc + (size_t)(l + 1) * (E + 1);
            for (int e = tid; e <= E; e += NT) {
                long long s = 0;
                if (e < E)
        #pragma unroll 1
            for (int q = 0; q < d_n; q++) s += router_fixed(rt[(size_t)q * E + e], xw[q]);
                else
        #pragma unroll 1
            for (int q = 0; q < d_n; q++) s += ss_fixed(xnext[q]);
                red_add_relaxed_u64(accn + e, CNT_UNIT + (unsigned long long)s);
            }
        }
        cta_sync();
        if (tid == 0) stamp(l, 7);
    }

    // ---------------------------------------------------------------- finish: last CTA advances the epoch
    if (tid == 0) {
        __threadfence();
        unsigned t = atomicAdd(P.ctl + 1, 1u);
        if (t == (unsigned)G - 1) {
            __threadfence();
            unsigned long long* last = P.acc + (size_t)(P.nL - 1) * (E + 1);
            for (int e = 0; e <= E; e++) last[e] = 0ull;
            P.ctl[1] = 0u;
            __threadfence();
            atomicAdd(P.ctl, 1u);
        }
    }
    return;

drain:
    // error path: let this CTA's own copies land before the shared memory goes away
    if (tid == PT) {
        const long long t0 = clock64();
        for (int u = 0; u < FUSED_MAX_GU; u++)
            if (pending >> u & 1u)
                while (!mbar_try_wait(mbar_gu + u, (unsigned)cur_l & 1u) && clock64() - t0 < WAIT_CYCLES) {
                }
        if (pending >> 4 & 1u)
            while (!mbar_try_wait(mbar_d, (unsigned)cur_l & 1u) && clock64() - t0 < WAIT_CYCLES) {
            }
        if (pending >> 5 & 1u)
            while (!mbar_try_wait(mbar_rt0, 0) && clock64() - t0 < WAIT_CYCLES) {
            }
    }
    cta_sync();
}

// ---------------------------------------------------------------- host side

int fused_plan(const Geom& g, int E, int k, int G, std::vector<uint16_t>& plan, size_t& arena_bytes,
               int& max_rows) {
    if (k > 16 || E > 1024 || G <= 0) return -1;
    const int n_gu_units = k * g.nbI;
    const size_t gu_b = 2 * 32 * g.row_gu;
    const size_t drow_b = (size_t)k * g.row_d + (size_t)E * 4;   // one down row of all k experts + router column
    std::vector<double> load(G, 0.0);
    std::vector<std::vector<int>> gu(G);
    for (int u = 0; u < n_gu_units; u++) {
        int best = 0;
        for (int c = 1; c < G; c++)
            if (load[c] < load[best]) best = c;
        gu[best].push_back(u);
        load[best] += (double)gu_b;
    }
    double total = (double)g.H * (double)drow_b;
    for (int c = 0; c < G; c++) total += load[c];
    const double target = total / G;
    std::vector<double> quota(G);
    double qs = 0;
    for (int c = 0; c < G; c++) {
        quota[c] = std::max(0.0, (target - load[c]) / (double)drow_b);
        qs += quota[c];
    }
    std::vector<int> rows(G);
    int assigned = 0;
    for (int c = 0; c < G; c++) {
        quota[c] = qs > 0 ? quota[c] * g.H / qs : (double)g.H / G;
        rows[c] = (int)quota[c];
        assigned += rows[c];
    }
    std::vector<int> order(G);
    for (int c = 0; c < G; c++) order[c] = c;
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return quota[a] - rows[a] > quota[b] - rows[b]; });
    for (int i = 0; assigned < g.H; i = (i + 1) % G, assigned++) rows[order[i]]++;
    plan.assign((size_t)G * FUSED_PLAN, 0);
    arena_bytes = 0;
    max_rows = 0;
    int lo = 0;
    for (int c = 0; c < G; c++) {
        if ((int)gu[c].size() > FUSED_MAX_GU || rows[c] > FUSED_MAX_ROWS) return -2;
        uint16_t* p = plan.data() + (size_t)c * FUSED_PLAN;
        p[0] = (uint16_t)gu[c].size();
        p[1] = (uint16_t)lo;
        p[2] = (uint16_t)rows[c];
        for (size_t i = 0; i < gu[c].size(); i++) p[3 + i] = (uint16_t)gu[c][i];
        lo += rows[c];
        arena_bytes = std::max(arena_bytes, gu[c].size() * gu_b + (size_t)rows[c] * k * g.row_d);
        max_rows = std::max(max_rows, rows[c]);
    }
    if (lo != g.H) return -3;
    arena_bytes = (arena_bytes + 15) & ~(size_t)15;
    return 0;
}

cudaError_t fused_prepare(const FusedParams& P) {
    cudaError_t e = cudaFuncSetAttribute(k_decode_fused<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)fused_smem_layout(P).total);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_decode_fused<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)fused_smem_layout(P).total);
}

cudaError_t fused_occupancy(const FusedParams& P, int* blocks_per_sm) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, k_decode_fused<false>, NT,
                                                         fused_smem_layout(P).total);
}

cudaError_t launch_decode_fused(const FusedParams& P, int G, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = fused_smem_layout(P).total;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (P.trace) return cudaLaunchKernelEx(&cfg, k_decode_fused<true>, P);
    return cudaLaunchKernelEx(&cfg, k_decode_fused<false>, P);
}

}  // namespace tg

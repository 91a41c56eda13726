// tg_decode.cu — the fused decode step: every MoE layer of one token in ONE
// persistent cooperative kernel (one CTA per SM).
//
// Per layer l (tinygiant/engine.py:229-258, attention excluded):
//   A  routing: wait until all CTAs' partial sums for layer l have landed in
//      acc[l] (count-tagged fixed point: R . (x * ffn_norm) per expert and sum x^2),
//      form the RMSNorm scale and the logits, top-k + softmax (engine.py:229-236);
//      every CTA computes the same result.
//   B  issue: one thread bulk-copies (cp.async.bulk, TMA) all of this CTA's
//      weight bytes for the layer into shared memory: its gate/up units
//      (32 rows of gate + up of one chosen expert) and its down units (4 output
//      rows x all k chosen experts), plus the next layer's router columns for
//      its rows.  Meanwhile every thread quantises RMSNorm(x_l) to Q8_0
//      (libtinygiant.c:322-340, 61-89).
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
// records an error in ctl[2], drains its own outstanding copies and returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "tg_decode.h"
#include "tg_device.cuh"

namespace tg {

namespace {

constexpr int NT = FUSED_THREADS;     // threads per CTA
constexpr int NW = NT / 32;
constexpr unsigned long long CNT_UNIT = 1ull << 56;   // count tag unit in acc words (<= 255 CTAs)
constexpr unsigned long long WAIT_NS = 1000000000ull; // 1 s per wait

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
__device__ __forceinline__ void red_add_release_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
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

__global__ void __launch_bounds__(NT, 1) k_decode_fused(FusedParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const FusedSmem S = fused_smem_layout(P);
    uint64_t* mbar_gu = reinterpret_cast<uint64_t*>(smem + S.mbar);     // [FUSED_MAX_GU]
    uint64_t* mbar_d = mbar_gu + FUSED_MAX_GU;                             // down + next-router columns
    uint64_t* mbar_rt0 = mbar_gu + FUSED_MAX_GU + 1;                       // first router columns
    uint16_t* plan = reinterpret_cast<uint16_t*>(smem + S.plan);
    long long* slog_fx = reinterpret_cast<long long*>(smem + S.slogfx);
    float* slog = reinterpret_cast<float*>(smem + S.slog);
    int* sidx = reinterpret_cast<int*>(smem + S.sidx);
    float* sw = reinterpret_cast<float*>(smem + S.sw);
    int* flags = reinterpret_cast<int*>(smem + S.flags);                   // [0] = error seen
    float* xs = reinterpret_cast<float*>(smem + S.xs);
    ActView xq = act_view(smem + S.xq, P.g.nbH);
    uint8_t* hq_base = smem + S.hq;
    uint8_t* rec = smem + S.rec;
    float* sh = reinterpret_cast<float*>(smem + S.sh);
    uint8_t* hrec = smem + S.hrec;
    float* xnext = reinterpret_cast<float*>(smem + S.xnext);   // x of the next layer, this CTA's rows
    float* xw = reinterpret_cast<float*>(smem + S.xw);         // the same rows times the next norm weight
    float* rt = reinterpret_cast<float*>(smem + S.rt);
    uint8_t* arena = smem + S.arena;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, cta = blockIdx.x;
    const Geom g = P.g;
    const int E = P.E, k = P.k, RD = P.rd, nbH = g.nbH, nbI = g.nbI;
    const size_t ab_i = act_bytes(nbI);
    const uint32_t gu_unit_bytes = (uint32_t)(32 * g.row_gu);   // one of gate / up
    const uint32_t d_chunk = (uint32_t)(RD * g.row_d);          // RD rows of one expert's down
    const uint32_t rt_chunk = (uint32_t)(RD * E * 4);

    if (tid < 2 + FUSED_MAX_GU + FUSED_MAX_D) plan[tid] = P.plan[(size_t)cta * P.plan_stride + tid];
    if (tid == 0) {
        for (int i = 0; i < FUSED_MAX_GU + 2; i++) mbar_init(mbar_gu + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        flags[0] = 0;
        flags[2] = 0;   // diagnostic word recorded with an error: (layer << 20) | (entry << 8) | count
    }
    __syncthreads();
    const int n_gu = plan[0], n_d = plan[1];
    const uint16_t* gu_units = plan + 2;
    const uint16_t* d_units = plan + 2 + FUSED_MAX_GU;
    const unsigned epoch = ld_relaxed_u32(P.ctl);
    const unsigned long long tag = (unsigned long long)(epoch % 65535u + 1u);
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const int nrows = n_d * RD;

    // outstanding-copy bookkeeping (thread 0 only) for the error path.  Every
    // mbarrier completes at most once per layer, so the parity to wait for in
    // layer l is l & 1 (0 for the one-off first router copy).
    unsigned pending_gu = 0;  // bit u: gu mbarrier armed in layer cur_l, not yet waited
    bool pending_d = false, pending_rt0 = false;
    int cur_l = 0;

    auto fail = [&](unsigned code) {
        if (atomicCAS(P.ctl + 2, 0u, code) == 0u) P.ctl[3] = (unsigned)flags[2];
        flags[0] = 1;
    };
    auto error_seen = [&]() -> bool { return ld_relaxed_u32(P.ctl + 2) != 0; };

    // ---------------------------------------------------------------- first routing partials
    if (tid == 0) {
        if (n_d > 0) {
            mbar_arrive_expect_tx(mbar_rt0, rt_chunk * n_d);
            for (int i = 0; i < n_d; i++)
                bulk_g2s(rt + (size_t)i * RD * E, P.RT + ((size_t)P.L0 * g.H + (size_t)d_units[i] * RD) * E, rt_chunk,
                         mbar_rt0, pol_keep);
            pending_rt0 = true;
        }
    }
    for (int q = tid; q < nrows; q += NT) {
        const int r = d_units[q / RD] * RD + (q % RD);
        const float xv = P.x_in[r];
        xnext[q] = xv;
        xw[q] = __fmul_rn(xv, P.normw[(size_t)P.L0 * g.H + r]);
    }
    if (n_d > 0) {
        unsigned long long t0 = gtime();
        while (!mbar_try_wait(mbar_rt0, 0)) {
            if (gtime() - t0 > WAIT_NS) {
                if (tid == 0) fail(1);
                break;
            }
        }
    }
    if (tid == 0) pending_rt0 = false;
    __syncthreads();
    if (flags[0]) goto drain;
    for (int e = tid; e <= E; e += NT) {
        long long s = 0;
        if (e < E)
            for (int q = 0; q < nrows; q++) s += router_fixed(rt[(size_t)q * E + e], xw[q]);
        else
            for (int q = 0; q < nrows; q++) s += ss_fixed(xnext[q]);
        atomicAdd(P.acc + e, CNT_UNIT + (unsigned long long)s);
    }

    for (int l = 0; l < P.nL; l++) {
        const int layer = P.L0 + l;
        cur_l = l;
        unsigned long long* accl = P.acc + (size_t)l * (E + 1);
        // ------------------------------------------------------------ A: routing
        {
            unsigned long long t0 = gtime();
            int spins = 0;
            while (true) {
                int ok = 1;
                for (int e = tid; e <= E; e += NT) {
                    unsigned long long v = ld_relaxed_u64(accl + e);
                    unsigned long long cnt = (v + (1ull << 55)) >> 56;
                    if (cnt != (unsigned long long)G) {
                        ok = 0;
                        flags[2] = (l << 20) | ((e & 0xfff) << 8) | (int)(cnt & 0xff);
                    } else {
                        slog_fx[e] = (long long)(v - (unsigned long long)G * CNT_UNIT);
                    }
                }
                if (__syncthreads_and(ok)) break;
                if (tid == 0 && ((++spins & 63) == 0) && (gtime() - t0 > WAIT_NS || error_seen())) fail(2);
                __syncthreads();
                if (flags[0]) goto drain;
            }
        }
        __threadfence();
        // decode logits in place (fixed -> float), then acc[l-1] can be recycled
        // logits of the normed input: scale * (R . (x * w)), scale = 1/sqrt(ss/H + eps)
        const float scale = rms_scale_from(slog_fx[E], g.H, P.eps);
        for (int e = tid; e < E; e += NT) slog[e] = __fmul_rn(scale, router_logit(slog_fx[e]));
        if (cta == 0 && l >= 1)
            for (int e = tid; e <= E; e += NT) accl[e - (E + 1)] = 0ull;
        __syncthreads();
        // top-k by rank: 4 threads per expert share the scan
        for (int base = 0; base < E; base += NT / 4) {
            int e = base + (tid >> 2), part = tid & 3;
            int rank = 0;
            if (e < E) {
                float le = slog[e];
                int chunk = (E + 3) / 4;
                int j0 = part * chunk, j1 = min(E, j0 + chunk);
                for (int j = j0; j < j1; j++) {
                    float lj = slog[j];
                    rank += (lj > le) || (lj == le && j > e);
                }
            }
            rank += __shfl_xor_sync(0xffffffffu, rank, 1);
            rank += __shfl_xor_sync(0xffffffffu, rank, 2);
            if (e < E && part == 0 && rank < k) sidx[k - 1 - rank] = e;
        }
        __syncthreads();
        if (tid == 0) {
            float m = slog[sidx[k - 1]];
            float ex[16];
            for (int j = 0; j < k; j++) ex[j] = tg_expf(__fsub_rn(slog[sidx[j]], m));
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
        __syncthreads();
        if (cta == 0) {
            if (tid < k) {
                P.idx_out[(size_t)layer * k + tid] = sidx[tid];
                P.w_out[(size_t)layer * k + tid] = sw[tid];
            }
            for (int e = tid; e < E; e += NT) P.logits_out[(size_t)layer * E + e] = slog[e];
        }

        // ------------------------------------------------------------ B: issue the layer's copies
        const uint8_t* lbase = P.weights + (size_t)layer * P.layer_bytes;
        if (tid == 0) {
            // the regions below were read by this CTA's threads in the previous layer
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            for (int u = 0; u < n_gu; u++) {
                int unit = gu_units[u];
                int j = unit / nbI, c = unit - j * nbI;
                const uint8_t* eb = lbase + (size_t)sidx[j] * g.expert_bytes;
                uint8_t* dst = arena + (size_t)u * 2 * gu_unit_bytes;
                mbar_arrive_expect_tx(mbar_gu + u, 2 * gu_unit_bytes);
                bulk_g2s(dst, eb + (size_t)c * gu_unit_bytes, gu_unit_bytes, mbar_gu + u, pol_stream);
                bulk_g2s(dst + gu_unit_bytes, eb + g.t_gu + (size_t)c * gu_unit_bytes, gu_unit_bytes, mbar_gu + u,
                         pol_stream);
                pending_gu |= 1u << u;
            }
            if (n_d > 0) {
                const bool next_rt = l + 1 < P.nL;
                uint32_t bytes = (uint32_t)n_d * k * d_chunk + (next_rt ? (uint32_t)n_d * rt_chunk : 0u);
                mbar_arrive_expect_tx(mbar_d, bytes);
                uint8_t* dbase = arena + (size_t)n_gu * 2 * gu_unit_bytes;
                for (int i = 0; i < n_d; i++)
                    for (int j = 0; j < k; j++) {
                        const uint8_t* src = lbase + (size_t)sidx[j] * g.expert_bytes + 2 * g.t_gu +
                                             (size_t)d_units[i] * d_chunk;
                        bulk_g2s(dbase + ((size_t)i * k + j) * d_chunk, src, d_chunk, mbar_d, pol_stream);
                    }
                if (next_rt)
                    for (int i = 0; i < n_d; i++)
                        bulk_g2s(rt + (size_t)i * RD * E,
                                 P.RT + ((size_t)(layer + 1) * g.H + (size_t)d_units[i] * RD) * E, rt_chunk, mbar_d,
                                 pol_keep);
                pending_d = true;
            }
        }
        // x_l -> shared (f32) and Q8_0 activation form, while the copies fly
        {
            const float* xsrc = l == 0 ? P.x_in : P.xbuf + (size_t)l * g.H;
            const float* nw = P.normw + (size_t)layer * g.H;
            for (int i = tid; i < g.H; i += NT) xs[i] = __ldcg(xsrc + i);
            __syncthreads();
            for (int b = warp; b < nbH; b += NW) {
                // expert input = RMSNorm(x) * w = (x * scale) * w  (libtinygiant.c:336-339)
                float v = __fmul_rn(__fmul_rn(xs[(size_t)b * 32 + lane], scale), __ldg(nw + (size_t)b * 32 + lane));
                float am = absmax_lane(v);
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
                Q8Scale sc = q8_scale(am);
                int q = q8_round(v, sc.id);
                xq.qs[(size_t)b * 32 + lane] = (int8_t)q;
                int s = q;
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                if (lane == 0) {
                    xq.d[b] = f16_bits_to_f32(sc.dh);
                    xq.s8[b] = 8 * s;
                }
            }
            __syncthreads();
        }

        // ------------------------------------------------------------ C: gate/up units
        for (int u = 0; u < n_gu; u++) {
            {
                unsigned long long t0 = gtime();
                int spins = 0;
                while (!mbar_try_wait(mbar_gu + u, (unsigned)l & 1u)) {
                    if ((++spins & 255) == 0 && gtime() - t0 > WAIT_NS) {
                        if (lane == 0) fail(3);
                        break;
                    }
                }
            }
            __syncthreads();
            if (flags[0]) goto drain;
            if (tid == 0) pending_gu &= ~(1u << u);
            const int unit = gu_units[u];
            const int j = unit / nbI, c = unit - j * nbI;
            const uint8_t* gate = arena + (size_t)u * 2 * gu_unit_bytes;
            const uint8_t* up = gate + gu_unit_bytes;
            const int r0 = warp * 2;   // two h rows per warp (NW * 2 == 32)
            float ag0 = 0.f, ag1 = 0.f, au0 = 0.f, au1 = 0.f;
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
            ag0 = warp_sum_butterfly(ag0);
            ag1 = warp_sum_butterfly(ag1);
            au0 = warp_sum_butterfly(au0);
            au1 = warp_sum_butterfly(au1);
            if (lane == 0) {
                sh[r0] = silu_mul(ag0, au0);
                sh[r0 + 1] = silu_mul(ag1, au1);
            }
            __syncthreads();
            if (warp == 0) {
                float hv = sh[lane];
                float am = absmax_lane(hv);
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
                Q8Scale sc = q8_scale(am);
                int q = q8_round(hv, sc.id);
                int s = q;
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                hrec[lane] = (uint8_t)(int8_t)q;
                if (lane == 0) {
                    hrec[32] = (uint8_t)(sc.dh & 0xff);
                    hrec[33] = (uint8_t)(sc.dh >> 8);
                    hrec[34] = (uint8_t)(s & 0xff);
                    hrec[35] = (uint8_t)((s >> 8) & 0xff);
                }
                __syncwarp();
                if (lane < 6) {
                    unsigned long long wv = tag << 48;
#pragma unroll
                    for (int t = 0; t < 6; t++) wv |= (unsigned long long)hrec[lane * 6 + t] << (8 * t);
                    unsigned long long* dst = P.hqt + (((size_t)l * k + j) * nbI + c) * 6 + lane;
                    st_relaxed_u64(dst, wv);
                }
                if (P.h_dbg && lane < 32) P.h_dbg[((size_t)layer * k + j) * g.I + c * 32 + lane] = hv;
            }
            __syncthreads();
        }

        // ------------------------------------------------------------ D: down rows + combine + next routing
        if (n_d > 0) {
            // gather all k * nbI h blocks (tagged words) into shared memory
            const int nwords = k * nbI * 6;
            {
                unsigned long long t0 = gtime();
                int spins = 0;
                while (true) {
                    int ok = 1;
                    for (int w = tid; w < nwords; w += NT) {
                        unsigned long long v = ld_relaxed_u64(P.hqt + (size_t)l * nwords + w);
                        if ((v >> 48) != tag) {
                            ok = 0;
                            flags[2] = (l << 20) | ((w / 6) & 0xfff) << 8 | (int)((v >> 48) & 0xff);
                        } else {
                            uint8_t* r = rec + (size_t)(w / 6) * 36 + (w % 6) * 6;
#pragma unroll
                            for (int t = 0; t < 6; t++) r[t] = (uint8_t)(v >> (8 * t));
                        }
                    }
                    if (__syncthreads_and(ok)) break;
                    if (tid == 0 && ((++spins & 63) == 0) && (gtime() - t0 > WAIT_NS || error_seen())) fail(4);
                    __syncthreads();
                    if (flags[0]) goto drain;
                }
            }
            // records -> activation form: codes, fp32 scale, 8*sum
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
            {
                unsigned long long t0 = gtime();
                int spins = 0;
                while (!mbar_try_wait(mbar_d, (unsigned)l & 1u)) {
                    if ((++spins & 255) == 0 && gtime() - t0 > WAIT_NS) {
                        if (lane == 0) fail(5);
                        break;
                    }
                }
            }
            __syncthreads();
            if (flags[0]) goto drain;
            if (tid == 0) pending_d = false;
            const uint8_t* dbase = arena + (size_t)n_gu * 2 * gu_unit_bytes;
            float* xout = (l + 1 == P.nL) ? P.x_out : P.xbuf + (size_t)(l + 1) * g.H;
            for (int q = warp; q < nrows; q += NW) {
                const int i = q / RD, rr = q - i * RD;
                const int r = d_units[i] * RD + rr;
                float a = 0.0f;
                for (int j = 0; j < k; j++) {
                    const uint8_t* row = dbase + ((size_t)i * k + j) * d_chunk + (size_t)rr * g.row_d;
                    ActView ha = act_view(hq_base + (size_t)j * ab_i, nbI);
                    float acc = 0.0f;
                    for (int b = lane; b < nbI; b += 32) {
                        uint4 wv = *reinterpret_cast<const uint4*>(row + 16 * b);
                        float dw = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(row + 16 * nbI + 2 * b));
                        XBlk xb = load_xblk_s(ha, b);
                        acc = __fadd_rn(acc, block_term(block_sumi(wv, xb), dw, xb.d));
                    }
                    float y = warp_sum_butterfly(acc);
                    a = __fadd_rn(a, __fmul_rn(sw[j], y));
                }
                if (lane == 0) {
                    float xn = __fadd_rn(xs[r], a);
                    xout[r] = xn;
                    xnext[q] = xn;
                    if (l + 1 < P.nL) xw[q] = __fmul_rn(xn, __ldg(P.normw + (size_t)(layer + 1) * g.H + r));
                }
            }
            __threadfence();
            __syncthreads();
        }
        if (l + 1 < P.nL) {
            unsigned long long* accn = P.acc + (size_t)(l + 1) * (E + 1);
            for (int e = tid; e <= E; e += NT) {
                long long s = 0;
                if (e < E)
                    for (int q = 0; q < nrows; q++) s += router_fixed(rt[(size_t)q * E + e], xw[q]);
                else
                    for (int q = 0; q < nrows; q++) s += ss_fixed(xnext[q]);
                red_add_release_u64(accn + e, CNT_UNIT + (unsigned long long)s);
            }
        }
        __syncthreads();
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
    if (tid == 0) {
        unsigned long long t0 = gtime();
        for (int u = 0; u < FUSED_MAX_GU; u++)
            if (pending_gu >> u & 1u)
                while (!mbar_try_wait(mbar_gu + u, (unsigned)cur_l & 1u) && gtime() - t0 < WAIT_NS) {
                }
        if (pending_d)
            while (!mbar_try_wait(mbar_d, (unsigned)cur_l & 1u) && gtime() - t0 < WAIT_NS) {
            }
        if (pending_rt0)
            while (!mbar_try_wait(mbar_rt0, 0) && gtime() - t0 < WAIT_NS) {
            }
    }
    __syncthreads();
}

// ---------------------------------------------------------------- host side

int fused_plan(const Geom& g, int E, int k, int G, int rd, std::vector<uint16_t>& plan, size_t& arena_bytes,
               int& plan_stride) {
    if (g.H % rd != 0 || k > 16 || E > 1024) return -1;
    const int n_gu_units = k * g.nbI;
    const int n_d_units = g.H / rd;
    const size_t gu_b = 2 * 32 * g.row_gu;
    const size_t d_b = (size_t)k * rd * g.row_d;
    const size_t rt_b = (size_t)rd * E * 4;
    std::vector<size_t> load(G, 0), arena(G, 0);
    std::vector<std::vector<int>> gu(G), dd(G);
    auto argmin = [&]() {
        int best = 0;
        for (int c = 1; c < G; c++)
            if (load[c] < load[best]) best = c;
        return best;
    };
    for (int u = 0; u < n_gu_units; u++) {
        int c = argmin();
        gu[c].push_back(u);
        load[c] += gu_b;
        arena[c] += gu_b;
    }
    for (int t = 0; t < n_d_units; t++) {
        int c = argmin();
        dd[c].push_back(t);
        load[c] += d_b + rt_b;
        arena[c] += d_b;
    }
    plan_stride = 2 + FUSED_MAX_GU + FUSED_MAX_D;
    plan.assign((size_t)G * plan_stride, 0);
    arena_bytes = 0;
    for (int c = 0; c < G; c++) {
        if ((int)gu[c].size() > FUSED_MAX_GU || (int)dd[c].size() > FUSED_MAX_D) return -2;
        uint16_t* p = plan.data() + (size_t)c * plan_stride;
        p[0] = (uint16_t)gu[c].size();
        p[1] = (uint16_t)dd[c].size();
        for (size_t i = 0; i < gu[c].size(); i++) p[2 + i] = (uint16_t)gu[c][i];
        for (size_t i = 0; i < dd[c].size(); i++) p[2 + FUSED_MAX_GU + i] = (uint16_t)dd[c][i];
        arena_bytes = std::max(arena_bytes, arena[c]);
    }
    return 0;
}

cudaError_t fused_prepare(const FusedParams& P) {
    return cudaFuncSetAttribute(k_decode_fused, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)fused_smem_layout(P).total);
}

cudaError_t fused_occupancy(const FusedParams& P, int* blocks_per_sm) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, k_decode_fused, NT,
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
    return cudaLaunchKernelEx(&cfg, k_decode_fused, P);
}

}  // namespace tg

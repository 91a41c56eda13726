// tg_decode.cu — the fused decode step: every MoE layer of one token in ONE
// persistent cooperative kernel (one CTA per SM: 16 compute warps + 1 producer warp).
//
// Per layer l (tinygiant/engine.py:229-258, attention excluded):
//   A  routing: each CTA gathers x_l (tagged words written by the row owners) and
//      the router sums R . (x * ffn_norm) and sum x^2 of all CTAs (count-tagged
//      fixed point, spread over FUSED_ACC copies) in one polling sweep, forms the
//      RMSNorm scale and the logits, and takes top-k + softmax (engine.py:229-236);
//      every CTA computes the same result.
//   B  the producer warp bulk-copies (cp.async.bulk) this CTA's gate/up units
//      (32 rows of gate + up of one chosen expert) into shared memory; the compute
//      warps quantise RMSNorm(x_l) to Q8_0 (libtinygiant.c:322-340, 61-89).
//   C  gate/up: per unit, 32 gate and 32 up row dots, h = silu(g)*u, Q8_0 of the
//      32 h values (libtinygiant.c:566-586), published as six tagged 64-bit words.
//      Once the CTA's last unit has landed, its down rows (all k experts), the next
//      layer's router columns and norm weights are copied in.
//   D  down: gather the h records (polling their tags) and compute the CTA's output
//      rows for all k experts, in two stages (early slots, then the late ones),
//      combine in slot order and add to x (libtinygiant.c:588-594, engine.py:240-258);
//      publish x_{l+1} as tagged words, and add the rows' products with the next
//      router and their squares (exact fixed point) into acc[l+1] with a count tag.
// Arithmetic is identical to the multi-kernel path and to the oracle's mirror
// order, so results are bit-identical.  No grid-wide barrier and no memory fence
// sits in the layer loop: every cross-CTA word validates itself.
//
// Every wait (mbarrier, tag poll) has a cycle limit (FusedParams::wait_cycles); on
// expiry the kernel records an error in ctl[2..3], drains its own outstanding copies
// and returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
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
// Wait limits are in SM cycles (FusedParams::wait_cycles; clock64 is a per-SM counter
// and cheap to read, unlike %globaltimer).

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
// The same, but the thread may be suspended (issuing nothing) until the phase
// completes or about hint_ns pass, so waiting warps leave the issue slots to the warps
// that compute.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
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
// system scope: words that other devices store over NVLink
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_add_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
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



// Gather the h records of slots [jlo, jlo + nwords / (6 * nbI)) of one layer (six
// tagged words each) straight into the activation form: codes, fp32 scale, 8 * sum
// of codes.  With lmap (experts sharded over devices) hw is the layer's first record
// and the records gathered are those of slots lmap[0 .. nwords / (6 * nbI)), stored
// in that order.  Each thread re-polls only its missing words.  False when the wait
// limit passed (error recorded) or another CTA reported an error.  Called from one
// place only, so the layer loop holds one copy of it.
__device__ __forceinline__ bool gather_h_records(const unsigned long long* hw, int nwords, int jlo, int nbI,
                                              uint8_t* hq_base, int ab_i, unsigned tag, unsigned* ctl, int* flags,
                                              int l, long long limit, const int* lmap = nullptr) {
    const int tid = threadIdx.x;
    unsigned mine = 0, done = 0;
    for (int i = 0; i * NT + tid < nwords; i++) mine |= 1u << i;
    // with a slot map, word w of record rec = w / 6 of local slot jl = rec / nbI lies at
    // (lmap[jl] - jl) * nbI * 6 + w; the first batch's offsets are worked out once, not
    // on every polling round
    auto source = [&](int w) -> int {
        if (!lmap || w >= nwords) return w;
        const int jl = w / (6 * nbI);
        return (lmap[jl] - jl) * nbI * 6 + w;
    };
    int src0[8];
#pragma unroll
    for (int t = 0; t < 8; t++) src0[t] = source(t * NT + tid);
    const long long t0 = clock64();
    int spins = 0;
    while (done != mine) {
#pragma unroll 1
        for (int i0 = 0; i0 * NT + tid < nwords; i0 += 8) {
            unsigned long long v[8];
#pragma unroll
            for (int t = 0; t < 8; t++) {
                const int i = i0 + t, w = i * NT + tid;
                const int src = i0 == 0 ? src0[t] : source(w);
                v[t] = (w < nwords && !(done >> i & 1u)) ? ld_relaxed_u64(hw + src) : 0ull;
            }
#pragma unroll
            for (int t = 0; t < 8; t++) {
                const int i = i0 + t, w = i * NT + tid;
                if (w >= nwords || (done >> i & 1u)) continue;
                if ((unsigned)(v[t] >> 48) != tag) continue;
                done |= 1u << i;
                const int rec = w / 6, part = w - rec * 6;
                const int jj = jlo + rec / nbI, c = rec % nbI;
                uint8_t* base = hq_base + (size_t)jj * ab_i;
                uint16_t* q16 = reinterpret_cast<uint16_t*>(base + (size_t)c * 32 + 6 * part);
                const unsigned long long pv = v[t];
                if (part < 5) {
                    q16[0] = (uint16_t)pv;
                    q16[1] = (uint16_t)(pv >> 16);
                    q16[2] = (uint16_t)(pv >> 32);
                } else {
                    q16[0] = (uint16_t)pv;   // codes 30, 31
                    reinterpret_cast<float*>(base + (size_t)nbI * 32)[c] = f16_bits_to_f32((uint16_t)(pv >> 16));
                    reinterpret_cast<int*>(base + (size_t)nbI * 36)[c] = 8 * (int)(int16_t)(uint16_t)(pv >> 32);
                }
            }
        }
        if (done == mine) break;
        if ((++spins & 63) == 0) {
            if (clock64() - t0 > limit) {
                const int i = __ffs(mine & ~done) - 1, w = i * NT + tid;
                flags[1] = (l << 20) | (((jlo * nbI + w / 6) & 0xfff) << 8);
                record_failure(ctl, flags, 4);
                return false;
            }
            if (ld_relaxed_u32(ctl + 2) != 0) return false;
        }
    }
    return true;
}

// Down values y_j of this CTA's rows for slots [jlo, jhi) into ys[j][q].  One task
// per warp: one slot and a group of at most 8 consecutive rows, enough groups per slot
// to occupy the warps.  The lanes hold the slot's h blocks b = lane, lane + 32, ... in
// registers across the group's rows (each h block is read from shared memory once per
// task, not once per row), lane partials in block order b = lane, lane + 32, ..., then
// one transposed reduction over the group's rows.  Each row's reduction is the same
// pairing tree as a butterfly over the lanes whatever the other values in the
// reduction, so the bits are the mirror order's.  Called from one place only.
// Experts sharded over devices: where the down values go besides ys (every rank's y
// buffer, this launch's half and layer), as soon as each warp has them.
struct DownPush {
    unsigned long long* const* ypeer;
    size_t ylay;        // this layer's words in every rank's buffer
    const int* lmap;    // local slot -> slot
    int d_lo, H, ep_size;
    unsigned ytag;
};

__device__ __forceinline__ void down_rows(const uint8_t* dbase, const uint8_t* hq_base, float* ys, uint32_t d_chunk,
                                          int row_d, int nbI, int ab_i, int d_n, int max_rows, int jlo, int jhi,
                                          const DownPush* push = nullptr) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ns = jhi - jlo;
    if (warp >= CW || ns <= 0 || d_n <= 0) return;
    int gps = CW / ns > 1 ? CW / ns : 1;         // row groups per slot
    int R = (d_n + gps - 1) / gps;               // rows per group
    if (R > 8) R = 8;
    gps = (d_n + R - 1) / R;
    for (int t = warp; t < ns * gps; t += CW) {
        const int js = t / gps, grp = t - js * gps, j = jlo + js;
        const int q0 = grp * R, nr = d_n - q0 < R ? d_n - q0 : R;
        const uint8_t* rows = dbase + (size_t)j * d_chunk + (size_t)q0 * row_d;
        const ActView hv = act_view(hq_base + (size_t)j * ab_i, nbI);
        float acc[8];
#pragma unroll
        for (int r = 0; r < 8; r++) acc[r] = 0.0f;
#pragma unroll 1
        for (int b = lane; b < nbI; b += 32) {
            const XBlk xb = load_xblk(hv, b);
#pragma unroll
            for (int r = 0; r < 8; r++) {
                if (r < nr) {
                    const uint8_t* row = rows + (size_t)r * row_d;
                    const uint4 w = *reinterpret_cast<const uint4*>(row + 16 * b);
                    const float dw = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(row + 16 * nbI + 2 * b));
                    acc[r] = __fadd_rn(acc[r], block_term(block_sumi(w, xb), dw, xb.d));
                }
            }
        }
        const float y = warp_sum8_transposed(acc, lane);   // row q0 + r in lanes 4r .. 4r+3
        const int r = lane >> 2;
        if ((lane & 3) == 0 && r < nr) {
            ys[(size_t)j * max_rows + q0 + r] = y;
            if (push) {
                const unsigned long long word = ((unsigned long long)push->ytag << 32) | __float_as_uint(y);
                const size_t at = push->ylay + (size_t)push->lmap[j] * push->H + push->d_lo + q0 + r;
                for (int rr = 0; rr < push->ep_size; rr++) st_relaxed_sys_u64(push->ypeer[rr] + at, word);
            }
        }
    }
}

}  // namespace

template <bool TRACE, bool EP>
__global__ void __launch_bounds__(NT, 1) k_decode_fused(FusedParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const FusedSmem S = fused_smem_layout(P);
    uint64_t* mbar_gu = reinterpret_cast<uint64_t*>(smem + S.mbar);     // [FUSED_MAX_GU]
    uint64_t* mbar_d = mbar_gu + FUSED_MAX_GU;                             // down rows + next router / norm
    uint64_t* mbar_rt0 = mbar_gu + FUSED_MAX_GU + 1;                       // first router columns + norm
    uint16_t* plan = reinterpret_cast<uint16_t*>(smem + S.plan);
    long long* slog_fx = reinterpret_cast<long long*>(smem + S.slogfx);   // [FUSED_ACC][E + 1]
    float* slog = reinterpret_cast<float*>(smem + S.slog);
    unsigned long long* skey = reinterpret_cast<unsigned long long*>(smem + S.skey);   // [E] rank keys
    int* sidx = reinterpret_cast<int*>(smem + S.sidx);
    int* lmap = reinterpret_cast<int*>(smem + S.lmap);     // EP: local slot -> slot
    int* flags = reinterpret_cast<int*>(smem + S.flags);   // [0] error seen, [1] error detail, [2] last CTA
    float* sscale = reinterpret_cast<float*>(flags + 4);   // RMSNorm scale of the current layer
    float* xs = reinterpret_cast<float*>(smem + S.xs);
    ActView xq = act_view(smem + S.xq, P.g.nbH);
    uint8_t* hq_base = smem + S.hq;
    float* sh = reinterpret_cast<float*>(smem + S.sh);      // [2][32] h of a unit, then [16] routing weights
    uint8_t* hrec = smem + S.hrec;                           // [2][64]
    float* xnext = reinterpret_cast<float*>(smem + S.xnext);  // x of the next layer, this CTA's rows
    float* xw = reinterpret_cast<float*>(smem + S.xw);        // the same rows times the next norm weight
    float* rt = reinterpret_cast<float*>(smem + S.rt);        // router columns of this CTA's rows [rows][E]
    float* snorm = reinterpret_cast<float*>(smem + S.snorm);  // [2][H]
    float* ys = reinterpret_cast<float*>(smem + S.ys);        // [k][max_rows] per-slot down values
    float* yr = reinterpret_cast<float*>(smem + S.yr);        // EP: [k][max_rows] as received
    uint8_t* arena = smem + S.arena;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, cta = blockIdx.x;
    const Geom g = P.g;
    const int E = P.E, k = P.k, nbH = g.nbH, nbI = g.nbI;
    const size_t ab_i = act_bytes(nbI);
    const uint32_t gu_unit_bytes = (uint32_t)(32 * g.row_gu);  // one of gate / up
    const uint32_t norm_bytes = (uint32_t)(4 * g.H);           // one layer's FFN norm weights
    const size_t acc_words = (size_t)FUSED_ACC * (E + 1);      // one layer's router accumulators

    if (tid < FUSED_PLAN) plan[tid] = P.plan[(size_t)cta * FUSED_PLAN + tid];
    if (tid == PT) {
        for (int i = 0; i < FUSED_MAX_GU + 2; i++) mbar_init(mbar_gu + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid < 4) flags[tid] = 0;
    cta_sync();
    // one device: the static plan; experts sharded over devices: n_gu, d_place and
    // dbase are set per layer from the slots whose expert is held here
    int n_gu = plan[0], d_place = plan[3];
    const int d_lo = plan[1], d_n = plan[2];
    const uint16_t* gu_units = plan + 4;
    const uint32_t d_chunk = (uint32_t)d_n * (uint32_t)g.row_d;   // this CTA's rows of one expert's down
    const uint32_t rt_bytes = (uint32_t)d_n * (uint32_t)E * 4u;  // their router columns
    // down rows: in unit 0's space once it is computed (placement 1), else after the units
    uint8_t* dbase = arena + (d_place ? (size_t)0 : (size_t)n_gu * 2 * gu_unit_bytes);
    const unsigned epoch = ld_relaxed_u32(P.ctl);
    const unsigned tag = epoch % 65535u + 1u;   // 1..65535; the tagged buffers are cleared before it repeats
    // EP: the y words carry the full launch count (never cleared; every rank launches
    // the same sequence) and alternate buffer halves by launch parity, so a rank one
    // launch ahead never overwrites a word another rank has still to read.  Every launch
    // rewrites every word of its half (each slot has one owner, which stores all rows), so
    // a half holds the tag of two launches before, never the initial 0: the 32-bit tag may
    // wrap.
    const unsigned ytag = epoch + 1u;
    int nloc = k;   // EP: slots whose expert is held here this layer
    // gate/up unit u of this CTA (slot * nbI + 32-row chunk): the static plan's, or with
    // experts sharded, unit cta + u * G of the local slots in slot order (the same
    // assignment the plan's greedy makes, u mod G, over nloc * nbI units)
    auto unit_of = [&](int u) -> int {
        if (!EP) return gu_units[u];
        const int U = cta + u * G, jl = U / nbI;
        return lmap[jl] * nbI + (U - jl * nbI);
    };
    auto expert_of = [&](int j) -> int { return EP ? sidx[j] - P.e_lo : sidx[j]; };
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();

    // Producer-lane bookkeeping of armed, not yet waited mbarriers (for the error
    // path).  Every mbarrier completes at most once per layer, so the parity to
    // wait for in layer l is l & 1 (0 for the one-off first router copy).
    unsigned pending = 0;  // bits 0..3: gate/up units, bit 4: down group, bit 5: first router copy
    int cur_l = 0;
    // phase parity of each gate/up unit's mbarrier (bit u), flipped every layer the unit
    // is used: with experts sharded over devices a CTA's unit count changes per layer,
    // so a unit's mbarrier does not complete once in every layer
    unsigned gu_par = 0;

    auto fail = [&](unsigned code) { record_failure(P.ctl, flags, code); };
    auto error_seen = [&]() -> bool { return ld_relaxed_u32(P.ctl + 2) != 0; };
    // trace stamp: %globaltimer (ns) for cross-SM alignment and clock64 for cycles
    auto stamp = [&](int l, int slot) {
        if (TRACE) {
            const unsigned long long t = gtime();
            const long long c1 = clock64();
            unsigned long long* row = P.trace + ((size_t)l * G + cta) * FUSED_TRACE;
            row[slot] = t;
            row[16 + slot] = (unsigned long long)c1;
        }
    };
    // bounded wait on an mbarrier phase by the calling thread; false (and an error
    // recorded) when the limit passes
    auto wait_bar = [&](uint64_t* bar, unsigned parity, unsigned code) -> bool {
        const long long t0 = clock64();
        while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
            if (clock64() - t0 > P.wait_cycles) {
                fail(code);
                return false;
            }
        }
        return true;
    };
    // Copies are cut into pieces of at most 16 KB (16-byte multiples), except the
    // gate / up halves, which go as one copy each (fewer copies issue faster); lane i
    // of the producer warp issues pieces i, i + 32, ..., so one warp instruction
    // starts up to 32 copies.
    auto pieces_of = [](uint32_t bytes) -> int { return (int)((bytes + 16383u) / 16384u); };
    auto piece_span = [](uint32_t bytes, int np, int p, uint32_t& off, uint32_t& n) {
        const uint32_t ps = ((bytes + np - 1) / np + 15u) & ~15u;
        off = (uint32_t)p * ps;
        n = off >= bytes ? 0u : (bytes - off < ps ? bytes - off : ps);
    };
    // producer warp: the gate and up halves of this CTA's units, one mbarrier per unit
    auto issue_gateup = [&](const uint8_t* lbase) {
        for (int pi = lane; pi < 2 * n_gu; pi += 32) {
            const int u = pi >> 1, half = pi & 1;
            const int unit = unit_of(u);
            const int j = unit / nbI, c = unit - j * nbI;
            const uint8_t* src = lbase + (size_t)expert_of(j) * g.expert_bytes + (half ? g.t_gu : 0) +
                                 (size_t)c * gu_unit_bytes;
            bulk_g2s(arena + ((size_t)u * 2 + half) * gu_unit_bytes, src, gu_unit_bytes, mbar_gu + u, pol_stream);
        }
    };
    // producer warp: this layer's down rows of all k experts (EP: of the nloc local
    // slots, in local order), plus the next layer's router columns and norm weights,
    // all on mbar_d
    auto issue_down = [&](int l, int layer, const uint8_t* lbase, bool next) {
        if (!(d_n > 0 || next)) return;
        const int ns = EP ? nloc : k;
        const uint32_t total = (uint32_t)ns * d_chunk + (next ? rt_bytes + norm_bytes : 0u);
        if (lane == 0) {
            mbar_arrive_expect_tx(mbar_d, total);
            pending |= 1u << 4;
        }
        __syncwarp();
        const int npd = d_n > 0 ? pieces_of(d_chunk) : 0;
        const int npr = (next && d_n > 0) ? pieces_of(rt_bytes) : 0;
        const int npn = next ? pieces_of(norm_bytes) : 0;
        const int nd = ns * npd;
        for (int pi = lane; pi < nd + npr + npn; pi += 32) {
            uint32_t off, n;
            const uint8_t* src;
            uint8_t* dst;
            uint64_t pol;
            if (pi < nd) {
                const int j = pi / npd, p = pi - j * npd;   // EP: j is the local slot
                piece_span(d_chunk, npd, p, off, n);
                src = lbase + (size_t)expert_of(EP ? lmap[j] : j) * g.expert_bytes + 2 * g.t_gu +
                      (size_t)d_lo * g.row_d + off;
                dst = dbase + (size_t)j * d_chunk + off;
                pol = pol_stream;
            } else if (pi < nd + npr) {
                piece_span(rt_bytes, npr, pi - nd, off, n);
                src = reinterpret_cast<const uint8_t*>(P.RT + ((size_t)(layer + 1) * g.H + d_lo) * E) + off;
                dst = reinterpret_cast<uint8_t*>(rt) + off;
                pol = pol_keep;
            } else {
                piece_span(norm_bytes, npn, pi - nd - npr, off, n);
                src = reinterpret_cast<const uint8_t*>(P.normw + (size_t)(layer + 1) * g.H) + off;
                dst = reinterpret_cast<uint8_t*>(snorm + (size_t)((l + 1) & 1) * g.H) + off;
                pol = pol_keep;
            }
            if (n) bulk_g2s(dst, src, n, mbar_d, pol);
        }
        __syncwarp();
    };
    // this CTA's rows' share of the next layer's router sums and sum of x^2, added with
    // a count tag into copy cta % FUSED_ACC: four threads per entry, exact int64 sums
    auto router_partials = [&](unsigned long long* accn) {
        accn += (size_t)(cta % FUSED_ACC) * (E + 1);
        for (int i0 = 0; i0 < 4 * (E + 1); i0 += NT) {
            const int i = i0 + tid, e = i >> 2, part = i & 3;
            long long s = 0;
            if (e < E) {
#pragma unroll 1
                for (int q = part; q < d_n; q += 4) s += router_fixed(rt[(size_t)q * E + e], xw[q]);
            } else if (e == E) {
#pragma unroll 1
                for (int q = part; q < d_n; q += 4) s += ss_fixed(xnext[q]);
            }
            __syncwarp();
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if (e <= E && part == 0) red_add_relaxed_u64(accn + e, CNT_UNIT + (unsigned long long)s);
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
    if (!cta_sync_and(wait_bar(mbar_rt0, 0, 1))) goto drain;
    if (tid == PT) pending &= ~(1u << 5);
    #pragma unroll 1
    for (int q = tid; q < d_n; q += NT) xw[q] = __fmul_rn(xnext[q], snorm[d_lo + q]);
    cta_sync();
    router_partials(P.acc);   // x_in is complete before the launch

    for (int l = 0; l < P.nL; l++) {
        const int layer = P.L0 + l;
        cur_l = l;
        unsigned long long* accl = P.acc + (size_t)l * acc_words;
        const bool next = l + 1 < P.nL;
        // one device: the unit count is static, so the arena fence and the units' mbarrier
        // arming come before the routing, off the path from top-k to the copies
        if (!EP && tid == PT) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            for (int u = 0; u < n_gu; u++) mbar_arrive_expect_tx(mbar_gu + u, 2 * gu_unit_bytes);
        }
        const uint8_t* lbase = P.weights + (size_t)layer * P.layer_bytes;
        // ------------------------------------------------------------ A: routing sums and x_l
        // Every word is validated on its own: x_l values carry the launch tag (x_in
        // needs none), router sums carry a count of contributing CTAs, so no fence is
        // needed.  Each thread re-polls only its missing words until all are in (or the
        // wait limit passes); one barrier ends the phase.
        {
            const int nwords = g.H + (int)acc_words;
            const unsigned long long* xl = P.xw + (size_t)l * g.H;
            unsigned mine = 0, done = 0;   // words tid + i * NT of this thread, and those taken
            for (int i = 0; i * NT + tid < nwords; i++) mine |= 1u << i;
            const long long t0 = clock64();
            int spins = 0;
            bool ok = true;
            while (done != mine) {
#pragma unroll 1
                for (int i0 = 0; i0 * NT + tid < nwords; i0 += 8) {
                    unsigned long long v[8];
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        const int i = i0 + t, w = i * NT + tid;
                        v[t] = 0ull;
                        if (w < nwords && !(done >> i & 1u)) {
                            if (w >= g.H)
                                v[t] = ld_relaxed_u64(accl + (w - g.H));
                            else if (l == 0)
                                v[t] = ((unsigned long long)tag << 32) | __float_as_uint(__ldcg(P.x_in + w));
                            else
                                v[t] = ld_relaxed_u64(xl + w);
                        }
                    }
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        const int i = i0 + t, w = i * NT + tid;
                        if (w >= nwords || (done >> i & 1u)) continue;
                        if (w < g.H) {
                            if ((unsigned)(v[t] >> 32) == tag) {
                                xs[w] = __uint_as_float((unsigned)v[t]);
                                done |= 1u << i;
                            }
                        } else {
                            // copy a holds the CTAs c with c % FUSED_ACC == a
                            const int a = (w - g.H) / (E + 1);
                            const unsigned long long want =
                                (unsigned long long)((G - a + FUSED_ACC - 1) / FUSED_ACC + (a == 0 ? P.missing : 0));
                            const unsigned long long cnt = (v[t] + (1ull << 55)) >> 56;
                            if (cnt == want) {
                                slog_fx[w - g.H] = (long long)(v[t] - want * CNT_UNIT);
                                done |= 1u << i;
                            }
                        }
                    }
                }
                if (done == mine) break;
                if ((++spins & 63) == 0) {
                    if (clock64() - t0 > P.wait_cycles) {
                        const int i = __ffs(mine & ~done) - 1, w = i * NT + tid;
                        flags[1] = (l << 20) | (((w < g.H ? w : w - g.H) & 0xfff) << 8) | (w < g.H ? 0xff : 0xfe);
                        fail(2);
                        ok = false;
                        break;
                    }
                    if (error_seen()) {
                        ok = false;
                        break;
                    }
                }
            }
            if (!cta_sync_and(ok)) goto drain;
        }
        if (tid == 0) stamp(l, 0);
        // logits of the normed input: scale * (R . (x * w)), scale = 1/sqrt(ss/H + eps);
        // each sum is the exact int64 total of the accumulator copies
        {
            auto total = [&](int e) {
                long long t = 0;
#pragma unroll
                for (int a = 0; a < FUSED_ACC; a++) t += slog_fx[(size_t)a * (E + 1) + e];
                return t;
            };
            const float scale = rms_scale_from(total(E), g.H, P.eps);
#pragma unroll 1
            for (int e = tid; e < E; e += NT) {
                // +0 for a zero logit, so equal logits get equal keys
                const float lg = __fadd_rn(__fmul_rn(scale, router_logit(total(e))), 0.0f);
                slog[e] = lg;
                // rank key: order-preserving bits of the logit, then the expert id, so
                // key_j > key_e exactly when l_j > l_e or (l_j == l_e and j > e)
                const unsigned b = __float_as_uint(lg);
                const unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
                skey[e] = ((unsigned long long)ord << 32) | (unsigned)e;
            }
            if (tid == 0) *sscale = scale;
            // every CTA has contributed to acc[l], so acc[l-1] is read by no one: recycle it
            if (cta == 0 && l >= 1)
                for (size_t i = tid; i < acc_words; i += NT) accl[i - acc_words] = 0ull;
        }
        cta_sync();
        // top-k by rank: 4 threads per expert share the scan, two keys per 16-byte
        // load (the four parts read neighbouring banks); the element beaten by fewer
        // than k others (larger logit, or equal logit and larger id) is kept
        for (int base = 0; base < E; base += NT / 4) {
            const int e = base + (tid >> 2), part = tid & 3;
            int rank = 0;
            if (e < E) {
                const unsigned long long ke = skey[e];
                const ulonglong2* kp = reinterpret_cast<const ulonglong2*>(skey);
#pragma unroll 4
                for (int j2 = part; 2 * j2 < E; j2 += 4) {
                    const ulonglong2 kk = kp[j2];
                    rank += (kk.x > ke) + (kk.y > ke);
                }
            }
            __syncwarp();
            rank += __shfl_xor_sync(0xffffffffu, rank, 1);
            rank += __shfl_xor_sync(0xffffffffu, rank, 2);
            if (e < E && part == 0 && rank < k) sidx[k - 1 - rank] = e;
        }
        cta_sync();
        if (tid == 0) stamp(l, 9);
        if (EP) {
            // the slots whose expert is held here, this CTA's share of their gate/up units
            // (units cta, cta + G, ... of nloc * nbI) and where its down rows go
            unsigned lmask = 0;
            for (int j = 0; j < k; j++)
                if ((unsigned)(sidx[j] - P.e_lo) < (unsigned)P.e_n) lmask |= 1u << j;
            nloc = __popc(lmask);
            const int nu = nloc * nbI;
            n_gu = cta < nu ? (nu - 1 - cta) / G + 1 : 0;
            d_place = (n_gu > 0 && (size_t)n_gu * 2 * gu_unit_bytes + (size_t)nloc * d_chunk > P.arena_bytes) ? 1 : 0;
            dbase = arena + (d_place ? (size_t)0 : (size_t)n_gu * 2 * gu_unit_bytes);
            // the producer warp writes the slot map; the compute warps read it after the
            // next barrier
            if (warp == CW) {
                if (lane < k && (lmask >> lane & 1u)) lmap[__popc(lmask & ((1u << lane) - 1u))] = lane;
                __syncwarp();
            }
        }

        // ------------------------------------------------------------ B: copies, softmax, x quantise
        if (warp == CW) {
            // producer warp: gate/up units now; the down rows once unit 0 is computed
            // (placement 1) or this CTA's last unit has landed (placement 0), so gate/up
            // bytes go first
            if (lane == 0) {
                // the regions below were read by this CTA's threads in the previous layer
                if (EP) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    for (int u = 0; u < n_gu; u++) mbar_arrive_expect_tx(mbar_gu + u, 2 * gu_unit_bytes);
                }
                pending |= (1u << n_gu) - 1u;
            }
            __syncwarp();
            issue_gateup(lbase);
            __syncwarp();
            if (lane == 0) stamp(l, 1);
            if (n_gu == 0) {
                issue_down(l, layer, lbase, next);
                if (lane == 0) stamp(l, 10);
            }
        } else {
            // softmax over the k chosen logits (engine.py:233-236), held by lane j of
            // every compute warp: w_j = exp(l_j - max) / sum, sum for k <= 8 as
            // ((e0+e1)+(e2+e3))+((e4+e5)+(e6+e7))
            const float m = slog[sidx[k - 1]];
            const float ex = lane < k ? tg_expf(__fsub_rn(slog[sidx[lane < k ? lane : 0]], m)) : 0.0f;
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
            const float wl = lane < k ? __fdiv_rn(ex, s) : 0.0f;
            if (cta == 0) {
                if (warp == 0 && lane < k) {
                    P.idx_out[(size_t)layer * k + lane] = sidx[lane];
                    P.w_out[(size_t)layer * k + lane] = wl;
                }
                for (int e = tid; e < E; e += CT) P.logits_out[(size_t)layer * E + e] = slog[e];
            }
            if (warp == 0 && lane < 16) sh[64 + lane] = wl;   // the routing weights, for the combine
            // Q8_0 of RMSNorm(x_l) * w (libtinygiant.c:336-339, 61-89): four blocks per
            // warp at a time, eight lanes per block, four values per lane
            const float scale = *sscale;
            const float* nw = snorm + (size_t)(l & 1) * g.H;
            for (int b0 = warp * 4; b0 < nbH; b0 += CW * 4) {
                const int b = b0 + (lane >> 3), sub = lane & 7;
                const float4 xv = reinterpret_cast<const float4*>(xs)[b * 8 + sub];
                const float4 wv = reinterpret_cast<const float4*>(nw)[b * 8 + sub];
                const float v0 = __fmul_rn(__fmul_rn(xv.x, scale), wv.x);
                const float v1 = __fmul_rn(__fmul_rn(xv.y, scale), wv.y);
                const float v2 = __fmul_rn(__fmul_rn(xv.z, scale), wv.z);
                const float v3 = __fmul_rn(__fmul_rn(xv.w, scale), wv.w);
                float am = fmaxf(fmaxf(absmax_lane(v0), absmax_lane(v1)), fmaxf(absmax_lane(v2), absmax_lane(v3)));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
                const Q8Scale sc = q8_scale(am);
                const int q0 = q8_round(v0, sc.id), q1 = q8_round(v1, sc.id);
                const int q2 = q8_round(v2, sc.id), q3 = q8_round(v3, sc.id);
                reinterpret_cast<uint32_t*>(xq.qs)[b * 8 + sub] =
                    (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
                    ((uint32_t)(q3 & 0xff) << 24);
                int qs = q0 + q1 + q2 + q3;
                qs += __shfl_xor_sync(0xffffffffu, qs, 4);
                qs += __shfl_xor_sync(0xffffffffu, qs, 2);
                qs += __shfl_xor_sync(0xffffffffu, qs, 1);
                if (sub == 0) {
                    xq.d[b] = f16_bits_to_f32(sc.dh);
                    xq.s8[b] = 8 * qs;
                }
            }
        }
        cta_sync();
        if (tid == 0) stamp(l, 2);

        // ------------------------------------------------------------ C: gate/up units
        // x blocks lane and lane + 32 stay in registers for all units when H <= 2048
        const bool xreg = nbH <= 64;
        XBlk xr0 = {}, xr1 = {};
        if (xreg && warp < CW) {
            if (lane < nbH) xr0 = load_xblk(xq, lane);
            if (lane + 32 < nbH) xr1 = load_xblk(xq, lane + 32);
        }
        for (int u = 0; u < n_gu; u++) {
            const bool ok = wait_bar(mbar_gu + u, gu_par >> u & 1u, 3);
            if (u == 0 && tid == 0) stamp(l, 8);
            const int unit = unit_of(u);
            const int j = unit / nbI, c = unit - j * nbI;
            float* shu = sh + (u & 1) * 32;
            if (warp == CW) {
                if (lane == 0) pending &= ~(1u << u);
                if (__all_sync(0xffffffffu, ok) && u == n_gu - 1 && !d_place) {
                    issue_down(l, layer, lbase, next);
                    if (lane == 0) stamp(l, 10);
                }
            } else if (ok) {
                const uint8_t* gate = arena + (size_t)u * 2 * gu_unit_bytes;
                const uint8_t* up = gate + gu_unit_bytes;
                const int r0 = warp * 2;   // two h rows per compute warp (CW * 2 == 32)
                const uint8_t* rg0 = gate + (size_t)r0 * g.row_gu;
                const uint8_t* rg1 = rg0 + g.row_gu;
                const uint8_t* ru0 = up + (size_t)r0 * g.row_gu;
                const uint8_t* ru1 = ru0 + g.row_gu;
                float ag0 = 0.f, ag1 = 0.f, au0 = 0.f, au1 = 0.f;
                // lane partials in block order b = lane, lane + 32, ... (the mirror order); x
                // from registers for the first two blocks of each lane when they are held there
#pragma unroll 1
                for (int it = 0; lane + 32 * it < nbH; it++) {
                    const int b = lane + 32 * it;
                    const XBlk xb = (xreg && it < 2) ? (it ? xr1 : xr0) : load_xblk(xq, b);
                    const uint4 wg0 = *reinterpret_cast<const uint4*>(rg0 + 16 * b);
                    const uint4 wg1 = *reinterpret_cast<const uint4*>(rg1 + 16 * b);
                    const uint4 wu0 = *reinterpret_cast<const uint4*>(ru0 + 16 * b);
                    const uint4 wu1 = *reinterpret_cast<const uint4*>(ru1 + 16 * b);
                    const float dg0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rg0 + 16 * nbH + 2 * b));
                    const float dg1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rg1 + 16 * nbH + 2 * b));
                    const float du0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ru0 + 16 * nbH + 2 * b));
                    const float du1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ru1 + 16 * nbH + 2 * b));
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
            if (!cta_sync_and(ok)) goto drain;
            // placement 1: the down rows go into unit 0's space, free from here on
            if (u == 0 && d_place && warp == CW) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_down(l, layer, lbase, next);
                if (lane == 0) stamp(l, 10);
            }
            // one warp (rotating) turns the 32 h values into a Q8_0 record and publishes
            // it as six tagged words; the others go on with the next unit
            if (warp == u % CW) {
                uint8_t* hr = hrec + (u & 1) * 64;
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
                    unsigned long long wv = (unsigned long long)tag << 48;
#pragma unroll
                    for (int t = 0; t < 6; t++) wv |= (unsigned long long)hr[lane * 6 + t] << (8 * t);
                    st_relaxed_u64(P.hqt + (((size_t)l * k + j) * nbI + c) * 6 + lane, wv);
                }
            }
            // the next unit writes the other sh / hrec buffer; the one after it is
            // ordered behind this publish by the next unit's barrier
        }
        gu_par ^= (1u << n_gu) - 1u;   // every unit used this layer has completed one phase
        if (tid == 0) stamp(l, 3);

        // ------------------------------------------------------------ D: down rows + combine + next routing
        // Two stages: slots [0, ke) were computed as the first gate/up unit of their
        // CTAs, so their h is complete early and their down values are computed while
        // the late units still stream; then slots [ke, k).  Per row and slot, y_j is the
        // mirror-order dot; the combine a = a + w_j * y_j runs in slot order at the end
        // (engine.py:240-258).
        const int ke = (P.k_early > 0 && P.k_early < k) ? P.k_early : k;
        const unsigned long long* hwl = P.hqt + (size_t)l * k * nbI * 6;
        auto gather_h = [&](int jlo, int jhi) -> bool {
            return gather_h_records(hwl + (size_t)jlo * nbI * 6, (jhi - jlo) * nbI * 6, jlo, nbI, hq_base, (int)ab_i,
                                    tag, P.ctl, flags, l, P.wait_cycles);
        };
        auto down_partial = [&](int jlo, int jhi) {
            down_rows(dbase, hq_base, ys, d_chunk, g.row_d, nbI, (int)ab_i, d_n, P.max_rows, jlo, jhi);
        };
        if (EP) {
            // the local slots' h records, down rows and per-slot down values, stored into
            // every rank's y buffer; then this CTA's rows of all k slots from its own
            const size_t ylay = ((size_t)(epoch & 1u) * P.Lmax + l) * k * g.H;
            if (d_n > 0 && nloc > 0) {
                if (!cta_sync_and(gather_h_records(hwl, nloc * nbI * 6, 0, nbI, hq_base, (int)ab_i, tag, P.ctl, flags,
                                                   l, P.wait_cycles, lmap)))
                    goto drain;
            }
            if (tid == 0) stamp(l, 4);
            if (!cta_sync_and(!(d_n > 0 || next) || wait_bar(mbar_d, (unsigned)l & 1u, 5))) goto drain;
            if (tid == PT) pending &= ~(1u << 4);
            if (tid == 0) stamp(l, 5);
            // each warp stores its rows' values into every rank's y buffer as it ends
            if (d_n > 0 && nloc > 0) {
                const DownPush push{P.ypeer, ylay, lmap, d_lo, g.H, P.ep_size, ytag};
                down_rows(dbase, hq_base, ys, d_chunk, g.row_d, nbI, (int)ab_i, d_n, P.max_rows, 0, nloc, &push);
            }
            if (tid == 0) stamp(l, 12);
            if (d_n > 0) {
                const unsigned long long* yown = P.ypeer[P.ep_rank] + ylay;
                const int npw = k * d_n;   // <= 16 * 64 words: at most 2 per thread
                unsigned mine = 0, done = 0;
                for (int i = 0; i * NT + tid < npw; i++) mine |= 1u << i;
                const long long t0 = clock64();
                int spins = 0;
                bool ok = true;
                while (done != mine) {
                    for (int i = 0; i * NT + tid < npw; i++) {
                        if (done >> i & 1u) continue;
                        const int w = i * NT + tid, j = w / d_n, q = w - j * d_n;
                        const unsigned long long v = ld_relaxed_sys_u64(yown + (size_t)j * g.H + d_lo + q);
                        if ((unsigned)(v >> 32) == ytag) {
                            yr[(size_t)j * P.max_rows + q] = __uint_as_float((unsigned)v);
                            done |= 1u << i;
                        }
                    }
                    if (done == mine) break;
                    if ((++spins & 63) == 0) {
                        if (clock64() - t0 > P.wait_cycles) {
                            const int w = (__ffs(mine & ~done) - 1) * NT + tid;
                            flags[1] = (l << 20) | (((w / d_n) & 0xfff) << 8) | 0xfd;
                            fail(6);
                            ok = false;
                            break;
                        }
                        if (error_seen()) {
                            ok = false;
                            break;
                        }
                    }
                }
                if (!cta_sync_and(ok)) goto drain;
            }
            if (tid == 0) stamp(l, 13);
        }
        // stage 0: slots [0, ke); stage 1: slots [ke, k) (empty when ke == k)
        for (int stage = 0; stage < (EP ? 0 : 2); stage++) {
            const int jlo = stage ? ke : 0, jhi = stage ? k : ke;
            if (jlo >= jhi) continue;
            if (d_n > 0) {
                if (!cta_sync_and(gather_h(jlo, jhi))) goto drain;
            }
            if (tid == 0) stamp(l, stage ? 11 : 4);
            if (stage == 0) {
                if (!cta_sync_and(!(d_n > 0 || next) || wait_bar(mbar_d, (unsigned)l & 1u, 5))) goto drain;
                if (tid == PT) pending &= ~(1u << 4);
                if (tid == 0) stamp(l, 5);
            }
            if (d_n > 0) down_partial(jlo, jhi);
        }
        if (d_n > 0) {
            cta_sync();
            // combine in slot order and the residual: x_{l+1} = x_l + sum_j w_j * y_j
            const float* nw1 = snorm + (size_t)((l + 1) & 1) * g.H;
            const float* yv = EP ? yr : ys;
            for (int q = tid; q < d_n; q += NT) {
                float a = 0.0f;
#pragma unroll 1
                for (int j = 0; j < k; j++) a = __fadd_rn(a, __fmul_rn(sh[64 + j], yv[(size_t)j * P.max_rows + q]));
                const int r = d_lo + q;
                const float xn = __fadd_rn(xs[r], a);
                if (next) {
                    st_relaxed_u64(P.xw + (size_t)(l + 1) * g.H + r, ((unsigned long long)tag << 32) | __float_as_uint(xn));
                    xnext[q] = xn;
                    xw[q] = __fmul_rn(xn, nw1[r]);
                } else {
                    P.x_out[r] = xn;
                }
            }
        }
        cta_sync();
        if (tid == 0) stamp(l, 6);
        if (next) router_partials(P.acc + (size_t)(l + 1) * acc_words);
        if (tid == 0) stamp(l, 7);
    }

    // ---------------------------------------------------------------- finish
    // The last CTA to finish recycles the last layer's sums, clears the tagged
    // buffers before their 16-bit tag can repeat, and advances the epoch.
    cta_sync();
    if (tid == 0) {
        __threadfence();
        const unsigned t = atomicAdd(P.ctl + 1, 1u);
        flags[2] = t == (unsigned)G - 1;
    }
    cta_sync();
    if (flags[2]) {
        __threadfence();
        unsigned long long* last = P.acc + (size_t)(P.nL - 1) * acc_words;
        for (size_t i = tid; i < acc_words; i += NT) last[i] = 0ull;
        if (tag == 65535u) {
            const size_t nh = (size_t)P.Lmax * k * nbI * 6, nx = (size_t)(P.Lmax + 1) * g.H;
            for (size_t i = tid; i < nh; i += NT) P.hqt[i] = 0ull;
            for (size_t i = tid; i < nx; i += NT) P.xw[i] = 0ull;
        }
        cta_sync();
        if (tid == 0) {
            __threadfence();
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
                while (!mbar_try_wait(mbar_gu + u, gu_par >> u & 1u) && clock64() - t0 < P.wait_cycles) {
                }
        if (pending >> 4 & 1u)
            while (!mbar_try_wait(mbar_d, (unsigned)cur_l & 1u) && clock64() - t0 < P.wait_cycles) {
            }
        if (pending >> 5 & 1u)
            while (!mbar_try_wait(mbar_rt0, 0) && clock64() - t0 < P.wait_cycles) {
            }
    }
    cta_sync();
}

// ---------------------------------------------------------------- host side

int fused_plan(const Geom& g, int E, int k, int G, std::vector<uint16_t>& plan, size_t& arena_bytes,
               int& max_rows, int& k_early) {
    if (k > 16 || E > 1024 || G <= 0) return -1;
    const int n_gu_units = k * g.nbI;
    const size_t gu_b = 2 * 32 * g.row_gu;
    std::vector<int> n_of(G, 0);
    std::vector<std::vector<int>> gu(G);
    for (int u = 0; u < n_gu_units; u++) {
        int best = 0;
        for (int c = 1; c < G; c++)
            if (n_of[c] < n_of[best]) best = c;
        gu[best].push_back(u);
        n_of[best]++;
    }
    std::vector<int> rows(G, g.H / G), order(G);
    for (int c = 0; c < G; c++) order[c] = c;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return n_of[a] < n_of[b]; });
    for (int i = 0; i < g.H % G; i++) rows[order[i]]++;
    plan.assign((size_t)G * FUSED_PLAN, 0);
    arena_bytes = 0;
    // the arena the units alone need; down rows that fit beside a CTA's units within it
    // go there (placement 0: copied as soon as the CTA's last unit has landed), the
    // others into the first unit's space once it is computed (placement 1)
    size_t cap = 0;
    for (int c = 0; c < G; c++) cap = std::max(cap, gu[c].size() * gu_b);
    max_rows = 0;
    int lo = 0;
    for (int c = 0; c < G; c++) {
        if ((int)gu[c].size() > FUSED_MAX_GU || rows[c] > FUSED_MAX_ROWS) return -2;
        const size_t down_b = (size_t)rows[c] * k * g.row_d;
        const int place = (!gu[c].empty() && down_b <= gu_b && gu[c].size() * gu_b + down_b > cap) ? 1 : 0;
        uint16_t* p = plan.data() + (size_t)c * FUSED_PLAN;
        p[0] = (uint16_t)gu[c].size();
        p[1] = (uint16_t)lo;
        p[2] = (uint16_t)rows[c];
        p[3] = (uint16_t)place;
        for (size_t i = 0; i < gu[c].size(); i++) p[4 + i] = (uint16_t)gu[c][i];
        lo += rows[c];
        arena_bytes = std::max(arena_bytes, std::max(gu[c].size() * gu_b, (place ? 0 : gu[c].size() * gu_b) + down_b));
        max_rows = std::max(max_rows, rows[c]);
    }
    if (lo != g.H) return -3;
    arena_bytes = (arena_bytes + 15) & ~(size_t)15;
    std::vector<char> first(n_gu_units, 0);
    for (int c = 0; c < G; c++)
        if (!gu[c].empty()) first[gu[c][0]] = 1;
    k_early = 0;
    while (k_early < k) {
        bool all = true;
        for (int c = 0; c < g.nbI; c++) all = all && first[k_early * g.nbI + c];
        if (!all) break;
        k_early++;
    }
    return 0;
}

// The attribute is per kernel and device, shared by every context on the device: only
// ever raise it, so a context with a smaller layout never lowers it below what another
// context's launches need.
cudaError_t fused_prepare(const FusedParams& P) {
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    const int bytes = (int)fused_smem_layout(P).total;
    for (auto fn : {k_decode_fused<false, false>, k_decode_fused<true, false>, k_decode_fused<false, true>,
                    k_decode_fused<true, true>}) {
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, fn);
        if (e != cudaSuccess) return e;
        if (fa.maxDynamicSharedSizeBytes >= bytes) continue;
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t fused_occupancy(const FusedParams& P, int* blocks_per_sm) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        blocks_per_sm, P.ypeer ? k_decode_fused<false, true> : k_decode_fused<false, false>, NT,
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
    if (P.ypeer) {
        if (P.trace) return cudaLaunchKernelEx(&cfg, k_decode_fused<true, true>, P);
        return cudaLaunchKernelEx(&cfg, k_decode_fused<false, true>, P);
    }
    if (P.trace) return cudaLaunchKernelEx(&cfg, k_decode_fused<true, false>, P);
    return cudaLaunchKernelEx(&cfg, k_decode_fused<false, false>, P);
}

}  // namespace tg

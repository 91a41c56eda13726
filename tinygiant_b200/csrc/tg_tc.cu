// tg_tc.cu — the batched expert matmuls on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in TMEM), for experts with many tokens.
//
// One Q4_0 block is exactly one K = 32 step of the MMA, so every MMA step gives the
// exact int32 block dots sumi[row][token] of one block (A = the weights' codes q - 8,
// B = the tokens' Q8_0 codes, both K-major int8 in shared memory, no swizzle).  The
// fp32 work then follows the single-token kernels' order bit for bit: per (row, token)
// the 32 lane classes l (blocks l, l + 32, ...) each chain term = (sumi * d_w) * d_x
// from 0 in increasing block order, and the 32 class sums meet in the xor-butterfly
// tree.  Visiting the classes in bit-reversed order (0, 16, 8, 24, ...) makes the
// tree's siblings consecutive, so a 6-slot stack per (row, token) evaluates it as the
// class sums arrive.
//
// EXACT = false: the fast epilogue.  Per (row, token) one fp32 accumulator takes
// acc = fma(float(sumi), d_w * d_x, acc) block after block in the K order above; no class
// chains, no tree.  The int32 block dots are the same exact values; only the fp32
// summation order differs, so the result stays within the reference's accumulation-order
// tolerance (1e-5 max-abs-rel before any Q8_0 requantisation), not bit-identical.
//
// Work item: 128 weight rows (one matrix of one expert) x a tile of 32 tokens; 16 warps,
// one persistent CTA per SM walking its items' K groups as one pipeline.
// Warp w reads TMEM lanes 32 (w % 4) .. + 31 (its rows) and owns tokens 8 (w / 4) .. + 7.
// K runs in groups of 8 steps through three shared stages and two TMEM accumulator sets
// (2 x 8 x 32 columns): while the epilogue reads group g, the tensor cores run group
// g + 1 and every thread's async copies (cp.async, into its own raw slots) for group
// g + 2 are in flight, converted into the MMA layout after the epilogue; thread 0 issues
// each group's MMAs and commits them to an mbarrier.  Every mbarrier wait is bounded; on
// expiry the CTA records the failure, drains its MMAs (bounded), frees its TMEM and returns.
#include <cuda_runtime.h>

#include "tg_device.cuh"
#include "tg_internal.h"

namespace tg {

namespace {

constexpr int TM = 128;          // weight rows per CTA (MMA M)
constexpr int TN = 32;           // tokens per tile (MMA N)
constexpr int KG = 8;            // K steps (blocks) per group
constexpr int TC_THREADS = 512;
constexpr int A_STEP = TM * 32;  // bytes of A per K step (4 KB)
constexpr int B_STEP = TN * 32;  // bytes of B per K step (1 KB)
// shared stage: A [KG][4 KB] | B [KG][1 KB] | dw [KG][TM] f32 | dx [KG][TN] f32
constexpr int ST_A = 0, ST_B = KG * A_STEP, ST_DW = ST_B + KG * B_STEP, ST_DX = ST_DW + KG * TM * 4;
constexpr int STAGE_BYTES = ST_DX + KG * TN * 4;
constexpr int NSTAGE = 3;        // shared stages: group g+2 is written while g+1 is in the MMA, g in the epilogue
// raw staging: each thread's own slots for its async copies of the next group's operands
// (A: 2 x 16 B codes + 2 x 4 B holding the f16 scale; B, threads < 256: 2 x 16 B + 4 B)
constexpr int RAW_A = NSTAGE * STAGE_BYTES, RAW_AS = RAW_A + TC_THREADS * 32, RAW_B = RAW_AS + TC_THREADS * 8,
              RAW_BD = RAW_B + TN * KG * 32, RAW_END = RAW_BD + TN * KG * 4;
constexpr int TC_SMEM = RAW_END + 1024;   // + alignment slack
constexpr uint32_t TMEM_COLS = 2 * KG * TN;       // 512
constexpr long long TC_WAIT_CYCLES = 2000000000ll;

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// K-major, no-swizzle shared-memory matrix descriptor (sm100 version 1): 8-row x 16-byte
// core matrices, rows 16 B apart, K chunks LBO apart, 8-row groups SBO apart.
__device__ __forceinline__ uint64_t kmajor_desc(const void* base) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr(base) & 0x3FFFF) >> 4);
    d |= (uint64_t)(128 >> 4) << 16;   // LBO: the second 16-byte K chunk of a row group
    d |= (uint64_t)(256 >> 4) << 32;   // SBO: the next 8-row group
    d |= (uint64_t)1 << 46;
    return d;
}
// kind::i8 instruction descriptor: D s32, A and B signed, both K-major, N = 32, M = 128
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);

__device__ __forceinline__ int rev5(int c) {
    return ((c & 1) << 4) | ((c & 2) << 2) | (c & 4) | ((c & 8) >> 2) | ((c & 16) >> 4);
}

// The K order: lane classes in bit-reversed order, each class's blocks ascending.
// steps[s] = block | class ordinal << 10 | (last block of its class) << 15.
constexpr int MAX_STEPS = 512;   // blocks per row: rows of up to 16384 values
__device__ __forceinline__ void build_steps(int nb, uint16_t* steps) {
    int s = 0;
    for (int c = 0; c < 32; c++) {
        const int l = rev5(c);
        for (int b = l; b < nb; b += 32) steps[s++] = (uint16_t)(b | (c << 10) | ((b + 32 >= nb) << 15));
    }
}

// Push the class sums v[t] (class ordinal c, the same for the whole warp) into the
// butterfly stacks: the trailing ones of c are the merges the tree makes at this leaf
// (siblings are earlier stack entries); st[t][5] ends as the total.
__device__ __forceinline__ void push8(float (&st)[8][6], const float (&v)[8], int c) {
    switch (__ffs(~c) - 1) {
        case 0:
#pragma unroll
            for (int t = 0; t < 8; t++) st[t][0] = v[t];
            break;
        case 1:
#pragma unroll
            for (int t = 0; t < 8; t++) st[t][1] = __fadd_rn(st[t][0], v[t]);
            break;
        case 2:
#pragma unroll
            for (int t = 0; t < 8; t++) st[t][2] = __fadd_rn(st[t][1], __fadd_rn(st[t][0], v[t]));
            break;
        case 3:
#pragma unroll
            for (int t = 0; t < 8; t++)
                st[t][3] = __fadd_rn(st[t][2], __fadd_rn(st[t][1], __fadd_rn(st[t][0], v[t])));
            break;
        case 4:
#pragma unroll
            for (int t = 0; t < 8; t++)
                st[t][4] = __fadd_rn(st[t][3], __fadd_rn(st[t][2], __fadd_rn(st[t][1], __fadd_rn(st[t][0], v[t]))));
            break;
        default:
#pragma unroll
            for (int t = 0; t < 8; t++)
                st[t][5] = __fadd_rn(st[t][4],
                                     __fadd_rn(st[t][3], __fadd_rn(st[t][2], __fadd_rn(st[t][1], __fadd_rn(st[t][0], v[t])))));
            break;
    }
}

// Q4_0 codes of four bytes' low (or, after >> 4, high) nibbles as four signed bytes
// q - 8: with bit 7 set first, the per-byte subtraction cannot borrow across bytes, and
// the xor clears it again.
__device__ __forceinline__ uint32_t nib_minus8(uint32_t x) {
    return (((x & 0x0F0F0F0Fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
}

// cp.async of 16 (cg: through L2 only) or 4 bytes; n = 0 copies nothing and zero-fills
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int n) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int n) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(saddr(dst)), "l"(src), "r"(n) : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t (&v)[8], uint32_t ta) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(ta));
}

struct TcParams {
    const uint8_t* layer;      // local routed experts (row-split), expert e_lo first
    const uint8_t* shared;     // shared expert (id E) or null
    int E, e_lo;
    Geom g;
    const int* off;            // pairs grouped by expert
    const int* list;
    const int* active;         // [0] count, [1..] experts
    const int* tile_pre;       // [count + 1]: 32-token tiles of the active experts, prefix sums
    int ks;                    // slots per token
    int down;                  // 0: gate (out0) and up (out1) of the rows of I; 1: down rows of H (out0)
    const uint8_t* act;        // gate/up: xq per token (act_bytes(nbH)); down: hq per pair (act_bytes(nbI))
    float* out0;               // [pair][rows]
    float* out1;
    unsigned* err;             // set when a bounded wait expired
};

constexpr int MAX_ACT = 1025;   // active experts (routed + shared)
constexpr int RING = 4;         // work items whose token lists are held at once

// Persistent: one CTA per SM takes work items w = blockIdx.x, + gridDim.x, ...; an item
// is (token tile of an active expert, 128-row tile of one matrix), token-tile-major so
// CTAs working at once share the tile's activations.  Its K groups are consecutive in
// the CTA's flattened group sequence f, so the pipeline (three shared stages, two TMEM
// sets) runs across item boundaries without restarting.
template <bool EXACT>
__global__ void __launch_bounds__(TC_THREADS, 1) k_q4_mma(TcParams P) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t mbar[2];
    __shared__ uint32_t s_taddr;
    __shared__ int s_fail;
    __shared__ uint16_t s_steps[MAX_STEPS];
    __shared__ int s_tp[MAX_ACT + 1];             // tile prefix per active expert
    __shared__ int s_e[MAX_ACT];                  // the active experts
    __shared__ int s_p0[MAX_ACT], s_n[MAX_ACT];   // their first pair and pair count
    __shared__ int s_pairs[RING][TN];             // token lists of the items in flight
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const Geom& g = P.g;
    const int n_act = P.active[0];
    const int rows = P.down ? g.H : g.I;
    const int tiles = rows / TM;
    const int MT = P.down ? tiles : 2 * tiles;       // matrix row tiles per token tile
    const int n_items = P.tile_pre[n_act] * MT;
    if ((int)blockIdx.x >= n_items) return;
    const int n_mine = (n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const int nb = P.down ? g.nbI : g.nbH;
    const size_t row_bytes = P.down ? g.row_d : g.row_gu;
    const size_t ab = act_bytes(nb);
    const int NG = (nb + KG - 1) / KG;
    const int F = n_mine * NG;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row = (warp & 3) * 32 + lane;          // this thread's TMEM lane / weight row
    const int cg = warp >> 2;                        // token group: tokens 8cg .. 8cg+7

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&s_taddr)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&mbar[0])), "r"(1));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&mbar[1])), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;");
        s_fail = 0;
        build_steps(nb, s_steps);
    }
    for (int a = tid; a <= n_act; a += TC_THREADS) s_tp[a] = P.tile_pre[a];
    for (int a = tid; a < n_act; a += TC_THREADS) {
        const int e = P.active[1 + a];
        s_e[a] = e;
        s_p0[a] = P.off[e];
        s_n[a] = P.off[e + 1] - P.off[e];
    }
    __syncthreads();

    // item i of this CTA: its expert slot a, token tile j, matrix, row tile
    struct Item {
        int a, j, nt, mat, r_base;
    };
    auto item = [&](int i) -> Item {
        Item it;
        const int w = (int)blockIdx.x + i * (int)gridDim.x;
        const int gt = w / MT, mt = w - gt * MT;
        int lo = 0, hi = n_act;                      // s_tp[lo] <= gt < s_tp[hi]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_tp[mid] <= gt) lo = mid; else hi = mid;
        }
        it.a = lo;
        it.j = gt - s_tp[lo];
        it.nt = min(TN, s_n[lo] - TN * it.j);
        it.mat = P.down ? 2 : mt / tiles;
        it.r_base = (mt % tiles) * TM;
        return it;
    };
    auto fill_ring = [&](int i) {   // token list of item i (threads < TN)
        if (i < n_mine && tid < TN) {
            const Item it = item(i);
            s_pairs[i & (RING - 1)][tid] = tid < it.nt ? P.list[s_p0[it.a] + TN * it.j + tid] : -1;
        }
    };
    for (int i = 0; i < 3; i++) fill_ring(i);

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tbase = s_taddr;
    uint32_t use0 = 0u, use1 = 0u;                   // completions consumed per mbarrier
    int fail_f = -1;
    bool failed = false;

    // operand staging: 2 A items (row, step) and 1 B item (token, step) per thread.
    // load_group issues the group's async copies into the thread's raw slots (they run
    // behind the epilogue: no register waits on them); store_group waits for them, then
    // converts the codes into the MMA layout.  A thread reads back only its own copies.
    uint8_t* const raw_a = smem + RAW_A + tid * 32;
    uint32_t* const raw_as = reinterpret_cast<uint32_t*>(smem + RAW_AS + tid * 8);
    uint8_t* const raw_b = smem + RAW_B + (tid & (TN * KG - 1)) * 32;
    float* const raw_bd = reinterpret_cast<float*>(smem + RAW_BD + (tid & (TN * KG - 1)) * 4);
    uint32_t a_odd = 0;         // bit u: item u's scale is the upper half of its 4 copied bytes
    int ld_i = -1;              // the loader's current item and where its rows start
    Item ld_it{};
    const uint8_t* ld_eb = nullptr;
    auto load_group = [&](int f) {
        const int i = f / NG, gi = f - i * NG;
        if (i != ld_i) {
            ld_i = i;
            ld_it = item(i);
            const int e = s_e[ld_it.a];
            ld_eb = (e == P.E ? P.shared : P.layer + (size_t)(e - P.e_lo) * g.expert_bytes) +
                    (size_t)ld_it.mat * g.t_gu + (size_t)ld_it.r_base * row_bytes;
        }
        const Item& it = ld_it;
        const uint8_t* eb = ld_eb;
        a_odd = 0;
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int x = tid + TC_THREADS * u, r = x & (TM - 1), jj = x >> 7;
            const int s = gi * KG + jj;
            const bool ok = s < nb;
            const int b = ok ? s_steps[s] & 1023 : 0;
            const uint8_t* rp = eb + (size_t)r * row_bytes;
            cp_async16(raw_a + 16 * u, rp + 16 * b, ok ? 16 : 0);
            // the f16 scale in an aligned 4-byte pair (the row's scales start 16-aligned,
            // and nb is even, so the pair stays inside them)
            cp_async4(raw_as + u, rp + 16 * (size_t)nb + 4 * (b >> 1), ok ? 4 : 0);
            a_odd |= (uint32_t)(b & 1) << u;
        }
        if (tid < TN * KG) {
            const int tk = tid & (TN - 1), jj = tid >> 5, s = gi * KG + jj;
            const bool ok = s < nb && tk < it.nt;
            const uint8_t* q = P.act;
            const float* d = reinterpret_cast<const float*>(P.act);
            if (ok) {
                const int b = s_steps[s] & 1023;
                const int p = s_pairs[i & (RING - 1)][tk];
                const ActView av = act_view(P.act + (size_t)(P.down ? p : p / P.ks) * ab, nb);
                q = reinterpret_cast<const uint8_t*>(av.qs) + (size_t)b * 32;
                d = av.d + b;
            }
            cp_async16(raw_b, q, ok ? 16 : 0);
            cp_async16(raw_b + 16, q + 16, ok ? 16 : 0);
            cp_async4(raw_bd, d, ok ? 4 : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto store_group = [&](int stg) {
        uint8_t* base = smem + (size_t)stg * STAGE_BYTES;
        asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int x = tid + TC_THREADS * u, r = x & (TM - 1), jj = x >> 7;
            uint8_t* a = base + ST_A + jj * A_STEP + (r >> 3) * 256 + (r & 7) * 16;
            const uint4 ra = *reinterpret_cast<const uint4*>(raw_a + 16 * u);
            const uint32_t sp = raw_as[u];
            uint4 lo, hi;   // element j < 16: low nibble of byte j; 16 + j: high nibble; both minus 8
            lo.x = nib_minus8(ra.x);
            lo.y = nib_minus8(ra.y);
            lo.z = nib_minus8(ra.z);
            lo.w = nib_minus8(ra.w);
            hi.x = nib_minus8(ra.x >> 4);
            hi.y = nib_minus8(ra.y >> 4);
            hi.z = nib_minus8(ra.z >> 4);
            hi.w = nib_minus8(ra.w >> 4);
            *reinterpret_cast<uint4*>(a) = lo;
            *reinterpret_cast<uint4*>(a + 128) = hi;
            reinterpret_cast<float*>(base + ST_DW)[jj * TM + r] =
                f16_bits_to_f32((uint16_t)(((a_odd >> u) & 1) ? sp >> 16 : sp & 0xFFFFu));
        }
        if (tid < TN * KG) {
            const int tk = tid & (TN - 1), jj = tid >> 5;
            uint8_t* bp = base + ST_B + jj * B_STEP + (tk >> 3) * 256 + (tk & 7) * 16;
            *reinterpret_cast<uint4*>(bp) = *reinterpret_cast<const uint4*>(raw_b);
            *reinterpret_cast<uint4*>(bp + 128) = *reinterpret_cast<const uint4*>(raw_b + 16);
            reinterpret_cast<float*>(base + ST_DX)[jj * TN + tk] = *raw_bd;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    };
    // MMAs of group f: operands in stage f % NSTAGE, accumulators in TMEM set f & 1
    auto issue_group = [&](int f) {
        const int gi = f % NG;
        const uint8_t* base = smem + (size_t)(f % NSTAGE) * STAGE_BYTES;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int jj = 0; jj < KG && gi * KG + jj < nb; jj++) {
            const uint64_t da = kmajor_desc(base + ST_A + jj * A_STEP);
            const uint64_t db = kmajor_desc(base + ST_B + jj * B_STEP);
            const uint32_t dt = tbase + (uint32_t)((f & 1) * KG * TN + jj * TN);
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(dt),
                "l"(da), "l"(db), "r"(IDESC), "r"(0));
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         saddr(&mbar[f & 1]))
                     : "memory");
    };
    auto try_group = [&](int f) -> bool {   // bounded wait for group f's commit
        const uint32_t parity = ((f & 1) ? use1 : use0) & 1u;
        const long long t_start = clock64();
        while (true) {
            uint32_t done;
            asm volatile(
                "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(done)
                : "r"(saddr(&mbar[f & 1])), "r"(parity)
                : "memory");
            if (done) return true;
            if (clock64() - t_start > TC_WAIT_CYCLES) return false;
        }
    };

    float leaf[8], st[8][6];
    const float zero8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    int next_cls = 0;   // class ordinal the stacks expect next (classes without blocks push 0)

    load_group(0);
    store_group(0);
    if (F > 1) {
        load_group(1);
        store_group(1);
    }
    __syncthreads();
    if (tid == 0) issue_group(0);
    for (int f = 0; f < F; f++) {
        const int i = f / NG, gi = f - i * NG;
        if (tid == 0 && f + 1 < F) issue_group(f + 1);
        if (f + 2 < F) load_group(f + 2);
        if (gi == 0) {   // a new item: fresh chains and stacks
#pragma unroll
            for (int t = 0; t < 8; t++) {
                leaf[t] = 0.0f;
#pragma unroll
                for (int q = 0; q < 6; q++) st[t][q] = 0.0f;
            }
            next_cls = 0;
        }
        const bool ok = try_group(f);
        if (!ok) {
            atomicExch(&s_fail, 1);
            fail_f = f;
        } else if (f & 1) {
            use1++;
        } else {
            use0++;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok) {
            const uint8_t* stage = smem + (size_t)(f % NSTAGE) * STAGE_BYTES;
            const float* dwp = reinterpret_cast<const float*>(stage + ST_DW);
            const float* dxp = reinterpret_cast<const float*>(stage + ST_DX);
            const uint32_t tcol = tbase + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((f & 1) * KG * TN + cg * 8);
            const int nsteps = min(KG, nb - gi * KG);
            uint32_t va[8], vb[8];
            tmem_ld8(va, tcol);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int jj = 0; jj < KG; jj++) {
                if (jj < nsteps) {
                    uint32_t (&cur)[8] = (jj & 1) ? vb : va;
                    uint32_t (&nxt)[8] = (jj & 1) ? va : vb;
                    if (jj + 1 < nsteps) tmem_ld8(nxt, tcol + (uint32_t)((jj + 1) * TN));
                    const float dw = dwp[jj * TM + row];
                    const float4 dxa = *reinterpret_cast<const float4*>(dxp + jj * TN + cg * 8);
                    const float4 dxb = *reinterpret_cast<const float4*>(dxp + jj * TN + cg * 8 + 4);
                    const float dx[8] = {dxa.x, dxa.y, dxa.z, dxa.w, dxb.x, dxb.y, dxb.z, dxb.w};
                    if constexpr (EXACT) {
                        const int code = s_steps[gi * KG + jj];
                        const int c = (code >> 10) & 31;
                        for (; next_cls < c; next_cls++) push8(st, zero8, next_cls);
#pragma unroll
                        for (int t = 0; t < 8; t++)
                            leaf[t] = __fadd_rn(leaf[t], __fmul_rn(__fmul_rn(__int2float_rn((int)cur[t]), dw), dx[t]));
                        if (code >> 15) {
                            push8(st, leaf, c);
#pragma unroll
                            for (int t = 0; t < 8; t++) leaf[t] = 0.0f;
                            next_cls = c + 1;
                        }
                    } else {   // leaf[t] is the token's single accumulator
#pragma unroll
                        for (int t = 0; t < 8; t++)
                            leaf[t] = __fmaf_rn(__int2float_rn((int)cur[t]), __fmul_rn(dw, dx[t]), leaf[t]);
                    }
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                }
            }
            if (gi == NG - 1) {   // the item's last group: finish the trees, write the sums
                if constexpr (EXACT)
                    for (; next_cls < 32; next_cls++) push8(st, zero8, next_cls);
                const Item it = item(i);
                float* out = it.mat == 1 ? P.out1 : P.out0;
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    const int tk = cg * 8 + t;
                    if (tk < it.nt)
                        out[(size_t)s_pairs[i & (RING - 1)][tk] * rows + it.r_base + row] = EXACT ? st[t][5] : leaf[t];
                }
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        if (f + 2 < F) store_group((f + 2) % NSTAGE);
        if (f + 3 < F && (f + 3) % NG == 0) fill_ring((f + 3) / NG);   // the token list of the item after
        __syncthreads();
        failed = s_fail != 0;
        if (failed) break;
    }
    if (failed) {
        // drain (bounded) the MMAs still in flight, the failed group's and the one issued
        // after it, before the TMEM is freed
        const long long t_start = clock64();
        for (int f = fail_f; f >= 0 && f <= fail_f + 1 && f < F; f++) {
            const uint32_t parity = ((f & 1) ? use1 : use0) & 1u;
            while (clock64() - t_start < TC_WAIT_CYCLES) {
                uint32_t done;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                    "selp.u32 %0, 1, 0, p;\n\t}"
                    : "=r"(done)
                    : "r"(saddr(&mbar[f & 1])), "r"(parity)
                    : "memory");
                if (done) break;
            }
        }
        if (tid == 0) atomicExch(P.err, 1u);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TMEM_COLS));
}

}  // namespace

bool q4_mma_supported(const Geom& g) { return g.I % TM == 0 && g.H % TM == 0; }
int q4_mma_tile_tokens() { return TN; }

cudaError_t launch_q4_mma(const uint8_t* layer, const uint8_t* shared, int E, int e_lo, Geom g, int down,
                          const int* off, const int* list, const int* active, const int* tile_pre, int n_act, int ks,
                          const uint8_t* act, float* out0, float* out1, unsigned* err, bool exact, cudaStream_t s) {
    if (n_act <= 0) return cudaSuccess;
    if (n_act > MAX_ACT) return cudaErrorInvalidValue;
    if (!q4_mma_supported(g)) return cudaErrorInvalidValue;
    TcParams P;
    P.layer = layer;
    P.shared = shared;
    P.E = E;
    P.e_lo = e_lo;
    P.g = g;
    P.off = off;
    P.list = list;
    P.active = active;
    P.tile_pre = tile_pre;
    P.ks = ks;
    P.down = down;
    P.act = act;
    P.out0 = out0;
    P.out1 = out1;
    P.err = err;
    auto kern = exact ? k_q4_mma<true> : k_q4_mma<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    kern<<<sms, TC_THREADS, TC_SMEM, s>>>(P);   // persistent: one CTA per SM
    return cudaGetLastError();
}

}  // namespace tg

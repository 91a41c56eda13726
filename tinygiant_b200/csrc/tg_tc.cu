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
// CTA: 128 weight rows (one matrix of one expert) x a tile of 32 tokens; 16 warps.
// Warp w reads TMEM lanes 32 (w % 4) .. + 31 (its rows) and owns tokens 8 (w / 4) .. + 7.
// K runs in groups of 8 steps: double-buffered shared-memory stages and TMEM
// accumulators (2 x 8 x 32 columns); every thread stages the next group's operands
// (global loads into registers before the current group's epilogue, shared stores
// after it), thread 0 issues the group's MMAs and commits them to an mbarrier.  Every
// mbarrier wait is bounded; on expiry the CTA records the failure, stops issuing, and
// frees its TMEM.
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
constexpr int TC_SMEM = 2 * STAGE_BYTES + 1024;   // + alignment slack
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

// push class sum v (class ordinal c) into the butterfly stack; st[5] is the total
__device__ __forceinline__ void stack_push(float (&st)[6], float v, int c) {
    bool done = false;
#pragma unroll
    for (int lv = 0; lv < 5; lv++) {
        if (!done) {
            if ((c >> lv) & 1) {
                v = __fadd_rn(st[lv], v);
            } else {
                st[lv] = v;
                done = true;
            }
        }
    }
    if (!done) st[5] = v;
}

struct TcParams {
    const uint8_t* layer;      // local routed experts (row-split), expert e_lo first
    const uint8_t* shared;     // shared expert (id E) or null
    int E, e_lo;
    Geom g;
    const int* off;            // pairs grouped by expert
    const int* list;
    const int* active;         // [0] count, [1..] experts
    int ks;                    // slots per token
    int down;                  // 0: gate (out0) and up (out1) of the rows of I; 1: down rows of H (out0)
    const uint8_t* act;        // gate/up: xq per token (act_bytes(nbH)); down: hq per pair (act_bytes(nbI))
    float* out0;               // [pair][rows]
    float* out1;
    unsigned* err;             // set when a bounded wait expired
};

__global__ void __launch_bounds__(TC_THREADS, 1) k_q4_mma(TcParams P) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t mbar[2];
    __shared__ uint32_t s_taddr;
    __shared__ int s_pair[TN];
    __shared__ int s_fail;
    __shared__ uint16_t s_steps[MAX_STEPS];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    if ((int)blockIdx.y >= P.active[0]) return;
    const int e = P.active[1 + blockIdx.y];
    const int p0 = P.off[e], n = P.off[e + 1] - p0;
    if (n == 0) return;
    const Geom& g = P.g;
    const int rows = P.down ? g.H : g.I;
    const int tiles = rows / TM;
    const int mat = P.down ? 2 : (int)blockIdx.x / tiles;          // 0 gate, 1 up, 2 down
    const int r_base = ((int)blockIdx.x % tiles) * TM;
    const int nb = P.down ? g.nbI : g.nbH;
    const size_t row_bytes = P.down ? g.row_d : g.row_gu;
    const uint8_t* eb = (e == P.E ? P.shared : P.layer + (size_t)(e - P.e_lo) * g.expert_bytes) +
                        (size_t)mat * g.t_gu + (size_t)r_base * row_bytes;
    const size_t ab = act_bytes(nb);
    float* out = mat == 1 ? P.out1 : P.out0;
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
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tbase = s_taddr;
    uint32_t uses[2] = {0u, 0u};                     // completions consumed per mbarrier
    const int NG = (nb + KG - 1) / KG;
    bool failed = false;

    for (int t0 = 0; t0 < n && !failed; t0 += TN) {
        const int nt = min(TN, n - t0);
        __syncthreads();
        if (tid < TN) s_pair[tid] = tid < nt ? P.list[p0 + t0 + tid] : -1;
        __syncthreads();

        // operand staging: 2 A items (row, step) and 1 B item (token, step) per thread
        uint4 ra[2];
        float rdw[2];
        uint4 rb0, rb1;
        float rdx = 0.0f;
        auto load_group = [&](int gi) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int it = tid + TC_THREADS * u, r = it & (TM - 1), jj = it >> 7;
                const int s = gi * KG + jj;
                ra[u] = make_uint4(0, 0, 0, 0);
                rdw[u] = 0.0f;
                if (s < nb) {
                    const int b = s_steps[s] & 1023;
                    const uint8_t* rp = eb + (size_t)r * row_bytes;
                    ra[u] = __ldg(reinterpret_cast<const uint4*>(rp + 16 * b));
                    rdw[u] = f16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t*>(rp + 16 * (size_t)nb + 2 * b)));
                }
            }
            rb0 = rb1 = make_uint4(0, 0, 0, 0);
            rdx = 0.0f;
            if (tid < TN * KG) {
                const int tk = tid & (TN - 1), jj = tid >> 5, s = gi * KG + jj;
                if (s < nb && tk < nt) {
                    const int b = s_steps[s] & 1023;
                    const int p = s_pair[tk];
                    const uint8_t* ap = P.act + (size_t)(P.down ? p : p / P.ks) * ab;
                    const ActView av = act_view(ap, nb);
                    const uint4* q = reinterpret_cast<const uint4*>(av.qs + (size_t)b * 32);
                    rb0 = __ldg(q);
                    rb1 = __ldg(q + 1);
                    rdx = __ldg(av.d + b);
                }
            }
        };
        auto store_group = [&](int stg) {
            uint8_t* base = smem + (size_t)stg * STAGE_BYTES;
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int it = tid + TC_THREADS * u, r = it & (TM - 1), jj = it >> 7;
                uint8_t* a = base + ST_A + jj * A_STEP + (r >> 3) * 256 + (r & 7) * 16;
                uint4 lo, hi;   // element j < 16: low nibble of byte j; 16 + j: high nibble; both minus 8
                lo.x = __vsub4(ra[u].x & 0x0F0F0F0Fu, 0x08080808u);
                lo.y = __vsub4(ra[u].y & 0x0F0F0F0Fu, 0x08080808u);
                lo.z = __vsub4(ra[u].z & 0x0F0F0F0Fu, 0x08080808u);
                lo.w = __vsub4(ra[u].w & 0x0F0F0F0Fu, 0x08080808u);
                hi.x = __vsub4((ra[u].x >> 4) & 0x0F0F0F0Fu, 0x08080808u);
                hi.y = __vsub4((ra[u].y >> 4) & 0x0F0F0F0Fu, 0x08080808u);
                hi.z = __vsub4((ra[u].z >> 4) & 0x0F0F0F0Fu, 0x08080808u);
                hi.w = __vsub4((ra[u].w >> 4) & 0x0F0F0F0Fu, 0x08080808u);
                *reinterpret_cast<uint4*>(a) = lo;
                *reinterpret_cast<uint4*>(a + 128) = hi;
                reinterpret_cast<float*>(base + ST_DW)[jj * TM + r] = rdw[u];
            }
            if (tid < TN * KG) {
                const int tk = tid & (TN - 1), jj = tid >> 5;
                uint8_t* bp = base + ST_B + jj * B_STEP + (tk >> 3) * 256 + (tk & 7) * 16;
                *reinterpret_cast<uint4*>(bp) = rb0;
                *reinterpret_cast<uint4*>(bp + 128) = rb1;
                reinterpret_cast<float*>(base + ST_DX)[jj * TN + tk] = rdx;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        };
        auto issue_group = [&](int gi) {
            const int stg = gi & 1;
            const uint8_t* base = smem + (size_t)stg * STAGE_BYTES;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int jj = 0; jj < KG && gi * KG + jj < nb; jj++) {
                const uint64_t da = kmajor_desc(base + ST_A + jj * A_STEP);
                const uint64_t db = kmajor_desc(base + ST_B + jj * B_STEP);
                const uint32_t dt = tbase + (uint32_t)(stg * KG * TN + jj * TN);
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(dt),
                    "l"(da), "l"(db), "r"(IDESC), "r"(0));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             saddr(&mbar[stg]))
                         : "memory");
        };
        auto wait_group = [&](int gi) -> bool {
            const int stg = gi & 1;
            const uint32_t parity = uses[stg] & 1u;
            const long long t_start = clock64();
            while (true) {
                uint32_t done;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                    "selp.u32 %0, 1, 0, p;\n\t}"
                    : "=r"(done)
                    : "r"(saddr(&mbar[stg])), "r"(parity)
                    : "memory");
                if (done) break;
                if (clock64() - t_start > TC_WAIT_CYCLES) return false;
            }
            uses[stg]++;
            return true;
        };

        float leaf[8], st[8][6];
#pragma unroll
        for (int t = 0; t < 8; t++) {
            leaf[t] = 0.0f;
#pragma unroll
            for (int q = 0; q < 6; q++) st[t][q] = 0.0f;
        }
        int next_cls = 0;   // class ordinal the stack expects next (empty classes are pushed as 0)

        load_group(0);
        store_group(0);
        __syncthreads();
        if (tid == 0) issue_group(0);
        for (int gi = 0; gi < NG; gi++) {
            if (gi + 1 < NG) load_group(gi + 1);
            const bool ok = wait_group(gi);
            if (!ok) {
                atomicExch(&s_fail, 1);
                uses[gi & 1]++;   // the completion, if it ever comes, belongs to this group
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (ok) {
                const float* dwp = reinterpret_cast<const float*>(smem + (size_t)(gi & 1) * STAGE_BYTES + ST_DW);
                const float* dxp = reinterpret_cast<const float*>(smem + (size_t)(gi & 1) * STAGE_BYTES + ST_DX);
                for (int jj = 0; jj < KG; jj++) {
                    const int s = gi * KG + jj;
                    if (s >= nb) break;
                    const int c = (s_steps[s] >> 10) & 31;
                    const bool lst = (s_steps[s] >> 15) != 0;
                    for (; next_cls < c; next_cls++)       // classes without blocks contribute +0
#pragma unroll
                        for (int t = 0; t < 8; t++) stack_push(st[t], 0.0f, next_cls);
                    uint32_t v[8];
                    const uint32_t ta = tbase + ((uint32_t)((warp & 3) * 32) << 16) +
                                        (uint32_t)((gi & 1) * KG * TN + jj * TN + cg * 8);
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                          "=r"(v[7])
                        : "r"(ta));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    const float dw = dwp[jj * TM + row];
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        const float term = __fmul_rn(__fmul_rn(__int2float_rn((int)v[t]), dw), dxp[jj * TN + cg * 8 + t]);
                        leaf[t] = __fadd_rn(leaf[t], term);
                    }
                    if (lst) {
#pragma unroll
                        for (int t = 0; t < 8; t++) {
                            stack_push(st[t], leaf[t], c);
                            leaf[t] = 0.0f;
                        }
                        next_cls = c + 1;
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            if (gi + 1 < NG) store_group((gi + 1) & 1);
            __syncthreads();
            failed = s_fail != 0;
            if (failed) break;
            if (tid == 0 && gi + 1 < NG) issue_group(gi + 1);
        }
        if (failed) break;
        for (; next_cls < 32; next_cls++)
#pragma unroll
            for (int t = 0; t < 8; t++) stack_push(st[t], 0.0f, next_cls);
#pragma unroll
        for (int t = 0; t < 8; t++) {
            const int tk = cg * 8 + t;
            if (tk < nt) out[(size_t)s_pair[tk] * rows + r_base + row] = st[t][5];
        }
    }
    if (failed) {
        // the failed group's MMAs may still be in flight: give them one more bounded wait
        // before the TMEM is freed
        const long long t_start = clock64();
        for (int b = 0; b < 2; b++) {
            const uint32_t parity = (uses[b] - 1u) & 1u;
            while (clock64() - t_start < TC_WAIT_CYCLES) {
                uint32_t done;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                    "selp.u32 %0, 1, 0, p;\n\t}"
                    : "=r"(done)
                    : "r"(saddr(&mbar[b])), "r"(parity)
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

cudaError_t launch_q4_mma(const uint8_t* layer, const uint8_t* shared, int E, int e_lo, Geom g, int down,
                          const int* off, const int* list, const int* active, int n_act, int ks, const uint8_t* act,
                          float* out0, float* out1, unsigned* err, cudaStream_t s) {
    if (n_act <= 0) return cudaSuccess;
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
    P.ks = ks;
    P.down = down;
    P.act = act;
    P.out0 = out0;
    P.out1 = out1;
    P.err = err;
    cudaError_t e = cudaFuncSetAttribute(k_q4_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    if (e != cudaSuccess) return e;
    const int gx = down ? g.H / TM : 2 * (g.I / TM);
    k_q4_mma<<<dim3(gx, n_act), TC_THREADS, TC_SMEM, s>>>(P);
    return cudaGetLastError();
}

}  // namespace tg

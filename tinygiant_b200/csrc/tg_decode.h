// tg_decode.h — the fused (one kernel per decode step) MoE path.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "tg_layout.h"

namespace tg {

constexpr int FUSED_MAX_GU = 4;          // gate/up units (32 rows of one expert) per CTA
constexpr int FUSED_MAX_ROWS = 64;       // contiguous down-projection output rows per CTA
constexpr int FUSED_COMPUTE_WARPS = 16;  // warps that compute (2 h rows each per gate/up unit)
constexpr int FUSED_THREADS = (FUSED_COMPUTE_WARPS + 1) * 32;  // + one producer warp issuing copies
constexpr int FUSED_PLAN = 4 + FUSED_MAX_GU;  // per CTA: n_gu, first down row, down rows, down placement, units
// phase stamps: 0 routing and x seen, 1 gate/up copies issued, 2 x quantised,
// 3 gate/up published, 4 early h gathered, 5 down data landed, 6 down rows done,
// 7 next-layer sums sent, 8 first gate/up unit landed, 9 top-k done,
// 10 down copies issued, 11 late h gathered, 12 down values stored to every rank,
// 13 every rank's down values received (12 and 13 with experts sharded over
// devices); slots 16..31 hold the SM's clock64 at the same events
constexpr int FUSED_TRACE = 32;
// router sums are spread over this many accumulator copies (CTA c adds into copy
// c % FUSED_ACC), so each word takes ~G / FUSED_ACC atomic adds instead of G
constexpr int FUSED_ACC = 8;
// default bounded-wait limit in SM cycles (~1 s at the B200's 1.9-2 GHz)
constexpr long long FUSED_WAIT_CYCLES = 2000000000ll;

struct FusedParams {
    const uint8_t* weights;   // [L][E] row-split experts
    size_t layer_bytes;
    Geom g;
    const float* RT;          // [L][H][E] routers, transposed
    const float* normw;       // [L][H] FFN RMSNorm weights
    float eps;                // RMSNorm epsilon
    int E, k, L0, nL;         // layers [L0, L0 + nL) of the model
    int max_rows;             // largest down-row range of any CTA
    int k_early;              // > 0: down in two stages, slots [0, k_early) (all their gate/up units
                              // first in their CTAs) before the rest; 0: one stage
    long long wait_cycles;    // limit of every bounded wait in the kernel, in SM cycles
    int missing;              // router-sum contributions to wait for that no CTA sends (0; > 0 makes
                              // the first routing wait run out: the failure path under test)
    const float* x_in;        // hidden state in
    float* x_out;             // hidden state out (may equal x_in when nL >= 2 or every CTA has a gate/up unit)
    unsigned long long* xw;   // [Lmax + 1][H] hidden states between layers: (tag << 32) | f32 bits
    unsigned long long* acc;  // [nL][FUSED_ACC][E + 1] count-tagged fixed-point router sums, then
                              // sum of x^2 (zero between launches)
    unsigned long long* hqt;  // [Lmax][k * nbI * 6] tagged requantised h words: (tag << 48) | 6 bytes
    int Lmax;                 // layers the xw / hqt buffers hold (cleared before the tag repeats)
    unsigned* ctl;            // [0] epoch, [1] finished CTAs, [2] error stage, [3] error detail
    const uint16_t* plan;     // [G][FUSED_PLAN]
    int* idx_out;             // [L][k] routing record (absolute layer index)
    float* w_out;             // [L][k]
    float* logits_out;        // [L][E]
    unsigned long long* trace;  // optional [nL][G][FUSED_TRACE] stamps per CTA and layer
    size_t arena_bytes;       // weight staging bytes per CTA
    // Experts sharded over devices (ypeer != nullptr): this device holds experts
    // [e_lo, e_lo + e_n) of every layer (weights / layer_bytes cover only them), routes
    // every token like the others, computes the gate/up and down rows of the slots whose
    // expert it holds, and stores each row's per-slot down value into every rank's y
    // buffer ([2][Lmax][k][H] words (tag << 32) | f32 bits, half = launch parity) over
    // NVLink; every rank then combines all k slots in slot order.  One device: 0, E, null.
    int e_lo, e_n;
    int ep_rank, ep_size;
    unsigned long long* const* ypeer;   // [ep_size] every rank's y buffer (device pointers)
};

// Shared-memory carve-up, identical on host and device.
struct FusedSmem {
    uint32_t mbar, plan, slogfx, slog, skey, sidx, lmap, flags, xs, xq, hq, sh, hrec, xnext, xw, rt, snorm, ys, yr,
        arena, total;
};

TG_HD uint32_t fused_take(uint32_t& o, size_t bytes) {
    uint32_t r = o;
    o += (uint32_t)((bytes + 127) & ~(size_t)127);
    return r;
}

TG_HD FusedSmem fused_smem_layout(const FusedParams& P) {
    FusedSmem s;
    uint32_t o = 0;
    s.mbar = fused_take(o, 8 * (FUSED_MAX_GU + 2));
    s.plan = fused_take(o, 2 * FUSED_PLAN);
    s.slogfx = fused_take(o, 8 * (size_t)FUSED_ACC * ((size_t)P.E + 1));   // per-copy router sums
    s.slog = fused_take(o, 4 * (size_t)P.E);
    s.skey = fused_take(o, 8 * (size_t)P.E);
    s.sidx = fused_take(o, 4 * 16);
    s.lmap = fused_take(o, 4 * 16);           // local slot -> slot (experts sharded over devices)
    s.flags = fused_take(o, 4 * 8);
    s.xs = fused_take(o, 4 * (size_t)P.g.H);
    s.xq = fused_take(o, act_bytes(P.g.nbH));
    s.hq = fused_take(o, act_bytes(P.g.nbI) * P.k);
    s.sh = fused_take(o, 4 * (2 * 32 + 16));  // h of a gate/up unit, double buffered; routing weights
    s.hrec = fused_take(o, 2 * 64);           // its Q8_0 record, double buffered
    s.xnext = fused_take(o, 4 * (size_t)P.max_rows);
    s.xw = fused_take(o, 4 * (size_t)P.max_rows);
    s.rt = fused_take(o, 4 * (size_t)P.max_rows * P.E);
    s.snorm = fused_take(o, 2 * 4 * (size_t)P.g.H);   // FFN norm weights, double buffered by layer parity
    s.ys = fused_take(o, 4 * 16 * (size_t)P.max_rows);  // per-slot down values of this CTA's rows
    // the same for all k slots as received from every rank (experts sharded over devices)
    s.yr = fused_take(o, P.ypeer ? 4 * 16 * (size_t)P.max_rows : 0);
    s.arena = fused_take(o, P.arena_bytes);
    s.total = o;
    return s;
}

// Static work split of one layer over G CTAs: gate/up units by longest-processing-
// time greedy, then contiguous down-row ranges of H/G or H/G + 1 rows (the extra
// rows to CTAs with fewer units).  A CTA's down rows go after its units (placement 0,
// fetched once its last unit has landed) when units and rows together fit the arena
// the largest unit set needs anyway, else into the space of its first gate/up unit
// once that unit is computed (placement 1).  k_early
// counts the leading slots whose units are all first units of their CTAs (their h
// is complete early).  Returns 0, or < 0 when the shape does not fit the limits.
int fused_plan(const Geom& g, int E, int k, int G, std::vector<uint16_t>& plan, size_t& arena_bytes,
               int& max_rows, int& k_early);
cudaError_t fused_prepare(const FusedParams& P);
cudaError_t fused_occupancy(const FusedParams& P, int* blocks_per_sm);
cudaError_t launch_decode_fused(const FusedParams& P, int G, cudaStream_t s);

}  // namespace tg

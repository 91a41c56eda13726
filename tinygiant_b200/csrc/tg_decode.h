// tg_decode.h — the fused (one kernel per decode step) MoE path.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "tg_layout.h"

namespace tg {

constexpr int FUSED_MAX_GU = 4;    // gate/up units (32 rows of one expert) per CTA
constexpr int FUSED_MAX_D = 16;    // down units (rd output rows, all k experts) per CTA
constexpr int FUSED_THREADS = 512;

struct FusedParams {
    const uint8_t* weights;   // [L][E] row-split experts
    size_t layer_bytes;
    Geom g;
    const float* RT;          // [L][H][E] routers, transposed
    const float* normw;       // [L][H] FFN RMSNorm weights
    float eps;                // RMSNorm epsilon
    int E, k, L0, nL, rd;     // layers [L0, L0 + nL) of the model
    const float* x_in;        // hidden state in
    float* x_out;             // hidden state out (may equal x_in when nL >= 2)
    float* xbuf;              // [nL + 1][H] intermediate hidden states
    unsigned long long* acc;  // [nL][E + 1] count-tagged fixed-point router sums, then sum of x^2
                              // (zero between launches)
    unsigned long long* hqt;  // [nL][k * nbI * 6] epoch-tagged requantised h words
    unsigned* ctl;            // [0] epoch, [1] finished CTAs, [2] error code
    const uint16_t* plan;     // per CTA: n_gu, n_d, gu units[FUSED_MAX_GU], d units[FUSED_MAX_D]
    int plan_stride;
    int* idx_out;             // [L][k] routing record (absolute layer index)
    float* w_out;             // [L][k]
    float* logits_out;        // [L][E]
    float* h_dbg;             // optional [L][k][I]
    size_t arena_bytes;       // weight staging bytes per CTA
};

// Shared-memory carve-up, identical on host and device.
struct FusedSmem {
    uint32_t mbar, plan, slogfx, slog, sidx, sw, flags, xs, xq, hq, rec, sh, hrec, xnext, xw, rt, arena, total;
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
    s.plan = fused_take(o, 2 * (2 + FUSED_MAX_GU + FUSED_MAX_D));
    s.slogfx = fused_take(o, 8 * ((size_t)P.E + 1));
    s.slog = fused_take(o, 4 * (size_t)P.E);
    s.sidx = fused_take(o, 4 * 16);
    s.sw = fused_take(o, 4 * 16);
    s.flags = fused_take(o, 16);
    s.xs = fused_take(o, 4 * (size_t)P.g.H);
    s.xq = fused_take(o, act_bytes(P.g.nbH));
    s.hq = fused_take(o, act_bytes(P.g.nbI) * P.k);
    s.rec = fused_take(o, 36 * (size_t)P.k * P.g.nbI);
    s.sh = fused_take(o, 4 * 32);
    s.hrec = fused_take(o, 64);
    s.xnext = fused_take(o, 4 * (size_t)FUSED_MAX_D * P.rd);
    s.xw = fused_take(o, 4 * (size_t)FUSED_MAX_D * P.rd);
    s.rt = fused_take(o, 4 * (size_t)FUSED_MAX_D * P.rd * P.E);
    s.arena = fused_take(o, P.arena_bytes);
    s.total = o;
    return s;
}

// Static work split of one layer over G CTAs (longest-processing-time greedy on bytes).
// Returns 0, or < 0 when the shape does not fit the per-CTA limits.
int fused_plan(const Geom& g, int E, int k, int G, int rd, std::vector<uint16_t>& plan, size_t& arena_bytes,
               int& plan_stride);
cudaError_t fused_prepare(const FusedParams& P);
cudaError_t fused_occupancy(const FusedParams& P, int* blocks_per_sm);
cudaError_t launch_decode_fused(const FusedParams& P, int G, cudaStream_t s);

}  // namespace tg

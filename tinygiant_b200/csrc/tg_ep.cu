// tg_ep.cu — experts sharded over devices (expert parallelism), one context per rank.
//
// Rank r of G holds experts [r * E/G, (r + 1) * E/G) of every layer; routers, norms and
// the optional shared expert (DeepSeek-V3-like: every token, weight 1, after the routed
// slots) are replicated.  A layer for T tokens is
//   tgx_ep_moe_partial   routing (the same on every rank), then y[(t, j)] for the
//                        pairs this rank owns (routed: their expert is local; shared:
//                        this rank holds the fewest of the token's routed experts),
//                        0 for the others
//   (caller)             sum of y over the ranks: an all-reduce (NCCL) or any exact sum
//   tgx_ep_combine       x[t] += sum_j w[t][j] * y[(t, j)] in slot order
// Every element of y has exactly one nonzero contribution and sums start from +0, so
// the all-reduce is exact and the result equals the single-device path bit for bit
// (tinygiant/engine.py:229-258 per token, the reference's sequential combine).
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/tinygiant.h"
#include "tg_decode.h"
#include "tg_device.cuh"
#include "tg_internal.h"

using tg::Geom;

struct tgx_ep {
    int device = 0, rank = 0, size = 1, e_lo = 0, e_n = 0, n_shared = 0;
    tgx_shape shape{};
    Geom g;
    float eps = 1e-6f;
    size_t layer_bytes = 0;       // e_n experts
    uint8_t* weights = nullptr;   // [L][e_n] local experts, row-split
    uint8_t* shared = nullptr;    // [L] shared expert (n_shared = 1), row-split
    float* routers = nullptr;     // [L][E][H]
    float* norms = nullptr;       // [L][H]
    uint8_t* staging = nullptr;
    size_t staging_bytes = 0;
    void* scratch = nullptr;      // partial-step scratch, grown on demand
    size_t scratch_bytes = 0;
    float* wts = nullptr;         // [T][k] routing weights of the last partial step
    size_t wts_bytes = 0;
    int last_T = 0;
    int kernels = 0;              // tg::BATCHED_AUTO / _DP4A / _MMA
    cudaStream_t s = nullptr;
    // NVLink exchange (tgx_ep_p2p_*): one region per rank, y[0] | y[1] | flags[G], shared
    // through CUDA IPC; y[b] receives the per-(token, slot) down sums of the exchange
    // calls whose epoch (calls exchanged before them) has parity b
    int p2p_T = 0;                // tokens per step the region holds
    uint8_t* region = nullptr;    // this rank's region
    float* ystage = nullptr;      // this rank's partial sums before the push (local, y_bytes)
    size_t y_bytes = 0, region_bytes = 0;
    void* peers[64] = {};         // opened peer regions (null for this rank)
    float** dst_dev = nullptr;    // [2][G]: rank q's y[b]
    unsigned** flag_dev = nullptr;  // [G]: rank q's flags
    unsigned* epoch = nullptr;    // layers exchanged so far (device)
    unsigned* p2p_err = nullptr;  // a bounded wait expired
    unsigned* p2p_count = nullptr;  // push CTAs finished this layer (zero between layers)
    int* owned = nullptr;         // [1 + T * ks]: count and list of the pairs this rank computed
    bool p2p_ready = false;
    // fused decode (tgx_ep_fused_*): the one-kernel-per-step path restricted to the local
    // experts; ybuf ([2][L][k][H] tagged words) receives every rank's per-slot down values
    bool fused_ready = false;
    int fG = 0;                         // CTAs = SMs
    float* RT = nullptr;                // [L][H][E] transposed routers
    unsigned long long* xw = nullptr;   // [L + 1][H]
    unsigned long long* facc = nullptr; // [L][FUSED_ACC][E + 1]
    unsigned long long* hqt = nullptr;  // [L][k * nbI * 6]
    unsigned* ctl = nullptr;            // epoch, finish count, error
    uint16_t* plan = nullptr;
    int* fidx = nullptr;                // [L][k] routing record of the last step
    float* fw = nullptr;                // [L][k]
    float* flogits = nullptr;           // [L][E]
    unsigned long long* ybuf = nullptr;
    size_t ybuf_bytes = 0;
    void* fpeers[64] = {};              // opened peer y buffers (null for this rank)
    unsigned long long** ypeer = nullptr;   // [G] device pointers to every rank's y buffer
    tg::FusedParams fp{};
    // token dispatch (tgx_ep_dispatch*): routing state of this rank's tokens between the
    // dispatch and the combine, and the receive side's activation rows and expert scratch
    void* dscratch = nullptr;
    size_t dscratch_bytes = 0;
    int d_T = 0;                        // tokens of the last tgx_ep_dispatch
    float* d_wts = nullptr;             // [T][ks] their routing weights
    int* d_slot = nullptr;              // [T][ks] each pair's record index in the send order
    // device-side token dispatch (tgx_ep_dispatch_p2p_*): one IPC region per rank (records
    // in, y rows back, flags), every buffer sized at set-up for dp_T tokens per call
    int dp_T = 0;
    size_t dp_cap = 0;                  // records per (buffer half, peer)
    uint8_t* dp_region = nullptr;
    size_t dp_region_bytes = 0;
    void* dp_peers[64] = {};
    uint8_t** dp_bases = nullptr;       // [G] every rank's region (device pointers)
    unsigned* dp_ctl = nullptr;         // [0] calls, [1..3] CTA counters, [4] error
    int* dp_meta = nullptr;             // [0..64] send prefix, [65..130] receive prefix, [131] received
    void* dp_work = nullptr;            // routing, receive side and expert scratch
    size_t dp_work_bytes = 0;
    bool dp_ready = false;
};

namespace {

int ep_fail(int code, const std::string& msg) { return tg::set_error(code, msg.c_str()); }

#define EP_CUDA(call)                                                                          \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return ep_fail(e_ == cudaErrorMemoryAllocation ? TG_ENOMEM : TG_ECUDA,              \
                           std::string(#call) + ": " + cudaGetErrorString(e_));                 \
    } while (0)
#define EP_CHECK(cond, code, msg) \
    do {                          \
        if (!(cond)) return ep_fail((code), (msg)); \
    } while (0)
#define EP_TRY(expr)                  \
    do {                              \
        int rc_ = (expr);             \
        if (rc_ != TG_OK) return rc_; \
    } while (0)

struct Dev {
    int prev = -1;
    explicit Dev(int d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(d);
    }
    ~Dev() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

void ep_free(tgx_ep* c) {
    if (!c) return;
    Dev dg(c->device);
    for (int q = 0; q < 64; q++) {
        if (c->peers[q]) cudaIpcCloseMemHandle(c->peers[q]);
        if (c->fpeers[q]) cudaIpcCloseMemHandle(c->fpeers[q]);
        if (c->dp_peers[q]) cudaIpcCloseMemHandle(c->dp_peers[q]);
    }
    for (void* p : {(void*)c->dp_region, (void*)c->dp_bases, (void*)c->dp_ctl, (void*)c->dp_meta, c->dp_work})
        if (p) cudaFree(p);
    for (void* p : {(void*)c->region, (void*)c->ystage, (void*)c->dst_dev, (void*)c->flag_dev, (void*)c->epoch, (void*)c->p2p_err,
                    (void*)c->p2p_count, (void*)c->owned})
        if (p) cudaFree(p);
    for (void* p : {(void*)c->RT, (void*)c->xw, (void*)c->facc, (void*)c->hqt, (void*)c->ctl, (void*)c->plan,
                    (void*)c->fidx, (void*)c->fw, (void*)c->flogits, (void*)c->ybuf, (void*)c->ypeer, c->dscratch})
        if (p) cudaFree(p);
    for (void* p : {(void*)c->weights, (void*)c->shared, (void*)c->routers, (void*)c->norms, (void*)c->staging,
                    c->scratch, (void*)c->wts})
        if (p) cudaFree(p);
    if (c->s) cudaStreamDestroy(c->s);
    delete c;
}

int ep_alloc(void** p, size_t n, const char* fn) {
    if (cudaMalloc(p, n) != cudaSuccess) {
        cudaGetLastError();
        return ep_fail(TG_ENOMEM, std::string(fn) + ": cudaMalloc of " + std::to_string(n) + " bytes failed");
    }
    return TG_OK;
}

// grow the partial-step scratch and the routing-weight buffer for T tokens
int ep_reserve(tgx_ep* c, int T, cudaStream_t s, const char* fn) {
    const tgx_shape& sh = c->shape;
    const size_t need = tg::batched_partial_bytes(c->g, sh.n_experts, c->n_shared, sh.top_k, T);
    const size_t wneed = sizeof(float) * (size_t)T * (sh.top_k + c->n_shared);
    if (need <= c->scratch_bytes && wneed <= c->wts_bytes) return TG_OK;
    EP_CUDA(cudaStreamSynchronize(s));
    if (need > c->scratch_bytes) {
        if (c->scratch) cudaFree(c->scratch);
        c->scratch = nullptr;
        c->scratch_bytes = 0;
        EP_TRY(ep_alloc(&c->scratch, need, fn));
        c->scratch_bytes = need;
        EP_CUDA(cudaMemset(c->scratch, 0, 256));   // the error flag
    }
    if (wneed > c->wts_bytes) {
        if (c->wts) cudaFree(c->wts);
        c->wts = nullptr;
        c->wts_bytes = 0;
        EP_TRY(ep_alloc((void**)&c->wts, wneed, fn));
        c->wts_bytes = wneed;
    }
    return TG_OK;
}

}  // namespace

extern "C" int tgx_ep_create(int device, const tgx_shape* shape, int n_shared, int ep_rank, int ep_size,
                             tgx_ep** out) {
    EP_CHECK(shape && out, TG_EINVAL, "tgx_ep_create: null argument");
    *out = nullptr;
    EP_CHECK(Geom::valid_dims(shape->embed, shape->inter), TG_EINVAL,
             "tgx_ep_create: embed/inter must be positive multiples of 256 (<= 16384)");
    EP_CHECK(shape->n_experts > 0 && shape->n_experts <= 1024 && shape->top_k > 0 && shape->top_k <= 16 &&
                 shape->top_k <= shape->n_experts && shape->n_layers > 0,
             TG_EINVAL, "tgx_ep_create: bad expert/top_k/layer counts");
    EP_CHECK(ep_size >= 1 && ep_rank >= 0 && ep_rank < ep_size && shape->n_experts % ep_size == 0, TG_EINVAL,
             "tgx_ep_create: need 0 <= ep_rank < ep_size and n_experts divisible by ep_size");
    EP_CHECK(n_shared == 0 || n_shared == 1, TG_EINVAL, "tgx_ep_create: n_shared must be 0 or 1");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) {
        cudaGetLastError();
        return ep_fail(TG_ENODEV, "no CUDA device");
    }
    EP_CHECK(device >= 0 && device < ndev, TG_EINVAL, "tgx_ep_create: bad device index");
    Dev dg(device);
    tgx_ep* c = new tgx_ep();
    c->device = device;
    c->rank = ep_rank;
    c->size = ep_size;
    c->shape = *shape;
    c->g = Geom::make(shape->embed, shape->inter);
    c->e_n = shape->n_experts / ep_size;
    c->e_lo = ep_rank * c->e_n;
    c->layer_bytes = c->g.expert_bytes * c->e_n;
    c->n_shared = n_shared;
    if (shape->rms_eps > 0.0f) c->eps = shape->rms_eps;
    const int L = shape->n_layers, E = shape->n_experts, H = shape->embed;
    c->staging_bytes = c->g.expert_bytes * 4;
    int rc;
    if ((rc = ep_alloc((void**)&c->weights, c->layer_bytes * L, "tgx_ep_create")) ||
        (rc = ep_alloc((void**)&c->routers, sizeof(float) * (size_t)L * E * H, "tgx_ep_create")) ||
        (rc = ep_alloc((void**)&c->norms, sizeof(float) * (size_t)L * H, "tgx_ep_create")) ||
        (rc = ep_alloc((void**)&c->staging, c->staging_bytes, "tgx_ep_create")) ||
        (n_shared && (rc = ep_alloc((void**)&c->shared, c->g.expert_bytes * L, "tgx_ep_create")))) {
        ep_free(c);
        return rc;
    }
    std::vector<float> ones((size_t)L * H, 1.0f);
    cudaError_t e = cudaMemcpy(c->norms, ones.data(), ones.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(c->routers, 0, sizeof(float) * (size_t)L * E * H);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->s, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        ep_free(c);
        return ep_fail(TG_ECUDA, std::string("tgx_ep_create: ") + cudaGetErrorString(e));
    }
    *out = c;
    return TG_OK;
}

extern "C" int tgx_ep_destroy(tgx_ep* ep) {
    ep_free(ep);
    return TG_OK;
}

extern "C" int tgx_ep_expert_range(const tgx_ep* ep, int* first, int* n) {
    EP_CHECK(ep && first && n, TG_EINVAL, "tgx_ep_expert_range: null argument");
    *first = ep->e_lo;
    *n = ep->e_n;
    return TG_OK;
}

extern "C" int tgx_ep_load_experts(tgx_ep* ep, int layer, int first, int n, const void* src, int src_on_device) {
    EP_CHECK(ep && src, TG_EINVAL, "tgx_ep_load_experts: null argument");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers && n >= 0 && first >= ep->e_lo && first + n <= ep->e_lo + ep->e_n,
             TG_EINVAL, "tgx_ep_load_experts: layer out of range or experts not held by this rank");
    Dev dg(ep->device);
    const Geom& g = ep->g;
    const int chunk = (int)(ep->staging_bytes / g.expert_bytes);
    for (int e0 = 0; e0 < n; e0 += chunk) {
        const int m = n - e0 < chunk ? n - e0 : chunk;
        EP_CUDA(cudaMemcpyAsync(ep->staging, (const uint8_t*)src + (size_t)e0 * g.expert_bytes, (size_t)m * g.expert_bytes,
                                src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ep->s));
        for (int e = 0; e < m; e++) {
            const uint8_t* raw = ep->staging + (size_t)e * g.expert_bytes;
            uint8_t* dst = ep->weights + (size_t)layer * ep->layer_bytes + (size_t)(first - ep->e_lo + e0 + e) * g.expert_bytes;
            EP_CUDA(tg::launch_repack_rows(raw, dst, 2LL * g.I, g.nbH, ep->s));
            EP_CUDA(tg::launch_repack_rows(raw + 2 * g.t_gu, dst + 2 * g.t_gu, g.H, g.nbI, ep->s));
        }
        EP_CUDA(cudaStreamSynchronize(ep->s));
    }
    return TG_OK;
}

extern "C" int tgx_ep_load_shared(tgx_ep* ep, int layer, const void* src, int src_on_device) {
    EP_CHECK(ep && src, TG_EINVAL, "tgx_ep_load_shared: null argument");
    EP_CHECK(ep->n_shared == 1, TG_EINVAL, "tgx_ep_load_shared: context has no shared expert");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_load_shared: layer out of range");
    Dev dg(ep->device);
    const Geom& g = ep->g;
    EP_CUDA(cudaMemcpyAsync(ep->staging, src, g.expert_bytes,
                            src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ep->s));
    uint8_t* dst = ep->shared + (size_t)layer * g.expert_bytes;
    EP_CUDA(tg::launch_repack_rows(ep->staging, dst, 2LL * g.I, g.nbH, ep->s));
    EP_CUDA(tg::launch_repack_rows(ep->staging + 2 * g.t_gu, dst + 2 * g.t_gu, g.H, g.nbI, ep->s));
    EP_CUDA(cudaStreamSynchronize(ep->s));
    return TG_OK;
}

extern "C" int tgx_ep_read_expert(tgx_ep* ep, int layer, int e, void* dst_host) {
    EP_CHECK(ep && dst_host, TG_EINVAL, "tgx_ep_read_expert: null argument");
    const bool is_shared = e == ep->shape.n_experts;
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers &&
                 ((e >= ep->e_lo && e < ep->e_lo + ep->e_n) || (is_shared && ep->n_shared)),
             TG_EINVAL, "tgx_ep_read_expert: layer out of range or expert not held by this rank");
    Dev dg(ep->device);
    const Geom& g = ep->g;
    const uint8_t* src = is_shared ? ep->shared + (size_t)layer * g.expert_bytes
                                   : ep->weights + (size_t)layer * ep->layer_bytes + (size_t)(e - ep->e_lo) * g.expert_bytes;
    EP_CUDA(tg::launch_unpack_rows(src, ep->staging, 2LL * g.I, g.nbH, ep->s));
    EP_CUDA(tg::launch_unpack_rows(src + 2 * g.t_gu, ep->staging + 2 * g.t_gu, g.H, g.nbI, ep->s));
    EP_CUDA(cudaMemcpyAsync(dst_host, ep->staging, g.expert_bytes, cudaMemcpyDeviceToHost, ep->s));
    EP_CUDA(cudaStreamSynchronize(ep->s));
    return TG_OK;
}

extern "C" int tgx_ep_set_router(tgx_ep* ep, int layer, const float* R, int src_on_device) {
    EP_CHECK(ep && R, TG_EINVAL, "tgx_ep_set_router: null argument");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_set_router: layer out of range");
    Dev dg(ep->device);
    const size_t n = (size_t)ep->shape.n_experts * ep->shape.embed;
    EP_CUDA(cudaMemcpyAsync(ep->routers + (size_t)layer * n, R, n * sizeof(float),
                            src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ep->s));
    if (ep->RT)   // the fused path's transposed copy
        EP_CUDA(tg::launch_transpose(ep->routers + (size_t)layer * n, ep->RT + (size_t)layer * n,
                                     ep->shape.n_experts, ep->shape.embed, ep->s));
    EP_CUDA(cudaStreamSynchronize(ep->s));
    return TG_OK;
}

extern "C" int tgx_ep_set_ffn_norm(tgx_ep* ep, int layer, const float* w, int src_on_device) {
    EP_CHECK(ep && w, TG_EINVAL, "tgx_ep_set_ffn_norm: null argument");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_set_ffn_norm: layer out of range");
    Dev dg(ep->device);
    EP_CUDA(cudaMemcpyAsync(ep->norms + (size_t)layer * ep->shape.embed, w, sizeof(float) * ep->shape.embed,
                            src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ep->s));
    EP_CUDA(cudaStreamSynchronize(ep->s));
    return TG_OK;
}

extern "C" int tgx_ep_fill_synthetic(tgx_ep* ep, uint64_t seed, float w_sigma, float r_sigma) {
    EP_CHECK(ep, TG_EINVAL, "tgx_ep_fill_synthetic: null context");
    Dev dg(ep->device);
    const Geom& g = ep->g;
    const tgx_shape& sh = ep->shape;
    const unsigned long long per_expert = 3ULL * g.H * g.I;
    for (int l = 0; l < sh.n_layers; l++) {
        // the values tgx_fill_synthetic gives experts e_lo .. e_lo + e_n - 1 of a full model
        const unsigned long long base = ((unsigned long long)l * sh.n_experts + ep->e_lo) * per_expert;
        EP_CUDA(tg::launch_fill_experts_q4_0(ep->weights + (size_t)l * ep->layer_bytes, ep->e_n, g, seed, base,
                                             w_sigma, ep->s));
        const size_t nr = (size_t)sh.n_experts * sh.embed;
        EP_CUDA(tg::launch_fill_normal(ep->routers + (size_t)l * nr, (long long)nr, seed ^ 0x5DEECE66Dull,
                                       (unsigned long long)l * nr * 2, r_sigma, ep->s));
        if (ep->n_shared)   // its own stream of values: layer l's shared expert at l * per_expert
            EP_CUDA(tg::launch_fill_experts_q4_0(ep->shared + (size_t)l * g.expert_bytes, 1, g, seed ^ 0xC2B2AE3D27D4EB4Full,
                                                 (unsigned long long)l * per_expert, w_sigma, ep->s));
        if (ep->RT)
            EP_CUDA(tg::launch_transpose(ep->routers + (size_t)l * nr, ep->RT + (size_t)l * nr, sh.n_experts,
                                         sh.embed, ep->s));
    }
    EP_CUDA(cudaStreamSynchronize(ep->s));
    return TG_OK;
}

extern "C" size_t tgx_ep_y_floats(const tgx_ep* ep, int T) {
    return ep && T > 0 ? (size_t)T * (ep->shape.top_k + ep->n_shared) * ep->shape.embed : 0;
}

extern "C" int tgx_ep_moe_partial(tgx_ep* ep, int layer, const float* x_dev, int T, float* y_dev, void* stream) {
    EP_CHECK(ep && x_dev && y_dev, TG_EINVAL, "tgx_ep_moe_partial: null argument");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_moe_partial: layer out of range");
    EP_CHECK(T >= 1 && T <= 65536 / ep->shape.top_k, TG_EINVAL, "tgx_ep_moe_partial: T must be in [1, 65536/top_k]");
    Dev dg(ep->device);
    cudaStream_t s = (cudaStream_t)stream;
    int optin = 0;
    EP_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ep->device));
    EP_CHECK(tg::batched_smem_bytes(ep->g) <= (size_t)optin, TG_EUNSUPPORTED,
             "tgx_ep_moe_partial: shape needs more shared memory per block than the device has");
    EP_TRY(ep_reserve(ep, T, s, "tgx_ep_moe_partial"));
    const tgx_shape& sh = ep->shape;
    const size_t nr = (size_t)sh.n_experts * sh.embed;
    const uint8_t* shared = ep->n_shared ? ep->shared + (size_t)layer * ep->g.expert_bytes : nullptr;
    EP_CUDA(tg::launch_moe_batched_partial(ep->weights + (size_t)layer * ep->layer_bytes, shared, ep->e_lo, ep->e_n,
                                           ep->rank, ep->size, ep->g, ep->routers + (size_t)layer * nr,
                                           ep->norms + (size_t)layer * sh.embed, ep->eps, sh.n_experts, ep->n_shared,
                                           sh.top_k, x_dev, T, ep->scratch, ep->scratch_bytes, y_dev, nullptr, ep->wts,
                                           nullptr, ep->kernels, s));
    ep->last_T = T;
    return TG_OK;
}

extern "C" int tgx_ep_combine(tgx_ep* ep, float* x_dev, int T, const float* y_dev, void* stream) {
    EP_CHECK(ep && x_dev && y_dev, TG_EINVAL, "tgx_ep_combine: null argument");
    EP_CHECK(T >= 1 && T == ep->last_T, TG_EINVAL, "tgx_ep_combine: T must match the last tgx_ep_moe_partial");
    Dev dg(ep->device);
    EP_CUDA(tg::launch_moe_batched_combine(x_dev, T, ep->shape.embed, ep->shape.top_k + ep->n_shared, ep->wts,
                                           y_dev, (cudaStream_t)stream));
    return TG_OK;
}

extern "C" int tgx_ep_set_kernels(tgx_ep* ep, int kernels) {
    EP_CHECK(ep && kernels >= 0 && kernels <= 3, TG_EINVAL,
             "tgx_ep_set_kernels: kernels must be 0 (auto), 1 (dp4a), 2 (tensor cores) or 3 (tensor cores, fast "
             "epilogue)");
    ep->kernels = kernels;
    return TG_OK;
}

extern "C" int tgx_ep_status(tgx_ep* ep, void* stream) {
    EP_CHECK(ep, TG_EINVAL, "tgx_ep_status: null context");
    Dev dg(ep->device);
    EP_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    // the partial step's flag and the token dispatch's
    for (void* f : {ep->scratch, ep->dscratch}) {
        if (!f) continue;
        unsigned flag = 0;
        EP_CUDA(cudaMemcpy(&flag, f, sizeof(flag), cudaMemcpyDeviceToHost));
        if (flag) {
            EP_CUDA(cudaMemset(f, 0, sizeof(flag)));
            return ep_fail(TG_ETIMEOUT, "tgx_ep: a tensor-core expert kernel's bounded wait expired");
        }
    }
    return TG_OK;
}

// ------------------------------------------------------------ the NVLink exchange

namespace {

constexpr long long EP_WAIT_CYCLES = 2000000000ll;   // ~1 s

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// grid = T * ks CTAs, after this rank's partial step on the same stream: CTA i < owned[0]
// copies the i-th pair this rank computed (its y row, H floats, contiguous) into buffer
// b = epoch & 1 of every rank, this one included, with 16-byte stores (over NVLink for
// the peers), fenced system-wide; the last CTA to finish publishes the next epoch in
// this rank's slot of every rank's flags.  The buffer follows the call count, not the
// layer, so consecutive calls alternate buffers for any layer count and under graph
// replay: a rank stores into buffer b again only after seeing every rank's flag of
// the call in between, which each rank publishes after its combine of this call.
__global__ void __launch_bounds__(256) k_ep_push_signal(const int* __restrict__ owned, const float* __restrict__ y,
                                                        float* const* __restrict__ dst, int G, int rank, int H,
                                                        unsigned* count, unsigned* epoch, unsigned* const* flags) {
    const int i = blockIdx.x;
    // every CTA reads the epoch before its atomicAdd below; the last CTA advances it
    // only after all of them have added
    const unsigned b = *(volatile unsigned*)epoch & 1u;
    if (i < owned[0]) {
        const int p = owned[1 + i];
        const float4* src = reinterpret_cast<const float4*>(y + (size_t)p * H);
        for (int q = 0; q < G; q++) {
            float4* d = reinterpret_cast<float4*>(dst[(size_t)b * G + q] + (size_t)p * H);
            for (int c = threadIdx.x; c < H / 4; c += blockDim.x) d[c] = __ldcg(src + c);
        }
        __threadfence_system();
    }
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(count, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence_system();
        *count = 0u;
        const unsigned e = *epoch + 1u;
        *epoch = e;
        for (int q = 0; q < G; q++) st_release_sys(flags[q] + rank, e);
    }
}

// grid T: wait (bounded) until every rank published this call's epoch e, then
// x[t] += sum_j w[t][j] * y[(t, j)] in slot order from this rank's buffer (e - 1) & 1,
// the one the push of this call filled.
__global__ void __launch_bounds__(256) k_ep_combine_p2p(float* __restrict__ X, int H, int ks,
                                                        const float* __restrict__ wts, const uint8_t* region,
                                                        size_t y_bytes, const unsigned* flags, const unsigned* epoch,
                                                        int G, unsigned* err) {
    __shared__ int ok;
    const unsigned e = *(const volatile unsigned*)epoch;
    const float* y = reinterpret_cast<const float*>(region + (size_t)((e - 1u) & 1u) * y_bytes);
    if (threadIdx.x == 0) {
        int good = 1;
        const long long t0 = clock64();
        for (int q = 0; q < G && good; q++)
            while ((int)(ld_acquire_sys(flags + q) - e) < 0)
                if (clock64() - t0 > EP_WAIT_CYCLES) {
                    good = 0;
                    break;
                }
        if (!good) atomicExch(err, 1u);
        ok = good;
    }
    __syncthreads();
    if (!ok) return;
    const int t = blockIdx.x;
    for (int r = threadIdx.x; r < H; r += blockDim.x) {
        float a = 0.0f;
        for (int j = 0; j < ks; j++)
            a = __fadd_rn(a, __fmul_rn(wts[(size_t)t * ks + j], __ldcg(y + ((size_t)t * ks + j) * H + r)));
        X[(size_t)t * H + r] = __fadd_rn(X[(size_t)t * H + r], a);
    }
}

}  // namespace

extern "C" int tgx_ep_p2p_init(tgx_ep* ep, int T_max, void* handle_out) {
    EP_CHECK(ep && handle_out, TG_EINVAL, "tgx_ep_p2p_init: null argument");
    EP_CHECK(T_max >= 1 && T_max <= 65536 / ep->shape.top_k, TG_EINVAL, "tgx_ep_p2p_init: T_max out of range");
    EP_CHECK(!ep->region, TG_EINVAL, "tgx_ep_p2p_init: already initialised");
    EP_CHECK(ep->size <= 64, TG_EINVAL, "tgx_ep_p2p_init: at most 64 ranks");
    Dev dg(ep->device);
    const size_t ks = (size_t)ep->shape.top_k + ep->n_shared;
    ep->p2p_T = T_max;
    ep->y_bytes = ((size_t)T_max * ks * ep->shape.embed * 4 + 255) & ~(size_t)255;
    ep->region_bytes = 2 * ep->y_bytes + 256;
    EP_TRY(ep_alloc((void**)&ep->region, ep->region_bytes, "tgx_ep_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->ystage, ep->y_bytes, "tgx_ep_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->dst_dev, sizeof(float*) * 2 * ep->size, "tgx_ep_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->flag_dev, sizeof(unsigned*) * ep->size, "tgx_ep_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->epoch, 256, "tgx_ep_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->p2p_err, 256, "tgx_ep_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->p2p_count, 256, "tgx_ep_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->owned, sizeof(int) * (1 + (size_t)T_max * ks), "tgx_ep_p2p_init"));
    EP_CUDA(cudaMemset(ep->region + 2 * ep->y_bytes, 0, 256));   // flags
    EP_CUDA(cudaMemset(ep->epoch, 0, 256));
    EP_CUDA(cudaMemset(ep->p2p_err, 0, 256));
    EP_CUDA(cudaMemset(ep->p2p_count, 0, 256));
    cudaIpcMemHandle_t h;
    EP_CUDA(cudaIpcGetMemHandle(&h, ep->region));
    memcpy(handle_out, &h, sizeof(h));
    return TG_OK;
}

extern "C" int tgx_ep_p2p_connect(tgx_ep* ep, const void* handles) {
    EP_CHECK(ep && handles, TG_EINVAL, "tgx_ep_p2p_connect: null argument");
    EP_CHECK(ep->region && !ep->p2p_ready, TG_EINVAL, "tgx_ep_p2p_connect: call tgx_ep_p2p_init first, once");
    Dev dg(ep->device);
    const int G = ep->size;
    std::vector<uint8_t*> base(G);
    for (int q = 0; q < G; q++) {
        if (q == ep->rank) {
            base[q] = ep->region;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t*)handles + (size_t)q * sizeof(h), sizeof(h));
        EP_CUDA(cudaIpcOpenMemHandle(&ep->peers[q], h, cudaIpcMemLazyEnablePeerAccess));
        base[q] = (uint8_t*)ep->peers[q];
    }
    std::vector<float*> dst(2 * G);
    std::vector<unsigned*> fl(G);
    for (int q = 0; q < G; q++) {
        dst[q] = (float*)base[q];
        dst[G + q] = (float*)(base[q] + ep->y_bytes);
        fl[q] = (unsigned*)(base[q] + 2 * ep->y_bytes);
    }
    EP_CUDA(cudaMemcpy(ep->dst_dev, dst.data(), sizeof(float*) * 2 * G, cudaMemcpyHostToDevice));
    EP_CUDA(cudaMemcpy(ep->flag_dev, fl.data(), sizeof(unsigned*) * G, cudaMemcpyHostToDevice));
    ep->p2p_ready = true;
    return TG_OK;
}

extern "C" size_t tgx_ep_p2p_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int tgx_ep_p2p_disconnect(tgx_ep* ep) {
    EP_CHECK(ep, TG_EINVAL, "tgx_ep_p2p_disconnect: null context");
    Dev dg(ep->device);
    EP_CUDA(cudaDeviceSynchronize());
    for (int q = 0; q < 64; q++) {
        if (ep->peers[q]) {
            EP_CUDA(cudaIpcCloseMemHandle(ep->peers[q]));
            ep->peers[q] = nullptr;
        }
        if (ep->fpeers[q]) {
            EP_CUDA(cudaIpcCloseMemHandle(ep->fpeers[q]));
            ep->fpeers[q] = nullptr;
        }
        if (ep->dp_peers[q]) {
            EP_CUDA(cudaIpcCloseMemHandle(ep->dp_peers[q]));
            ep->dp_peers[q] = nullptr;
        }
    }
    ep->p2p_ready = false;
    ep->fused_ready = false;
    ep->dp_ready = false;
    return TG_OK;
}

extern "C" int tgx_ep_moe_layer_p2p(tgx_ep* ep, int layer, float* x_dev, int T, void* stream) {
    EP_CHECK(ep && x_dev, TG_EINVAL, "tgx_ep_moe_layer_p2p: null argument");
    EP_CHECK(ep->p2p_ready, TG_EINVAL, "tgx_ep_moe_layer_p2p: exchange not connected (tgx_ep_p2p_connect)");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_moe_layer_p2p: layer out of range");
    EP_CHECK(T >= 1 && T <= ep->p2p_T, TG_EINVAL, "tgx_ep_moe_layer_p2p: T must be in [1, the T_max of p2p_init]");
    Dev dg(ep->device);
    cudaStream_t s = (cudaStream_t)stream;
    int optin = 0;
    EP_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ep->device));
    EP_CHECK(tg::batched_smem_bytes(ep->g) <= (size_t)optin, TG_EUNSUPPORTED,
             "tgx_ep_moe_layer_p2p: shape needs more shared memory per block than the device has");
    EP_TRY(ep_reserve(ep, T, s, "tgx_ep_moe_layer_p2p"));
    const tgx_shape& sh = ep->shape;
    const size_t nr = (size_t)sh.n_experts * sh.embed;
    const int G = ep->size, ks = sh.top_k + ep->n_shared;
    const uint8_t* shared = ep->n_shared ? ep->shared + (size_t)layer * ep->g.expert_bytes : nullptr;
    float* y = ep->ystage;
    EP_CUDA(tg::launch_moe_batched_partial(ep->weights + (size_t)layer * ep->layer_bytes, shared, ep->e_lo, ep->e_n,
                                           ep->rank, G, ep->g, ep->routers + (size_t)layer * nr,
                                           ep->norms + (size_t)layer * sh.embed, ep->eps, sh.n_experts, ep->n_shared,
                                           sh.top_k, x_dev, T, ep->scratch, ep->scratch_bytes, y, nullptr, ep->wts,
                                           nullptr, ep->kernels, s, false, ep->owned));
    k_ep_push_signal<<<T * ks, 256, 0, s>>>(ep->owned, y, ep->dst_dev, G, ep->rank, sh.embed, ep->p2p_count,
                                            ep->epoch, ep->flag_dev);
    EP_CUDA(cudaGetLastError());
    k_ep_combine_p2p<<<T, 256, 0, s>>>(x_dev, sh.embed, ks, ep->wts, ep->region, ep->y_bytes,
                                        (const unsigned*)(ep->region + 2 * ep->y_bytes), ep->epoch, G, ep->p2p_err);
    EP_CUDA(cudaGetLastError());
    ep->last_T = T;
    return TG_OK;
}

extern "C" int tgx_ep_p2p_status(tgx_ep* ep, void* stream) {
    EP_CHECK(ep, TG_EINVAL, "tgx_ep_p2p_status: null context");
    if (!ep->p2p_err) return TG_OK;
    Dev dg(ep->device);
    EP_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    unsigned flag = 0;
    EP_CUDA(cudaMemcpy(&flag, ep->p2p_err, sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag) {
        EP_CUDA(cudaMemset(ep->p2p_err, 0, sizeof(flag)));
        return ep_fail(TG_ETIMEOUT, "tgx_ep_moe_layer_p2p: a peer's exchange flag did not arrive within the wait limit");
    }
    return TG_OK;
}

// ------------------------------------------------------------ fused decode, experts sharded

// The one-kernel decode step (k_decode_fused) with this rank's experts: every rank
// routes every layer, streams the gate/up and down rows of the slots whose expert it
// holds, and stores each output row's per-slot down value into every rank's y buffer
// over NVLink (tagged 64-bit words, no flag, no fence); each rank then combines all
// k slots of its rows in slot order, so every rank ends each layer with the same
// hidden state, bit-identical to one device (tinygiant/engine.py:229-258 per layer).
extern "C" int tgx_ep_fused_init(tgx_ep* ep, void* handle_out) {
    EP_CHECK(ep && handle_out, TG_EINVAL, "tgx_ep_fused_init: null argument");
    EP_CHECK(!ep->ybuf, TG_EINVAL, "tgx_ep_fused_init: already initialised");
    EP_CHECK(ep->n_shared == 0, TG_EUNSUPPORTED, "tgx_ep_fused_init: the fused path has no shared expert");
    EP_CHECK(ep->size <= 64, TG_EINVAL, "tgx_ep_fused_init: at most 64 ranks");
    Dev dg(ep->device);
    const tgx_shape& sh = ep->shape;
    const int L = sh.n_layers, E = sh.n_experts, k = sh.top_k, H = sh.embed;
    int sms = 0, smem_optin = 0;
    EP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ep->device));
    EP_CUDA(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ep->device));
    // the limits of the one-device fused path (count tags, fixed-point sums, 16-byte
    // router columns, at most 32 polled words per thread)
    EP_CHECK(sms <= 255 && H <= 16384 && E % 4 == 0 &&
                 (size_t)H + (size_t)tg::FUSED_ACC * (E + 1) <= 32u * tg::FUSED_THREADS &&
                 (size_t)k * ep->g.nbI * 6 <= 32u * tg::FUSED_THREADS,
             TG_EUNSUPPORTED, "tgx_ep_fused_init: shape outside the fused path's limits");
    std::vector<uint16_t> plan;
    size_t arena = 0;
    int max_rows = 0, k_early = 0;
    EP_CHECK(tg::fused_plan(ep->g, E, k, sms, plan, arena, max_rows, k_early) == 0, TG_EUNSUPPORTED,
             "tgx_ep_fused_init: shape does not fit one CTA per SM");
    // The kernel assigns a layer's units per CTA from the number of local slots (units
    // c, c + G, ... of nloc * nbI) and puts the local down rows after them, or into the
    // first unit's space when they do not fit the arena: check every CTA and count.
    {
        const size_t gu_b = 2 * 32 * ep->g.row_gu;
        for (int c = 0; c < sms; c++) {
            const size_t rows = plan[(size_t)c * tg::FUSED_PLAN + 2];
            for (int nloc = 0; nloc <= k; nloc++) {
                const int nu = nloc * ep->g.nbI, n = c < nu ? (nu - 1 - c) / sms + 1 : 0;
                const size_t down = (size_t)nloc * rows * ep->g.row_d;
                const bool fits = n * gu_b + down <= arena || (n > 0 && down <= gu_b);
                EP_CHECK(n <= tg::FUSED_MAX_GU && fits, TG_EUNSUPPORTED,
                         "tgx_ep_fused_init: a CTA's units and down rows do not fit its arena");
            }
        }
    }
    const size_t nr = (size_t)L * E * H;
    ep->ybuf_bytes = sizeof(unsigned long long) * 2 * (size_t)L * k * H;
    EP_TRY(ep_alloc((void**)&ep->RT, sizeof(float) * nr, "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->xw, sizeof(unsigned long long) * (size_t)(L + 1) * H, "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->facc, sizeof(unsigned long long) * (size_t)L * tg::FUSED_ACC * (E + 1),
                    "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->hqt, sizeof(unsigned long long) * (size_t)L * k * ep->g.nbI * 6, "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->ctl, 256, "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->plan, plan.size() * sizeof(uint16_t), "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->fidx, sizeof(int) * (size_t)L * k, "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->fw, sizeof(float) * (size_t)L * k, "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->flogits, sizeof(float) * (size_t)L * E, "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->ybuf, ep->ybuf_bytes, "tgx_ep_fused_init"));
    EP_TRY(ep_alloc((void**)&ep->ypeer, sizeof(void*) * ep->size, "tgx_ep_fused_init"));
    EP_CUDA(cudaMemset(ep->xw, 0, sizeof(unsigned long long) * (size_t)(L + 1) * H));
    EP_CUDA(cudaMemset(ep->facc, 0, sizeof(unsigned long long) * (size_t)L * tg::FUSED_ACC * (E + 1)));
    EP_CUDA(cudaMemset(ep->hqt, 0, sizeof(unsigned long long) * (size_t)L * k * ep->g.nbI * 6));
    EP_CUDA(cudaMemset(ep->ctl, 0, 256));
    EP_CUDA(cudaMemset(ep->ybuf, 0, ep->ybuf_bytes));
    EP_CUDA(cudaMemcpy(ep->plan, plan.data(), plan.size() * sizeof(uint16_t), cudaMemcpyHostToDevice));
    for (int l = 0; l < L; l++)
        EP_CUDA(tg::launch_transpose(ep->routers + (size_t)l * E * H, ep->RT + (size_t)l * E * H, E, H, ep->s));
    EP_CUDA(cudaStreamSynchronize(ep->s));
    tg::FusedParams& P = ep->fp;
    P = tg::FusedParams{};
    P.weights = ep->weights;
    P.layer_bytes = ep->layer_bytes;
    P.g = ep->g;
    P.RT = ep->RT;
    P.normw = ep->norms;
    P.eps = ep->eps;
    P.E = E;
    P.k = k;
    P.L0 = 0;
    P.nL = L;
    P.max_rows = max_rows;
    P.k_early = 0;
    P.wait_cycles = tg::FUSED_WAIT_CYCLES;
    P.missing = 0;
    P.xw = ep->xw;
    P.acc = ep->facc;
    P.hqt = ep->hqt;
    P.Lmax = L;
    P.ctl = ep->ctl;
    P.plan = ep->plan;
    P.idx_out = ep->fidx;
    P.w_out = ep->fw;
    P.logits_out = ep->flogits;
    P.trace = nullptr;
    P.arena_bytes = arena;
    P.e_lo = ep->e_lo;
    P.e_n = ep->e_n;
    P.ep_rank = ep->rank;
    P.ep_size = ep->size;
    P.ypeer = ep->ypeer;
    EP_CHECK(tg::fused_smem_layout(P).total <= (uint32_t)smem_optin, TG_EUNSUPPORTED,
             "tgx_ep_fused_init: shape needs more shared memory per block than the device has");
    EP_CUDA(tg::fused_prepare(P));
    int per_sm = 0;
    EP_CUDA(tg::fused_occupancy(P, &per_sm));
    EP_CHECK(per_sm >= 1, TG_EUNSUPPORTED, "tgx_ep_fused_init: the kernel does not fit one CTA per SM");
    ep->fG = sms;
    cudaIpcMemHandle_t h;
    EP_CUDA(cudaIpcGetMemHandle(&h, ep->ybuf));
    memcpy(handle_out, &h, sizeof(h));
    return TG_OK;
}

extern "C" int tgx_ep_fused_connect(tgx_ep* ep, const void* handles) {
    EP_CHECK(ep && handles, TG_EINVAL, "tgx_ep_fused_connect: null argument");
    EP_CHECK(ep->ybuf && !ep->fused_ready, TG_EINVAL, "tgx_ep_fused_connect: call tgx_ep_fused_init first, once");
    Dev dg(ep->device);
    const int G = ep->size;
    std::vector<unsigned long long*> base(G);
    for (int q = 0; q < G; q++) {
        if (q == ep->rank) {
            base[q] = ep->ybuf;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t*)handles + (size_t)q * sizeof(h), sizeof(h));
        EP_CUDA(cudaIpcOpenMemHandle(&ep->fpeers[q], h, cudaIpcMemLazyEnablePeerAccess));
        base[q] = (unsigned long long*)ep->fpeers[q];
    }
    EP_CUDA(cudaMemcpy(ep->ypeer, base.data(), sizeof(void*) * G, cudaMemcpyHostToDevice));
    ep->fused_ready = true;
    return TG_OK;
}

namespace {
int ep_fused_launch(tgx_ep* ep, const tg::FusedParams& base, float* x_dev, cudaStream_t s) {
    tg::FusedParams P = base;
    P.x_in = x_dev;
    P.x_out = x_dev;   // in place: nL >= 2, or a one-layer model whose CTAs all read x first
    EP_CHECK(ep->shape.n_layers >= 2 || ep->shape.top_k * ep->g.nbI >= ep->fG, TG_EUNSUPPORTED,
             "tgx_ep_decode_step: a one-layer model needs a gate/up unit in every CTA");
    EP_CUDA(tg::launch_decode_fused(P, ep->fG, s));
    return TG_OK;
}
}  // namespace

extern "C" int tgx_ep_decode_step(tgx_ep* ep, float* x_dev, void* stream) {
    EP_CHECK(ep && x_dev, TG_EINVAL, "tgx_ep_decode_step: null argument");
    EP_CHECK(ep->fused_ready, TG_EINVAL, "tgx_ep_decode_step: call tgx_ep_fused_init and tgx_ep_fused_connect first");
    Dev dg(ep->device);
    return ep_fused_launch(ep, ep->fp, x_dev, (cudaStream_t)stream);
}

extern "C" int tgx_ep_fused_trace(tgx_ep* ep, float* x_dev, uint64_t* stamps_host, void* stream) {
    EP_CHECK(ep && x_dev && stamps_host, TG_EINVAL, "tgx_ep_fused_trace: null argument");
    EP_CHECK(ep->fused_ready, TG_EINVAL, "tgx_ep_fused_trace: call tgx_ep_fused_init and tgx_ep_fused_connect first");
    Dev dg(ep->device);
    const size_t n = (size_t)ep->shape.n_layers * ep->fG * tg::FUSED_TRACE;
    unsigned long long* buf = nullptr;
    EP_TRY(ep_alloc((void**)&buf, n * 8, "tgx_ep_fused_trace"));
    tg::FusedParams P = ep->fp;
    P.trace = buf;
    cudaError_t e = cudaMemset(buf, 0, n * 8);
    int rc = e == cudaSuccess ? ep_fused_launch(ep, P, x_dev, (cudaStream_t)stream)
                              : ep_fail(TG_ECUDA, std::string("tgx_ep_fused_trace: ") + cudaGetErrorString(e));
    if (rc == TG_OK) {
        e = cudaStreamSynchronize((cudaStream_t)stream);
        if (e == cudaSuccess) e = cudaMemcpy(stamps_host, buf, n * 8, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = ep_fail(TG_ECUDA, std::string("tgx_ep_fused_trace: ") + cudaGetErrorString(e));
    }
    cudaFree(buf);
    return rc;
}

extern "C" int tgx_ep_fused_info(tgx_ep* ep, int* ctas, int* smem_bytes) {
    EP_CHECK(ep, TG_EINVAL, "tgx_ep_fused_info: null context");
    if (ctas) *ctas = ep->ybuf ? ep->fG : 0;
    if (smem_bytes) *smem_bytes = ep->ybuf ? (int)tg::fused_smem_layout(ep->fp).total : 0;
    return TG_OK;
}

extern "C" int tgx_ep_set_wait_limit(tgx_ep* ep, long long cycles) {
    EP_CHECK(ep, TG_EINVAL, "tgx_ep_set_wait_limit: null context");
    EP_CHECK(cycles == 0 || cycles >= 1000, TG_EINVAL, "tgx_ep_set_wait_limit: cycles must be 0 (default) or >= 1000");
    ep->fp.wait_cycles = cycles ? cycles : tg::FUSED_WAIT_CYCLES;
    return TG_OK;
}

extern "C" int tgx_ep_fused_last_routing(tgx_ep* ep, int layer, int32_t* idx, float* w) {
    EP_CHECK(ep && ep->fidx, TG_EINVAL, "tgx_ep_fused_last_routing: null context or fused path not initialised");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_fused_last_routing: layer out of range");
    Dev dg(ep->device);
    EP_CUDA(cudaDeviceSynchronize());
    const int k = ep->shape.top_k;
    if (idx) EP_CUDA(cudaMemcpy(idx, ep->fidx + (size_t)layer * k, sizeof(int) * k, cudaMemcpyDeviceToHost));
    if (w) EP_CUDA(cudaMemcpy(w, ep->fw + (size_t)layer * k, sizeof(float) * k, cudaMemcpyDeviceToHost));
    return TG_OK;
}

// An expired wait inside the fused step: TG_ETIMEOUT with where it happened.  The
// state stays as it was; recover with tgx_ep_fused_reset on every rank.
extern "C" int tgx_ep_fused_status(tgx_ep* ep, void* stream) {
    EP_CHECK(ep, TG_EINVAL, "tgx_ep_fused_status: null context");
    if (!ep->ctl) return TG_OK;
    Dev dg(ep->device);
    EP_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    unsigned ctl[4];
    EP_CUDA(cudaMemcpy(ctl, ep->ctl, sizeof(ctl), cudaMemcpyDeviceToHost));
    if (ctl[2] == 0) return TG_OK;
    return ep_fail(TG_ETIMEOUT, "tgx_ep_decode_step: a bounded device wait expired (stage " + std::to_string(ctl[2]) +
                                    ", layer " + std::to_string(ctl[3] >> 20) + ", entry " +
                                    std::to_string((ctl[3] >> 8) & 0xfff) + ")");
}

// Steps this rank has completed (the launch count that tags the y words).
extern "C" int tgx_ep_fused_epoch(tgx_ep* ep, unsigned* epoch) {
    EP_CHECK(ep && epoch && ep->ctl, TG_EINVAL, "tgx_ep_fused_epoch: null argument or fused path not initialised");
    Dev dg(ep->device);
    EP_CUDA(cudaDeviceSynchronize());
    EP_CUDA(cudaMemcpy(epoch, ep->ctl, sizeof(unsigned), cudaMemcpyDeviceToHost));
    return TG_OK;
}

// Recovery after a failed step (an expired wait, or a rank that did not take part):
// clear this rank's cross-CTA state and restart the launch count at `epoch`.  Every
// rank calls it with the same value, above every rank's tgx_ep_fused_epoch (so the
// y words stored by the failed step, tagged at most with the old count + 1, are
// never taken), once no rank has a step in flight.
extern "C" int tgx_ep_fused_reset(tgx_ep* ep, unsigned epoch) {
    EP_CHECK(ep && ep->ctl, TG_EINVAL, "tgx_ep_fused_reset: null context or fused path not initialised");
    Dev dg(ep->device);
    EP_CUDA(cudaDeviceSynchronize());
    const tgx_shape& sh = ep->shape;
    EP_CUDA(cudaMemset(ep->facc, 0, sizeof(unsigned long long) * (size_t)sh.n_layers * tg::FUSED_ACC * (sh.n_experts + 1)));
    EP_CUDA(cudaMemset(ep->xw, 0, sizeof(unsigned long long) * (size_t)(sh.n_layers + 1) * sh.embed));
    EP_CUDA(cudaMemset(ep->hqt, 0, sizeof(unsigned long long) * (size_t)sh.n_layers * sh.top_k * ep->g.nbI * 6));
    const unsigned fresh[4] = {epoch, 0, 0, 0};
    EP_CUDA(cudaMemcpy(ep->ctl, fresh, sizeof(fresh), cudaMemcpyHostToDevice));
    return TG_OK;
}

// ------------------------------------------------------------ token dispatch

// Every rank holds its own tokens.  Per layer:
//   tgx_ep_dispatch          route this rank's T tokens (the batched path's routing and
//                            Q8_0 activation rows), then one record per (token, slot) pair
//                            in destination-rank order: a routed slot goes to its
//                            expert's holder, the shared slot stays here; per-rank counts
//   (caller)                 exchange the counts, then the records (any all-to-all)
//   tgx_ep_dispatch_experts  the received records' expert FFNs: y [n][H], record order
//   (caller)                 send each y row back to the record's sender (the reverse
//                            all-to-all, so rows return in send order)
//   tgx_ep_dispatch_combine  x[t] += sum_j w[t][j] * y[(t, j)] in slot order
// A record carries the pair's Q8_0 activation row in ggml form (nbH blocks of fp16 scale +
// 32 codes) behind 16 bytes of header (expert id).  The expert kernels are the batched
// path's and each pair's arithmetic is independent of the others, so the result is the
// single-device batched path's bit for bit (tinygiant/engine.py:229-258 per token).

namespace {

using tg::ActView;
using tg::act_bytes;
using tg::act_view;
using tg::f16_bits_to_f32;
using tg::f32_to_f16_bits;

constexpr int REC_HDR = 16;

size_t rec_bytes(const Geom& g) { return REC_HDR + (size_t)g.nbH * 34; }
size_t r256(size_t n) { return (n + 255) & ~(size_t)255; }

// one CTA of 1024 threads: destination of every pair, counts per rank, and a record
// index per pair (destination-major; the order inside a destination does not affect
// any result); send_map[record] = pair
__global__ void __launch_bounds__(1024) k_dispatch_plan(const int* __restrict__ idx, int n_pairs, int ks, int k,
                                                        int e_n, int rank, int G, int* __restrict__ counts,
                                                        int* __restrict__ pair_slot, int* __restrict__ send_map) {
    __shared__ int cnt[64], base[65];
    for (int q = threadIdx.x; q < G; q += blockDim.x) cnt[q] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < n_pairs; p += blockDim.x) {
        const int j = p % ks;
        atomicAdd(&cnt[j < k ? idx[p] / e_n : rank], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int a = 0;
        for (int q = 0; q < G; q++) {
            base[q] = a;
            counts[q] = cnt[q];
            a += cnt[q];
            cnt[q] = 0;
        }
        base[G] = a;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < n_pairs; p += blockDim.x) {
        const int j = p % ks, q = j < k ? idx[p] / e_n : rank;
        const int slot = base[q] + atomicAdd(&cnt[q], 1);
        pair_slot[p] = slot;
        send_map[slot] = p;
    }
}

// grid n_records, 128 threads: record i = pair p = send_map[i] of token t: header (expert
// id, p) and the token's Q8_0 row in ggml form (the fp16 scale is the activation's own, exact)
__global__ void __launch_bounds__(128) k_dispatch_pack(const int* __restrict__ send_map, const int* __restrict__ idx,
                                                       int ks, int nb, const uint8_t* __restrict__ xq,
                                                       uint8_t* __restrict__ out, size_t rec) {
    const int i = blockIdx.x, p = send_map[i], t = p / ks;
    uint8_t* r = out + (size_t)i * rec;
    if (threadIdx.x < 4) reinterpret_cast<int*>(r)[threadIdx.x] = threadIdx.x == 0 ? idx[p] : threadIdx.x == 1 ? p : 0;
    const ActView a = act_view(const_cast<uint8_t*>(xq) + (size_t)t * act_bytes(nb), nb);
    // a 34-byte block starts on a 2-byte boundary (records are 16-byte aligned): the scale
    // and the codes go as 17 little-endian 16-bit words
    uint16_t* blk = reinterpret_cast<uint16_t*>(r + REC_HDR);
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
        uint16_t* o = blk + (size_t)b * 17;
        o[0] = f32_to_f16_bits(a.d[b]);
        const uint8_t* q = reinterpret_cast<const uint8_t*>(a.qs) + (size_t)b * 32;
        for (int c = 0; c < 16; c++) o[1 + c] = (uint16_t)(q[2 * c] | (q[2 * c + 1] << 8));
    }
}

// grid n_records, 128 threads: a received record into the activation form (codes, fp32 of
// the fp16 scale, 8 * sum of codes) and its expert id
__global__ void __launch_bounds__(128) k_dispatch_unpack(const uint8_t* __restrict__ in, size_t rec, int nb,
                                                         uint8_t* __restrict__ xq, int* __restrict__ idx) {
    const int i = blockIdx.x;
    const uint8_t* r = in + (size_t)i * rec;
    if (threadIdx.x == 0) idx[i] = reinterpret_cast<const int*>(r)[0];
    ActView a = act_view(xq + (size_t)i * act_bytes(nb), nb);
    const uint16_t* blk = reinterpret_cast<const uint16_t*>(r + REC_HDR);
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
        const uint16_t* o = blk + (size_t)b * 17;
        a.d[b] = f16_bits_to_f32(o[0]);
        int sum = 0;
        for (int c = 0; c < 16; c++) {
            const uint16_t w = o[1 + c];
            const int8_t q0 = (int8_t)(w & 0xff), q1 = (int8_t)(w >> 8);
            a.qs[(size_t)b * 32 + 2 * c] = q0;
            a.qs[(size_t)b * 32 + 2 * c + 1] = q1;
            sum += q0 + q1;
        }
        a.s8[b] = 8 * sum;
    }
}

// grid T, 256 threads: x[t][r] += sum over slots j in order of w[t][j] * y_back[pair_slot[t*ks+j]][r]
__global__ void __launch_bounds__(256) k_dispatch_combine(float* __restrict__ X, int H, int ks,
                                                          const float* __restrict__ wts,
                                                          const int* __restrict__ pair_slot,
                                                          const float* __restrict__ y) {
    const int t = blockIdx.x;
    for (int r = threadIdx.x; r < H; r += blockDim.x) {
        float a = 0.0f;
        for (int j = 0; j < ks; j++)
            a = __fadd_rn(a, __fmul_rn(wts[(size_t)t * ks + j], __ldg(y + (size_t)pair_slot[(size_t)t * ks + j] * H + r)));
        X[(size_t)t * H + r] = __fadd_rn(X[(size_t)t * H + r], a);
    }
}

// The dispatch scratch: an error flag for the expert step's tensor-core kernels, the
// routing buffers of T own tokens (S, xq, idx, wts, pair_slot, send_map: offsets that
// depend on T only), then the receive side for n_recv records (activation rows,
// expert ids, the expert step's scratch).
struct DispatchLayout {
    size_t S, xq, idx, wts, slot, map, route_end, rxq, ridx, xs, total;
};
DispatchLayout dispatch_layout(const tgx_ep* ep, int T, int n_recv) {
    const Geom& g = ep->g;
    const int E = ep->shape.n_experts, ks = ep->shape.top_k + ep->n_shared;
    DispatchLayout L;
    size_t o = 256;
    auto take = [&](size_t n) {
        const size_t r = o;
        o += r256(n);
        return r;
    };
    L.S = take((size_t)T * E * 8);
    L.xq = take((size_t)T * tg::act_bytes(g.nbH));
    L.idx = take((size_t)T * ks * 4);
    L.wts = take((size_t)T * ks * 4);
    L.slot = take((size_t)T * ks * 4);
    L.map = take((size_t)T * ks * 4);
    L.route_end = o;
    L.rxq = take((size_t)n_recv * tg::act_bytes(g.nbH));
    L.ridx = take((size_t)n_recv * 4);
    L.xs = take(tg::experts_scratch_bytes(g, E, ep->n_shared, (size_t)(n_recv > 0 ? n_recv : 1)));
    L.total = o;
    return L;
}

// grow the dispatch scratch to L, keeping the first `keep` bytes (the flag and a
// pending dispatch's routing buffers)
int dispatch_reserve(tgx_ep* ep, const DispatchLayout& L, size_t keep, cudaStream_t s, const char* fn) {
    if (L.total <= ep->dscratch_bytes) return TG_OK;
    EP_CUDA(cudaStreamSynchronize(s));
    void* fresh = nullptr;
    EP_TRY(ep_alloc(&fresh, L.total, fn));
    if (ep->dscratch && keep)
        EP_CUDA(cudaMemcpy(fresh, ep->dscratch, keep < ep->dscratch_bytes ? keep : ep->dscratch_bytes,
                           cudaMemcpyDeviceToDevice));
    else
        EP_CUDA(cudaMemset(fresh, 0, 256));   // the error flag
    if (ep->dscratch) cudaFree(ep->dscratch);
    ep->dscratch = fresh;
    ep->dscratch_bytes = L.total;
    return TG_OK;
}

}  // namespace

extern "C" size_t tgx_ep_record_bytes(const tgx_ep* ep) { return ep ? rec_bytes(ep->g) : 0; }

extern "C" int tgx_ep_dispatch(tgx_ep* ep, int layer, const float* x_dev, int T, void* send_dev, int* counts_dev,
                               void* stream) {
    EP_CHECK(ep && x_dev && send_dev && counts_dev, TG_EINVAL, "tgx_ep_dispatch: null argument");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_dispatch: layer out of range");
    EP_CHECK(T >= 1 && T <= 65536 / ep->shape.top_k, TG_EINVAL, "tgx_ep_dispatch: T must be in [1, 65536/top_k]");
    EP_CHECK(ep->size <= 64, TG_EINVAL, "tgx_ep_dispatch: at most 64 ranks");
    Dev dg(ep->device);
    cudaStream_t s = (cudaStream_t)stream;
    const tgx_shape& sh = ep->shape;
    const int ks = sh.top_k + ep->n_shared;
    const DispatchLayout L = dispatch_layout(ep, T, 0);
    EP_TRY(dispatch_reserve(ep, L, 256, s, "tgx_ep_dispatch"));
    uint8_t* base = (uint8_t*)ep->dscratch;
    auto* S = (unsigned long long*)(base + L.S);
    uint8_t* xq = base + L.xq;
    int* idx = (int*)(base + L.idx);
    float* wts = (float*)(base + L.wts);
    int* slot = (int*)(base + L.slot);
    int* map = (int*)(base + L.map);
    const size_t nr = (size_t)sh.n_experts * sh.embed;
    EP_CUDA(tg::launch_batched_route(ep->g, ep->routers + (size_t)layer * nr, ep->norms + (size_t)layer * sh.embed,
                                     ep->eps, sh.n_experts, ep->n_shared, sh.top_k, x_dev, T, S, idx, wts, nullptr, xq,
                                     s));
    k_dispatch_plan<<<1, 1024, 0, s>>>(idx, T * ks, ks, sh.top_k, ep->e_n, ep->rank, ep->size, counts_dev, slot, map);
    EP_CUDA(cudaGetLastError());
    k_dispatch_pack<<<T * ks, 128, 0, s>>>(map, idx, ks, ep->g.nbH, xq, (uint8_t*)send_dev, rec_bytes(ep->g));
    EP_CUDA(cudaGetLastError());
    ep->d_T = T;
    ep->d_wts = wts;
    ep->d_slot = slot;
    return TG_OK;
}

extern "C" int tgx_ep_dispatch_experts(tgx_ep* ep, int layer, const void* recv_dev, int n_recv, float* y_dev,
                                       void* stream) {
    EP_CHECK(ep && (n_recv == 0 || (recv_dev && y_dev)), TG_EINVAL, "tgx_ep_dispatch_experts: null argument");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_dispatch_experts: layer out of range");
    EP_CHECK(ep->d_T > 0, TG_EINVAL, "tgx_ep_dispatch_experts: call tgx_ep_dispatch first");
    EP_CHECK(n_recv >= 0 && n_recv <= 65536 * 64, TG_EINVAL, "tgx_ep_dispatch_experts: bad record count");
    if (n_recv == 0) return TG_OK;
    Dev dg(ep->device);
    cudaStream_t s = (cudaStream_t)stream;
    int optin = 0;
    EP_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ep->device));
    EP_CHECK(tg::batched_smem_bytes(ep->g) <= (size_t)optin, TG_EUNSUPPORTED,
             "tgx_ep_dispatch_experts: shape needs more shared memory per block than the device has");
    const DispatchLayout L = dispatch_layout(ep, ep->d_T, n_recv);
    EP_TRY(dispatch_reserve(ep, L, L.route_end, s, "tgx_ep_dispatch_experts"));
    uint8_t* base = (uint8_t*)ep->dscratch;
    ep->d_wts = (float*)(base + L.wts);
    ep->d_slot = (int*)(base + L.slot);
    uint8_t* rxq = base + L.rxq;
    int* ridx = (int*)(base + L.ridx);
    k_dispatch_unpack<<<n_recv, 128, 0, s>>>((const uint8_t*)recv_dev, rec_bytes(ep->g), ep->g.nbH, rxq, ridx);
    EP_CUDA(cudaGetLastError());
    const tgx_shape& sh = ep->shape;
    const uint8_t* shared = ep->n_shared ? ep->shared + (size_t)layer * ep->g.expert_bytes : nullptr;
    const int E_tot = sh.n_experts + ep->n_shared;
    // every received record is computed here: rank 0 of one with all experts "owned"
    EP_CUDA(tg::launch_batched_experts(ep->weights + (size_t)layer * ep->layer_bytes, shared, sh.n_experts, ep->e_lo,
                                       E_tot, 0, 1, ep->g, ep->n_shared, 1, 1, ridx, n_recv, rxq, base + L.xs,
                                       L.total - L.xs, y_dev, nullptr, ep->kernels, ep->e_n + ep->n_shared, s,
                                       (unsigned*)base));
    return TG_OK;
}

extern "C" int tgx_ep_dispatch_combine(tgx_ep* ep, float* x_dev, int T, const float* y_back_dev, void* stream) {
    EP_CHECK(ep && x_dev && y_back_dev, TG_EINVAL, "tgx_ep_dispatch_combine: null argument");
    EP_CHECK(T >= 1 && T == ep->d_T, TG_EINVAL, "tgx_ep_dispatch_combine: T must match the last tgx_ep_dispatch");
    Dev dg(ep->device);
    k_dispatch_combine<<<T, 256, 0, (cudaStream_t)stream>>>(x_dev, ep->shape.embed, ep->shape.top_k + ep->n_shared,
                                                            ep->d_wts, ep->d_slot, y_back_dev);
    EP_CUDA(cudaGetLastError());
    return TG_OK;
}

// ------------------------------------------------------------ token dispatch over NVLink

// The same exchange as tgx_ep_dispatch*, device-side: no host sync, capturable in a
// CUDA graph.  Rank r's region: records in [2][G][cap][rec] (half, source, position),
// y rows back [2][G][cap][H] (half, destination, position), record flags [2][G] and
// y flags [2][G] (64-bit: (call + 1) << 32 | count).  Per call (one layer), with
// e = calls so far and half e & 1:
//   route, plan             this rank's tokens, records grouped by destination
//   k_dp_pack_push          record i of destination q's group at position pos into q's
//                           region [half][r][pos] (NVLink for peers); fence, and the last
//                           CTA stores every destination's flag with its count
//   k_dp_wait               wait (bounded) for all G record flags; counts -> receive prefix
//   k_dp_unpack             records -> activation rows, expert ids, (source, position)
//   experts                 the batched expert kernels, the pair count read on the device
//   k_dp_return             y row of received record (q, pos) into q's region [half][r][pos];
//                           fence, the last CTA stores every source's y flag
//   k_dp_combine            wait (bounded) for all G y flags, x[t] += sum_j w_j * y_j in slot
//                           order; the last CTA advances the call count
// A rank reaches call e + 2 (the same half) only after every rank's y flags of call e + 1,
// which each rank stores after finishing call e: a half is never rewritten while read.

namespace {

struct DpGeom {
    size_t rec, cap, off_yb, off_rflag, off_yflag;
    int G, H;
};
DpGeom dp_geom(const tgx_ep* ep) {
    DpGeom d;
    d.G = ep->size;
    d.H = ep->shape.embed;
    d.rec = rec_bytes(ep->g);
    d.cap = ep->dp_cap;
    size_t o = r256(2 * (size_t)d.G * d.cap * d.rec);
    d.off_yb = o;
    o += r256(2 * (size_t)d.G * d.cap * d.H * 4);
    d.off_rflag = o;
    o += r256(2 * (size_t)d.G * 8);
    d.off_yflag = o;
    return d;
}
size_t dp_region_bytes(const DpGeom& d) { return d.off_yflag + r256(2 * (size_t)d.G * 8); }

__device__ __forceinline__ uint8_t* dp_rec(uint8_t* base, const DpGeom& d, unsigned half, int src, size_t pos) {
    return base + (((size_t)half * d.G + src) * d.cap + pos) * d.rec;
}
__device__ __forceinline__ float* dp_yb(uint8_t* base, const DpGeom& d, unsigned half, int dst, size_t pos) {
    return reinterpret_cast<float*>(base + d.off_yb) + (((size_t)half * d.G + dst) * d.cap + pos) * d.H;
}
__device__ __forceinline__ unsigned long long* dp_flag(uint8_t* base, size_t off, const DpGeom& d, unsigned half,
                                                       int q) {
    return reinterpret_cast<unsigned long long*>(base + off) + (size_t)half * d.G + q;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// the group a sorted index i falls in: pre[q] <= i < pre[q + 1]
__device__ __forceinline__ int dp_group(const int* pre, int G, int i) {
    int q = 0;
    while (q + 1 < G && pre[q + 1] <= i) q++;
    return q;
}

// one thread: the send order's group starts, pre[q] = records for ranks < q (pre[G] = all)
__global__ void k_dp_prefix(const int* __restrict__ counts, int G, int* __restrict__ pre) {
    if (threadIdx.x == 0) {
        int a = 0;
        for (int q = 0; q < G; q++) {
            pre[q] = a;
            a += counts[q];
        }
        pre[G] = a;
    }
}

// grid n_records, 128 threads (the plan's send order): pack record i into its
// destination's region, then the last CTA publishes every destination's flag
__global__ void __launch_bounds__(128) k_dp_pack_push(const int* __restrict__ send_map, const int* __restrict__ idx,
                                                      int ks, int nb, const uint8_t* __restrict__ xq,
                                                      const int* __restrict__ counts, const int* __restrict__ pre,
                                                      uint8_t* const* __restrict__ bases, int rank, DpGeom d,
                                                      unsigned* ctl) {
    __shared__ int last;
    const unsigned e = *(volatile unsigned*)ctl, half = e & 1u;
    const int i = blockIdx.x, p = send_map[i], t = p / ks;
    const int q = dp_group(pre, d.G, i);
    uint8_t* r = dp_rec(bases[q], d, half, rank, (size_t)(i - pre[q]));
    if (threadIdx.x < 4) reinterpret_cast<int*>(r)[threadIdx.x] = threadIdx.x == 0 ? idx[p] : threadIdx.x == 1 ? p : 0;
    const ActView a = act_view(const_cast<uint8_t*>(xq) + (size_t)t * act_bytes(nb), nb);
    uint16_t* blk = reinterpret_cast<uint16_t*>(r + REC_HDR);
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
        uint16_t* o = blk + (size_t)b * 17;
        o[0] = f32_to_f16_bits(a.d[b]);
        const uint8_t* c = reinterpret_cast<const uint8_t*>(a.qs) + (size_t)b * 32;
        for (int u = 0; u < 16; u++) o[1 + u] = (uint16_t)(c[2 * u] | (c[2 * u + 1] << 8));
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(ctl + 1, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last) {
        __threadfence_system();
        if ((int)threadIdx.x < d.G)
            st_release_sys_u64(dp_flag(bases[threadIdx.x], d.off_rflag, d, half, rank),
                               ((unsigned long long)(e + 1u) << 32) | (unsigned)counts[threadIdx.x]);
        if (threadIdx.x == 0) ctl[1] = 0u;
    }
}

// one CTA of 64 threads: wait (bounded) for every source's record flag of this call;
// receive prefix and count into meta[65 ..]
__global__ void __launch_bounds__(64) k_dp_wait(uint8_t* own, DpGeom d, unsigned* ctl, int* meta, long long limit) {
    __shared__ int cnt[64];
    __shared__ int bad;
    const unsigned e = *(volatile unsigned*)ctl, half = e & 1u;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    const int q = threadIdx.x;
    if (q < d.G) {
        const unsigned long long* f = dp_flag(own, d.off_rflag, d, half, q);
        const long long t0 = clock64();
        unsigned long long v = ld_acquire_sys_u64(f);
        while ((unsigned)(v >> 32) != e + 1u) {
            if (clock64() - t0 > limit) {
                atomicExch(&bad, 1);
                break;
            }
            v = ld_acquire_sys_u64(f);
        }
        cnt[q] = (unsigned)(v >> 32) == e + 1u ? (int)(unsigned)v : 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int a = 0;
        for (int s = 0; s < d.G; s++) {
            meta[65 + s] = a;
            a += cnt[s];
        }
        meta[65 + d.G] = a;
        meta[131] = bad ? 0 : a;
        if (bad) atomicExch(ctl + 4, 1u);
    }
}

// grid-stride over the received records: activation rows, expert ids, (source, position)
__global__ void __launch_bounds__(128) k_dp_unpack(uint8_t* own, DpGeom d, const unsigned* ctl,
                                                   const int* __restrict__ meta, int nb, uint8_t* __restrict__ xq,
                                                   int* __restrict__ idx, int* __restrict__ rsrc,
                                                   int* __restrict__ rpos) {
    const unsigned half = *(volatile const unsigned*)ctl & 1u;
    const int n = meta[131];
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        const int q = dp_group(meta + 65, d.G, i), pos = i - meta[65 + q];
        const uint8_t* r = dp_rec(own, d, half, q, (size_t)pos);
        if (threadIdx.x == 0) {
            idx[i] = __ldcg(reinterpret_cast<const int*>(r));
            rsrc[i] = q;
            rpos[i] = pos;
        }
        ActView a = act_view(xq + (size_t)i * act_bytes(nb), nb);
        const unsigned short* blk = reinterpret_cast<const unsigned short*>(r + REC_HDR);
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            const unsigned short* o = blk + (size_t)b * 17;
            a.d[b] = f16_bits_to_f32(__ldcg(o));
            int sum = 0;
            for (int c = 0; c < 16; c++) {
                const unsigned short w = __ldcg(o + 1 + c);
                const int8_t q0 = (int8_t)(w & 0xff), q1 = (int8_t)(w >> 8);
                a.qs[(size_t)b * 32 + 2 * c] = q0;
                a.qs[(size_t)b * 32 + 2 * c + 1] = q1;
                sum += q0 + q1;
            }
            a.s8[b] = 8 * sum;
        }
    }
}

// grid-stride over the received records: y row i back into its source's region at the
// record's position; then the last CTA publishes every source's y flag
__global__ void __launch_bounds__(256) k_dp_return(const float* __restrict__ y, const int* __restrict__ meta,
                                                   const int* __restrict__ rsrc, const int* __restrict__ rpos,
                                                   uint8_t* const* __restrict__ bases, int rank, DpGeom d,
                                                   unsigned* ctl) {
    __shared__ int last;
    const unsigned e = *(volatile unsigned*)ctl, half = e & 1u;
    const int n = meta[131];
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        float4* dst = reinterpret_cast<float4*>(dp_yb(bases[rsrc[i]], d, half, rank, (size_t)rpos[i]));
        const float4* src = reinterpret_cast<const float4*>(y + (size_t)i * d.H);
        for (int c = threadIdx.x; c < d.H / 4; c += blockDim.x) dst[c] = __ldcg(src + c);
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(ctl + 2, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last) {
        __threadfence_system();
        if ((int)threadIdx.x < d.G)
            st_release_sys_u64(dp_flag(bases[threadIdx.x], d.off_yflag, d, half, rank),
                               (unsigned long long)(e + 1u) << 32);
        if (threadIdx.x == 0) ctl[2] = 0u;
    }
}

// grid T, 256 threads: wait (bounded) for every destination's y flag of this call, then
// x[t] += sum over slots j in order of w[t][j] * y[(t, j)] (y from this rank's region at
// the pair's destination and position); the last CTA advances the call count
__global__ void __launch_bounds__(256) k_dp_combine(float* __restrict__ X, int ks, const float* __restrict__ wts,
                                                    const int* __restrict__ pair_slot, const int* __restrict__ pre,
                                                    uint8_t* own, DpGeom d, unsigned* ctl, long long limit) {
    __shared__ int ok, last;
    __shared__ const float* yp[32];
    const unsigned e = *(volatile unsigned*)ctl, half = e & 1u;
    const int t = blockIdx.x;
    if (threadIdx.x == 0) {
        int good = 1;
        const long long t0 = clock64();
        for (int q = 0; q < d.G && good; q++) {
            const unsigned long long* f = dp_flag(own, d.off_yflag, d, half, q);
            while ((unsigned)(ld_acquire_sys_u64(f) >> 32) != e + 1u)
                if (clock64() - t0 > limit) {
                    good = 0;
                    break;
                }
        }
        if (!good) atomicExch(ctl + 4, 1u);
        ok = good;
    }
    if ((int)threadIdx.x < ks) {
        const int s = pair_slot[(size_t)t * ks + threadIdx.x];
        const int q = dp_group(pre, d.G, s);
        yp[threadIdx.x] = dp_yb(own, d, half, q, (size_t)(s - pre[q]));
    }
    __syncthreads();
    if (ok) {
        for (int r = threadIdx.x; r < d.H; r += blockDim.x) {
            float a = 0.0f;
            for (int j = 0; j < ks; j++) a = __fadd_rn(a, __fmul_rn(wts[(size_t)t * ks + j], __ldcg(yp[j] + r)));
            X[(size_t)t * d.H + r] = __fadd_rn(X[(size_t)t * d.H + r], a);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(ctl + 3, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        ctl[3] = 0u;
        __threadfence();
        *(volatile unsigned*)ctl = e + 1u;
    }
}

// the work area for T tokens per call and N = G * cap received records at most
struct DpWork {
    size_t S, xq, idx, wts, slot, map, counts, rxq, ridx, rsrc, rpos, y, xs, total;
};
DpWork dp_work(const tgx_ep* ep) {
    const Geom& g = ep->g;
    const int E = ep->shape.n_experts, ks = ep->shape.top_k + ep->n_shared, T = ep->dp_T;
    const size_t N = (size_t)ep->size * ep->dp_cap;
    DpWork w;
    size_t o = 256;   // the expert step's error flag
    auto take = [&](size_t n) {
        const size_t r = o;
        o += r256(n);
        return r;
    };
    w.S = take((size_t)T * E * 8);
    w.xq = take((size_t)T * act_bytes(g.nbH));
    w.idx = take((size_t)T * ks * 4);
    w.wts = take((size_t)T * ks * 4);
    w.slot = take((size_t)T * ks * 4);
    w.map = take((size_t)T * ks * 4);
    w.counts = take(64 * 4);
    w.rxq = take(N * act_bytes(g.nbH));
    w.ridx = take(N * 4);
    w.rsrc = take(N * 4);
    w.rpos = take(N * 4);
    w.y = take(N * (size_t)g.H * 4);
    w.xs = take(tg::experts_scratch_bytes(g, E, ep->n_shared, N));
    w.total = o;
    return w;
}

}  // namespace

extern "C" int tgx_ep_dispatch_p2p_init(tgx_ep* ep, int T_max, void* handle_out) {
    EP_CHECK(ep && handle_out, TG_EINVAL, "tgx_ep_dispatch_p2p_init: null argument");
    EP_CHECK(!ep->dp_region, TG_EINVAL, "tgx_ep_dispatch_p2p_init: already initialised");
    EP_CHECK(T_max >= 1 && T_max <= 65536 / ep->shape.top_k, TG_EINVAL, "tgx_ep_dispatch_p2p_init: T_max out of range");
    EP_CHECK(ep->size <= 32, TG_EINVAL, "tgx_ep_dispatch_p2p_init: at most 32 ranks");
    EP_CHECK(ep->shape.top_k + ep->n_shared <= 32, TG_EINVAL, "tgx_ep_dispatch_p2p_init: at most 32 slots");
    Dev dg(ep->device);
    ep->dp_T = T_max;
    ep->dp_cap = (size_t)T_max * (ep->shape.top_k + ep->n_shared);
    const DpGeom d = dp_geom(ep);
    ep->dp_region_bytes = dp_region_bytes(d);
    const DpWork w = dp_work(ep);
    ep->dp_work_bytes = w.total;
    EP_TRY(ep_alloc((void**)&ep->dp_region, ep->dp_region_bytes, "tgx_ep_dispatch_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->dp_bases, sizeof(void*) * ep->size, "tgx_ep_dispatch_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->dp_ctl, 256, "tgx_ep_dispatch_p2p_init"));
    EP_TRY(ep_alloc((void**)&ep->dp_meta, 256 * 4, "tgx_ep_dispatch_p2p_init"));
    EP_TRY(ep_alloc(&ep->dp_work, ep->dp_work_bytes, "tgx_ep_dispatch_p2p_init"));
    // flags start at call 0 (no flag matches call 0 + 1); the records and y rows need no clearing
    EP_CUDA(cudaMemset(ep->dp_region + d.off_rflag, 0, ep->dp_region_bytes - d.off_rflag));
    EP_CUDA(cudaMemset(ep->dp_ctl, 0, 256));
    EP_CUDA(cudaMemset(ep->dp_meta, 0, 256 * 4));
    EP_CUDA(cudaMemset(ep->dp_work, 0, 256));
    cudaIpcMemHandle_t h;
    EP_CUDA(cudaIpcGetMemHandle(&h, ep->dp_region));
    memcpy(handle_out, &h, sizeof(h));
    return TG_OK;
}

extern "C" int tgx_ep_dispatch_p2p_connect(tgx_ep* ep, const void* handles) {
    EP_CHECK(ep && handles, TG_EINVAL, "tgx_ep_dispatch_p2p_connect: null argument");
    EP_CHECK(ep->dp_region && !ep->dp_ready, TG_EINVAL,
             "tgx_ep_dispatch_p2p_connect: call tgx_ep_dispatch_p2p_init first, once");
    Dev dg(ep->device);
    std::vector<uint8_t*> base(ep->size);
    for (int q = 0; q < ep->size; q++) {
        if (q == ep->rank) {
            base[q] = ep->dp_region;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t*)handles + (size_t)q * sizeof(h), sizeof(h));
        EP_CUDA(cudaIpcOpenMemHandle(&ep->dp_peers[q], h, cudaIpcMemLazyEnablePeerAccess));
        base[q] = (uint8_t*)ep->dp_peers[q];
    }
    EP_CUDA(cudaMemcpy(ep->dp_bases, base.data(), sizeof(void*) * ep->size, cudaMemcpyHostToDevice));
    ep->dp_ready = true;
    return TG_OK;
}

extern "C" int tgx_ep_moe_layer_dispatch_p2p(tgx_ep* ep, int layer, float* x_dev, int T, void* stream) {
    EP_CHECK(ep && x_dev, TG_EINVAL, "tgx_ep_moe_layer_dispatch_p2p: null argument");
    EP_CHECK(ep->dp_ready, TG_EINVAL, "tgx_ep_moe_layer_dispatch_p2p: call tgx_ep_dispatch_p2p_init / _connect first");
    EP_CHECK(layer >= 0 && layer < ep->shape.n_layers, TG_EINVAL, "tgx_ep_moe_layer_dispatch_p2p: layer out of range");
    EP_CHECK(T >= 1 && T <= ep->dp_T, TG_EINVAL, "tgx_ep_moe_layer_dispatch_p2p: T must be in [1, the T_max of init]");
    Dev dg(ep->device);
    cudaStream_t s = (cudaStream_t)stream;
    int optin = 0;
    EP_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ep->device));
    EP_CHECK(tg::batched_smem_bytes(ep->g) <= (size_t)optin, TG_EUNSUPPORTED,
             "tgx_ep_moe_layer_dispatch_p2p: shape needs more shared memory per block than the device has");
    const tgx_shape& sh = ep->shape;
    const int ks = sh.top_k + ep->n_shared, G = ep->size;
    const DpGeom d = dp_geom(ep);
    const DpWork w = dp_work(ep);
    uint8_t* b = (uint8_t*)ep->dp_work;
    const size_t N = (size_t)G * ep->dp_cap;
    int* counts = (int*)(b + w.counts);
    int* pre = ep->dp_meta;   // send prefix [0 .. G]
    const size_t nr = (size_t)sh.n_experts * sh.embed;
    EP_CUDA(tg::launch_batched_route(ep->g, ep->routers + (size_t)layer * nr, ep->norms + (size_t)layer * sh.embed,
                                     ep->eps, sh.n_experts, ep->n_shared, sh.top_k, x_dev, T,
                                     (unsigned long long*)(b + w.S), (int*)(b + w.idx), (float*)(b + w.wts), nullptr,
                                     b + w.xq, s));
    k_dispatch_plan<<<1, 1024, 0, s>>>((int*)(b + w.idx), T * ks, ks, sh.top_k, ep->e_n, ep->rank, G, counts,
                                       (int*)(b + w.slot), (int*)(b + w.map));
    EP_CUDA(cudaGetLastError());
    k_dp_prefix<<<1, 32, 0, s>>>(counts, G, pre);
    EP_CUDA(cudaGetLastError());
    k_dp_pack_push<<<T * ks, 128, 0, s>>>((int*)(b + w.map), (int*)(b + w.idx), ks, ep->g.nbH, b + w.xq, counts, pre,
                                          ep->dp_bases, ep->rank, d, ep->dp_ctl);
    EP_CUDA(cudaGetLastError());
    k_dp_wait<<<1, 64, 0, s>>>(ep->dp_region, d, ep->dp_ctl, ep->dp_meta, EP_WAIT_CYCLES);
    EP_CUDA(cudaGetLastError());
    const unsigned grid_n = (unsigned)(N < 1184 ? N : 1184);
    k_dp_unpack<<<grid_n, 128, 0, s>>>(ep->dp_region, d, ep->dp_ctl, ep->dp_meta, ep->g.nbH, b + w.rxq,
                                       (int*)(b + w.ridx), (int*)(b + w.rsrc), (int*)(b + w.rpos));
    EP_CUDA(cudaGetLastError());
    const uint8_t* shared = ep->n_shared ? ep->shared + (size_t)layer * ep->g.expert_bytes : nullptr;
    // the expected received pairs per local expert picks the kernels (both give the same bits)
    EP_CUDA(tg::launch_batched_experts(ep->weights + (size_t)layer * ep->layer_bytes, shared, sh.n_experts, ep->e_lo,
                                       sh.n_experts + ep->n_shared, 0, 1, ep->g, ep->n_shared, 1, 1,
                                       (int*)(b + w.ridx), (int)N, b + w.rxq, b + w.xs, w.total - w.xs,
                                       (float*)(b + w.y), nullptr, ep->kernels,
                                       (int)((size_t)ep->e_n * N / ((size_t)T * ks) + ep->n_shared), s,
                                       (unsigned*)b, ep->dp_meta + 131));
    k_dp_return<<<grid_n, 256, 0, s>>>((float*)(b + w.y), ep->dp_meta, (int*)(b + w.rsrc), (int*)(b + w.rpos),
                                       ep->dp_bases, ep->rank, d, ep->dp_ctl);
    EP_CUDA(cudaGetLastError());
    k_dp_combine<<<T, 256, 0, s>>>(x_dev, ks, (float*)(b + w.wts), (int*)(b + w.slot), pre, ep->dp_region, d,
                                   ep->dp_ctl, EP_WAIT_CYCLES);
    EP_CUDA(cudaGetLastError());
    return TG_OK;
}

// Records and y rows this rank received and sent in its last call (synchronises).
extern "C" int tgx_ep_dispatch_p2p_counts(tgx_ep* ep, int* received, int* sent) {
    EP_CHECK(ep && ep->dp_meta, TG_EINVAL, "tgx_ep_dispatch_p2p_counts: null context or not initialised");
    Dev dg(ep->device);
    EP_CUDA(cudaDeviceSynchronize());
    int meta[132];
    EP_CUDA(cudaMemcpy(meta, ep->dp_meta, sizeof(meta), cudaMemcpyDeviceToHost));
    if (received) *received = meta[131];
    if (sent) *sent = meta[ep->size];
    return TG_OK;
}

extern "C" int tgx_ep_dispatch_p2p_status(tgx_ep* ep, void* stream) {
    EP_CHECK(ep, TG_EINVAL, "tgx_ep_dispatch_p2p_status: null context");
    if (!ep->dp_ctl) return TG_OK;
    Dev dg(ep->device);
    EP_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    unsigned flag = 0;
    EP_CUDA(cudaMemcpy(&flag, ep->dp_ctl + 4, sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag) {
        EP_CUDA(cudaMemset(ep->dp_ctl + 4, 0, sizeof(flag)));
        return ep_fail(TG_ETIMEOUT, "tgx_ep_moe_layer_dispatch_p2p: a peer's flag did not arrive within the wait limit");
    }
    return TG_OK;
}

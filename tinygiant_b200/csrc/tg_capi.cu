// tg_capi.cu — the C ABI declared in include/tinygiant.h.
//
// tg_*  : the reference library's entry points (csrc/libtinygiant.c) on host
//         pointers.  They share one device workspace per process (grown on
//         demand, guarded by a mutex) and are synchronous like the reference's.
// tgx_* : a context that owns an L x E expert model and L routers in HBM and
//         runs the routed MoE decode on caller streams.
#include <cuda_runtime.h>
#include <algorithm>
#include <sys/mman.h>
#include <cerrno>
#include <unistd.h>

#include <mutex>
#include <string>
#include <vector>

#include "../../include/tinygiant.h"
#include "tg_decode.h"
#include "tg_internal.h"

using tg::ActView;
using tg::Geom;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

#define TG_CUDA(call)                                                                         \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess)                                                                \
            return fail(e_ == cudaErrorMemoryAllocation ? TG_ENOMEM : TG_ECUDA,               \
                        std::string(#call) + ": " + cudaGetErrorString(e_));                  \
    } while (0)

#define TG_CHECK(cond, code, msg) \
    do {                          \
        if (!(cond)) return fail((code), (msg)); \
    } while (0)

int have_device() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

struct DevBuf {
    void* p = nullptr;
    size_t n = 0;
};

int ensure(DevBuf& b, size_t n) {
    if (b.n >= n && b.p) return TG_OK;
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.n = 0;
    size_t want = n < 256 ? 256 : n;
    if (cudaMalloc(&b.p, want) != cudaSuccess) {
        cudaGetLastError();
        return fail(TG_ENOMEM, "cudaMalloc of " + std::to_string(want) + " bytes failed");
    }
    b.n = want;
    return TG_OK;
}

// Device workspace of the host-pointer entry points.
struct HostWS {
    std::mutex mu;
    int device = -1;
    cudaStream_t s = nullptr;
    DevBuf raw, w, x, out, act, hq, ptrs, wts, i32, kqs, att;   // kqs: down counters must stay zero

    int bind() {
        int dev = 0;
        if (!have_device()) return fail(TG_ENODEV, "no CUDA device");
        if (cudaGetDevice(&dev) != cudaSuccess) return fail(TG_ECUDA, "cudaGetDevice failed");
        if (dev != device) {
            release();
            device = dev;
        }
        if (!s && cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
            return fail(TG_ECUDA, "cudaStreamCreate failed");
        return TG_OK;
    }
    void release() {
        for (DevBuf* b : {&raw, &w, &x, &out, &act, &hq, &ptrs, &wts, &i32, &kqs, &att}) {
            if (b->p) cudaFree(b->p);
            b->p = nullptr;
            b->n = 0;
        }
        if (s) cudaStreamDestroy(s);
        s = nullptr;
    }
};

HostWS& ws() {
    static HostWS* w = new HostWS();  // never destroyed: safe at process exit
    return *w;
}

#define TG_TRY(expr)            \
    do {                        \
        int rc_ = (expr);       \
        if (rc_ != TG_OK) return rc_; \
    } while (0)

// Copy a ggml expert blob already on the device (raw) into row-split form (dst).
cudaError_t repack_expert(const uint8_t* raw, uint8_t* dst, const Geom& g, cudaStream_t s) {
    cudaError_t e = tg::launch_repack_rows(raw, dst, 2LL * g.I, g.nbH, s);
    if (e != cudaSuccess) return e;
    return tg::launch_repack_rows(raw + 2 * g.t_gu, dst + 2 * g.t_gu, g.H, g.nbI, s);
}
cudaError_t unpack_expert(const uint8_t* src, uint8_t* raw, const Geom& g, cudaStream_t s) {
    cudaError_t e = tg::launch_unpack_rows(src, raw, 2LL * g.I, g.nbH, s);
    if (e != cudaSuccess) return e;
    return tg::launch_unpack_rows(src + 2 * g.t_gu, raw + 2 * g.t_gu, g.H, g.nbI, s);
}

// Expert forward of n experts already row-split on the device in ws.w
// (expert e at w + e * expert_bytes), on input ws.x, into ws.out.
int run_experts(HostWS& W, const Geom& g, int n, const float* weights_host, float w_scalar,
                int accumulate) {
    std::vector<const uint8_t*> ptrs(n);
    for (int e = 0; e < n; e++) ptrs[e] = (const uint8_t*)W.w.p + (size_t)e * g.expert_bytes;
    TG_TRY(ensure(W.ptrs, sizeof(void*) * n));
    TG_TRY(ensure(W.hq, tg::act_bytes(g.nbI) * n));
    TG_CUDA(cudaMemcpyAsync(W.ptrs.p, ptrs.data(), sizeof(void*) * n, cudaMemcpyHostToDevice, W.s));
    const float* wdev = nullptr;
    if (weights_host) {
        TG_TRY(ensure(W.wts, sizeof(float) * n));
        TG_CUDA(cudaMemcpyAsync(W.wts.p, weights_host, sizeof(float) * n, cudaMemcpyHostToDevice, W.s));
        wdev = (const float*)W.wts.p;
    }
    TG_CUDA(tg::prepare_kernels(g, n));
    TG_CUDA(tg::launch_gateup((const uint8_t* const*)W.ptrs.p, n, (const float*)W.x.p, nullptr, nullptr, g,
                              (uint8_t*)W.hq.p, nullptr, nullptr, W.s));
    TG_CUDA(tg::launch_down_combine((const uint8_t* const*)W.ptrs.p, n, (const uint8_t*)W.hq.p, wdev, w_scalar,
                                    g, nullptr, (float*)W.out.p, accumulate, nullptr, W.s));
    return TG_OK;
}

}  // namespace

namespace tg {
int set_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace tg

// ============================================================ reference-shaped

extern "C" const char* tg_last_error(void) { return g_err.c_str(); }
extern "C" int tg_version(void) { return 1; }
extern "C" int tg_device_count(void) { return have_device(); }

extern "C" int tg_quantize_q8_0(const float* x, void* out, int n) {
    TG_CHECK(x && out && n > 0 && n % 32 == 0, TG_EINVAL, "tg_quantize_q8_0: bad arguments");
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    int nb = n / 32;
    TG_TRY(ensure(W.x, sizeof(float) * n));
    TG_TRY(ensure(W.act, tg::act_bytes(nb)));
    TG_TRY(ensure(W.raw, (size_t)nb * tg::Q8_0_BYTES));
    TG_CUDA(cudaMemcpyAsync(W.x.p, x, sizeof(float) * n, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(tg::launch_quantize_act((const float*)W.x.p, n, tg::act_view(W.act.p, nb), (uint8_t*)W.raw.p, W.s));
    TG_CUDA(cudaMemcpyAsync(out, W.raw.p, (size_t)nb * tg::Q8_0_BYTES, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

extern "C" int tg_quantize_q4_0(const float* x, void* out, long long n) {
    TG_CHECK(x && out && n > 0 && n % 32 == 0, TG_EINVAL, "tg_quantize_q4_0: bad arguments");
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    long long nb = n / 32;
    TG_TRY(ensure(W.x, sizeof(float) * (size_t)n));
    TG_TRY(ensure(W.raw, (size_t)nb * tg::Q4_0_BYTES));
    TG_CUDA(cudaMemcpyAsync(W.x.p, x, sizeof(float) * (size_t)n, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(tg::launch_quantize_q4_0((const float*)W.x.p, n, (uint8_t*)W.raw.p, W.s));
    TG_CUDA(cudaMemcpyAsync(out, W.raw.p, (size_t)nb * tg::Q4_0_BYTES, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

extern "C" int tg_block_dots_q4_0(const uint8_t* Wq, const void* xq, int32_t* out, int nrows, int ncols) {
    TG_CHECK(Wq && xq && out && nrows > 0 && ncols > 0 && ncols % 256 == 0, TG_EINVAL,
             "tg_block_dots_q4_0: bad arguments (ncols must be a multiple of 256)");
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    int nb = ncols / 32;
    size_t wb = (size_t)nrows * nb * tg::Q4_0_BYTES;
    TG_TRY(ensure(W.raw, wb));
    TG_TRY(ensure(W.w, wb));
    TG_TRY(ensure(W.x, (size_t)nb * tg::Q8_0_BYTES));
    TG_TRY(ensure(W.act, tg::act_bytes(nb)));
    TG_TRY(ensure(W.i32, sizeof(int32_t) * (size_t)nrows * nb));
    TG_CUDA(cudaMemcpyAsync(W.raw.p, Wq, wb, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(cudaMemcpyAsync(W.x.p, xq, (size_t)nb * tg::Q8_0_BYTES, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(tg::launch_repack_rows((const uint8_t*)W.raw.p, (uint8_t*)W.w.p, nrows, nb, W.s));
    ActView a = tg::act_view(W.act.p, nb);
    TG_CUDA(tg::launch_q8_0_to_act((const uint8_t*)W.x.p, nb, a, W.s));
    TG_CUDA(tg::launch_block_dots((const uint8_t*)W.w.p, a, (int32_t*)W.i32.p, nrows, nb, W.s));
    TG_CUDA(cudaMemcpyAsync(out, W.i32.p, sizeof(int32_t) * (size_t)nrows * nb, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

extern "C" int tg_matmul_q4_0(const uint8_t* Wq, const float* input, float* output, int nrows, int ncols) {
    TG_CHECK(Wq && input && output && nrows > 0 && ncols > 0 && ncols % 256 == 0, TG_EINVAL,
             "tg_matmul_q4_0: bad arguments (ncols must be a multiple of 256)");
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    int nb = ncols / 32;
    size_t wb = (size_t)nrows * nb * tg::Q4_0_BYTES;
    TG_TRY(ensure(W.raw, wb));
    TG_TRY(ensure(W.w, wb));
    TG_TRY(ensure(W.x, sizeof(float) * ncols));
    TG_TRY(ensure(W.act, tg::act_bytes(nb)));
    TG_TRY(ensure(W.out, sizeof(float) * nrows));
    TG_CUDA(cudaMemcpyAsync(W.raw.p, Wq, wb, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(cudaMemcpyAsync(W.x.p, input, sizeof(float) * ncols, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(tg::launch_repack_rows((const uint8_t*)W.raw.p, (uint8_t*)W.w.p, nrows, nb, W.s));
    ActView a = tg::act_view(W.act.p, nb);
    TG_CUDA(tg::launch_quantize_act((const float*)W.x.p, ncols, a, nullptr, W.s));
    TG_CUDA(tg::launch_matvec((const uint8_t*)W.w.p, a, (float*)W.out.p, nrows, nb, W.s));
    TG_CUDA(cudaMemcpyAsync(output, W.out.p, sizeof(float) * nrows, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

static int expert_forward_parts(const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* input,
                                float* output, float weight, int embed, int inter) {
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    Geom g = Geom::make(embed, inter);
    TG_TRY(ensure(W.raw, g.expert_bytes));
    TG_TRY(ensure(W.w, g.expert_bytes));
    TG_TRY(ensure(W.x, sizeof(float) * embed));
    TG_TRY(ensure(W.out, sizeof(float) * embed));
    uint8_t* raw = (uint8_t*)W.raw.p;
    TG_CUDA(cudaMemcpyAsync(raw, gate, g.t_gu, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(cudaMemcpyAsync(raw + g.t_gu, up, g.t_gu, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(cudaMemcpyAsync(raw + 2 * g.t_gu, down, g.t_d, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(repack_expert(raw, (uint8_t*)W.w.p, g, W.s));
    TG_CUDA(cudaMemcpyAsync(W.x.p, input, sizeof(float) * embed, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(cudaMemcpyAsync(W.out.p, output, sizeof(float) * embed, cudaMemcpyHostToDevice, W.s));
    TG_TRY(run_experts(W, g, 1, nullptr, weight, 1));
    TG_CUDA(cudaMemcpyAsync(output, W.out.p, sizeof(float) * embed, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

extern "C" int tg_expert_forward_q4_0(const uint8_t* q4_data, const float* input, float* output, float weight,
                                      int embed_dim, int inter_dim) {
    TG_CHECK(q4_data && input && output, TG_EINVAL, "tg_expert_forward_q4_0: null pointer");
    TG_CHECK(Geom::valid_dims(embed_dim, inter_dim), TG_EINVAL,
             "tg_expert_forward_q4_0: embed/inter must be positive multiples of 256");
    Geom g = Geom::make(embed_dim, inter_dim);
    return expert_forward_parts(q4_data, q4_data + g.t_gu, q4_data + 2 * g.t_gu, input, output, weight,
                                embed_dim, inter_dim);
}

// ------------------------------------------------------------ the reference's own formats
// (csrc/libtinygiant.c: Q4_K, Q6_K, f16, f32, RMSNorm; kernels in tg_kquant.cu)

static size_t r256(size_t n) { return (n + 255) & ~(size_t)255; }

// Copy a host matrix in the reference's byte layout to dst in device layout (Q6_K is
// split through W.raw; the other formats are copied as they are).
static int kq_put(HostWS& W, int fmt, const void* src, long long rows, int cols, uint8_t* dst) {
    size_t nb = tg::kq_matrix_bytes(fmt, rows, cols);
    if (fmt == tg::KQ_Q6K) {
        TG_TRY(ensure(W.raw, nb));
        TG_CUDA(cudaMemcpyAsync(W.raw.p, src, nb, cudaMemcpyHostToDevice, W.s));
        TG_CUDA(tg::launch_kq_split_q6k((const uint8_t*)W.raw.p, dst, rows * (cols / 256), W.s));
    } else {
        TG_CUDA(cudaMemcpyAsync(dst, src, nb, cudaMemcpyHostToDevice, W.s));
    }
    return TG_OK;
}

static int kq_matvec_host(int fmt, const void* A, const float* x, float* out, int nrows, int ncols, const char* fn) {
    TG_CHECK(A && x && out, TG_EINVAL, std::string(fn) + ": null pointer");
    TG_CHECK(tg::kq_valid(fmt, nrows, ncols), TG_EINVAL,
             std::string(fn) + ": bad shape (rows > 0; ncols a multiple of 256 for Q4_K/Q6_K, of 8 for f16/f32)");
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    TG_TRY(ensure(W.w, tg::kq_matrix_bytes(fmt, nrows, ncols)));
    TG_TRY(ensure(W.x, sizeof(float) * ncols));
    TG_TRY(ensure(W.out, sizeof(float) * nrows));
    TG_TRY(kq_put(W, fmt, A, nrows, ncols, (uint8_t*)W.w.p));
    TG_CUDA(cudaMemcpyAsync(W.x.p, x, sizeof(float) * ncols, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(tg::launch_kq_matvec(fmt, (const uint8_t*)W.w.p, (const float*)W.x.p, (float*)W.out.p, nrows, ncols,
                                 W.s));
    TG_CUDA(cudaMemcpyAsync(out, W.out.p, sizeof(float) * nrows, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

extern "C" int tg_matmul_q4k(const uint8_t* q4_matrix, const float* input, float* output, int nrows, int ncols) {
    return kq_matvec_host(tg::KQ_Q4K, q4_matrix, input, output, nrows, ncols, "tg_matmul_q4k");
}
extern "C" int tg_matmul_q6k(const uint8_t* q6_matrix, const float* input, float* output, int nrows, int ncols) {
    return kq_matvec_host(tg::KQ_Q6K, q6_matrix, input, output, nrows, ncols, "tg_matmul_q6k");
}
extern "C" int tg_f16_matvec(const uint16_t* A, const float* x, float* out, int nrows, int ncols) {
    return kq_matvec_host(tg::KQ_F16, A, x, out, nrows, ncols, "tg_f16_matvec");
}
extern "C" int tg_f32_matvec(const float* A, const float* x, float* out, int nrows, int ncols) {
    return kq_matvec_host(tg::KQ_F32, A, x, out, nrows, ncols, "tg_f32_matvec");
}

extern "C" int tg_rms_norm(const float* x, const float* weight, float* out, int dim, float eps) {
    TG_CHECK(x && weight && out, TG_EINVAL, "tg_rms_norm: null pointer");
    TG_CHECK(dim > 0 && dim % 4 == 0, TG_EINVAL, "tg_rms_norm: dim must be a positive multiple of 4");
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    TG_TRY(ensure(W.x, sizeof(float) * dim));
    TG_TRY(ensure(W.wts, sizeof(float) * dim));
    TG_TRY(ensure(W.out, sizeof(float) * dim));
    TG_CUDA(cudaMemcpyAsync(W.x.p, x, sizeof(float) * dim, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(cudaMemcpyAsync(W.wts.p, weight, sizeof(float) * dim, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(tg::launch_rms_norm_ref((const float*)W.x.p, (const float*)W.wts.p, (float*)W.out.p, dim, eps, W.s));
    TG_CUDA(cudaMemcpyAsync(out, W.out.p, sizeof(float) * dim, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

// tg_attention_decode / tg_attention_decode_q4 on host buffers (csrc/libtinygiant.c:
// 364-551): the weights, the cached rows 0 .. kv_len - 1 and the rope rows of pos go
// to the device; the output and the appended cache row (kv_len) come back.
static int attention_host(int q4, const void* wq, const void* wk, const void* wv, const void* wo,
                          const float* q_norm_w, const float* k_norm_w, float* kv_k, float* kv_v, int kv_len,
                          int kv_max, const float* rope_cos, const float* rope_sin, const float* input,
                          float* output, int embed, int n_heads, int n_kv, int head_dim, int pos, const char* fn) {
    TG_CHECK(wq && wk && wv && wo && q_norm_w && k_norm_w && kv_k && kv_v && rope_cos && rope_sin && input && output,
             TG_EINVAL, std::string(fn) + ": null pointer");
    TG_CHECK(kv_len >= 0 && kv_len < kv_max && pos >= 0, TG_EINVAL,
             std::string(fn) + ": need 0 <= kv_len < kv_max and pos >= 0");
    const int seq = kv_len + 1;
    TG_CHECK(tg::attention_valid(q4, embed, n_heads, n_kv, head_dim, seq), TG_EINVAL,
             std::string(fn) + ": bad shape (head_dim a multiple of 8 in [8, 256]; n_heads a multiple of "
                               "n_kv_heads, at most 32 per kv head; kv_len < 32768)");
    const int qd = n_heads * head_dim, kvd = n_kv * head_dim, half = head_dim / 2;
    const int fq = q4 ? tg::KQ_Q4K : tg::KQ_F32, fv = q4 ? tg::KQ_F16 : tg::KQ_F32;
    auto r16 = [](size_t n) { return (n + 15) & ~(size_t)15; };
    const size_t bq = tg::kq_matrix_bytes(fq, qd, embed), bk = tg::kq_matrix_bytes(fq, kvd, embed),
                 bv = tg::kq_matrix_bytes(fv, kvd, embed), bo = tg::kq_matrix_bytes(fq, embed, qd);
    const size_t cache = (size_t)n_kv * seq * head_dim * sizeof(float);
    const size_t small = r16(sizeof(float) * (2 * head_dim + 2 * half + embed));
    const size_t scratch = tg::attention_scratch_bytes(n_heads, n_kv, head_dim, seq);
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    TG_TRY(ensure(W.w, r16(bq) + r16(bk) + r16(bv) + r16(bo)));
    TG_TRY(ensure(W.att, 2 * r16(cache) + small + scratch));
    TG_TRY(ensure(W.out, sizeof(float) * embed));
    uint8_t* wdev = (uint8_t*)W.w.p;
    uint8_t *dq = wdev, *dk = dq + r16(bq), *dv = dk + r16(bk), *dw = dv + r16(bv);
    uint8_t* sdev = (uint8_t*)W.att.p;
    float* ck = (float*)sdev;
    float* cv = (float*)(sdev + r16(cache));
    float* fs = (float*)(sdev + 2 * r16(cache));   // q_norm | k_norm | cos row | sin row | input
    void* scr = sdev + 2 * r16(cache) + small;
    cudaStream_t s = W.s;
    TG_CUDA(cudaMemcpyAsync(dq, wq, bq, cudaMemcpyHostToDevice, s));
    TG_CUDA(cudaMemcpyAsync(dk, wk, bk, cudaMemcpyHostToDevice, s));
    TG_CUDA(cudaMemcpyAsync(dv, wv, bv, cudaMemcpyHostToDevice, s));
    TG_CUDA(cudaMemcpyAsync(dw, wo, bo, cudaMemcpyHostToDevice, s));
    TG_CUDA(cudaMemcpyAsync(fs, q_norm_w, sizeof(float) * head_dim, cudaMemcpyHostToDevice, s));
    TG_CUDA(cudaMemcpyAsync(fs + head_dim, k_norm_w, sizeof(float) * head_dim, cudaMemcpyHostToDevice, s));
    TG_CUDA(cudaMemcpyAsync(fs + 2 * head_dim, rope_cos + (size_t)pos * half, sizeof(float) * half,
                            cudaMemcpyHostToDevice, s));
    TG_CUDA(cudaMemcpyAsync(fs + 2 * head_dim + half, rope_sin + (size_t)pos * half, sizeof(float) * half,
                            cudaMemcpyHostToDevice, s));
    float* xd = fs + 2 * head_dim + 2 * half;
    TG_CUDA(cudaMemcpyAsync(xd, input, sizeof(float) * embed, cudaMemcpyHostToDevice, s));
    const size_t hpitch = (size_t)kv_max * head_dim * sizeof(float), dpitch = (size_t)seq * head_dim * sizeof(float);
    if (kv_len > 0) {
        const size_t width = (size_t)kv_len * head_dim * sizeof(float);
        TG_CUDA(cudaMemcpy2DAsync(ck, dpitch, kv_k, hpitch, width, n_kv, cudaMemcpyHostToDevice, s));
        TG_CUDA(cudaMemcpy2DAsync(cv, dpitch, kv_v, hpitch, width, n_kv, cudaMemcpyHostToDevice, s));
    }
    // the device caches hold seq rows per head; the rope rows of pos sit at row 0
    TG_CUDA(tg::launch_attention(q4, dq, dk, dv, dw, fs, fs + head_dim, ck, cv, kv_len, seq, fs + 2 * head_dim,
                                 fs + 2 * head_dim + half, xd, (float*)W.out.p, embed, n_heads, n_kv, head_dim, 0,
                                 nullptr, scr, s));
    TG_CUDA(cudaMemcpyAsync(output, W.out.p, sizeof(float) * embed, cudaMemcpyDeviceToHost, s));
    const size_t row = (size_t)head_dim * sizeof(float);
    TG_CUDA(cudaMemcpy2DAsync(kv_k + (size_t)kv_len * head_dim, hpitch, ck + (size_t)kv_len * head_dim, dpitch, row,
                              n_kv, cudaMemcpyDeviceToHost, s));
    TG_CUDA(cudaMemcpy2DAsync(kv_v + (size_t)kv_len * head_dim, hpitch, cv + (size_t)kv_len * head_dim, dpitch, row,
                              n_kv, cudaMemcpyDeviceToHost, s));
    TG_CUDA(cudaStreamSynchronize(s));
    return TG_OK;
}

extern "C" int tg_attention_decode(const float* wq, const float* wk, const float* wv, const float* wo,
                                   const float* q_norm_w, const float* k_norm_w, float* kv_k, float* kv_v, int kv_len,
                                   int kv_max, const float* rope_cos, const float* rope_sin, const float* input,
                                   float* output, int embed_dim, int n_heads, int n_kv_heads, int head_dim, int pos) {
    return attention_host(0, wq, wk, wv, wo, q_norm_w, k_norm_w, kv_k, kv_v, kv_len, kv_max, rope_cos, rope_sin, input,
                          output, embed_dim, n_heads, n_kv_heads, head_dim, pos, "tg_attention_decode");
}

extern "C" int tg_attention_decode_q4(const uint8_t* wq_q4, const uint8_t* wk_q4, const uint16_t* wv_f16,
                                      const uint8_t* wo_q4, const float* q_norm_w, const float* k_norm_w, float* kv_k,
                                      float* kv_v, int kv_len, int kv_max, const float* rope_cos,
                                      const float* rope_sin, const float* input, float* output, int embed_dim,
                                      int n_heads, int n_kv_heads, int head_dim, int pos) {
    return attention_host(1, wq_q4, wk_q4, wv_f16, wo_q4, q_norm_w, k_norm_w, kv_k, kv_v, kv_len, kv_max, rope_cos,
                          rope_sin, input, output, embed_dim, n_heads, n_kv_heads, head_dim, pos,
                          "tg_attention_decode_q4");
}

// n experts with Q4_K gate/up and a down matrix of format fmt (host pointers):
// out = (accumulate ? output : 0) + sum_e w_e * expert_e(input), experts in order.
static int kq_experts_host(const uint8_t* const* gate, const uint8_t* const* up, const void* const* down, int fmt,
                           int n, const float* weights, float w_scalar, const float* input, float* output, int embed,
                           int inter, int accumulate, const char* fn) {
    TG_CHECK(n >= 1 && n <= 64, TG_EINVAL, std::string(fn) + ": 1 <= n_experts <= 64");
    for (int e = 0; e < n; e++)
        TG_CHECK(gate[e] && up[e] && down[e], TG_EINVAL, std::string(fn) + ": null expert pointer");
    TG_CHECK(Geom::valid_dims(embed, inter), TG_EINVAL,
             std::string(fn) + ": embed/inter must be positive multiples of 256 (<= 16384)");
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    const size_t gb = r256(tg::kq_matrix_bytes(tg::KQ_Q4K, inter, embed));
    const size_t db = r256(tg::kq_matrix_bytes(fmt, embed, inter));
    const size_t stride = 2 * gb + db;
    TG_TRY(ensure(W.w, stride * n));
    TG_TRY(ensure(W.x, sizeof(float) * embed));
    TG_TRY(ensure(W.out, sizeof(float) * embed));
    TG_TRY(ensure(W.hq, sizeof(float) * (size_t)n * inter));
    const size_t dsb = tg::kq_down_scratch_bytes(n, embed, inter);
    if (W.kqs.n < dsb) {   // the row-block counters start at zero; every launch leaves them zero
        TG_TRY(ensure(W.kqs, dsb));
        TG_CUDA(cudaMemsetAsync(W.kqs.p, 0, W.kqs.n, W.s));
    }
    TG_TRY(ensure(W.ptrs, sizeof(void*) * 3 * n));
    TG_TRY(ensure(W.wts, sizeof(float) * n));
    std::vector<const uint8_t*> ptrs(3 * n);
    for (int e = 0; e < n; e++) {
        uint8_t* base = (uint8_t*)W.w.p + stride * e;
        ptrs[e] = base;
        ptrs[n + e] = base + gb;
        ptrs[2 * n + e] = base + 2 * gb;
        TG_TRY(kq_put(W, tg::KQ_Q4K, gate[e], inter, embed, base));
        TG_TRY(kq_put(W, tg::KQ_Q4K, up[e], inter, embed, base + gb));
        TG_TRY(kq_put(W, fmt, down[e], embed, inter, base + 2 * gb));
    }
    std::vector<float> wv(n, w_scalar);
    if (weights)
        for (int e = 0; e < n; e++) wv[e] = weights[e];
    TG_CUDA(cudaMemcpyAsync(W.ptrs.p, ptrs.data(), sizeof(void*) * 3 * n, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(cudaMemcpyAsync(W.wts.p, wv.data(), sizeof(float) * n, cudaMemcpyHostToDevice, W.s));
    TG_CUDA(cudaMemcpyAsync(W.x.p, input, sizeof(float) * embed, cudaMemcpyHostToDevice, W.s));
    if (accumulate) TG_CUDA(cudaMemcpyAsync(W.out.p, output, sizeof(float) * embed, cudaMemcpyHostToDevice, W.s));
    const uint8_t* const* dp = (const uint8_t* const*)W.ptrs.p;
    TG_CUDA(tg::launch_kq_gateup(dp, dp + n, n, (const float*)W.x.p, embed, inter, (float*)W.hq.p, false, W.s));
    TG_CUDA(tg::launch_kq_down(fmt, dp + 2 * n, n, (const float*)W.hq.p, (const float*)W.wts.p, embed, inter,
                               (float*)W.out.p, accumulate, W.kqs.p, W.s));
    TG_CUDA(cudaMemcpyAsync(output, W.out.p, sizeof(float) * embed, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

extern "C" int tg_expert_forward(const uint8_t* q4_data, const float* input, float* output, float weight,
                                 int embed_dim, int inter_dim) {
    TG_CHECK(q4_data && input && output, TG_EINVAL, "tg_expert_forward: null pointer");
    TG_CHECK(Geom::valid_dims(embed_dim, inter_dim), TG_EINVAL,
             "tg_expert_forward: embed/inter must be positive multiples of 256 (<= 16384)");
    const size_t gb = tg::kq_matrix_bytes(tg::KQ_Q4K, inter_dim, embed_dim);
    const uint8_t* g = q4_data;
    const uint8_t* u = q4_data + gb;
    const void* d = q4_data + 2 * gb;
    return kq_experts_host(&g, &u, &d, tg::KQ_Q4K, 1, nullptr, weight, input, output, embed_dim, inter_dim, 1,
                           "tg_expert_forward");
}

extern "C" int tg_expert_forward_mixed(const uint8_t* gate_q4, const uint8_t* up_q4, const void* down_data,
                                       int down_format, const float* input, float* output, float weight,
                                       int embed_dim, int inter_dim) {
    TG_CHECK(gate_q4 && up_q4 && down_data && input && output, TG_EINVAL, "tg_expert_forward_mixed: null pointer");
    TG_CHECK(Geom::valid_dims(embed_dim, inter_dim), TG_EINVAL,
             "tg_expert_forward_mixed: embed/inter must be positive multiples of 256 (<= 16384)");
    if (down_format == TG_FMT_Q4_0)
        return expert_forward_parts(gate_q4, up_q4, (const uint8_t*)down_data, input, output, weight, embed_dim,
                                    inter_dim);
    int fmt;
    switch (down_format) {
        case TG_FMT_Q4_K: fmt = tg::KQ_Q4K; break;
        case TG_FMT_F16: fmt = tg::KQ_F16; break;
        case TG_FMT_Q6_K: fmt = tg::KQ_Q6K; break;
        default: return fail(TG_EINVAL, "tg_expert_forward_mixed: down_format must be 0 (Q4_K), 1 (f16), 2 (Q6_K) or 3 (Q4_0)");
    }
    return kq_experts_host(&gate_q4, &up_q4, &down_data, fmt, 1, nullptr, weight, input, output, embed_dim,
                           inter_dim, 1, "tg_expert_forward_mixed");
}

// One whole decoder layer on host buffers, csrc/libtinygiant.c:662-702: RMSNorm (eps
// 1e-6), the fp32-weight attention step (appending row kv_len of the caches), x += attn;
// RMSNorm with the FFN weight, then the n_active experts accumulated into a zeroed
// moe_out in order with tg_expert_forward_mixed (down format down_is_f16[e]: 0 Q4_K,
// 1 f16, 2 Q6_K, 3 Q4_0), x += moe_out.  The same calls in the same order as the
// reference, each on the GPU; the two residual adds are single fp32 additions per
// element on the host buffers.
extern "C" int tg_transformer_layer(const float* wq, const float* wk, const float* wv, const float* wo,
                                    const float* attn_norm_w, const float* q_norm_w, const float* k_norm_w,
                                    const float* ffn_norm_w, float* kv_k, float* kv_v, int kv_len, int kv_max,
                                    const float* rope_cos, const float* rope_sin, const uint8_t** gate_ptrs,
                                    const uint8_t** up_ptrs, const void** down_ptrs, const int* down_is_f16,
                                    const float* expert_weights, int n_active, float* x, int embed_dim,
                                    int inter_dim, int n_heads, int n_kv_heads, int head_dim, int pos) {
    TG_CHECK(wq && wk && wv && wo && attn_norm_w && q_norm_w && k_norm_w && ffn_norm_w && kv_k && kv_v && rope_cos &&
                 rope_sin && x,
             TG_EINVAL, "tg_transformer_layer: null pointer");
    TG_CHECK(n_active >= 0 && n_active <= 64, TG_EINVAL, "tg_transformer_layer: 0 <= n_active <= 64");
    TG_CHECK(n_active == 0 || (gate_ptrs && up_ptrs && down_ptrs && down_is_f16 && expert_weights), TG_EINVAL,
             "tg_transformer_layer: null expert table");
    TG_CHECK(embed_dim > 0 && embed_dim % 4 == 0, TG_EINVAL, "tg_transformer_layer: embed_dim must be a positive "
                                                             "multiple of 4");
    std::vector<float> normed(embed_dim), part(embed_dim);
    TG_TRY(tg_rms_norm(x, attn_norm_w, normed.data(), embed_dim, 1e-6f));
    TG_TRY(tg_attention_decode(wq, wk, wv, wo, q_norm_w, k_norm_w, kv_k, kv_v, kv_len, kv_max, rope_cos, rope_sin,
                               normed.data(), part.data(), embed_dim, n_heads, n_kv_heads, head_dim, pos));
    for (int i = 0; i < embed_dim; i++) x[i] = x[i] + part[i];
    TG_TRY(tg_rms_norm(x, ffn_norm_w, normed.data(), embed_dim, 1e-6f));
    std::fill(part.begin(), part.end(), 0.0f);
    for (int e = 0; e < n_active; e++)
        TG_TRY(tg_expert_forward_mixed(gate_ptrs[e], up_ptrs[e], down_ptrs[e], down_is_f16[e], normed.data(),
                                       part.data(), expert_weights[e], embed_dim, inter_dim));
    for (int i = 0; i < embed_dim; i++) x[i] = x[i] + part[i];
    return TG_OK;
}

extern "C" int tg_moe_forward(const uint8_t** expert_ptrs, const float* weights, int n_experts, const float* input,
                              float* output, int embed_dim, int inter_dim) {
    TG_CHECK(expert_ptrs && weights && input && output, TG_EINVAL, "tg_moe_forward: null pointer");
    TG_CHECK(n_experts >= 1 && n_experts <= 64, TG_EINVAL, "tg_moe_forward: 1 <= n_experts <= 64");
    TG_CHECK(Geom::valid_dims(embed_dim, inter_dim), TG_EINVAL,
             "tg_moe_forward: embed/inter must be positive multiples of 256 (<= 16384)");
    const size_t gb = tg::kq_matrix_bytes(tg::KQ_Q4K, inter_dim, embed_dim);
    std::vector<const uint8_t*> g(n_experts), u(n_experts);
    std::vector<const void*> d(n_experts);
    for (int e = 0; e < n_experts; e++) {
        TG_CHECK(expert_ptrs[e], TG_EINVAL, "tg_moe_forward: null expert");
        g[e] = expert_ptrs[e];
        u[e] = expert_ptrs[e] + gb;
        d[e] = expert_ptrs[e] + 2 * gb;
    }
    return kq_experts_host(g.data(), u.data(), d.data(), tg::KQ_Q4K, n_experts, weights, 0.0f, input, output,
                           embed_dim, inter_dim, 0, "tg_moe_forward");
}

extern "C" int tg_moe_forward_q4_0(const uint8_t** expert_ptrs, const float* weights, int n_experts,
                                   const float* input, float* output, int embed_dim, int inter_dim) {
    TG_CHECK(expert_ptrs && weights && input && output && n_experts > 0 && n_experts <= 16, TG_EINVAL,
             "tg_moe_forward_q4_0: bad arguments (1 <= n_experts <= 16)");
    for (int e = 0; e < n_experts; e++) TG_CHECK(expert_ptrs[e], TG_EINVAL, "tg_moe_forward_q4_0: null expert");
    TG_CHECK(Geom::valid_dims(embed_dim, inter_dim), TG_EINVAL,
             "tg_moe_forward_q4_0: embed/inter must be positive multiples of 256");
    HostWS& W = ws();
    std::lock_guard<std::mutex> lk(W.mu);
    TG_TRY(W.bind());
    Geom g = Geom::make(embed_dim, inter_dim);
    size_t tot = g.expert_bytes * n_experts;
    TG_TRY(ensure(W.raw, tot));
    TG_TRY(ensure(W.w, tot));
    TG_TRY(ensure(W.x, sizeof(float) * embed_dim));
    TG_TRY(ensure(W.out, sizeof(float) * embed_dim));
    for (int e = 0; e < n_experts; e++) {
        uint8_t* raw = (uint8_t*)W.raw.p + (size_t)e * g.expert_bytes;
        TG_CUDA(cudaMemcpyAsync(raw, expert_ptrs[e], g.expert_bytes, cudaMemcpyHostToDevice, W.s));
        TG_CUDA(repack_expert(raw, (uint8_t*)W.w.p + (size_t)e * g.expert_bytes, g, W.s));
    }
    TG_CUDA(cudaMemcpyAsync(W.x.p, input, sizeof(float) * embed_dim, cudaMemcpyHostToDevice, W.s));
    TG_TRY(run_experts(W, g, n_experts, weights, 0.0f, 0));
    TG_CUDA(cudaMemcpyAsync(output, W.out.p, sizeof(float) * embed_dim, cudaMemcpyDeviceToHost, W.s));
    TG_CUDA(cudaStreamSynchronize(W.s));
    return TG_OK;
}

extern "C" int tg_mlock(const void* addr, size_t len) {
    uintptr_t page = (uintptr_t)sysconf(_SC_PAGESIZE);
    uintptr_t a = (uintptr_t)addr & ~(page - 1);
    size_t l = len + ((uintptr_t)addr - a);
    return mlock((const void*)a, l);
}

// posix_madvise(WILLNEED) over the pages of [addr, addr + len): the reference's page
// hint ahead of reading a cold expert (csrc/libtinygiant.c:745-750); here the host
// tier's pinned copies make it a hint for relayout files mapped from disk.  Returns
// posix_madvise's result (0 or an errno value).
extern "C" int tg_prefetch(const void* addr, size_t len) {
    if (!addr || !len) return 0;
    const uintptr_t page = (uintptr_t)sysconf(_SC_PAGESIZE);
    const uintptr_t a = (uintptr_t)addr & ~(page - 1);
    return posix_madvise((void*)a, len + ((uintptr_t)addr - a), POSIX_MADV_WILLNEED);
}

// tg_prefetch over count ranges (csrc/libtinygiant.c:752-759); the first nonzero result.
extern "C" int tg_prefetch_batch(const void** addrs, const size_t* lens, int count) {
    if (!addrs || !lens || count <= 0) return count < 0 ? EINVAL : 0;
    int rc = 0;
    for (int i = 0; i < count; i++) {
        const int r = tg_prefetch(addrs[i], lens[i]);
        if (r && !rc) rc = r;
    }
    return rc;
}

// ============================================================ device-resident

struct tgx_ctx {
    int device = 0;
    tgx_shape shape{};
    Geom g;
    size_t layer_bytes = 0;
    uint8_t* weights = nullptr;   // [L][E] experts, row-split
    float* routers = nullptr;     // [L][E][H]
    float eps = 1e-6f;            // FFN RMSNorm epsilon
    float* norms = nullptr;       // [L][H] FFN RMSNorm weights (default 1)
    float* nscale = nullptr;      // RMSNorm scale of the current layer (multi-kernel path)
    long long* acc = nullptr;     // [E + 1] router / sum-of-squares accumulators (kept zero)
    unsigned* counter = nullptr;  // router block counter (kept zero)
    float* logits = nullptr;      // [L][E]
    int* idx = nullptr;           // [L][k]
    float* wts = nullptr;         // [L][k]
    const uint8_t** eptrs = nullptr;  // [L][k]
    uint8_t* hq = nullptr;        // k activation blocks of I/32
    uint8_t* staging = nullptr;   // ggml blobs in transit
    size_t staging_bytes = 0;
    cudaStream_t s = nullptr;     // loads, synthetic fill, graph capture
    cudaGraphExec_t gexec = nullptr;
    const float* gx = nullptr;
    // fused (one kernel per step) path
    bool fused_ok = false;
    int G = 0;                          // CTAs = SMs
    float* RT = nullptr;                // [L][H][E] transposed routers
    unsigned long long* xw = nullptr;   // [L + 1][H] tagged hidden states between layers
    float* xbuf = nullptr;              // [H] output of a one-layer launch
    unsigned long long* facc = nullptr; // [L][FUSED_ACC][E + 1]
    unsigned long long* hqt = nullptr;  // [L][k * nbI * 6]
    unsigned* ctl = nullptr;            // epoch, finish count, error
    uint16_t* plan = nullptr;
    tg::FusedParams fp{};
    void* bscratch = nullptr;           // batched path scratch, grown on demand
    size_t bscratch_bytes = 0;
    int batched_kernels = 0;            // tg::BATCHED_AUTO / _DP4A / _MMA
    const uint8_t** eall = nullptr;     // [L][E] pointers to every expert (tgx_expert_forward)
    uint8_t* ehq = nullptr;             // its requantised h (one expert)
    // tgx_experts_forward: up to 16 expert pointers and weights, their h blocks, the norm scale
    const uint8_t** lptrs = nullptr;
    float* lwts = nullptr;
    uint8_t* lhq = nullptr;
    float* lscale = nullptr;
    cudaGraphExec_t fexec = nullptr;
    const float* fx = nullptr;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

void ctx_free(tgx_ctx* c) {
    if (!c) return;
    DeviceGuard dg(c->device);
    if (c->gexec) cudaGraphExecDestroy(c->gexec);
    if (c->fexec) cudaGraphExecDestroy(c->fexec);
    for (void* p : {(void*)c->weights, (void*)c->routers, (void*)c->norms, (void*)c->nscale, (void*)c->acc,
                    (void*)c->counter, (void*)c->logits,
                    (void*)c->idx, (void*)c->wts, (void*)c->eptrs, (void*)c->hq, (void*)c->staging, (void*)c->RT,
                    (void*)c->xw, (void*)c->xbuf, (void*)c->bscratch, (void*)c->lptrs, (void*)c->lwts,
                    (void*)c->lhq, (void*)c->lscale, (void*)c->facc, (void*)c->hqt, (void*)c->ctl, (void*)c->plan,
                    (void*)c->eall, (void*)c->ehq})
        if (p) cudaFree(p);
    if (c->s) cudaStreamDestroy(c->s);
    delete c;
}

int moe_layer_launch(tgx_ctx* c, int layer, float* x, cudaStream_t s) {
    const tgx_shape& sh = c->shape;
    const int E = sh.n_experts, k = sh.top_k, H = sh.embed;
    const uint8_t* lb = c->weights + (size_t)layer * c->layer_bytes;
    const uint8_t** ep = c->eptrs + (size_t)layer * k;
    float* w = c->wts + (size_t)layer * k;
    const float* nw = c->norms + (size_t)layer * H;
    TG_CUDA(tg::launch_router_topk(c->routers + (size_t)layer * E * H, x, nw, c->eps, E, H, k, c->acc, c->counter,
                                   c->logits + (size_t)layer * E, c->idx + (size_t)layer * k, w, c->nscale, lb,
                                   c->g.expert_bytes, ep, s));
    TG_CUDA(tg::launch_gateup(ep, k, x, nw, c->nscale, c->g, c->hq, nullptr, nullptr, s));
    TG_CUDA(tg::launch_down_combine(ep, k, c->hq, w, 0.0f, c->g, x, x, 0, nullptr, s));
    return TG_OK;
}

// Allocate the fused path's state and plan its work split; the fused path is
// disabled (fused_ok = false) when the shape does not fit one CTA per SM.
int fused_setup(tgx_ctx* c) {
    const tgx_shape& sh = c->shape;
    const int L = sh.n_layers, E = sh.n_experts, k = sh.top_k, H = sh.embed;
    int dev = c->device, sms = 0, smem_optin = 0;
    TG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    TG_CUDA(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    auto A = [&](void** p, size_t n) -> int {
        if (cudaMalloc(p, n) != cudaSuccess) {
            cudaGetLastError();
            return fail(TG_ENOMEM, "tgx_ctx_create: cudaMalloc of " + std::to_string(n) + " bytes failed");
        }
        return TG_OK;
    };
    int rc;
    if ((rc = A((void**)&c->RT, sizeof(float) * (size_t)L * E * H)) ||
        (rc = A((void**)&c->xw, sizeof(unsigned long long) * (size_t)(L + 1) * H)) ||
        (rc = A((void**)&c->xbuf, sizeof(float) * (size_t)H)) ||
        (rc = A((void**)&c->facc, sizeof(unsigned long long) * (size_t)L * tg::FUSED_ACC * (E + 1))) ||
        (rc = A((void**)&c->hqt, sizeof(unsigned long long) * (size_t)L * k * c->g.nbI * 6)) ||
        (rc = A((void**)&c->ctl, sizeof(unsigned) * 4)))
        return rc;
    TG_CUDA(cudaMemset(c->RT, 0, sizeof(float) * (size_t)L * E * H));
    TG_CUDA(cudaMemset(c->xw, 0, sizeof(unsigned long long) * (size_t)(L + 1) * H));
    TG_CUDA(cudaMemset(c->facc, 0, sizeof(unsigned long long) * (size_t)L * tg::FUSED_ACC * (E + 1)));
    TG_CUDA(cudaMemset(c->hqt, 0, sizeof(unsigned long long) * (size_t)L * k * c->g.nbI * 6));
    TG_CUDA(cudaMemset(c->ctl, 0, sizeof(unsigned) * 4));
    std::vector<uint16_t> plan;
    size_t arena = 0;
    int max_rows = 0, k_early = 0;
    if (sms > 255 || c->g.H > 16384) return TG_OK;  // count tags and fixed-point bounds
    if (E % 4 != 0) return TG_OK;                   // router columns are bulk-copied in 16-byte units
    // each thread of a CTA polls at most 32 words (x and router sums; h records)
    if ((size_t)H + (size_t)tg::FUSED_ACC * (E + 1) > 32u * tg::FUSED_THREADS ||
        (size_t)k * c->g.nbI * 6 > 32u * tg::FUSED_THREADS)
        return TG_OK;
    if (tg::fused_plan(c->g, E, k, sms, plan, arena, max_rows, k_early) != 0) return TG_OK;  // fused path off
    tg::FusedParams& P = c->fp;
    P.weights = c->weights;
    P.layer_bytes = c->layer_bytes;
    P.g = c->g;
    P.RT = c->RT;
    P.normw = c->norms;
    P.eps = c->eps;
    P.E = E;
    P.k = k;
    P.L0 = 0;
    P.nL = L;
    P.max_rows = max_rows;
    P.k_early = k_early;
    // The down phase can run in two stages (early slots while late gate/up units
    // still stream); at the Qwen3 shape one stage measured faster, so it is the default.
    P.k_early = 0;
    P.xw = c->xw;
    P.acc = c->facc;
    P.hqt = c->hqt;
    P.Lmax = L;
    P.ctl = c->ctl;
    P.idx_out = c->idx;
    P.w_out = c->wts;
    P.logits_out = c->logits;
    P.trace = nullptr;
    P.wait_cycles = tg::FUSED_WAIT_CYCLES;
    P.missing = 0;
    P.arena_bytes = arena;
    if (tg::fused_smem_layout(P).total > (uint32_t)smem_optin) return TG_OK;
    if ((rc = A((void**)&c->plan, plan.size() * sizeof(uint16_t)))) return rc;
    TG_CUDA(cudaMemcpy(c->plan, plan.data(), plan.size() * sizeof(uint16_t), cudaMemcpyHostToDevice));
    P.plan = c->plan;
    TG_CUDA(tg::fused_prepare(P));
    int per_sm = 0;
    TG_CUDA(tg::fused_occupancy(P, &per_sm));
    if (per_sm < 1) return TG_OK;
    c->G = sms;
    c->fused_ok = true;
    return TG_OK;
}

// Launch the fused kernel for layers [L0, L0 + nL) on x (in place).
int fused_launch(tgx_ctx* c, int L0, int nL, float* x, cudaStream_t s) {
    tg::FusedParams P = c->fp;
    P.L0 = L0;
    P.nL = nL;
    P.x_in = x;
    // In place is safe when every read of x_in precedes the first write of x_out: with
    // nL >= 2, or when every CTA owns a gate/up unit (x_out is written after all h
    // records are gathered, and each CTA reads x_in before computing its units).
    const bool inplace = nL >= 2 || c->fp.k * c->g.nbI >= c->G;
    P.x_out = inplace ? x : c->xbuf;
    TG_CUDA(tg::launch_decode_fused(P, c->G, s));
    if (!inplace)
        TG_CUDA(cudaMemcpyAsync(x, P.x_out, sizeof(float) * c->g.H, cudaMemcpyDeviceToDevice, s));
    return TG_OK;
}

int transpose_router(tgx_ctx* c, int layer) {
    const size_t n = (size_t)c->shape.n_experts * c->shape.embed;
    TG_CUDA(tg::launch_transpose(c->routers + (size_t)layer * n, c->RT + (size_t)layer * n, c->shape.n_experts,
                                 c->shape.embed, c->s));
    return TG_OK;
}

}  // namespace

extern "C" int tgx_ctx_create(int device, const tgx_shape* shape, tgx_ctx** out) {
    TG_CHECK(shape && out, TG_EINVAL, "tgx_ctx_create: null argument");
    *out = nullptr;
    TG_CHECK(Geom::valid_dims(shape->embed, shape->inter), TG_EINVAL,
             "tgx_ctx_create: embed/inter must be positive multiples of 256");
    TG_CHECK(shape->n_experts > 0 && shape->n_experts <= 1024 && shape->top_k > 0 && shape->top_k <= 16 &&
                 shape->top_k <= shape->n_experts && shape->n_layers > 0,
             TG_EINVAL, "tgx_ctx_create: bad expert/top_k/layer counts");
    int ndev = have_device();
    TG_CHECK(ndev > 0, TG_ENODEV, "no CUDA device");
    TG_CHECK(device >= 0 && device < ndev, TG_EINVAL, "tgx_ctx_create: bad device index");
    DeviceGuard dg(device);
    tgx_ctx* c = new tgx_ctx();
    c->device = device;
    c->shape = *shape;
    c->g = Geom::make(shape->embed, shape->inter);
    c->layer_bytes = c->g.expert_bytes * shape->n_experts;
    const int L = shape->n_layers, E = shape->n_experts, k = shape->top_k, H = shape->embed;
    c->staging_bytes = c->g.expert_bytes * 8;
    auto A = [&](void** p, size_t n) -> int {
        if (cudaMalloc(p, n) != cudaSuccess) {
            cudaGetLastError();
            return fail(TG_ENOMEM, "tgx_ctx_create: cudaMalloc of " + std::to_string(n) + " bytes failed");
        }
        return TG_OK;
    };
    int rc = TG_OK;
    if ((rc = A((void**)&c->weights, c->layer_bytes * L)) || (rc = A((void**)&c->routers, sizeof(float) * L * E * H)) ||
        (rc = A((void**)&c->norms, sizeof(float) * L * H)) || (rc = A((void**)&c->nscale, sizeof(float))) ||
        (rc = A((void**)&c->acc, sizeof(long long) * (E + 1))) || (rc = A((void**)&c->counter, sizeof(unsigned))) ||
        (rc = A((void**)&c->logits, sizeof(float) * L * E)) || (rc = A((void**)&c->idx, sizeof(int) * L * k)) ||
        (rc = A((void**)&c->wts, sizeof(float) * L * k)) || (rc = A((void**)&c->eptrs, sizeof(void*) * L * k)) ||
        (rc = A((void**)&c->hq, tg::act_bytes(c->g.nbI) * k)) || (rc = A((void**)&c->staging, c->staging_bytes))) {
        ctx_free(c);
        return rc;
    }
    if (shape->rms_eps > 0.0f) c->eps = shape->rms_eps;
    {
        std::vector<float> ones((size_t)L * H, 1.0f);
        if (cudaMemcpy(c->norms, ones.data(), ones.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
            ctx_free(c);
            return fail(TG_ECUDA, "tgx_ctx_create: norm weight init failed");
        }
    }
    cudaError_t e = cudaMemset(c->acc, 0, sizeof(long long) * (E + 1));
    if (e == cudaSuccess) e = cudaMemset(c->counter, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(c->routers, 0, sizeof(float) * L * E * H);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->s, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = tg::prepare_kernels(c->g, k);
    if (e != cudaSuccess) {
        ctx_free(c);
        return fail(TG_ECUDA, std::string("tgx_ctx_create: ") + cudaGetErrorString(e));
    }
    if ((rc = fused_setup(c)) != TG_OK) {
        ctx_free(c);
        return rc;
    }
    *out = c;
    return TG_OK;
}

extern "C" int tgx_ctx_destroy(tgx_ctx* ctx) {
    if (!ctx) return TG_OK;
    ctx_free(ctx);
    return TG_OK;
}

extern "C" size_t tgx_expert_bytes(const tgx_ctx* ctx) { return ctx ? ctx->g.expert_bytes : 0; }

// out += weight * expert(x) for expert `expert` of layer `layer`, resident in the
// context: tg_expert_forward_q4_0 (csrc/libtinygiant.c:555-595) on device memory, the
// gate/up and down kernels of the multi-kernel path with one expert.  The first call
// allocates the context's table of expert pointers and an h buffer; later calls only
// enqueue the two kernels on `stream`.
extern "C" int tgx_expert_forward(tgx_ctx* ctx, int layer, int expert, const float* x_dev, float* out_dev,
                                  float weight, void* stream) {
    TG_CHECK(ctx && x_dev && out_dev, TG_EINVAL, "tgx_expert_forward: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers && expert >= 0 && expert < ctx->shape.n_experts, TG_EINVAL,
             "tgx_expert_forward: layer/expert out of range");
    DeviceGuard dg(ctx->device);
    const int L = ctx->shape.n_layers, E = ctx->shape.n_experts;
    if (!ctx->eall) {
        std::vector<const uint8_t*> ptrs((size_t)L * E);
        for (size_t i = 0; i < ptrs.size(); i++) ptrs[i] = ctx->weights + i * ctx->g.expert_bytes;
        const uint8_t** t = nullptr;
        uint8_t* h = nullptr;
        if (cudaMalloc((void**)&t, sizeof(void*) * ptrs.size()) != cudaSuccess ||
            cudaMalloc((void**)&h, tg::act_bytes(ctx->g.nbI)) != cudaSuccess) {
            cudaGetLastError();
            if (t) cudaFree((void*)t);
            return fail(TG_ENOMEM, "tgx_expert_forward: cudaMalloc failed");
        }
        TG_CUDA(cudaMemcpy(t, ptrs.data(), sizeof(void*) * ptrs.size(), cudaMemcpyHostToDevice));
        TG_CUDA(tg::prepare_kernels(ctx->g, 1));
        ctx->eall = t;
        ctx->ehq = h;
    }
    cudaStream_t s = (cudaStream_t)stream;
    const uint8_t* const* ep = ctx->eall + (size_t)layer * E + expert;
    TG_CUDA(tg::launch_gateup(ep, 1, x_dev, nullptr, nullptr, ctx->g, ctx->ehq, nullptr, nullptr, s));
    TG_CUDA(tg::launch_down_combine(ep, 1, ctx->ehq, nullptr, weight, ctx->g, nullptr, out_dev, 1, nullptr, s));
    return TG_OK;
}

extern "C" int tgx_load_experts(tgx_ctx* ctx, int layer, int first, int n, const void* src, int src_on_device) {
    TG_CHECK(ctx && src, TG_EINVAL, "tgx_load_experts: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers && first >= 0 && n >= 0 && first + n <= ctx->shape.n_experts,
             TG_EINVAL, "tgx_load_experts: layer/expert range out of bounds");
    DeviceGuard dg(ctx->device);
    const Geom& g = ctx->g;
    const int chunk = (int)(ctx->staging_bytes / g.expert_bytes);
    for (int e0 = 0; e0 < n; e0 += chunk) {
        int m = n - e0 < chunk ? n - e0 : chunk;
        const uint8_t* s = (const uint8_t*)src + (size_t)e0 * g.expert_bytes;
        TG_CUDA(cudaMemcpyAsync(ctx->staging, s, (size_t)m * g.expert_bytes,
                                src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->s));
        for (int e = 0; e < m; e++) {
            uint8_t* dst = ctx->weights + (size_t)layer * ctx->layer_bytes + (size_t)(first + e0 + e) * g.expert_bytes;
            TG_CUDA(repack_expert(ctx->staging + (size_t)e * g.expert_bytes, dst, g, ctx->s));
        }
        TG_CUDA(cudaStreamSynchronize(ctx->s));
    }
    return TG_OK;
}

extern "C" int tgx_load_experts_rows(tgx_ctx* ctx, int layer, int first, int n, const void* src,
                                     int src_on_device) {
    TG_CHECK(ctx && src, TG_EINVAL, "tgx_load_experts_rows: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers && first >= 0 && n >= 0 && first + n <= ctx->shape.n_experts,
             TG_EINVAL, "tgx_load_experts_rows: layer/expert range out of bounds");
    DeviceGuard dg(ctx->device);
    const Geom& g = ctx->g;
    uint8_t* dst = ctx->weights + (size_t)layer * ctx->layer_bytes + (size_t)first * g.expert_bytes;
    TG_CUDA(cudaMemcpyAsync(dst, src, (size_t)n * g.expert_bytes,
                            src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->s));
    TG_CUDA(cudaStreamSynchronize(ctx->s));
    return TG_OK;
}

extern "C" int tgx_read_experts(tgx_ctx* ctx, int layer, int first, int n, void* dst_host) {
    TG_CHECK(ctx && dst_host, TG_EINVAL, "tgx_read_experts: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers && first >= 0 && n >= 0 && first + n <= ctx->shape.n_experts,
             TG_EINVAL, "tgx_read_experts: layer/expert range out of bounds");
    DeviceGuard dg(ctx->device);
    const Geom& g = ctx->g;
    const int chunk = (int)(ctx->staging_bytes / g.expert_bytes);
    for (int e0 = 0; e0 < n; e0 += chunk) {
        int m = n - e0 < chunk ? n - e0 : chunk;
        for (int e = 0; e < m; e++) {
            const uint8_t* src = ctx->weights + (size_t)layer * ctx->layer_bytes + (size_t)(first + e0 + e) * g.expert_bytes;
            TG_CUDA(unpack_expert(src, ctx->staging + (size_t)e * g.expert_bytes, g, ctx->s));
        }
        TG_CUDA(cudaMemcpyAsync((uint8_t*)dst_host + (size_t)e0 * g.expert_bytes, ctx->staging,
                                (size_t)m * g.expert_bytes, cudaMemcpyDeviceToHost, ctx->s));
        TG_CUDA(cudaStreamSynchronize(ctx->s));
    }
    return TG_OK;
}

extern "C" int tgx_set_router(tgx_ctx* ctx, int layer, const float* R, int src_on_device) {
    TG_CHECK(ctx && R, TG_EINVAL, "tgx_set_router: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers, TG_EINVAL, "tgx_set_router: layer out of range");
    DeviceGuard dg(ctx->device);
    size_t n = (size_t)ctx->shape.n_experts * ctx->shape.embed;
    TG_CUDA(cudaMemcpyAsync(ctx->routers + (size_t)layer * n, R, n * sizeof(float),
                            src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->s));
    TG_TRY(transpose_router(ctx, layer));
    TG_CUDA(cudaStreamSynchronize(ctx->s));
    return TG_OK;
}

extern "C" int tgx_set_ffn_norm(tgx_ctx* ctx, int layer, const float* w, int src_on_device) {
    TG_CHECK(ctx && w, TG_EINVAL, "tgx_set_ffn_norm: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers, TG_EINVAL, "tgx_set_ffn_norm: layer out of range");
    DeviceGuard dg(ctx->device);
    size_t n = (size_t)ctx->shape.embed;
    TG_CUDA(cudaMemcpyAsync(ctx->norms + (size_t)layer * n, w, n * sizeof(float),
                            src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->s));
    TG_CUDA(cudaStreamSynchronize(ctx->s));
    return TG_OK;
}

extern "C" int tgx_fill_synthetic(tgx_ctx* ctx, uint64_t seed, float w_sigma, float r_sigma) {
    TG_CHECK(ctx, TG_EINVAL, "tgx_fill_synthetic: null context");
    DeviceGuard dg(ctx->device);
    const Geom& g = ctx->g;
    const tgx_shape& sh = ctx->shape;
    const unsigned long long per_expert = 3ULL * g.H * g.I;  // weights per expert
    for (int l = 0; l < sh.n_layers; l++) {
        unsigned long long base = (unsigned long long)l * sh.n_experts * per_expert;
        TG_CUDA(tg::launch_fill_experts_q4_0(ctx->weights + (size_t)l * ctx->layer_bytes, sh.n_experts, g, seed,
                                             base, w_sigma, ctx->s));
        size_t nr = (size_t)sh.n_experts * sh.embed;
        TG_CUDA(tg::launch_fill_normal(ctx->routers + (size_t)l * nr, (long long)nr, seed ^ 0x5DEECE66Dull,
                                       (unsigned long long)l * nr * 2, r_sigma, ctx->s));
        TG_TRY(transpose_router(ctx, l));
    }
    TG_CUDA(cudaStreamSynchronize(ctx->s));
    return TG_OK;
}

extern "C" int tgx_moe_layer(tgx_ctx* ctx, int layer, float* x_dev, void* stream) {
    TG_CHECK(ctx && x_dev, TG_EINVAL, "tgx_moe_layer: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers, TG_EINVAL, "tgx_moe_layer: layer out of range");
    DeviceGuard dg(ctx->device);
    if (ctx->fused_ok) return fused_launch(ctx, layer, 1, x_dev, (cudaStream_t)stream);
    return moe_layer_launch(ctx, layer, x_dev, (cudaStream_t)stream);
}

namespace {
// Run MoE blocks [l0, l1) for T tokens on x_dev[T][embed] with the batched kernels.
int batched_run(tgx_ctx* ctx, int l0, int l1, float* x_dev, int T, cudaStream_t s, const char* fn) {
    const tgx_shape& sh = ctx->shape;
    TG_CHECK(T >= 1 && T <= 65536 / sh.top_k, TG_EINVAL, std::string(fn) + ": T must be in [1, 65536/top_k]");
    int optin = 0;
    TG_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device));
    TG_CHECK(tg::batched_smem_bytes(ctx->g) <= (size_t)optin, TG_EUNSUPPORTED,
             std::string(fn) + ": shape needs more shared memory per block than the device has");
    const size_t need = tg::batched_scratch_bytes(ctx->g, sh.n_experts, sh.top_k, T);
    if (need > ctx->bscratch_bytes) {
        TG_CUDA(cudaStreamSynchronize(s));
        if (ctx->bscratch) cudaFree(ctx->bscratch);
        ctx->bscratch = nullptr;
        ctx->bscratch_bytes = 0;
        if (cudaMalloc(&ctx->bscratch, need) != cudaSuccess) {
            cudaGetLastError();
            return fail(TG_ENOMEM, std::string(fn) + ": cudaMalloc of " + std::to_string(need) + " bytes failed");
        }
        ctx->bscratch_bytes = need;
        TG_CUDA(cudaMemset(ctx->bscratch, 0, 256));   // the error flag
    }
    const size_t n = (size_t)sh.n_experts * sh.embed;
    for (int l = l0; l < l1; l++)
        TG_CUDA(tg::launch_moe_batched(ctx->weights + (size_t)l * ctx->layer_bytes, ctx->g, ctx->routers + (size_t)l * n,
                                       ctx->norms + (size_t)l * sh.embed, ctx->eps, sh.n_experts, sh.top_k, x_dev, T,
                                       ctx->bscratch, ctx->bscratch_bytes, nullptr, nullptr, nullptr,
                                       ctx->batched_kernels, s));
    return TG_OK;
}
}  // namespace

extern "C" int tgx_moe_batched(tgx_ctx* ctx, int layer, float* x_dev, int T, void* stream) {
    TG_CHECK(ctx && x_dev, TG_EINVAL, "tgx_moe_batched: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers, TG_EINVAL, "tgx_moe_batched: layer out of range");
    DeviceGuard dg(ctx->device);
    return batched_run(ctx, layer, layer + 1, x_dev, T, (cudaStream_t)stream, "tgx_moe_batched");
}

// Up to this many tokens, a whole-model step runs the fused single-token kernel once per
// token (same bits as the batched kernels, which equal single-token calls): few tokens
// touch few shared experts, and at the Qwen3 shape 8 fused tokens took 5.6 ms against
// 6.1 ms for the batched kernels.
constexpr int FUSED_PER_TOKEN_MAX_T = 8;

extern "C" int tgx_decode_batched(tgx_ctx* ctx, float* x_dev, int T, void* stream) {
    TG_CHECK(ctx && x_dev, TG_EINVAL, "tgx_decode_batched: null argument");
    DeviceGuard dg(ctx->device);
    if (ctx->fused_ok && ctx->batched_kernels == tg::BATCHED_AUTO && T >= 1 && T <= FUSED_PER_TOKEN_MAX_T) {
        for (int t = 0; t < T; t++)
            TG_TRY(fused_launch(ctx, 0, ctx->shape.n_layers, x_dev + (size_t)t * ctx->shape.embed,
                                (cudaStream_t)stream));
        return TG_OK;
    }
    return batched_run(ctx, 0, ctx->shape.n_layers, x_dev, T, (cudaStream_t)stream, "tgx_decode_batched");
}

extern "C" int tgx_experts_forward(tgx_ctx* ctx, int layer, const void* const* experts, const float* weights, int n,
                                   float* x_dev, void* stream) {
    TG_CHECK(ctx && experts && weights && x_dev, TG_EINVAL, "tgx_experts_forward: null argument");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers, TG_EINVAL, "tgx_experts_forward: layer out of range");
    TG_CHECK(n >= 1 && n <= 16, TG_EINVAL, "tgx_experts_forward: n must be in [1, 16]");
    for (int j = 0; j < n; j++) TG_CHECK(experts[j], TG_EINVAL, "tgx_experts_forward: null expert pointer");
    DeviceGuard dg(ctx->device);
    const Geom& g = ctx->g;
    if (!ctx->lptrs) {
        if (cudaMalloc((void**)&ctx->lptrs, 16 * sizeof(void*)) != cudaSuccess ||
            cudaMalloc((void**)&ctx->lwts, 16 * sizeof(float)) != cudaSuccess ||
            cudaMalloc((void**)&ctx->lhq, 16 * tg::act_bytes(g.nbI)) != cudaSuccess ||
            cudaMalloc((void**)&ctx->lscale, sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return fail(TG_ENOMEM, "tgx_experts_forward: cudaMalloc of its small buffers failed");
        }
    }
    cudaStream_t s = (cudaStream_t)stream;
    // pageable sources: the copies are staged before the calls return, so the
    // caller's arrays may be reused at once
    TG_CUDA(cudaMemcpyAsync(ctx->lptrs, experts, n * sizeof(void*), cudaMemcpyHostToDevice, s));
    TG_CUDA(cudaMemcpyAsync(ctx->lwts, weights, n * sizeof(float), cudaMemcpyHostToDevice, s));
    const float* nw = ctx->norms + (size_t)layer * g.H;
    TG_CUDA(tg::prepare_kernels(g, n));
    TG_CUDA(tg::launch_rms_scale(x_dev, g.H, ctx->eps, ctx->lscale, s));
    TG_CUDA(tg::launch_gateup(ctx->lptrs, n, x_dev, nw, ctx->lscale, g, ctx->lhq, nullptr, nullptr, s));
    TG_CUDA(tg::launch_down_combine(ctx->lptrs, n, ctx->lhq, ctx->lwts, 0.0f, g, x_dev, x_dev, 0, nullptr, s));
    return TG_OK;
}

extern "C" int tgx_repack_experts(tgx_ctx* ctx, const void* raw_dev, void* dst_dev, int n, void* stream) {
    TG_CHECK(ctx && raw_dev && dst_dev && n >= 0, TG_EINVAL, "tgx_repack_experts: bad arguments");
    DeviceGuard dg(ctx->device);
    const Geom& g = ctx->g;
    for (int e = 0; e < n; e++)
        TG_CUDA(repack_expert((const uint8_t*)raw_dev + (size_t)e * g.expert_bytes, (uint8_t*)dst_dev + (size_t)e * g.expert_bytes,
                              g, (cudaStream_t)stream));
    return TG_OK;
}

extern "C" int tgx_decode_step(tgx_ctx* ctx, float* x_dev, void* stream, int flags) {
    TG_CHECK(ctx && x_dev, TG_EINVAL, "tgx_decode_step: null argument");
    DeviceGuard dg(ctx->device);
    cudaStream_t s = (cudaStream_t)stream;
    const bool fused = ctx->fused_ok && !(flags & TGX_MULTI);
    if (flags & TGX_EAGER) {
        if (fused) return fused_launch(ctx, 0, ctx->shape.n_layers, x_dev, s);
        for (int l = 0; l < ctx->shape.n_layers; l++) TG_TRY(moe_layer_launch(ctx, l, x_dev, s));
        return TG_OK;
    }
    cudaGraphExec_t& exec = fused ? ctx->fexec : ctx->gexec;
    const float*& gx = fused ? ctx->fx : ctx->gx;
    if (!exec || gx != x_dev) {
        if (exec) cudaGraphExecDestroy(exec);
        exec = nullptr;
        gx = nullptr;
        cudaGraph_t graph = nullptr;
        TG_CUDA(cudaStreamBeginCapture(ctx->s, cudaStreamCaptureModeThreadLocal));
        int rc = TG_OK;
        if (fused) {
            rc = fused_launch(ctx, 0, ctx->shape.n_layers, x_dev, ctx->s);
        } else {
            for (int l = 0; l < ctx->shape.n_layers && rc == TG_OK; l++) rc = moe_layer_launch(ctx, l, x_dev, ctx->s);
        }
        cudaError_t e = cudaStreamEndCapture(ctx->s, &graph);
        if (rc != TG_OK) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        TG_CUDA(e);
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        TG_CUDA(e);
        gx = x_dev;
    }
    TG_CUDA(cudaGraphLaunch(exec, s));
    return TG_OK;
}

// The fused kernel's parameters are baked into the step graph at capture: drop it so
// the next replay captures the new ones.
static void drop_fused_graph(tgx_ctx* ctx) {
    if (ctx->fexec) cudaGraphExecDestroy(ctx->fexec);
    ctx->fexec = nullptr;
    ctx->fx = nullptr;
}

extern "C" int tgx_set_wait_limit(tgx_ctx* ctx, long long cycles) {
    TG_CHECK(ctx, TG_EINVAL, "tgx_set_wait_limit: null context");
    TG_CHECK(cycles == 0 || cycles >= 1000, TG_EINVAL, "tgx_set_wait_limit: cycles must be 0 (default) or >= 1000");
    DeviceGuard dg(ctx->device);
    TG_CUDA(cudaDeviceSynchronize());
    ctx->fp.wait_cycles = cycles ? cycles : tg::FUSED_WAIT_CYCLES;
    drop_fused_graph(ctx);
    return TG_OK;
}

extern "C" int tgx_fused_inject_missing(tgx_ctx* ctx, int n) {
    TG_CHECK(ctx && n >= 0 && n <= 16, TG_EINVAL, "tgx_fused_inject_missing: 0 <= n <= 16");
    TG_CHECK(ctx->fused_ok, TG_EUNSUPPORTED, "tgx_fused_inject_missing: fused path not available for this shape");
    DeviceGuard dg(ctx->device);
    TG_CUDA(cudaDeviceSynchronize());
    ctx->fp.missing = n;
    drop_fused_graph(ctx);
    return TG_OK;
}

extern "C" int tgx_set_batched_kernels(tgx_ctx* ctx, int kernels) {
    TG_CHECK(ctx && kernels >= 0 && kernels <= 3, TG_EINVAL,
             "tgx_set_batched_kernels: kernels must be 0 (auto), 1 (dp4a), 2 (tensor cores) or 3 (tensor cores, "
             "fast epilogue)");
    ctx->batched_kernels = kernels;
    return TG_OK;
}

extern "C" int tgx_sync_status(tgx_ctx* ctx) {
    TG_CHECK(ctx, TG_EINVAL, "tgx_sync_status: null context");
    DeviceGuard dg(ctx->device);
    TG_CUDA(cudaDeviceSynchronize());
    if (ctx->bscratch) {   // the batched path's tensor-core kernels
        unsigned flag = 0;
        TG_CUDA(cudaMemcpy(&flag, ctx->bscratch, sizeof(flag), cudaMemcpyDeviceToHost));
        if (flag) {
            TG_CUDA(cudaMemset(ctx->bscratch, 0, sizeof(flag)));
            return fail(TG_ETIMEOUT, "batched path: a tensor-core expert kernel's bounded wait expired");
        }
    }
    if (!ctx->ctl) return TG_OK;
    unsigned ctl[4];
    TG_CUDA(cudaMemcpy(ctl, ctx->ctl, sizeof(ctl), cudaMemcpyDeviceToHost));
    if (ctl[2] == 0) return TG_OK;
    // a bounded wait expired inside the fused kernel: reset its cross-CTA state
    const tgx_shape& sh = ctx->shape;
    TG_CUDA(cudaMemset(ctx->facc, 0,
                       sizeof(unsigned long long) * (size_t)sh.n_layers * tg::FUSED_ACC * (sh.n_experts + 1)));
    TG_CUDA(cudaMemset(ctx->xw, 0, sizeof(unsigned long long) * (size_t)(sh.n_layers + 1) * sh.embed));
    TG_CUDA(cudaMemset(ctx->hqt, 0, sizeof(unsigned long long) * (size_t)sh.n_layers * sh.top_k * ctx->g.nbI * 6));
    unsigned fresh[4] = {ctl[0] + 1, 0, 0, 0};
    TG_CUDA(cudaMemcpy(ctx->ctl, fresh, sizeof(fresh), cudaMemcpyHostToDevice));
    return fail(TG_ETIMEOUT, "fused decode: a bounded device wait expired (stage " + std::to_string(ctl[2]) +
                                 ", layer " + std::to_string(ctl[3] >> 20) + ", entry " +
                                 std::to_string((ctl[3] >> 8) & 0xfff) + ", seen " + std::to_string(ctl[3] & 0xff) +
                                 ", finished blocks " + std::to_string(ctl[1]) + ")");
}

extern "C" int tgx_fused_debug(tgx_ctx* ctx, uint32_t* ctl4, uint64_t* acc, size_t n_acc) {
    TG_CHECK(ctx && ctl4, TG_EINVAL, "tgx_fused_debug: null argument");
    DeviceGuard dg(ctx->device);
    TG_CUDA(cudaDeviceSynchronize());
    TG_CUDA(cudaMemcpy(ctl4, ctx->ctl, 4 * sizeof(uint32_t), cudaMemcpyDeviceToHost));
    size_t have = (size_t)ctx->shape.n_layers * tg::FUSED_ACC * (ctx->shape.n_experts + 1);
    if (acc && n_acc) TG_CUDA(cudaMemcpy(acc, ctx->facc, (n_acc < have ? n_acc : have) * 8, cudaMemcpyDeviceToHost));
    return TG_OK;
}

extern "C" int tgx_fused_trace(tgx_ctx* ctx, float* x_dev, uint64_t* stamps_host, void* stream) {
    TG_CHECK(ctx && x_dev && stamps_host, TG_EINVAL, "tgx_fused_trace: null argument");
    TG_CHECK(ctx->fused_ok, TG_EUNSUPPORTED, "tgx_fused_trace: fused path not available for this shape");
    DeviceGuard dg(ctx->device);
    const size_t n = (size_t)ctx->shape.n_layers * ctx->G * tg::FUSED_TRACE;
    unsigned long long* buf = nullptr;
    TG_CUDA(cudaMalloc(&buf, n * 8));
    TG_CUDA(cudaMemset(buf, 0, n * 8));
    tg::FusedParams saved = ctx->fp;
    ctx->fp.trace = buf;
    int rc = fused_launch(ctx, 0, ctx->shape.n_layers, x_dev, (cudaStream_t)stream);
    ctx->fp = saved;
    if (rc == TG_OK) {
        cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
        if (e == cudaSuccess) e = cudaMemcpy(stamps_host, buf, n * 8, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = fail(TG_ECUDA, std::string("tgx_fused_trace: ") + cudaGetErrorString(e));
    }
    cudaFree(buf);
    return rc;
}

extern "C" int tgx_fused_info(tgx_ctx* ctx, int* ctas, int* smem_bytes, int* arena_bytes) {
    TG_CHECK(ctx, TG_EINVAL, "tgx_fused_info: null context");
    if (ctas) *ctas = ctx->fused_ok ? ctx->G : 0;
    if (smem_bytes) *smem_bytes = ctx->fused_ok ? (int)tg::fused_smem_layout(ctx->fp).total : 0;
    if (arena_bytes) *arena_bytes = ctx->fused_ok ? (int)ctx->fp.arena_bytes : 0;
    return TG_OK;
}

extern "C" int tgx_last_routing(tgx_ctx* ctx, int layer, int32_t* idx, float* w, float* logits) {
    TG_CHECK(ctx, TG_EINVAL, "tgx_last_routing: null context");
    TG_CHECK(layer >= 0 && layer < ctx->shape.n_layers, TG_EINVAL, "tgx_last_routing: layer out of range");
    DeviceGuard dg(ctx->device);
    TG_CUDA(cudaDeviceSynchronize());
    const int k = ctx->shape.top_k, E = ctx->shape.n_experts;
    if (idx) TG_CUDA(cudaMemcpy(idx, ctx->idx + (size_t)layer * k, sizeof(int) * k, cudaMemcpyDeviceToHost));
    if (w) TG_CUDA(cudaMemcpy(w, ctx->wts + (size_t)layer * k, sizeof(float) * k, cudaMemcpyDeviceToHost));
    if (logits)
        TG_CUDA(cudaMemcpy(logits, ctx->logits + (size_t)layer * E, sizeof(float) * E, cudaMemcpyDeviceToHost));
    return TG_OK;
}

// ============================================================ reference formats on device pointers

extern "C" size_t tgx_kq_matrix_bytes(int fmt, long long rows, int cols) {
    return tg::kq_valid(fmt, rows > 0 && rows < (1LL << 31) ? (int)rows : 0, cols) ? tg::kq_matrix_bytes(fmt, rows, cols)
                                                                                   : 0;
}

extern "C" int tgx_kq_prepare(int fmt, const void* src_dev, void* dst_dev, long long rows, int cols, void* stream) {
    TG_CHECK(src_dev && dst_dev && src_dev != dst_dev, TG_EINVAL, "tgx_kq_prepare: null or aliased pointers");
    TG_CHECK(rows > 0 && rows < (1LL << 31) && tg::kq_valid(fmt, (int)rows, cols), TG_EINVAL,
             "tgx_kq_prepare: bad format or shape");
    cudaStream_t s = (cudaStream_t)stream;
    if (fmt == tg::KQ_Q6K)
        TG_CUDA(tg::launch_kq_split_q6k((const uint8_t*)src_dev, (uint8_t*)dst_dev, rows * (cols / 256), s));
    else
        TG_CUDA(cudaMemcpyAsync(dst_dev, src_dev, tg::kq_matrix_bytes(fmt, rows, cols), cudaMemcpyDeviceToDevice, s));
    return TG_OK;
}

extern "C" int tgx_kq_matvec(int fmt, const void* W_dev, const float* x_dev, float* y_dev, int rows, int cols,
                             void* stream) {
    TG_CHECK(W_dev && x_dev && y_dev, TG_EINVAL, "tgx_kq_matvec: null pointer");
    TG_CHECK(tg::kq_valid(fmt, rows, cols), TG_EINVAL, "tgx_kq_matvec: bad format or shape");
    TG_CUDA(tg::launch_kq_matvec(fmt, (const uint8_t*)W_dev, x_dev, y_dev, rows, cols, (cudaStream_t)stream));
    return TG_OK;
}

extern "C" int tgx_rms_norm(const float* x_dev, const float* w_dev, float* out_dev, int dim, float eps, void* stream) {
    TG_CHECK(x_dev && w_dev && out_dev, TG_EINVAL, "tgx_rms_norm: null pointer");
    TG_CHECK(dim > 0 && dim % 4 == 0, TG_EINVAL, "tgx_rms_norm: dim must be a positive multiple of 4");
    TG_CUDA(tg::launch_rms_norm_ref(x_dev, w_dev, out_dev, dim, eps, (cudaStream_t)stream));
    return TG_OK;
}

extern "C" size_t tgx_kq_scratch_bytes(int n, int embed, int inter) {
    if (n < 1 || n > 65535 || !Geom::valid_dims(embed, inter)) return 0;
    return r256(tg::kq_down_scratch_bytes(n, embed, inter)) + sizeof(float) * (size_t)n * inter;
}

extern "C" int tgx_kq_experts_forward(const void* const* gate_dev, const void* const* up_dev,
                                      const void* const* down_dev, int down_format, int n, const float* w_dev,
                                      const float* x_dev, float* out_dev, int embed, int inter, int accumulate,
                                      void* scratch, size_t scratch_bytes, int flags, void* stream) {
    TG_CHECK(gate_dev && up_dev && down_dev && w_dev && x_dev && out_dev && scratch, TG_EINVAL,
             "tgx_kq_experts_forward: null pointer");
    TG_CHECK(n >= 1 && n <= 65535, TG_EINVAL, "tgx_kq_experts_forward: 1 <= n <= 65535");
    TG_CHECK(Geom::valid_dims(embed, inter), TG_EINVAL,
             "tgx_kq_experts_forward: embed/inter must be positive multiples of 256 (<= 16384)");
    TG_CHECK(scratch_bytes >= tgx_kq_scratch_bytes(n, embed, inter), TG_EINVAL,
             "tgx_kq_experts_forward: scratch smaller than tgx_kq_scratch_bytes(n, embed, inter)");
    TG_CHECK(((uintptr_t)scratch & 255) == 0, TG_EINVAL, "tgx_kq_experts_forward: scratch must be 256-byte aligned");
    int fmt;
    switch (down_format) {
        case TG_FMT_Q4_K: fmt = tg::KQ_Q4K; break;
        case TG_FMT_F16: fmt = tg::KQ_F16; break;
        case TG_FMT_Q6_K: fmt = tg::KQ_Q6K; break;
        default: return fail(TG_EINVAL, "tgx_kq_experts_forward: down_format must be 0 (Q4_K), 1 (f16) or 2 (Q6_K)");
    }
    cudaStream_t s = (cudaStream_t)stream;
    void* ds = scratch;
    float* h = (float*)((uint8_t*)scratch + r256(tg::kq_down_scratch_bytes(n, embed, inter)));
    TG_CUDA(tg::launch_kq_gateup((const uint8_t* const*)gate_dev, (const uint8_t* const*)up_dev, n, x_dev, embed,
                                 inter, h, (flags & TGX_KQ_CHAINED) != 0, s));
    TG_CUDA(tg::launch_kq_down(fmt, (const uint8_t* const*)down_dev, n, h, w_dev, embed, inter, out_dev,
                               accumulate, ds, s));
    return TG_OK;
}

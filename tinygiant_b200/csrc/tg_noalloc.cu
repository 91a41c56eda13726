// tg_noalloc.cu — tg_expert_forward_q4_0_noalloc: the expert forward of
// tg_expert_forward_q4_0 on device pointers and a caller stream, with no
// device or host allocation anywhere on the call path.
//
// Who needs it: a caller whose device memory is already fully committed (a
// serving process that has carved HBM into its own weight and cache pools and
// cannot have a library grow a workspace behind its back), and a caller on a
// latency-bound decode loop, where cudaMalloc/cudaFree may block on other
// work of the device and a failed allocation mid-step has no recovery.  The
// host-pointer entry points cannot serve them: they grow a shared workspace
// with cudaMalloc on demand.
//
// Scratch: one file-scope __device__ array of TG_NOALLOC_SCRATCH_BYTES per
// device (the module's own static storage, created with the module).  Its
// address is taken once per device with cudaGetSymbolAddress, by the first
// call made while that device is current; that first call also writes a
// one-entry pointer table at the start of the scratch (a synchronous copy).
// Make the first call on each device before any stream capture.
//
// Layout of the scratch (offsets in bytes):
//   [0, 256)              device pointer table of one entry: the expert copy below
//   [256, 256 + EB)       the expert repacked into the row-split layout (EB = expert bytes)
//   [256 + EB', + A)      Q8_0 activation form of h (A = 40 bytes per 32 values of I),
//                         EB' = EB rounded up to 256
// Nothing in it needs to start at zero: every byte a call reads was written
// earlier by the same call, or by the set-up (the pointer table).
//
// Calls share the one scratch of their device, so calls that overlap in time
// on one device (two streams, or two host threads without ordering) race and
// corrupt each other's results; order them on one stream or with events.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "../../include/tinygiant.h"
#include "tg_internal.h"

using tg::Geom;

namespace {

constexpr size_t kTableBytes = 256;
constexpr int kMaxDevices = 64;

static_assert(TG_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size must be a multiple of 256");

static __device__ __align__(256) unsigned char g_noalloc_scratch[TG_NOALLOC_SCRATCH_BYTES];

std::mutex g_setup_mu;
uint8_t* g_scratch_ptr[kMaxDevices];  // per device, set once by setup_scratch

size_t round256(size_t n) { return (n + 255) & ~(size_t)255; }

size_t scratch_needed(const Geom& g) {
    return kTableBytes + round256(g.expert_bytes) + tg::act_bytes(g.nbI);
}

// Address of this device's scratch; the first call per device takes it with
// cudaGetSymbolAddress and stores the pointer table.
int setup_scratch(int dev, uint8_t** out) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        uint8_t* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr)
            return tg::set_error(TG_ECUDA, (std::string("tg_expert_forward_q4_0_noalloc: cudaGetSymbolAddress: ") +
                                            cudaGetErrorString(e)).c_str());
        const uint8_t* expert = ptr + kTableBytes;
        e = cudaMemcpy(ptr, &expert, sizeof(expert), cudaMemcpyHostToDevice);
        if (e != cudaSuccess)
            return tg::set_error(TG_ECUDA, (std::string("tg_expert_forward_q4_0_noalloc: pointer table: ") +
                                            cudaGetErrorString(e)).c_str());
        g_scratch_ptr[dev] = ptr;
    }
    *out = g_scratch_ptr[dev];
    return TG_OK;
}

bool on_device(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace

extern "C" int tg_expert_forward_q4_0_noalloc(const uint8_t* q4_data, const float* input, float* output,
                                              float weight, int embed_dim, int inter_dim, void* stream) {
    static const char* fn = "tg_expert_forward_q4_0_noalloc: ";
    if (!q4_data || !input || !output)
        return tg::set_error(TG_EINVAL, (std::string(fn) + "null pointer").c_str());
    if (!Geom::valid_dims(embed_dim, inter_dim))
        return tg::set_error(TG_EINVAL, (std::string(fn) + "embed/inter must be positive multiples of 256").c_str());
    Geom g = Geom::make(embed_dim, inter_dim);
    size_t need = scratch_needed(g);
    if (need > (size_t)TG_NOALLOC_SCRATCH_BYTES)
        return tg::set_error(TG_EINVAL, (std::string(fn) + "an expert of embed " + std::to_string(embed_dim) +
                                         " x inter " + std::to_string(inter_dim) + " needs " + std::to_string(need) +
                                         " bytes of scratch; the fixed scratch holds " +
                                         std::to_string((size_t)TG_NOALLOC_SCRATCH_BYTES))
                                            .c_str());
    if (((uintptr_t)q4_data & 1) || ((uintptr_t)input & 3) || ((uintptr_t)output & 3))
        return tg::set_error(TG_EINVAL, (std::string(fn) + "q4_data must be 2-byte and input/output 4-byte aligned").c_str());
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return tg::set_error(TG_ENODEV, "no CUDA device");
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return tg::set_error(TG_ECUDA, (std::string(fn) + "no usable current device").c_str());
    if (!on_device(q4_data) || !on_device(input) || !on_device(output))
        return tg::set_error(TG_EINVAL, (std::string(fn) + "q4_data, input and output must be device memory").c_str());

    uint8_t* scratch = nullptr;
    int rc = setup_scratch(dev, &scratch);
    if (rc != TG_OK) return rc;
    const uint8_t* const* table = (const uint8_t* const*)scratch;
    uint8_t* expert = scratch + kTableBytes;
    uint8_t* hq = expert + round256(g.expert_bytes);
    cudaStream_t s = (cudaStream_t)stream;

    cudaError_t e = tg::prepare_kernels(g, 1);
    if (e == cudaSuccess) e = tg::launch_repack_rows(q4_data, expert, 2LL * g.I, g.nbH, s);
    if (e == cudaSuccess) e = tg::launch_repack_rows(q4_data + 2 * g.t_gu, expert + 2 * g.t_gu, g.H, g.nbI, s);
    if (e == cudaSuccess) e = tg::launch_gateup(table, 1, input, nullptr, nullptr, g, hq, nullptr, nullptr, s);
    if (e == cudaSuccess)
        e = tg::launch_down_combine(table, 1, hq, nullptr, weight, g, nullptr, output, 1, nullptr, s);
    if (e != cudaSuccess)
        return tg::set_error(TG_ECUDA, (std::string(fn) + cudaGetErrorString(e)).c_str());
    return TG_OK;
}

// tg_layout.h — byte layout of Q4_0 experts in HBM, shared by host and device code.
//
// On disk and at the C-ABI an expert is the reference's expert-contiguous blob
// (tinygiant/relayout.py:142-157): gate | up | down, each a row-major matrix of
// ggml Q4_0 blocks (18 B: fp16 d, 16 B nibbles), rows contiguous.
//
// In HBM each row is stored "row-split": the 16-byte nibble groups of all its
// blocks first, then the fp16 scales of all its blocks.  The row keeps its
// ggml byte length (18 * nb) and position, so an expert keeps its size and
// offsets, but every nibble group starts on a 16-byte boundary and a lane
// fetches a whole block with one 128-bit load.  Rows must hold a multiple of 8
// blocks (row length a multiple of 256 values) so rows stay 16-byte aligned.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#define TG_HD __host__ __device__ __forceinline__
#else
#define TG_HD inline
#endif

namespace tg {

constexpr int QK = 32;            // block length of Q4_0 and Q8_0
constexpr int Q4_0_BYTES = 18;    // ggml Q4_0 block: fp16 d | u8 qs[16]
constexpr int Q8_0_BYTES = 34;    // ggml Q8_0 block: fp16 d | i8 qs[32]

struct Geom {
    int H = 0;        // hidden (embed) size: gate/up input, down output
    int I = 0;        // expert intermediate size
    int nbH = 0;      // H / 32 blocks per gate/up row
    int nbI = 0;      // I / 32 blocks per down row
    size_t row_gu = 0;  // bytes per gate/up row
    size_t row_d = 0;   // bytes per down row
    size_t t_gu = 0;    // bytes of the gate (or up) matrix
    size_t t_d = 0;     // bytes of the down matrix
    size_t expert_bytes = 0;

    static bool valid_dims(int H, int I) {
        return H > 0 && I > 0 && H % 256 == 0 && I % 256 == 0 && H <= 16384 && I <= 16384;
    }
    static Geom make(int H, int I) {
        Geom g;
        g.H = H;
        g.I = I;
        g.nbH = H / 32;
        g.nbI = I / 32;
        g.row_gu = (size_t)g.nbH * 18;
        g.row_d = (size_t)g.nbI * 18;
        g.t_gu = (size_t)I * g.row_gu;
        g.t_d = (size_t)H * g.row_d;
        g.expert_bytes = 2 * g.t_gu + g.t_d;
        return g;
    }
};

// Activation vector quantised to Q8_0, in the kernels' working form:
// codes [nb][32] int8, then fp32 value of each stored fp16 scale, then 8*sum(codes).
struct ActView {
    int8_t* qs;
    float* d;
    int* s8;
};
TG_HD size_t act_bytes(int nb) { return (size_t)nb * 32 + (size_t)nb * 8; }
template <typename P>
TG_HD ActView act_view(P* base, int nb) {
    ActView a;
    uint8_t* b = (uint8_t*)base;
    a.qs = (int8_t*)b;
    a.d = (float*)(b + (size_t)nb * 32);
    a.s8 = (int*)(b + (size_t)nb * 36);
    return a;
}

}  // namespace tg

// Pruned 16-point DFTs: compile-time masks tell which inputs can be non-zero and which outputs
// are needed, so truncated spectra (the kept FNO modes) cost only the arithmetic they need.
//
//   dft16_m<INV, IN, OUT>(a): a[n] for n with bit n of IN set are inputs (others are zero and not
//   read); on return a[k] holds output k for every bit k of OUT (other entries are unspecified).
//
// Same factorisation as fft::dft16 (n = 4 n1 + n2, k = k1 + 4 k2): column DFTs over n1, twiddles
// W16^(n2 k1), row DFTs over n2.  Zero columns are skipped; rows compute only the needed outputs
// (direct sums of +-1 / +-i multiples when fewer than three are needed).
#pragma once

#include "fft_core.cuh"

namespace nop {
namespace fft {

// a * W4^m (m folded to 0..3 at compile time after inlining)
template <bool INV>
__device__ __forceinline__ float2 rot4(float2 a, int m) {
    m &= 3;
    if (m == 0) return a;
    if (m == 1) return mul_rot<INV>(a);
    if (m == 2) return make_float2(-a.x, -a.y);
    return mul_rot<!INV>(a);
}

// cos(2 pi m / 16) and sin(2 pi m / 16) as constant expressions
__host__ __device__ constexpr float cos16(int m) {
    constexpr float c1 = 0.92387953251128674f, c2 = 0.70710678118654757f, c3 = 0.38268343236508978f;
    switch (m & 15) {
        case 0: return 1.0f;
        case 1: return c1;
        case 2: return c2;
        case 3: return c3;
        case 4: return 0.0f;
        case 5: return -c3;
        case 6: return -c2;
        case 7: return -c1;
        case 8: return -1.0f;
        case 9: return -c1;
        case 10: return -c2;
        case 11: return -c3;
        case 12: return 0.0f;
        case 13: return c3;
        case 14: return c2;
        default: return c1;
    }
}
__host__ __device__ constexpr float sin16(int m) { return cos16(m - 4); }

// a * W16^m with m a constant after inlining
template <bool INV>
__device__ __forceinline__ float2 tw16r(float2 a, int m) {
    m &= 15;
    if ((m & 3) == 0) return rot4<INV>(a, m >> 2);
    const float c = cos16(m);
    const float s = INV ? sin16(m) : -sin16(m);
    return make_float2(fmaf(a.x, c, -a.y * s), fmaf(a.x, s, a.y * c));
}

__host__ __device__ constexpr int popc4(unsigned v) { return (v & 1) + ((v >> 1) & 1) + ((v >> 2) & 1) + ((v >> 3) & 1); }

// 4-point DFT of (x0..x3) with non-zero input mask NZ; outputs with bit k of NEED are written to y[k]
template <bool INV>
__device__ __forceinline__ void dft4_m(const float2* x, unsigned NZ, unsigned NEED, float2* y) {
    if (NZ == 15 && popc4(NEED) >= 3) {
        float2 x0 = x[0], x1 = x[1], x2 = x[2], x3 = x[3];
        dft4<INV>(x0, x1, x2, x3);
        y[0] = x0;
        y[1] = x1;
        y[2] = x2;
        y[3] = x3;
        return;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if (!((NEED >> k) & 1)) continue;
        bool first = true;
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (!((NZ >> j) & 1)) continue;
            const float2 term = rot4<INV>(x[j], j * k);
            acc = first ? term : cadd(acc, term);
            first = false;
        }
        y[k] = acc;
    }
}

template <bool INV, unsigned IN, unsigned OUT>
__device__ __forceinline__ void dft16_m(float2* a) {
    float2 A[4][4];  // A[n2][k1]
    unsigned colnz = 0;
    // k1 values whose outputs are needed by some k2
    constexpr unsigned need_k1 = ((OUT | (OUT >> 4) | (OUT >> 8) | (OUT >> 12)) & 15u);
#pragma unroll
    for (int n2 = 0; n2 < 4; ++n2) {
        const unsigned nz = ((IN >> n2) & 1u) | (((IN >> (n2 + 4)) & 1u) << 1) | (((IN >> (n2 + 8)) & 1u) << 2) |
                            (((IN >> (n2 + 12)) & 1u) << 3);
        if (nz == 0) continue;
        colnz |= 1u << n2;
        const float2 x[4] = {a[n2], a[n2 + 4], a[n2 + 8], a[n2 + 12]};
        dft4_m<INV>(x, nz, need_k1, A[n2]);
#pragma unroll
        for (int k1 = 1; k1 < 4; ++k1)
            if ((need_k1 >> k1) & 1) A[n2][k1] = tw16r<INV>(A[n2][k1], n2 * k1);
    }
#pragma unroll
    for (int k1 = 0; k1 < 4; ++k1) {
        const unsigned need = ((OUT >> k1) & 1u) | (((OUT >> (k1 + 4)) & 1u) << 1) | (((OUT >> (k1 + 8)) & 1u) << 2) |
                              (((OUT >> (k1 + 12)) & 1u) << 3);
        if (need == 0) continue;
        const float2 x[4] = {A[0][k1], A[1][k1], A[2][k1], A[3][k1]};
        float2 y[4];
        dft4_m<INV>(x, colnz, need, y);
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2)
            if ((need >> k2) & 1) a[k1 + 4 * k2] = y[k2];
    }
}

}  // namespace fft
}  // namespace nop

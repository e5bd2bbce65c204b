// Register-blocked Stockham FFT for one line of length N (power of two, 16..512), computed by a
// group of G = N/16 consecutive lanes of one warp.  Every lane holds 16 complex values; passes of
// radix 16 (and one final pass of radix 2, 4 or 8) exchange data through a padded shared-memory
// line buffer, one exchange per pass.  Decimation in time, self-sorting (Stockham):
//
//   pass with radix R after passes whose radices multiply to NS, butterfly j in [0, N/R):
//     v[r] = in[j + r N/R] * W_{NS R}^{r (j mod NS)},  v = DFT_R(v),
//     out[(j / NS) NS R + (j mod NS) + r NS] = v[r]
//
// The first pass reads through a caller functor (global memory, a sparse spectrum, ...) and the
// last pass writes through another, so truncation and epilogues fuse into the transform.
#pragma once

#include <cuda_runtime.h>

namespace nop {
namespace fft {

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }

// multiply by -i (forward transform) or +i (inverse transform)
template <bool INV>
__device__ __forceinline__ float2 mul_rot(float2 a) {
    return INV ? make_float2(-a.y, a.x) : make_float2(a.y, -a.x);
}

// cos(2 pi m / 16), sin(2 pi m / 16)
constexpr float kC16[16] = {1.0f, 0.92387953251128674f, 0.70710678118654757f, 0.38268343236508978f,
                            0.0f, -0.38268343236508978f, -0.70710678118654757f, -0.92387953251128674f,
                            -1.0f, -0.92387953251128674f, -0.70710678118654757f, -0.38268343236508978f,
                            0.0f, 0.38268343236508978f, 0.70710678118654757f, 0.92387953251128674f};
constexpr float kS16[16] = {0.0f, 0.38268343236508978f, 0.70710678118654757f, 0.92387953251128674f,
                            1.0f, 0.92387953251128674f, 0.70710678118654757f, 0.38268343236508978f,
                            0.0f, -0.38268343236508978f, -0.70710678118654757f, -0.92387953251128674f,
                            -1.0f, -0.92387953251128674f, -0.70710678118654757f, -0.38268343236508978f};

// a * W16^m  (W = e^{-2 pi i/16} forward, e^{+2 pi i/16} inverse), m a compile-time constant
template <bool INV, int M>
__device__ __forceinline__ float2 tw16(float2 a) {
    constexpr int m = M & 15;
    if constexpr (m == 0) {
        return a;
    } else if constexpr (m == 4) {
        return mul_rot<INV>(a);
    } else if constexpr (m == 8) {
        return make_float2(-a.x, -a.y);
    } else if constexpr (m == 12) {
        return mul_rot<!INV>(a);
    } else {
        constexpr float c = kC16[m];
        constexpr float s = INV ? kS16[m] : -kS16[m];
        return make_float2(fmaf(a.x, c, -a.y * s), fmaf(a.x, s, a.y * c));
    }
}

template <bool INV>
__device__ __forceinline__ void dft2(float2& a, float2& b) {
    float2 t = a;
    a = cadd(t, b);
    b = csub(t, b);
}

template <bool INV>
__device__ __forceinline__ void dft4(float2& a0, float2& a1, float2& a2, float2& a3) {
    float2 s02 = cadd(a0, a2), d02 = csub(a0, a2);
    float2 s13 = cadd(a1, a3), d13 = mul_rot<INV>(csub(a1, a3));
    a0 = cadd(s02, s13);
    a2 = csub(s02, s13);
    a1 = cadd(d02, d13);
    a3 = csub(d02, d13);
}

// 8-point DFT in natural order (n = 2 n1 + n2, k = k1 + 4 k2)
template <bool INV>
__device__ __forceinline__ void dft8(float2* a) {
    dft4<INV>(a[0], a[2], a[4], a[6]);
    dft4<INV>(a[1], a[3], a[5], a[7]);
    a[3] = tw16<INV, 2>(a[3]);
    a[5] = tw16<INV, 4>(a[5]);
    a[7] = tw16<INV, 6>(a[7]);
    dft2<INV>(a[0], a[1]);
    dft2<INV>(a[2], a[3]);
    dft2<INV>(a[4], a[5]);
    dft2<INV>(a[6], a[7]);
    // X[k1 + 4 k2] sits at a[2 k1 + k2]
    float2 t[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = a[2 * (k & 3) + (k >> 2)];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = t[k];
}

template <bool INV, int N2>
__device__ __forceinline__ void dft16_twiddle_row(float2* a) {
    a[4 * 1 + N2] = tw16<INV, N2 * 1>(a[4 * 1 + N2]);
    a[4 * 2 + N2] = tw16<INV, N2 * 2>(a[4 * 2 + N2]);
    a[4 * 3 + N2] = tw16<INV, N2 * 3>(a[4 * 3 + N2]);
}

// 16-point DFT in natural order (n = 4 n1 + n2, k = k1 + 4 k2)
template <bool INV>
__device__ __forceinline__ void dft16(float2* a) {
#pragma unroll
    for (int n2 = 0; n2 < 4; ++n2) dft4<INV>(a[n2], a[4 + n2], a[8 + n2], a[12 + n2]);
    dft16_twiddle_row<INV, 1>(a);
    dft16_twiddle_row<INV, 2>(a);
    dft16_twiddle_row<INV, 3>(a);
#pragma unroll
    for (int k1 = 0; k1 < 4; ++k1) dft4<INV>(a[4 * k1], a[4 * k1 + 1], a[4 * k1 + 2], a[4 * k1 + 3]);
    // X[k1 + 4 k2] sits at a[4 k1 + k2]
    float2 t[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) t[k] = a[4 * (k & 3) + (k >> 2)];
#pragma unroll
    for (int k = 0; k < 16; ++k) a[k] = t[k];
}

template <int R, bool INV>
__device__ __forceinline__ void dft_r(float2* a) {
    if constexpr (R == 2) {
        dft2<INV>(a[0], a[1]);
    } else if constexpr (R == 4) {
        dft4<INV>(a[0], a[1], a[2], a[3]);
    } else if constexpr (R == 8) {
        dft8<INV>(a);
    } else {
        dft16<INV>(a);
    }
}

__host__ __device__ constexpr int ilog2(int n) { return n <= 1 ? 0 : 1 + ilog2(n / 2); }

// padded index inside a line buffer: one spare slot every 16 entries (conflict-free exchanges)
__device__ __forceinline__ int pad(int i) { return i + (i >> 4); }

template <int N>
struct LineShape {
    static constexpr int G = N / 16;                  // lanes per line
    static constexpr int P = ilog2(N);
    static constexpr int N16 = P / 4;                 // radix-16 passes
    static constexpr int RLAST = 1 << (P % 4);        // final small radix (1: none)
    static constexpr int BUF = N + N / 16;            // padded line length
    static_assert(N >= 16 && N <= 512 && (N & (N - 1)) == 0, "line length must be a power of two in 16..512");
};

// twiddle from the shared table tw[k] = (cos 2 pi k / N, sin 2 pi k / N)
template <bool INV>
__device__ __forceinline__ float2 table_tw(const float2* tw, int k) {
    float2 w = tw[k];
    return INV ? w : make_float2(w.x, -w.y);
}

// One line transform.  Lane t in [0, G) of the group; `buf` is the group's padded line buffer
// (LineShape<N>::BUF entries, may alias the data the loader reads -- the first pass finishes
// every load before it writes).  load(i) returns input element i; store(k, v) receives output k.
// A group with no line to transform passes active = false: it still reaches every warp barrier
// but writes nothing to `buf` (which may then point at another group's line).
// line_fft with the first pass's inputs already in registers: v[r] = element t + r G.
template <int N, bool INV, class Store>
__device__ __forceinline__ void line_fft_regs(float2 (&v)[16], float2* buf, const float2* tw, int t, bool active,
                                              Store&& store) {
    using S = LineShape<N>;
    constexpr int G = S::G;
    // ---- pass 1: radix 16, NS = 1 ----
    dft16<INV>(v);
    if constexpr (S::N16 == 1 && S::RLAST == 1) {
#pragma unroll
        for (int r = 0; r < 16; ++r) store(16 * t + r, v[r]);
        return;
    } else {
        __syncwarp();
        if (active) {
#pragma unroll
            for (int r = 0; r < 16; ++r) buf[pad(16 * t + r)] = v[r];
        }
        __syncwarp();
        // ---- further radix-16 passes ----
        constexpr int NS16_LAST = (S::RLAST == 1) ? S::N16 - 1 : -1;  // index of a radix-16 final pass
#pragma unroll
        for (int s = 1; s < S::N16; ++s) {
            const int NS = 1 << (4 * s);
            const int k = t & (NS - 1);
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = buf[pad(t + r * G)];
            const int step = k * (N / (NS * 16));
#pragma unroll
            for (int r = 1; r < 16; ++r) v[r] = cmul(v[r], table_tw<INV>(tw, r * step));
            dft16<INV>(v);
            __syncwarp();
            const int base = (t / NS) * NS * 16 + k;
            if (s == NS16_LAST) {
#pragma unroll
                for (int r = 0; r < 16; ++r) store(base + r * NS, v[r]);
            } else {
                if (active) {
#pragma unroll
                    for (int r = 0; r < 16; ++r) buf[pad(base + r * NS)] = v[r];
                }
                __syncwarp();
            }
        }
        // ---- final small-radix pass ----
        if constexpr (S::RLAST > 1) {
            constexpr int R = S::RLAST;
            constexpr int NB = 16 / R;
            constexpr int NS = N / R;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const int j = t + G * b;
#pragma unroll
                for (int r = 0; r < R; ++r) v[b * R + r] = buf[pad(j + r * NS)];
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const int j = t + G * b;
                const int k = j & (NS - 1);
                // step = k * N / (NS * R) = k
#pragma unroll
                for (int r = 1; r < R; ++r) v[b * R + r] = cmul(v[b * R + r], table_tw<INV>(tw, r * k));
                dft_r<R, INV>(v + b * R);
            }
            __syncwarp();
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const int j = t + G * b;
#pragma unroll
                for (int r = 0; r < R; ++r) store(j + r * NS, v[b * R + r]);
            }
        }
    }
}

template <int N, bool INV, class Load, class Store>
__device__ __forceinline__ void line_fft(float2* buf, const float2* tw, int t, bool active, Load&& load,
                                         Store&& store) {
    constexpr int G = LineShape<N>::G;
    float2 v[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) v[r] = load(t + r * G);
    line_fft_regs<N, INV>(v, buf, tw, t, active, store);
}

}  // namespace fft
}  // namespace nop

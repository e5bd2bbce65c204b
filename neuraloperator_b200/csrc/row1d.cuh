// Fused 1D kernels for long real lines with few kept bins (the Burgers configuration: N = 8192,
// 9 kept rFFT bins).  With K << N a full FFT wastes work, so each line is decimated by 16:
//
//   forward  X[k] = sum_{n1 < Q} W_N^{k n1} D_{n1}[k mod 16],   D_{n1} = DFT16 { x[n1 + Q j] }_j,  Q = N/16
//   inverse  y[n1 + Q j] = Re sum_k c_k Z_k W_N^{-k n1} w16^{k j}  =  IDFT16(H_{n1})[j]
//
// Two subsequences (n1 and n1 + Q/2) share one complex DFT16 (real/imaginary packing); H is the
// Hermitian part of the twiddled bins so the packed inverse returns both real subsequences.
// 64 lanes work on one line; the forward partial sums are reduced with shuffles and shared memory.
// Output / input spectra use the mode-blocked layout [Q8][lines][8] of the contraction.
#pragma once

#include "fft_core.cuh"
#include "l2_hints.cuh"
#include "nop_internal.cuh"

namespace nop {
namespace r1d {

constexpr int THREADS = 256;
constexpr int TPR = 64;                 // lanes per line
constexpr int LINES = THREADS / TPR;    // lines per CTA

template <int N, int K>
__global__ void __launch_bounds__(THREADS)
k_fwd(const float* __restrict__ x, float2* __restrict__ out, const float2* __restrict__ tw, int64_t L, float scale,
      int64_t blk_stride) {
    static_assert(K >= 1 && K <= 32, "kept bins per line must be in 1..32");
    constexpr int Q = N / 16;
    constexpr int PAIRS = Q / 2;
    constexpr int PER = PAIRS / TPR;  // pairs per lane
    static_assert(PER >= 1 && PAIRS % TPR == 0, "line too short for 64 lanes");
    __shared__ float2 part[LINES][TPR / 32][K];
    const int lane64 = threadIdx.x % TPR;
    const int lr = threadIdx.x / TPR;
    const int64_t line = (int64_t)blockIdx.x * LINES + lr;
    const bool active = line < L;
    const float* xl = x + (active ? line : 0) * (int64_t)N;
    const uint64_t pol_x = l2::evict_first();  // x is read once
    float2 acc[K];
#pragma unroll
    for (int k = 0; k < K; ++k) acc[k] = make_float2(0.f, 0.f);
#pragma unroll 1
    for (int s = 0; s < PER; ++s) {
        const int na = lane64 + TPR * s, nb = na + PAIRS;
        float2 z[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
            z[j] = active ? make_float2(l2::ld(xl + na + Q * j, pol_x), l2::ld(xl + nb + Q * j, pol_x))
                          : make_float2(0.f, 0.f);
        fft::dft16<false>(z);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const float2 zk = z[k & 15], zn = z[(16 - k) & 15];
            const float2 da = make_float2(0.5f * (zk.x + zn.x), 0.5f * (zk.y - zn.y));
            const float2 db = make_float2(0.5f * (zk.y + zn.y), 0.5f * (zn.x - zk.x));
            const float2 wa = __ldg(tw + ((k * na) & (N - 1)));
            const float2 wb = __ldg(tw + ((k * nb) & (N - 1)));
            // acc += conj(wa) da + conj(wb) db   (forward twiddles e^{-i theta})
            acc[k].x = fmaf(wa.x, da.x, fmaf(wa.y, da.y, acc[k].x));
            acc[k].y = fmaf(wa.x, da.y, fmaf(-wa.y, da.x, acc[k].y));
            acc[k].x = fmaf(wb.x, db.x, fmaf(wb.y, db.y, acc[k].x));
            acc[k].y = fmaf(wb.x, db.y, fmaf(-wb.y, db.x, acc[k].y));
        }
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            acc[k].x += __shfl_xor_sync(0xffffffffu, acc[k].x, off);
            acc[k].y += __shfl_xor_sync(0xffffffffu, acc[k].y, off);
        }
    }
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
        for (int k = 0; k < K; ++k) part[lr][lane64 / 32][k] = acc[k];
    }
    __syncthreads();
    constexpr int QB = (K + 7) / 8;
    if (active && lane64 < 8 * QB) {
        const int k = lane64;
        float2 v = make_float2(0.f, 0.f);
        if (k < K) {
#pragma unroll
            for (int w = 0; w < TPR / 32; ++w) {
                v.x += part[lr][w][k].x;
                v.y += part[lr][w][k].y;
            }
            v = fft::cscale(v, scale);
        }
        l2::st2(out + (k >> 3) * blk_stride + line * 8 + (k & 7), v, l2::evict_last());
    }
}

struct Epi1 {
    const float* bias;
    const float* addend;
    int apply_gelu;
    int C;
};

template <int N, int K>
__global__ void __launch_bounds__(THREADS)
k_inv(const float2* __restrict__ in, float* __restrict__ y, const float2* __restrict__ tw, int64_t L, float scale,
      int64_t blk_stride, Epi1 ep) {
    static_assert(K >= 1 && K <= 32, "kept bins per line must be in 1..32");
    constexpr int Q = N / 16;
    constexpr int PAIRS = Q / 2;
    constexpr int PER = PAIRS / TPR;
    __shared__ float2 zs[LINES][K];
    const int lane64 = threadIdx.x % TPR;
    const int lr = threadIdx.x / TPR;
    const int64_t line = (int64_t)blockIdx.x * LINES + lr;
    const bool active = line < L;
    if (active && lane64 < K) {
        float2 v = l2::ld2(in + (lane64 >> 3) * blk_stride + line * 8 + (lane64 & 7), l2::evict_first());
        if (lane64 == 0) v.y = 0.f;                      // bin 0 contributes its real part only
        zs[lr][lane64] = lane64 == 0 ? v : fft::cscale(v, 2.f);  // Hermitian weights 1, 2, 2, ...
    }
    __syncthreads();
    if (!active) return;
    float2 Z[K];
#pragma unroll
    for (int k = 0; k < K; ++k) Z[k] = zs[lr][k];
    const float bias = ep.bias ? ep.bias[line % ep.C] : 0.f;
    float* yl = y + line * (int64_t)N;
    const float* al = ep.addend ? ep.addend + line * (int64_t)N : nullptr;
    const uint64_t pol_y = l2::evict_first();  // y (and the skip addend) stream through
#pragma unroll 1
    for (int s = 0; s < PER; ++s) {
        const int na = lane64 + TPR * s, nb = na + PAIRS;
        float2 va[16], vb[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) va[m] = vb[m] = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < K; ++k) {  // V_k = c_k Z_k e^{+i theta k n1}, folded onto k mod 16
            const float2 wa = __ldg(tw + ((k * na) & (N - 1)));
            const float2 wb = __ldg(tw + ((k * nb) & (N - 1)));
            if (k < 16) {
                va[k] = fft::cmul(Z[k], wa);
                vb[k] = fft::cmul(Z[k], wb);
            } else {
                va[k & 15] = fft::cadd(va[k & 15], fft::cmul(Z[k], wa));
                vb[k & 15] = fft::cadd(vb[k & 15], fft::cmul(Z[k], wb));
            }
        }
        // U = H(va) + i H(vb), H(v)[m] = (v[m] + conj v[-m]) / 2
        float2 u[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const int mm = (16 - m) & 15;
            const float2 ha = make_float2(0.5f * (va[m].x + va[mm].x), 0.5f * (va[m].y - va[mm].y));
            const float2 hb = make_float2(0.5f * (vb[m].x + vb[mm].x), 0.5f * (vb[m].y - vb[mm].y));
            u[m] = make_float2(ha.x - hb.y, ha.y + hb.x);
        }
        fft::dft16<true>(u);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            float ra = u[j].x * scale + bias;
            float rb = u[j].y * scale + bias;
            if (al) {
                ra += l2::ld(al + na + Q * j, pol_y);
                rb += l2::ld(al + nb + Q * j, pol_y);
            }
            if (ep.apply_gelu) {
                ra = gelu_erf(ra);
                rb = gelu_erf(rb);
            }
            l2::st(yl + na + Q * j, ra, pol_y);
            l2::st(yl + nb + Q * j, rb, pol_y);
        }
    }
}

}  // namespace r1d
}  // namespace nop

// Outer-axis transforms of the 3D spectral block.  After the (y, z) plane kernels, the kept plane
// modes of every x-plane sit in the mode-blocked layout P[qp][(bc, x)][j] (8 modes per block).
// For one (qp, bc) the 8 lines (j) over x are N * 8 complex values; these kernels transform them
// along x (keeping MX centred bins forward, expanding them inverse) and write / read the
// contraction's mode-blocked layout with total mode (mx, plane mode):
//     X^[(mx * QP + qp)][bc][j]        QP = plane-mode blocks handled here
// The x lines may be split into segments of nx_seg planes that lie seg_stride complex values apart
// (one segment per source rank after the slab exchange); element (qp, bc, x, j) is at
//     seg(x) * seg_stride + ((qp * BC + bc) * nx_seg + x mod nx_seg) * 8 + j.
#pragma once

#include "fft_core.cuh"
#include "nop_internal.cuh"

namespace nop {
namespace axis {

constexpr int N = 256;
constexpr int LANES = 16;        // lanes per line
constexpr int THREADS = 8 * LANES;
constexpr int LINE = N + N / 16;

template <int MX>
__global__ void __launch_bounds__(THREADS)
k_fwd(const float2* __restrict__ P, float2* __restrict__ Xh, const float2* __restrict__ twg, int QP, int64_t BC,
      int nx_seg, int64_t seg_stride) {
    __shared__ float2 tw[N];
    __shared__ __align__(16) float2 lines[8][LINE];
    __shared__ __align__(16) float2 stage[MX][8];
    const int64_t qp = blockIdx.x % QP;
    const int64_t bc = blockIdx.x / QP;
    const int j = threadIdx.x / LANES, t = threadIdx.x % LANES;
    for (int i = threadIdx.x; i < N; i += THREADS) tw[i] = twg[i];
    const float2* blk = P + (qp * BC + bc) * nx_seg * 8;
    for (int e = threadIdx.x; e < N * 4; e += THREADS) {  // (x, j pair)
        const int x = e >> 2, jj = 2 * (e & 3);
        const float4 v = __ldg(reinterpret_cast<const float4*>(blk + (x / nx_seg) * seg_stride + (x % nx_seg) * 8 + jj));
        lines[jj][fft::pad(x)] = make_float2(v.x, v.y);
        lines[jj + 1][fft::pad(x)] = make_float2(v.z, v.w);
    }
    __syncthreads();
    float2* buf = lines[j];
    fft::line_fft<N, false>(
        buf, tw, t, true, [&](int i) { return buf[fft::pad(i)]; },
        [&](int k, float2 v) {
            const int m = (k + MX / 2) & (N - 1);
            if (m < MX) stage[m][j] = v;
        });
    __syncthreads();
    for (int e = threadIdx.x; e < MX * 4; e += THREADS) {
        const int mx = e >> 2, jj = 2 * (e & 3);
        float2* dst = Xh + ((mx * (int64_t)QP + qp) * BC + bc) * 8 + jj;
        *reinterpret_cast<float4*>(dst) = make_float4(stage[mx][jj].x, stage[mx][jj].y, stage[mx][jj + 1].x,
                                                      stage[mx][jj + 1].y);
    }
}

template <int MX>
__global__ void __launch_bounds__(THREADS)
k_inv(const float2* __restrict__ Yh, float2* __restrict__ P, const float2* __restrict__ twg, int QP, int64_t BC,
      int nx_seg, int64_t seg_stride) {
    __shared__ float2 tw[N];
    __shared__ __align__(16) float2 lines[8][LINE];
    __shared__ __align__(16) float2 stage[MX][8];
    const int64_t qp = blockIdx.x % QP;
    const int64_t bc = blockIdx.x / QP;
    const int j = threadIdx.x / LANES, t = threadIdx.x % LANES;
    for (int i = threadIdx.x; i < N; i += THREADS) tw[i] = twg[i];
    for (int e = threadIdx.x; e < MX * 4; e += THREADS) {
        const int mx = e >> 2, jj = 2 * (e & 3);
        const float4 v = __ldg(reinterpret_cast<const float4*>(Yh + ((mx * (int64_t)QP + qp) * BC + bc) * 8 + jj));
        stage[mx][jj] = make_float2(v.x, v.y);
        stage[mx][jj + 1] = make_float2(v.z, v.w);
    }
    __syncthreads();
    float2* buf = lines[j];
    fft::line_fft<N, true>(
        buf, tw, t, true,
        [&](int i) {
            const int m = (i + MX / 2) & (N - 1);
            return m < MX ? stage[m][j] : make_float2(0.f, 0.f);
        },
        [&](int x, float2 v) { buf[fft::pad(x)] = v; });
    __syncthreads();
    float2* blk = P + (qp * BC + bc) * nx_seg * 8;
    for (int e = threadIdx.x; e < N * 4; e += THREADS) {
        const int x = e >> 2, jj = 2 * (e & 3);
        const float2 a = lines[jj][fft::pad(x)], b = lines[jj + 1][fft::pad(x)];
        *reinterpret_cast<float4*>(blk + (x / nx_seg) * seg_stride + (x % nx_seg) * 8 + jj) =
            make_float4(a.x, a.y, b.x, b.y);
    }
}

}  // namespace axis
}  // namespace nop

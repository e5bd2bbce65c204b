// Plane kernels for 512 x 512 grids (kept KX rFFT bins on the last axis, MY centred bins on the first),
// built from the 256-point machinery of plane256.cuh:
//   * a 512-sample real row is ONE 256-point complex FFT of z[m] = x[2m] + i x[2m+1] (8-byte loads),
//     followed by X[k] = E[k] + W512^k O[k], E = (Z_k + conj Z_{256-k}) / 2, O = (Z_k - conj Z_{256-k}) / 2i;
//   * the 512-point column transform is split by row parity: Y[f] = C_even[f] + W512^f C_odd[f], where
//     C_e is the 256-point transform over the rows of parity e.  The forward runs the even rows and their
//     columns, parks C_even in the output slot, runs the odd rows and columns, and combines.  The
//     inverse pre-twiddles the kept spectrum by W512^(-e f) for output rows of parity e, so every phase
//     needs only a 256-row column store: the shared-memory footprint stays that of the 256 x 256 kernels
//     (two CTAs per SM).
// W512 = e^{-2 pi i / 512} (forward); the inverse uses the conjugates.
#pragma once

#include "plane256.cuh"

namespace nop {
namespace p512 {

using p256::G;
using p256::GROUPS;
using p256::ipad;
using p256::LINE;
using p256::THREADS;
using p256::TPITCH;
using p256::TWP;

constexpr int NH = 256;  // half length: the FFTs are 256-point
constexpr int W64 = 64;  // W512^k for k < 64 (row bins < 33, centred column bins |f| <= 32)

template <int KX>
__host__ __device__ constexpr size_t w_offset() {
    return ((size_t)NH + (size_t)G * TWP + (size_t)KX * TPITCH + 1) & ~(size_t)1;
}

template <int KX>
__host__ __device__ constexpr size_t x_offset() {
    return w_offset<KX>() + W64;
}

template <int KX, int MY>
__host__ __device__ constexpr size_t smem_bytes() {
    constexpr size_t stage = (size_t)MY * KX;
    constexpr size_t x = (size_t)GROUPS * LINE;
    return sizeof(float2) * (x_offset<KX>() + (x > stage ? x : stage));
}

// tables from the 512-point table: tw[i] = W^(2i) for the 256-point FFTs, lane twiddles, w512[k] = W^k
__device__ __forceinline__ void init_tables(float2* tw, float2* twp, float2* w512, const float2* twg512) {
    for (int i = threadIdx.x; i < NH; i += THREADS) tw[i] = twg512[2 * i];
    for (int i = threadIdx.x; i < W64; i += THREADS) w512[i] = twg512[i];
    __syncthreads();
    for (int i = threadIdx.x; i < G * 16; i += THREADS) {
        const int t = i >> 4, r = i & 15;
        twp[t * TWP + r] = tw[(r * t) & (NH - 1)];
    }
    __syncthreads();
}

// e^{-2 pi i f / 512} (forward) or its conjugate, for |f| < 64
template <bool INV>
__device__ __forceinline__ float2 w512_at(const float2* w512, int f) {
    const float2 w = w512[f < 0 ? -f : f];
    const bool conj_ = (f < 0) != INV;  // table holds e^{+2 pi i k / 512}
    return conj_ ? w : make_float2(w.x, -w.y);
}

// ------------------------------------------------------------------------------------------
// forward: x [L, 512, 512] real -> mode-blocked spectrum [Q][L][8] (kept modes MY x KX)
// ------------------------------------------------------------------------------------------
template <int KX, int MY>
__global__ void __launch_bounds__(THREADS, 2)
k_fwd(const float* __restrict__ x, float2* __restrict__ out, const float2* __restrict__ twg512, float scale,
      int64_t blk_stride) {
    constexpr int N = 512;
    constexpr unsigned OUT_ROW = p256::row_out_mask(KX);
    constexpr unsigned OUT_COL = p256::col_mask(MY);
    constexpr int Mt = MY * KX;
    constexpr int Q = (Mt + 7) / 8;
    extern __shared__ float2 smem[];
    float2* tw = smem;
    float2* twp = tw + NH;
    float2* T = twp + G * TWP;
    float2* w512 = smem + w_offset<KX>();
    float2* X = smem + x_offset<KX>();
    const int64_t plane = blockIdx.x;
    const int g = threadIdx.x / G;
    const int t = threadIdx.x % G;
    const float* xp = x + plane * (int64_t)N * N;
    float2* buf = X + g * LINE;
    float2* stage = X;
    float2* op = out + plane * 8;
    const int warp_first_group = (threadIdx.x & ~31) / G;

    // row R as one complex line: nxt[r] = (x[R][2 m], x[R][2 m + 1]), m = t + 16 r
    float2 nxt[16];
    const uint64_t pol_x = l2::evict_first();  // x is read once
    auto load_row = [&](int R) {
        const float2* rp = reinterpret_cast<const float2*>(xp + (int64_t)R * N) + t;
#pragma unroll
        for (int r = 0; r < 16; ++r) nxt[r] = l2::ld2(rp + 16 * r, pol_x);
    };
    load_row(2 * g);  // in flight while the tables are built
    init_tables(tw, twp, w512, twg512);
    float2 twr[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) twr[r] = twp[t * TWP + r];

#pragma unroll 1
    for (int e = 0; e < 2; ++e) {
        // ---- rows of parity e: j -> row 2 j + e; kept bins X[k], k < KX, into the column store ----
#pragma unroll 1
        for (int base = 0; base < NH; base += GROUPS) {
            const int j = base + g;
            float2 v[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = nxt[r];
            if (base + GROUPS < NH)
                load_row(2 * (j + GROUPS) + e);
            else if (e == 0)
                load_row(2 * g + 1);  // the odd phase's first row
            fft::dft16<false>(v);
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; r += 2)
                *reinterpret_cast<float4*>(buf + 18 * t + r) = make_float4(v[r].x, v[r].y, v[r + 1].x, v[r + 1].y);
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = buf[t + 18 * r];
            p256::pass2_twiddle_reg<false>(v, twr);
            fft::dft16_m<false, 0xFFFFu, OUT_ROW>(v);
            // E = (Z_k + conj Z_{256-k}) / 2, O = (Z_k - conj Z_{256-k}) / 2i, X_k = E + W512^k O
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                if (16 * r >= KX) continue;
                const float2 sh = make_float2(__shfl_sync(0xffffffffu, v[15 - r].x, (16 - t) & 15, 16),
                                              __shfl_sync(0xffffffffu, v[15 - r].y, (16 - t) & 15, 16));
                const float2 zn = t == 0 ? v[(16 - r) & 15] : sh;
                const float2 zk = v[r];
                const int k = t + 16 * r;
                if (16 * r + 15 < KX || k < KX) {
                    const float2 E = make_float2(0.5f * (zk.x + zn.x), 0.5f * (zk.y - zn.y));
                    const float2 O = make_float2(0.5f * (zk.y + zn.y), 0.5f * (zn.x - zk.x));
                    T[k * TPITCH + ipad(j)] = fft::cadd(E, fft::cmul(O, w512_at<false>(w512, k)));
                }
            }
        }
        __syncthreads();

        // ---- columns over the rows of parity e: keep MY centred bins ----
#pragma unroll 1
        for (int base = 0; base < KX; base += GROUPS) {
            if (base + warp_first_group >= KX) break;
            const int c = base + g;
            const bool active = c < KX;
            float2* col = T + (active ? c : 0) * TPITCH;
            // odd phase: this lane's parked C_even values, loaded before the column transform
            float2 ce[16];
            if (e == 1 && active) {
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    if (!((OUT_COL >> r) & 1)) continue;
                    const int idx = ((t + 16 * r + MY / 2) & (NH - 1)) * KX + c;
                    ce[r] = op[(idx >> 3) * blk_stride + (idx & 7)];
                }
            }
            float2 v[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = col[t + 17 * r];
            fft::dft16<false>(v);
            __syncwarp();
            if (active) {
#pragma unroll
                for (int r = 0; r < 16; ++r) col[17 * t + r] = v[r];
            }
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = col[t + 17 * r];
            p256::pass2_twiddle_reg<false>(v, twr);
            fft::dft16_m<false, 0xFFFFu, OUT_COL>(v);
            if (active) {
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    if (!((OUT_COL >> r) & 1)) continue;
                    const int m = (t + 16 * r + MY / 2) & (NH - 1);  // stage row; frequency m - MY/2
                    const int idx = m * KX + c;
                    if (e == 0) {
                        stage[idx] = v[r];
                    } else {
                        // Y = C_even + W512^f C_odd, C_even parked in this plane's output slot
                        stage[idx] = fft::cscale(fft::cadd(ce[r], fft::cmul(v[r], w512_at<false>(w512, m - MY / 2))),
                                                 scale);
                    }
                }
            }
        }
        __syncthreads();
        // the stage region is the next phase's exchange lines: park (e = 0) or write (e = 1) the modes
        for (int ee = threadIdx.x; ee < Q * 4; ee += THREADS) {
            const int q = ee >> 2, m = 8 * q + 2 * (ee & 3);
            const float2 a = m < Mt ? stage[m] : make_float2(0.f, 0.f);
            const float2 b = m + 1 < Mt ? stage[m + 1] : make_float2(0.f, 0.f);
            l2::st4(op + q * blk_stride + 2 * (ee & 3), make_float4(a.x, a.y, b.x, b.y), l2::evict_last());
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------
// inverse: mode-blocked spectrum [Q][L][8] -> y [L, 512, 512] real with bias / skip / GELU
// ------------------------------------------------------------------------------------------
template <int KX, int MY>
__global__ void __launch_bounds__(THREADS, 2)
k_inv(const float2* __restrict__ in, float* __restrict__ y, const float2* __restrict__ twg512, float scale,
      int64_t blk_stride, p256::Epi ep) {
    constexpr int N = 512;
    constexpr unsigned IN_COL = p256::col_mask(MY);
    constexpr unsigned IN_ROW = p256::row_in_mask(KX);
    constexpr int Mt = MY * KX;
    constexpr int Q = (Mt + 7) / 8;
    constexpr int NPF = (Q * 4 + THREADS - 1) / THREADS;
    extern __shared__ float2 smem[];
    float2* tw = smem;
    float2* twp = tw + NH;
    float2* T = twp + G * TWP;
    float2* w512 = smem + w_offset<KX>();
    float2* X = smem + x_offset<KX>();
    const int64_t plane = blockIdx.x;
    const int g = threadIdx.x / G;
    const int t = threadIdx.x % G;
    float2* stage = X;
    float2* buf = X + g * LINE;
    const float2* ip = in + plane * 8;
    const uint64_t pol_y = l2::evict_first();  // y (and the skip addend) stream through
    float4 pf[NPF];  // the kept spectrum; read again for the odd phase (the stage region is reused)
    auto fetch = [&]() {
#pragma unroll
        for (int k = 0; k < NPF; ++k) {
            const int e = threadIdx.x + k * THREADS;
            if (e < Q * 4) pf[k] = __ldg(reinterpret_cast<const float4*>(ip + (e >> 2) * blk_stride + 2 * (e & 3)));
        }
    };
    auto put = [&]() {
#pragma unroll
        for (int k = 0; k < NPF; ++k) {
            const int e = threadIdx.x + k * THREADS;
            const int m = 8 * (e >> 2) + 2 * (e & 3);
            if (e < Q * 4 && m < Mt) stage[m] = make_float2(pf[k].x, pf[k].y);
            if (e < Q * 4 && m + 1 < Mt) stage[m + 1] = make_float2(pf[k].z, pf[k].w);
        }
    };
    fetch();
    init_tables(tw, twp, w512, twg512);
    const float2* twl = twp + t * TWP;
    const float2 twb[6] = {twl[1], twl[2], twl[3], twl[4], twl[8], twl[12]};
    const int warp_first_group = (threadIdx.x & ~31) / G;
    const float bias = ep.bias ? ep.bias[(plane / ep.chan_div) % ep.C] : 0.f;
    float* yp = y + plane * (int64_t)N * N;
    const float* ap = ep.addend ? ep.addend + plane * (int64_t)N * N : nullptr;

#pragma unroll 1
    for (int e = 0; e < 2; ++e) {
        put();
        __syncthreads();
        // ---- columns: kept bins (pre-twiddled by W512^(-e f)) -> rows j of parity e ----
#pragma unroll 1
        for (int base = 0; base < KX; base += GROUPS) {
            if (base + warp_first_group >= KX) break;
            const int c = base + g;
            const bool active = c < KX;
            float2* col = T + (active ? c : 0) * TPITCH;
            float2 v[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                if (!((IN_COL >> r) & 1)) continue;
                const int m = (t + 16 * r + MY / 2) & (NH - 1);
                float2 val = active ? stage[m * KX + c] : make_float2(0.f, 0.f);
                if (e == 1) val = fft::cmul(val, w512_at<true>(w512, m - MY / 2));
                v[r] = val;
            }
            fft::dft16_m<true, IN_COL, 0xFFFFu>(v);
            if (active) {
#pragma unroll
                for (int r = 0; r < 16; ++r) col[17 * t + r] = v[r];
            }
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = col[t + 17 * r];
            p256::pass2_twiddle_6<true>(v, twb);
            fft::dft16<true>(v);
            __syncwarp();
            if (active) {
#pragma unroll
                for (int r = 0; r < 16; ++r) col[t + 17 * r] = v[r];
            }
        }
        __syncthreads();
        if (e == 0) fetch();  // the odd phase's copy of the spectrum, in flight during the rows

        // ---- rows 2 j + e: Z'[k] = X_k (1 + i W512^-k) (k < KX), conj X_{k'} (1 - i W512^-k) at
        // k = 256 - k'; z = IDFT256(Z') gives (x[2m], x[2m+1]); epilogue ----
#pragma unroll 1
        for (int base = 0; base < NH; base += GROUPS) {
            const int j = base + g;
            const int R = 2 * j + e;
            float2 v[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                if (!((IN_ROW >> r) & 1)) continue;
                const int i = t + 16 * r;
                float2 z = make_float2(0.f, 0.f);
                if (16 * r < KX) {  // direct bins
                    if (16 * r + 15 < KX || i < KX) {
                        float2 Xk = T[i * TPITCH + ipad(j)];
                        if (i == 0) Xk.y = 0.f;
                        const float2 wk = w512_at<true>(w512, i);           // W512^-k
                        const float2 iw = make_float2(-wk.y, wk.x);         // i W512^-k
                        z = fft::cmul(Xk, make_float2(1.f + iw.x, iw.y));
                    }
                } else {  // k = 256 - k'
                    const int kp = NH - i;
                    if (kp < KX) {
                        const float2 Xc = T[kp * TPITCH + ipad(j)];
                        const float2 cx = make_float2(Xc.x, -Xc.y);
                        const float2 wk = w512_at<true>(w512, i - NH);      // W512^-(k) with k = 256 - k', |.| < 64
                        // W512^-k for k = 256 - k' is -W512^(k') ... handled as e^{+2 pi i k / 512}
                        const float2 wf = make_float2(-wk.x, -wk.y);         // e^{i pi} W512^{+k'} = W512^{-(256 - k')}
                        const float2 iw = make_float2(-wf.y, wf.x);
                        z = fft::cmul(cx, make_float2(1.f - iw.x, -iw.y));
                    }
                }
                v[r] = z;
            }
            fft::dft16_m<true, IN_ROW, 0xFFFFu>(v);
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; r += 2)
                *reinterpret_cast<float4*>(buf + 18 * t + r) = make_float4(v[r].x, v[r].y, v[r + 1].x, v[r + 1].y);
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = buf[t + 18 * r];
            p256::pass2_twiddle_6<true>(v, twb);
            fft::dft16<true>(v);
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                const int m = t + 16 * r;
                float a0 = v[r].x * scale + bias;
                float a1 = v[r].y * scale + bias;
                if (ap) {
                    const float2 s = l2::ld2(reinterpret_cast<const float2*>(ap + (int64_t)R * N) + m, pol_y);
                    a0 += s.x;
                    a1 += s.y;
                }
                if (ep.apply_gelu) {
                    a0 = gelu_erf(a0);
                    a1 = gelu_erf(a1);
                }
                l2::st2(reinterpret_cast<float2*>(yp + (int64_t)R * N) + m, make_float2(a0, a1), pol_y);
            }
            __syncwarp();  // buf is rewritten by the next row
        }
        __syncthreads();  // the odd phase's spectrum goes into the exchange lines' region
    }
}

}  // namespace p512
}  // namespace nop

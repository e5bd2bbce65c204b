// Plane kernels for 256 x 256 grids specialised on the kept mode counts (KX rFFT bins on the last
// axis, MY centred bins on the first axis, offset MY/2).  Same data flow as the generic plane
// kernels in fast.cu, with the truncation known at compile time:
//   * forward: the last radix-16 pass of every line computes only the outputs that are kept (and
//     their Hermitian partners); the two packed real rows are separated with warp shuffles;
//   * inverse: the first radix-16 pass reads only the non-zero (kept) inputs;
//   * pass-2 twiddles: the forward kernel keeps its lane's 16 in registers; the inverse keeps six
//     and forms the rest as one product each (fewer registers next to its spectrum prefetch);
//   * the forward kernel issues its first row loads before it builds the twiddle tables; an inverse
//     CTA transforms `ppc` consecutive planes, with the kept spectrum of its next plane in flight
//     while it finishes the current one (the first one's while the tables are built).
// Lane t of a 16-lane group owns elements t + 16 r (first pass) and outputs t + 16 r (last pass).
#pragma once

#include "fft_masked.cuh"
#include "l2_hints.cuh"
#include "nop_internal.cuh"

namespace nop {
namespace p256 {

constexpr int N = 256;
constexpr int G = 16;             // lanes per line
constexpr int THREADS = 256;      // 16 groups
constexpr int GROUPS = THREADS / G;
constexpr int LINE = 288;         // per-group exchange line (index i -> i + 2 (i / 16), 16-byte aligned rows)
constexpr int TPITCH = 273;       // odd pitch of the column store
constexpr int TWP = 18;           // per-lane twiddle row pitch (float2), 16-byte multiple

// outputs r (k = t + 16 r) of the forward row transform that are kept or are partners of kept bins
__host__ __device__ constexpr unsigned row_out_mask(int KX) {
    unsigned m = 0;
    for (int r = 0; r < 16; ++r) {
        if (16 * r < KX) {
            m |= 1u << r;                    // kept bin k = t + 16 r (some t)
            m |= 1u << ((16 - r) & 15);      // partner of lane 0: 256 - 16 r
            if (16 * r + 1 < KX) m |= 1u << (15 - r);  // partner of lanes t >= 1
        }
    }
    return m;
}

// bins r (k = t + 16 r) of a column transform holding centred kept modes: m = (k + MY/2) mod 256 < MY
__host__ __device__ constexpr unsigned col_mask(int MY) {
    unsigned m = 0;
    for (int r = 0; r < 16; ++r)
        for (int t = 0; t < 16; ++t)
            if (((t + 16 * r + MY / 2) & 255) < MY) m |= 1u << r;
    return m;
}

// non-zero inputs r (i = t + 16 r) of the inverse row transform: i < KX or a mirror 256 - i < KX
__host__ __device__ constexpr unsigned row_in_mask(int KX) {
    unsigned m = 0;
    for (int r = 0; r < 16; ++r)
        for (int t = 0; t < 16; ++t) {
            const int i = t + 16 * r;
            if (i < KX || (256 - i < KX && 2 * i > 256)) m |= 1u << r;
        }
    return m;
}

__host__ __device__ constexpr int ipad(int i) { return i + (i >> 4); }

// float2 offset of the exchange / stage region: after tw, twp and the column store, rounded up to
// an even count so the region is 16-byte aligned (128-bit stores into the exchange lines)
template <int KX>
__host__ __device__ constexpr size_t x_offset() {
    return ((size_t)N + (size_t)G * TWP + (size_t)KX * TPITCH + 1) & ~(size_t)1;
}

template <int KX, int MY>
__host__ __device__ constexpr size_t smem_bytes() {
    constexpr size_t stage = (size_t)MY * KX;
    constexpr size_t x = (size_t)GROUPS * LINE;
    return sizeof(float2) * (x_offset<KX>() + (x > stage ? x : stage));
}

// per-lane pass-2 twiddles W^(r t) of a 256-point transform, conjugated for the forward direction
template <bool INV>
__device__ __forceinline__ void pass2_twiddle(float2* v, const float2* twp_lane) {
#pragma unroll
    for (int r = 0; r < 16; r += 2) {
        const float4 w = *reinterpret_cast<const float4*>(twp_lane + r);
        if (r > 0) v[r] = fft::cmul(v[r], INV ? make_float2(w.x, w.y) : make_float2(w.x, -w.y));
        v[r + 1] = fft::cmul(v[r + 1], INV ? make_float2(w.z, w.w) : make_float2(w.z, -w.w));
    }
}

// the same with the lane's 16 twiddles held in registers
template <bool INV>
__device__ __forceinline__ void pass2_twiddle_reg(float2* v, const float2* w) {
#pragma unroll
    for (int r = 1; r < 16; ++r) v[r] = fft::cmul(v[r], INV ? w[r] : make_float2(w[r].x, -w[r].y));
}

// the same from six per-lane base twiddles W^(r t), r in {1, 2, 3, 4, 8, 12}: W^((4a + c) t) is one
// product of two exactly-rounded table values (at most about one extra rounding)
template <bool INV>
__device__ __forceinline__ void pass2_twiddle_6(float2* v, const float2 (&b)[6]) {
#pragma unroll
    for (int r = 1; r < 16; ++r) {
        const int a = r >> 2, c = r & 3;
        const float2 wa = a == 1 ? b[3] : a == 2 ? b[4] : b[5];
        const float2 wc = c == 1 ? b[0] : c == 2 ? b[1] : b[2];
        const float2 w = a == 0 ? wc : c == 0 ? wa : fft::cmul(wa, wc);
        v[r] = fft::cmul(v[r], INV ? w : make_float2(w.x, -w.y));
    }
}

__device__ __forceinline__ void init_tables(float2* tw, float2* twp, const float2* twg) {
    for (int i = threadIdx.x; i < N; i += THREADS) tw[i] = twg[i];
    __syncthreads();
    for (int i = threadIdx.x; i < G * 16; i += THREADS) {
        const int t = i >> 4, r = i & 15;
        twp[t * TWP + r] = tw[(r * t) & (N - 1)];
    }
    __syncthreads();
}

// ------------------------------------------------------------------------------------------
// forward: x [L, 256, 256] real -> mode-blocked spectrum [Q][L][8] (kept modes MY x KX)
// ------------------------------------------------------------------------------------------
template <int KX, int MY>
__global__ void __launch_bounds__(THREADS, 2)
k_fwd(const float* __restrict__ x, float2* __restrict__ out, const float2* __restrict__ twg, float scale,
      int64_t blk_stride) {
    constexpr unsigned OUT_ROW = row_out_mask(KX);
    constexpr unsigned OUT_COL = col_mask(MY);
    extern __shared__ float2 smem[];
    float2* tw = smem;
    float2* twp = tw + N;
    float2* T = twp + G * TWP;
    float2* X = smem + x_offset<KX>();
    const int64_t plane = blockIdx.x;
    const int g = threadIdx.x / G;
    const int t = threadIdx.x % G;
    const float* xp = x + plane * (int64_t)N * N;
    float2* buf = X + g * LINE;

    // ---- rows: pairs (2p, 2p+1) as one complex line, kept bins to the column store ----
    // The next pair's 32 loads are issued before the current pair is transformed; the first pair's
    // loads are in flight while the twiddle tables are built.
    const uint64_t pol_x = l2::evict_first();   // x is read once
    float2 nxt[16];
    {
        const float* ra = xp + (int64_t)(2 * g) * N + t;
#pragma unroll
        for (int r = 0; r < 16; ++r) nxt[r] = make_float2(l2::ld(ra + 16 * r, pol_x), l2::ld(ra + N + 16 * r, pol_x));
    }
    init_tables(tw, twp, twg);
    float2 twr[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) twr[r] = twp[t * TWP + r];
#pragma unroll 1
    for (int base = 0; base < N / 2; base += GROUPS) {
        const int pr = base + g;
        float2 v[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) v[r] = nxt[r];
        if (base + GROUPS < N / 2) {
            const float* ra = xp + (int64_t)(2 * (pr + GROUPS)) * N + t;
#pragma unroll
            for (int r = 0; r < 16; ++r)
                nxt[r] = make_float2(l2::ld(ra + 16 * r, pol_x), l2::ld(ra + N + 16 * r, pol_x));
        }
        fft::dft16<false>(v);
        __syncwarp();
#pragma unroll
        for (int r = 0; r < 16; r += 2)
            *reinterpret_cast<float4*>(buf + 18 * t + r) = make_float4(v[r].x, v[r].y, v[r + 1].x, v[r + 1].y);
        __syncwarp();
#pragma unroll
        for (int r = 0; r < 16; ++r) v[r] = buf[t + 18 * r];
        pass2_twiddle_reg<false>(v, twr);
        fft::dft16_m<false, 0xFFFFu, OUT_ROW>(v);
        // separate the two real rows: A[k] = (Z_k + conj Z_{N-k}) / 2, B[k] = (Z_k - conj Z_{N-k}) / 2i
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            if (16 * r >= KX) continue;
            const float2 sh = make_float2(__shfl_sync(0xffffffffu, v[15 - r].x, (16 - t) & 15, 16),
                                          __shfl_sync(0xffffffffu, v[15 - r].y, (16 - t) & 15, 16));
            const float2 zn = t == 0 ? v[(16 - r) & 15] : sh;
            const float2 zk = v[r];
            const int k = t + 16 * r;
            if (16 * r + 15 < KX || k < KX) {
                T[k * TPITCH + ipad(2 * pr)] = make_float2(0.5f * (zk.x + zn.x), 0.5f * (zk.y - zn.y));
                T[k * TPITCH + ipad(2 * pr + 1)] = make_float2(0.5f * (zk.y + zn.y), 0.5f * (zn.x - zk.x));
            }
        }
    }
    __syncthreads();

    // ---- columns: keep MY centred bins ----
    float2* stage = X;
    const int warp_first_group = (threadIdx.x & ~31) / G;
#pragma unroll 1
    for (int base = 0; base < KX; base += GROUPS) {
        if (base + warp_first_group >= KX) break;
        const int c = base + g;
        const bool active = c < KX;
        float2* col = T + (active ? c : 0) * TPITCH;
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
        pass2_twiddle_reg<false>(v, twr);
        fft::dft16_m<false, 0xFFFFu, OUT_COL>(v);
        if (active) {
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                if (!((OUT_COL >> r) & 1)) continue;
                const int m = (t + 16 * r + MY / 2) & (N - 1);
                stage[m * KX + c] = fft::cscale(v[r], scale);
            }
        }
    }
    __syncthreads();
    constexpr int Mt = MY * KX;
    constexpr int Q = (Mt + 7) / 8;
    float2* op = out + plane * 8;
    const uint64_t pol_s = l2::evict_last();  // the kept spectrum is read back by the next kernel
    for (int e = threadIdx.x; e < Q * 4; e += THREADS) {
        const int q = e >> 2, m = 8 * q + 2 * (e & 3);
        const float2 a = m < Mt ? stage[m] : make_float2(0.f, 0.f);
        const float2 b = m + 1 < Mt ? stage[m + 1] : make_float2(0.f, 0.f);
        l2::st4(op + q * blk_stride + 2 * (e & 3), make_float4(a.x, a.y, b.x, b.y), pol_s);
    }
}

struct Epi {
    const float* bias;
    const float* addend;
    int apply_gelu;
    int C;
    int64_t chan_div;
};

// ------------------------------------------------------------------------------------------
// inverse: mode-blocked spectrum [Q][L][8] -> y [L, 256, 256] real with bias / skip / GELU
// ------------------------------------------------------------------------------------------
template <int KX, int MY>
__global__ void __launch_bounds__(THREADS, 2)
k_inv(const float2* __restrict__ in, float* __restrict__ y, const float2* __restrict__ twg, float scale,
      int64_t blk_stride, Epi ep, int64_t L, int ppc) {
    constexpr unsigned IN_COL = col_mask(MY);
    constexpr unsigned IN_ROW = row_in_mask(KX);
    const uint64_t pol_s = l2::evict_first();  // the kept spectrum is read once
    const uint64_t pol_y = l2::evict_first();  // y (and the skip addend) stream through
    constexpr int Mt = MY * KX;
    constexpr int Q = (Mt + 7) / 8;
    constexpr int NPF = (Q * 4 + THREADS - 1) / THREADS;  // 16-byte pieces of the spectrum per thread
    extern __shared__ float2 smem[];
    float2* tw = smem;
    float2* twp = tw + N;
    float2* T = twp + G * TWP;
    float2* X = smem + x_offset<KX>();
    const int g = threadIdx.x / G;
    const int t = threadIdx.x % G;
    const int64_t first = (int64_t)blockIdx.x * ppc;
    const int64_t last = first + ppc < L ? first + ppc : L;  // planes [first, last)
    float2* stage = X;
    float4 pf[NPF];  // the next plane's kept spectrum, in flight
    auto fetch = [&](int64_t pl) {
        const float2* ip = in + pl * 8;
#pragma unroll
        for (int k = 0; k < NPF; ++k) {
            const int e = threadIdx.x + k * THREADS;
            if (e < Q * 4) pf[k] = l2::ld4(ip + (e >> 2) * blk_stride + 2 * (e & 3), pol_s);
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
    if (first < last) fetch(first);  // overlaps the table set-up
    init_tables(tw, twp, twg);
    const float2* twl = twp + t * TWP;
    const float2 twb[6] = {twl[1], twl[2], twl[3], twl[4], twl[8], twl[12]};
    const int warp_first_group = (threadIdx.x & ~31) / G;
    float2* buf = X + g * LINE;
#pragma unroll 1
    for (int64_t plane = first; plane < last; ++plane) {
        put();
        __syncthreads();
        // ---- columns: kept bins -> full y lines ----
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
                const int m = (t + 16 * r + MY / 2) & (N - 1);
                v[r] = active ? stage[m * KX + c] : make_float2(0.f, 0.f);
            }
            fft::dft16_m<true, IN_COL, 0xFFFFu>(v);
            if (active) {
#pragma unroll
                for (int r = 0; r < 16; ++r) col[17 * t + r] = v[r];
            }
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = col[t + 17 * r];
            pass2_twiddle_6<true>(v, twb);
            fft::dft16<true>(v);
            __syncwarp();
            if (active) {
#pragma unroll
                for (int r = 0; r < 16; ++r) col[t + 17 * r] = v[r];
            }
        }
        __syncthreads();
        if (plane + 1 < last) fetch(plane + 1);

        // ---- rows: Z = A + iB (k < KX), conj(A) + i conj(B) at 256 - k; inverse; epilogue ----
        const float bias = ep.bias ? ep.bias[(plane / ep.chan_div) % ep.C] : 0.f;
        float* yp = y + plane * (int64_t)N * N;
        const float* ap = ep.addend ? ep.addend + plane * (int64_t)N * N : nullptr;
#pragma unroll 1
        for (int base = 0; base < N / 2; base += GROUPS) {
            const int pr = base + g;
            const int na = 2 * pr, nb = 2 * pr + 1;
            float2 v[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                if (!((IN_ROW >> r) & 1)) continue;
                const int i = t + 16 * r;
                if (16 * r < KX) {  // direct bins
                    float2 z = make_float2(0.f, 0.f);
                    if (16 * r + 15 < KX || i < KX) {
                        float2 A = T[i * TPITCH + ipad(na)];
                        float2 B = T[i * TPITCH + ipad(nb)];
                        if (i == 0) {
                            A.y = 0.f;
                            B.y = 0.f;
                        }
                        z = make_float2(A.x - B.y, A.y + B.x);
                    }
                    v[r] = z;
                } else {  // mirrored bins k = 256 - i
                    const int k = N - i;
                    float2 z = make_float2(0.f, 0.f);
                    if (k < KX) {
                        const float2 A = T[k * TPITCH + ipad(na)];
                        const float2 B = T[k * TPITCH + ipad(nb)];
                        z = make_float2(A.x + B.y, B.x - A.y);
                    }
                    v[r] = z;
                }
            }
            fft::dft16_m<true, IN_ROW, 0xFFFFu>(v);
            if (t == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // buf's last rows read
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; r += 2)
                *reinterpret_cast<float4*>(buf + 18 * t + r) = make_float4(v[r].x, v[r].y, v[r + 1].x, v[r + 1].y);
            __syncwarp();
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] = buf[t + 18 * r];
            pass2_twiddle_6<true>(v, twb);
            fft::dft16<true>(v);
            // rows na, nb (contiguous in y) staged in the group's exchange line, written by one bulk copy;
            // odd groups stage 64 bytes further in, off the banks of the even group of their warp
            __syncwarp();  // every lane has read its exchange values
            float* ob = reinterpret_cast<float*>(buf) + 16 * (g & 1);
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                const int n = t + 16 * r;
                float va = v[r].x * scale + bias;
                float vb = v[r].y * scale + bias;
                if (ap) {
                    va += l2::ld(ap + (int64_t)na * N + n, pol_y);
                    vb += l2::ld(ap + (int64_t)nb * N + n, pol_y);
                }
                if (ep.apply_gelu) {
                    va = gelu_erf(va);
                    vb = gelu_erf(vb);
                }
                ob[n] = va;
                ob[N + n] = vb;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the bulk copy
            __syncwarp();
            if (t == 0) {
                asm volatile("cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;" ::"l"(
                                 yp + (int64_t)na * N),
                             "r"((uint32_t)__cvta_generic_to_shared(ob)), "r"(2 * N * 4), "l"(pol_y)
                             : "memory");
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
        }
        // the next plane's spectrum goes into the exchange lines' region
        if (t == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncthreads();
    }
    if (t == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

}  // namespace p256
}  // namespace nop

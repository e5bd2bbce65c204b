// Weight gradient of the per-mode contraction on the tensor cores (tcgen05, sm_100a).
//
//   dL/dW[i][o][t] = d_t * sum_b conj(Xh[b][i][t]) * Gh[b][o][t]        (mode t = 8 q + j)
//
// on mode-blocked spectra ([Q][B][C][8], fused engine): Xh from the forward, Gh from the adjoint
// forward (see grad.cu for the derivation and d_t).  It is the forward contraction (mix_tc.cuh) with the
// roles of batch and input channel exchanged: for each mode ONE real GEMM with M = 128, N = 2 CO, K = batch,
//
//   A rows: in every 32-row quadrant, 16 input channels of Re Xh^T followed by the same 16 of Im Xh^T
//   B = [Re Gh | Im Gh]
//   D row (Re, i) = [Xr^T Gr, Xr^T Gi],  D row (Im, i) = [Xi^T Gr, Xi^T Gi]   (16 lanes apart)
//
// so  Re dW = Xr^T Gr + Xi^T Gi  and  Im dW = Xr^T Gi - Xi^T Gr  combine with lane shuffles.  A producer
// unit (input channel or output channel, K half) copies the same float4 mode pairs as the forward's
// units, so the raw ring, the tf32 hi / lo conversion (store_step), the stages, the MMA issuer and the
// bounded waits are the forward's; only the gather addresses, the K extent (batch) and the epilogue's
// combination and output (dW[i][o][t], 32 bytes = 4 modes per (i, o)) differ.
#pragma once

#include "mix_tc.cuh"

namespace nop {
namespace wgtc {

using tc::BT;
using tc::EPI_WARPS;
using tc::MMA_WARP;
using tc::MODES;
using tc::PROD_THREADS;
using tc::PROD_WARPS;
using tc::THREADS;

struct Problem {
    const float2* X;   // [Q][B][Ci][8]
    const float2* G;   // [Q][B][Co][8]
    float2* W;         // [Ci][Co][Mt]
    int B, Ci, Co, Q;
    int64_t Mt;
    int it, ot;        // input-channel tiles (64), output-channel tiles (CO)
    int kl, nyq, dbl;  // per-mode factor d_t (see grad.cu)
};

struct Tile {
    int h, i0, o0, q;
};

// tile t: mode half fastest, then output tile, input tile, mode block
__device__ __forceinline__ Tile tile_at(const Problem& pr, int t, int co_tile) {
    Tile r;
    r.h = t & 1;
    int rest = t >> 1;
    r.o0 = (rest % pr.ot) * co_tile;
    rest /= pr.ot;
    r.i0 = (rest % pr.it) * BT;
    r.q = rest / pr.it;
    return r;
}

// raw copies of producer thread p for the K step starting at batch entry b0.  A unit (p < 128): input
// channel i = p / 2, batch half kh = p % 2; B unit: output channel o = u % CO, batch half u / CO.
// Value c of a unit is batch entry b0 + 4 kh + c; its two float4 are modes (4h, 4h+1) and (4h+2, 4h+3).
template <int CO>
__device__ __forceinline__ void issue_step(float4* slot, const Problem& pr, const Tile& tl, int b0, int p,
                                           uint64_t pol) {
    if (p < 128) {
        const int il = p >> 1, kh = p & 1;
        const bool iok = tl.i0 + il < pr.Ci;
        const float2* src = pr.X + ((int64_t)tl.q * pr.B * pr.Ci + tl.i0 + il) * 8 + 4 * tl.h;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int b = b0 + 4 * kh + c;
            const bool ok = iok && b < pr.B;
            const float2* sc = ok ? src + (int64_t)b * pr.Ci * 8 : pr.X;
            l2::cp_async16(slot + (2 * c) * PROD_THREADS + p, sc, ok, pol);
            l2::cp_async16(slot + (2 * c + 1) * PROD_THREADS + p, ok ? sc + 2 : pr.X, ok, pol);
        }
    } else if (p < 128 + 2 * CO) {
        const int u = p - 128;
        const int o = u % CO, kh = u / CO;
        const bool ook = tl.o0 + o < pr.Co;
        const float2* src = pr.G + ((int64_t)tl.q * pr.B * pr.Co + tl.o0 + o) * 8 + 4 * tl.h;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int b = b0 + 4 * kh + c;
            const bool ok = ook && b < pr.B;
            const float2* sc = ok ? src + (int64_t)b * pr.Co * 8 : pr.G;
            l2::cp_async16(slot + (2 * c) * PROD_THREADS + p, sc, ok, pol);
            l2::cp_async16(slot + (2 * c + 1) * PROD_THREADS + p, ok ? sc + 2 : pr.G, ok, pol);
        }
    }
}

__device__ __forceinline__ float mode_factor(int64_t t, int kl, int nyq, int dbl) {
    if (!dbl) return 1.f;
    const int m = (int)(t % kl);
    return (m == 0 || m == nyq) ? 1.f : 2.f;
}

template <int CO>
__global__ void __maxnreg__(128)
k_wgrad_tc(Problem pr, int* __restrict__ status) {
    using C = tc::Cfg<CO, false>;
    constexpr int NS = C::NS, NACC = C::NACC;
    extern __shared__ __align__(1024) char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BODY);
    uint64_t* empty = full + NS;
    uint64_t* acc_full = empty + NS;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int tiles = 2 * pr.Q * pr.it * pr.ot;
    const int my_tiles = tiles > (int)blockIdx.x ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nk = (pr.B + C::KS - 1) / C::KS;
    auto tile_k = [&](int k) { return tile_at(pr, (int)blockIdx.x + k * (int)gridDim.x, CO); };

    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            tc::mbar_init(&full[i], PROD_WARPS);
            tc::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&acc_full[i], 1);
            tc::mbar_init(&acc_empty[i], EPI_WARPS);
        }
        tc::mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort_flag = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(tmem_slot)),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    auto give_up = [&]() {
        *abort_flag = 1;
        atomicExch(status, tc::kStatusMmaTimeout);
    };

    if (warp >= EPI_WARPS && warp < MMA_WARP) {
        // ------------------------------ producers ------------------------------
        const int p = tid - 32 * EPI_WARPS;
        const uint64_t pol_in = l2::evict_first();  // both spectra are read once
        constexpr int RS = C::RS;
        float4* raw = reinterpret_cast<float4*>(smem + C::RAW_OFF);
        constexpr int SLOT_F4 = PROD_THREADS * C::RAWF4;
        int lk = 0, lkc = 0;
        Tile ltile;
        if (my_tiles > 0) ltile = tile_k(0);
        int slot_in = 0, slot_out = 0;
        auto issue_next = [&]() {
            if (lk < my_tiles) {
                issue_step<CO>(raw + slot_in * SLOT_F4, pr, ltile, lkc * C::KS, p, pol_in);
                if (++lkc == nk) {
                    lkc = 0;
                    if (++lk < my_tiles) ltile = tile_k(lk);
                }
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
            if (++slot_in == RS) slot_in = 0;
        };
#pragma unroll
        for (int d = 0; d < RS - 1; ++d) issue_next();
        tc::Step<false> cur;
        int s = 0;
        uint32_t upar = 0;
        bool reuse = false;
        for (int k = 0; k < my_tiles; ++k) {
            for (int kc = 0; kc < nk; ++kc) {
                issue_next();
                asm volatile("cp.async.wait_group %0;\n" ::"n"(RS - 1) : "memory");
                const float4* mine = raw + slot_out * SLOT_F4 + p;
#pragma unroll
                for (int c = 0; c < C::RAWF4; ++c) cur.v[c] = mine[c * PROD_THREADS];
                if (++slot_out == RS) slot_out = 0;
                if (reuse && !tc::mbar_wait(&empty[s], upar ^ 1, abort_flag)) {
                    give_up();
                    k = my_tiles;
                    break;
                }
                tc::store_step<CO, false>(cur, smem + s * C::STAGE, p);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&full[s]);
                if (++s == NS) {
                    s = 0;
                    upar ^= 1;
                    reuse = true;
                }
            }
        }
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    } else if (warp == MMA_WARP) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t upar = 0;
            bool ok = true;
            for (int k = 0; k < my_tiles && ok; ++k) {
                const int a = k % NACC;
                const int v = k / NACC;
                if (v > 0 && !tc::mbar_wait(&acc_empty[a], (uint32_t)((v - 1) & 1), abort_flag)) {
                    give_up();
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dacc = tmem + a * C::ACC_COLS;
                for (int kc = 0; kc < nk; ++kc) {
                    if (!tc::mbar_wait(&full[s], upar, abort_flag)) {
                        give_up();
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a0 = tc::smem_u32(smem + s * C::STAGE);
                    const uint32_t bq = a0 + MODES * C::SPLITS * C::A_TILE;
#pragma unroll
                    for (int jl = 0; jl < MODES; ++jl) {
                        const uint32_t d = dacc + jl * C::N;
                        const uint64_t ahi = tc::smem_desc(a0 + (jl * 2) * C::A_TILE);
                        const uint64_t alo = tc::smem_desc(a0 + (jl * 2 + 1) * C::A_TILE);
                        const uint64_t bhi = tc::smem_desc(bq + (jl * 2) * C::B_TILE);
                        const uint64_t blo = tc::smem_desc(bq + (jl * 2 + 1) * C::B_TILE);
                        tc::mma_tf32(d, ahi, bhi, C::IDESC, kc > 0);
                        tc::mma_tf32(d, ahi, blo, C::IDESC, 1);
                        tc::mma_tf32(d, alo, bhi, C::IDESC, 1);
                    }
                    tc::mma_commit(&empty[s]);
                    if (++s == NS) {
                        s = 0;
                        upar ^= 1;
                    }
                }
                if (!ok) break;
                tc::mma_commit(&acc_full[a]);
            }
            tc::mma_commit(drain);
            if (!tc::mbar_wait(drain, 0, nullptr)) give_up();
        }
    } else {
        // ------------------------------ epilogue (warps 0..3) ------------------------------
        const int qd = warp;
        const bool im = lane >= 16;            // this lane holds the Im row of its input channel
        const int il = qd * 16 + (lane & 15);  // input channel within the tile
        const uint64_t pol_out = l2::evict_first();
        for (int k = 0; k < my_tiles; ++k) {
            const int a = k % NACC;
            if (!tc::mbar_wait(&acc_full[a], (uint32_t)((k / NACC) & 1), abort_flag)) {
                give_up();
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const Tile tl = tile_k(k);
            const uint32_t tbase = tmem + ((uint32_t)(qd * 32) << 16) + a * C::ACC_COLS;
            const int i = tl.i0 + il;
            const int64_t t0 = 8 * (int64_t)tl.q + 4 * tl.h;  // first mode of the tile
            float f[MODES];
#pragma unroll
            for (int jl = 0; jl < MODES; ++jl) f[jl] = mode_factor(t0 + jl, pr.kl, pr.nyq, pr.dbl);
            const bool vec = pr.Mt % 4 == 0 && t0 + MODES <= pr.Mt;  // four modes, 32-byte aligned
            for (int cb = 0; cb < CO; cb += 8) {
                float P[MODES][8], Qv[MODES][8];
#pragma unroll
                for (int jl = 0; jl < MODES; ++jl) {
                    tc::tmem_ld8(tbase + jl * C::N + cb, P[jl]);
                    tc::tmem_ld8(tbase + jl * C::N + CO + cb, Qv[jl]);
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (cb + 8 >= CO) {
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&acc_empty[a]);
                }
                // Re lanes finish columns 0..3 of this group, Im lanes columns 4..7
                float out[4][2 * MODES];
#pragma unroll
                for (int jl = 0; jl < MODES; ++jl) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float sp = im ? P[jl][c] : P[jl][4 + c];
                        const float sq = im ? Qv[jl][c] : Qv[jl][4 + c];
                        const float rp = __shfl_xor_sync(0xffffffffu, sp, 16);
                        const float rq = __shfl_xor_sync(0xffffffffu, sq, 16);
                        float re, imv;
                        if (!im) {  // own Re row: P = Xr Gr, Q = Xr Gi; partner: Xi Gr, Xi Gi
                            re = P[jl][c] + rq;
                            imv = Qv[jl][c] - rp;
                        } else {    // own Im row; partner: Xr Gr, Xr Gi of columns 4..7
                            re = rp + Qv[jl][4 + c];
                            imv = rq - P[jl][4 + c];
                        }
                        out[c][2 * jl] = f[jl] * re;
                        out[c][2 * jl + 1] = f[jl] * imv;
                    }
                }
                if (i < pr.Ci) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int o = tl.o0 + cb + (im ? 4 : 0) + c;
                        if (o >= pr.Co) continue;
                        float2* dst = pr.W + ((int64_t)i * pr.Co + o) * pr.Mt + t0;
                        if (vec) {
                            l2::st8(dst, make_float4(out[c][0], out[c][1], out[c][2], out[c][3]),
                                    make_float4(out[c][4], out[c][5], out[c][6], out[c][7]), pol_out);
                        } else {
#pragma unroll
                            for (int jl = 0; jl < MODES; ++jl)
                                if (t0 + jl < pr.Mt) dst[jl] = make_float2(out[c][2 * jl], out[c][2 * jl + 1]);
                        }
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
}

}  // namespace wgtc
}  // namespace nop

// Fused per-pixel channel MLP on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Same function as the CUDA-core kernel in pointwise.cu (u = [x ; grid], h = act1(W1 u + b1),
// y = act2(W2 h + b2 + g * r + gb), z = W3 y), with every layer one GEMM per tile of 128 points:
//
//   D[p][n] = sum_k A[p][k] W[n][k]        M = 128 points, N = output channels (padded to 16), K = 8 per MMA
//
// Both operands are K-major in shared memory (canonical no-swizzle layout: 8-row x 16-byte core
// matrices, K-adjacent core matrices 128 B apart, 8-row groups 256 B apart): A = activations with the
// points as rows, W = weights [out][in].  x arrives by cp.async into a staging buffer in its HBM order
// (one 128-point row per channel, rows padded to 544 B) and a split pass transposes it into A: every
// warp step moves an 8-point x 4-channel block, so both the staging reads and the A writes are
// bank-conflict free.  Epilogues write h and y back as A with one 16-byte store per 4 channels.
//
// fp32 accuracy from tf32 MMAs (three-pass split): every operand is stored as hi = tf32(x) and
// lo = x - hi, and D = A_hi W_hi + A_hi W_lo + A_lo W_hi accumulates in fp32 in tensor memory (the
// dropped lo * lo term is below 2^-22 relative).
//
// Selected with NOP_POINTWISE=tc.  Measured on B200 it is slower than the CUDA-core kernel (C4 TFNO model
// 42.6 vs 40.1 ms): the hi / lo operand copies of one tile, the weights and the staging buffers fill the
// CTA's shared memory, so each SM runs a single serialized GEMM -> epilogue chain (tensor pipe ~5% busy);
// a faster version needs several tiles in flight (warp-specialised stages, operands in tensor memory).
//
// One persistent CTA per SM (256 threads), tiles walked in grid stride.  Per tile: wait for x ->
// split into A (hi, lo) -> the staging buffer is free: the next tile's x starts loading -> GEMM 1 ->
// epilogue 1 (bias, act1) writes h as A, in chunks of hidden channels when h does not fit at once ->
// GEMM 2 per chunk -> epilogue 2 (bias, gate * residual, act2) stores y and writes it as A -> GEMM 3
// -> epilogue 3 stores z.  The eight warps split every epilogue: warp w reads tensor-memory lane
// quadrant w % 4 (points 32 (w % 4) ..) and half w / 4 of the columns.  MMAs are issued by one thread
// and signal completion through one mbarrier whose phase every thread tracks; every wait is bounded
// (status word, no trap).
#pragma once

#include "mix_tc.cuh"

namespace nop {
namespace pwtc {

constexpr int THREADS = 256;
constexpr int TP = 128;          // points per tile (MMA M)
constexpr int KSB = TP * 32;     // bytes of one 8-channel K step of an A tile (4096)
constexpr int SROW = 544;        // bytes per channel row of the x staging buffer (128 points + 32 B pad)

__host__ __device__ inline int up8(int v) { return (v + 7) & ~7; }
__host__ __device__ inline int up16(int v) { return (v + 15) & ~15; }
__host__ __device__ inline int act_bytes(int k) { return (k / 8) * KSB; }

// byte offset of element (point p, channel k) in a K-major A tile, or (out n, in k) in a K-major W
// operand with R rows (R = 128 for A)
__device__ __forceinline__ uint32_t kmaj_off(int r, int k, int R) {
    return (k >> 3) * (R * 32) + (r >> 3) * 256 + ((k >> 2) & 1) * 128 + (r & 7) * 16 + (k & 3) * 4;
}

struct Layout {
    int K1, N1, K2, N2, K3, N3;  // padded dims: layer 1 (K1 x N1), 2 (K2 x N2), 3 (K3 x N3)
    int chunk;                   // hidden channels staged per GEMM-2 pass (multiple of 16, divides N1)
    // byte offsets in dynamic shared memory
    int o_w1h, o_w1l, o_w2h, o_w2l, o_w3h, o_w3l, o_stg, o_rstg, o_ah, o_al, o_h, o_vec, o_bar;
    int h_lo;                    // offset of the lo half inside the h region
    int d1, d2, d3;              // tensor-memory column offsets of the accumulators
    uint32_t idesc1, idesc2, idesc3;
    int smem;
};

__host__ __device__ inline uint32_t make_idesc(int N) {
    // D f32, A and B tf32, both K-major, N >> 3, M >> 4
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TP >> 4) << 24);
}

// Host-side layout: returns false when the shapes do not fit (the CUDA-core kernel runs instead).
inline bool plan_layout(const pw::Params& p, Layout* L) {
    Layout l{};
    const bool has1 = p.Ch > 0;
    l.K1 = up8(p.Ku);
    l.N1 = has1 ? up16(p.Ch) : 0;
    l.K2 = has1 ? l.N1 : l.K1;
    l.N2 = up16(p.Cy);
    l.K3 = p.Cz > 0 ? l.N2 : 0;
    l.N3 = p.Cz > 0 ? up16(p.Cz) : 0;
    if (l.N1 > 256 || l.N2 > 256 || l.N3 > 256 || l.N1 + l.N2 + l.N3 > 512) return false;
    const int wbytes = 8 * ((has1 ? l.K1 * l.N1 : 0) + l.K2 * l.N2 + l.K3 * l.N3);
    const int stg = l.K1 * SROW;
    const int a = act_bytes(l.K1 > l.K3 ? l.K1 : l.K3);  // x as A (hi, lo), later y as A
    bool ok = false;
    for (int chunk : {128, 64, 32, 16}) {
        if (has1 && (chunk > l.N1 || l.N1 % chunk)) continue;
        if (!has1 && chunk != 16) continue;
        const int h = has1 ? 2 * act_bytes(chunk) : 0;
        int off = 0;
        auto take = [&](int n) {
            const int at = off;
            off += (n + 127) & ~127;
            return at;
        };
        l.o_w1h = take(has1 ? 4 * l.K1 * l.N1 : 0);
        l.o_w1l = take(has1 ? 4 * l.K1 * l.N1 : 0);
        l.o_w2h = take(4 * l.K2 * l.N2);
        l.o_w2l = take(4 * l.K2 * l.N2);
        l.o_w3h = take(4 * l.K3 * l.N3);
        l.o_w3l = take(4 * l.K3 * l.N3);
        l.o_stg = take(stg);
        l.o_rstg = take(p.r ? p.Cy * SROW : 0);  // the gate's residual, staged like x
        l.o_ah = take(a);
        l.o_al = take(a);
        l.o_h = take(h);
        l.o_vec = take(4 * (l.N1 + 3 * l.N2));  // b1, then b2 + gb, g (zero padded)
        l.o_bar = take(64);
        (void)wbytes;
        if (off <= 227 * 1024) {
            ok = true;
            l.chunk = has1 ? chunk : 0;
            l.h_lo = has1 ? act_bytes(chunk) : 0;
            l.smem = off < 120 * 1024 ? 120 * 1024 : off;  // > half the SM: one CTA per SM (all of TMEM)
            break;
        }
    }
    if (!ok) return false;
    l.d1 = 0;
    l.d2 = l.N1;
    l.d3 = l.N1 + l.N2;
    l.idesc1 = has1 ? make_idesc(l.N1) : 0;
    l.idesc2 = make_idesc(l.N2);
    l.idesc3 = l.N3 ? make_idesc(l.N3) : 0;
    *L = l;
    return true;
}

// K-major hi / lo copies of W [rows x cols] (row-major, out x in) padded to N x K with zeros
__device__ __forceinline__ void load_weight(char* sm, int o_hi, int o_lo, const float* w, int rows, int cols, int N,
                                            int K) {
    for (int e = threadIdx.x; e < N * K; e += THREADS) {
        const int n = e / K, k = e % K;
        const float v = (n < rows && k < cols) ? __ldg(w + (int64_t)n * cols + k) : 0.f;
        const float hi = tc::tf32_round(v);
        const float lo = tc::tf32_round(v - hi);
        const uint32_t o = kmaj_off(n, k, N);
        *reinterpret_cast<float*>(sm + o_hi + o) = hi;
        *reinterpret_cast<float*>(sm + o_lo + o) = lo;
    }
}

// issue the copies of tile t's x into the staging buffer (one 544-byte row per channel, 16-byte
// chunks of 4 points) and write the grid channels; always commits a group (empty past the last tile),
// so the wait counts of the x and residual groups stay in step
__device__ __forceinline__ void stage_x(const pw::Params& p, const Layout& L, char* sm, int64_t t) {
    if (t >= p.tiles) {
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        return;
    }
    const int64_t tiles_per_sample = p.P / TP;
    const int64_t b = t / tiles_per_sample;
    const int64_t pix0 = (t % tiles_per_sample) * TP;
    char* stg = sm + L.o_stg;
    for (int e = threadIdx.x; e < p.Cx * (TP / 4); e += THREADS) {
        const int c = e / (TP / 4), q = e % (TP / 4);
        const unsigned s = tc::smem_u32(stg + c * SROW + 16 * q);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s),
                     "l"(p.x + (b * p.Cx + c) * p.P + pix0 + 4 * q)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    for (int e = threadIdx.x; e < p.nd * TP; e += THREADS) {
        const int j = e / TP, q = e % TP;
        int64_t idx = pix0 + q;
        int64_t ij = 0;
        for (int a = p.nd - 1; a >= 0; --a) {
            const int64_t ia = idx % p.sp[a];
            idx /= p.sp[a];
            if (a == j) ij = ia;
        }
        *reinterpret_cast<float*>(stg + (p.Cx + j) * SROW + 4 * q) = p.glo[j] + (float)ij * p.gstep[j];
    }
}

// the gate's residual of tile t into its staging buffer (rows of Cy channels); always commits a group
__device__ __forceinline__ void stage_r(const pw::Params& p, const Layout& L, char* sm, int64_t t) {
    if (p.r && t < p.tiles) {
        const int64_t tiles_per_sample = p.P / TP;
        const int64_t b = t / tiles_per_sample;
        const int64_t pix0 = (t % tiles_per_sample) * TP;
        char* rs = sm + L.o_rstg;
        for (int e = threadIdx.x; e < p.Cy * (TP / 4); e += THREADS) {
            const int c = e / (TP / 4), q = e % (TP / 4);
            const unsigned s = tc::smem_u32(rs + c * SROW + 16 * q);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s),
                         "l"(p.r + (b * p.Cy + c) * p.P + pix0 + 4 * q)
                         : "memory");
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// hi / lo of 4 consecutive channels of one point, stored as A (one 16-byte store each)
__device__ __forceinline__ void store_a4(char* ahi, char* alo, int p, int k, const float* v) {
    float4 h, l;
    h.x = tc::tf32_round(v[0]);
    h.y = tc::tf32_round(v[1]);
    h.z = tc::tf32_round(v[2]);
    h.w = tc::tf32_round(v[3]);
    l = make_float4(v[0] - h.x, v[1] - h.y, v[2] - h.z, v[3] - h.w);
    const uint32_t o = kmaj_off(p, k, TP);
    *reinterpret_cast<float4*>(ahi + o) = h;
    *reinterpret_cast<float4*>(alo + o) = l;
}

__global__ void __launch_bounds__(THREADS, 1) k_pointwise_tc(pw::Params p, Layout L, int* status) {
    extern __shared__ __align__(1024) char sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, half = warp >> 2;
    const int pt = quad * 32 + lane;  // this thread's point (tensor-memory lane) in every epilogue
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L.o_bar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L.o_bar + 16);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L.o_bar + 24);
    const bool has1 = p.Ch > 0;

    if (tid == 0) {
        tc::mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort_flag = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // weights (hi / lo, zero padded) and a zeroed staging buffer (padding channels stay zero)
    if (has1) load_weight(sm, L.o_w1h, L.o_w1l, p.w1, p.Ch, p.Ku, L.N1, L.K1);
    load_weight(sm, L.o_w2h, L.o_w2l, p.w2, p.Cy, has1 ? p.Ch : p.Ku, L.N2, L.K2);
    if (L.N3) load_weight(sm, L.o_w3h, L.o_w3l, p.w3, p.Cz, p.Cy, L.N3, L.K3);
    for (int e = tid; e < L.K1 * SROW / 16; e += THREADS)
        reinterpret_cast<float4*>(sm + L.o_stg)[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    float* vb1 = reinterpret_cast<float*>(sm + L.o_vec);
    float* vb2 = vb1 + L.N1;  // b2 + gb
    float* vg = vb2 + L.N2;
    for (int c = tid; c < L.N1; c += THREADS) vb1[c] = (c < p.Ch && p.b1) ? __ldg(p.b1 + c) : 0.f;
    for (int c = tid; c < L.N2; c += THREADS) {
        vb2[c] = c < p.Cy ? (p.b2 ? __ldg(p.b2 + c) : 0.f) + (p.gb ? __ldg(p.gb + c) : 0.f) : 0.f;
        vg[c] = (c < p.Cy && p.g) ? __ldg(p.g + c) : 0.f;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t tlane = (uint32_t)(quad * 32) << 16;

    uint32_t phase = 0;  // completions of `bar` so far (every thread counts the same)
    bool ok = true;
    // one thread issues a GEMM: ksteps x 3 tf32 MMAs into columns dcol; `first` clears the accumulator
    auto gemm = [&](uint32_t a_hi, uint32_t a_lo, uint32_t w_hi, uint32_t w_lo, int N, int ksteps, uint32_t dcol,
                    uint32_t idesc, bool first) {
        for (int ks = 0; ks < ksteps; ++ks) {
            const uint64_t ah = tc::smem_desc(a_hi + ks * KSB), al = tc::smem_desc(a_lo + ks * KSB);
            const uint64_t bh = tc::smem_desc(w_hi + ks * N * 32), bl = tc::smem_desc(w_lo + ks * N * 32);
            const uint32_t d = tmem + dcol;
            tc::mma_tf32(d, ah, bh, idesc, (first && ks == 0) ? 0u : 1u);
            tc::mma_tf32(d, ah, bl, idesc, 1u);
            tc::mma_tf32(d, al, bh, idesc, 1u);
        }
    };
    // one warp waits for the MMAs; the others sleep in the barrier instead of polling
    auto commit_wait = [&]() -> bool {
        if (tid == 0) tc::mma_commit(bar);
        if (warp == 0 && !tc::mbar_wait(bar, phase & 1, abort_flag)) {
            if (lane == 0) {
                *abort_flag = 1;
                atomicExch(status, tc::kStatusMmaTimeout);
            }
        }
        __syncthreads();
        ++phase;
        if (*abort_flag) {
            ok = false;
            return false;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        return true;
    };
    auto sync_for_mma = [&]() {  // generic-proxy smem writes -> visible to the tensor cores
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    };

    const uint32_t s_w1h = tc::smem_u32(sm + L.o_w1h), s_w1l = tc::smem_u32(sm + L.o_w1l);
    const uint32_t s_w2h = tc::smem_u32(sm + L.o_w2h), s_w2l = tc::smem_u32(sm + L.o_w2l);
    const uint32_t s_w3h = tc::smem_u32(sm + L.o_w3h), s_w3l = tc::smem_u32(sm + L.o_w3l);
    char* stg = sm + L.o_stg;
    char* ah = sm + L.o_ah;
    char* al = sm + L.o_al;
    char* hh = sm + L.o_h;
    char* hl = sm + L.o_h + L.h_lo;
    const uint32_t s_ah = tc::smem_u32(ah), s_al = tc::smem_u32(al);
    const uint32_t s_hh = tc::smem_u32(hh), s_hl = tc::smem_u32(hl);
    const int64_t tiles_per_sample = p.P / TP;

    const char* rstg = sm + L.o_rstg;
    // cp.async groups in issue order: x(t0), r(t0), then per tile x(t + grid) after the split and
    // r(t + grid) after epilogue 2 -- "wait_group 1" always leaves only the newest group pending
    int64_t t = blockIdx.x;
    stage_x(p, L, sm, t);
    stage_r(p, L, sm, t);
    for (; t < p.tiles && ok; t += gridDim.x) {
        const int64_t nt = t + gridDim.x;
        const int64_t b = t / tiles_per_sample;
        const int64_t pix0 = (t % tiles_per_sample) * TP;

        // ---- x has landed: split into A (hi, lo); warp step = 8 points x 4 channels ----
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        __syncthreads();
        {
            const int pl = lane >> 2, kl = lane & 3;
            const int blocks = (TP / 8) * (L.K1 / 4);
            for (int blk = warp; blk < blocks; blk += THREADS / 32) {
                const int pp = (blk % (TP / 8)) * 8 + pl, k = (blk / (TP / 8)) * 4 + kl;
                const float v = *reinterpret_cast<const float*>(stg + k * SROW + 4 * pp);
                const float h = tc::tf32_round(v);
                const uint32_t o = kmaj_off(pp, k, TP);
                *reinterpret_cast<float*>(ah + o) = h;
                *reinterpret_cast<float*>(al + o) = v - h;
            }
        }
        sync_for_mma();
        stage_x(p, L, sm, nt);  // the staging buffer is free: the next tile's x loads now

        // ---- layer 1 ----
        if (has1) {
            if (tid == 0) gemm(s_ah, s_al, s_w1h, s_w1l, L.N1, L.K1 / 8, L.d1, L.idesc1, true);
            if (!commit_wait()) break;
        }

        // ---- layer 2 (per hidden chunk) ----
        if (has1) {
            const int nchunks = L.N1 / L.chunk;
            const int hc = L.chunk / 2;
            for (int ch = 0; ch < nchunks && ok; ++ch) {
                const int c0 = ch * L.chunk;
                for (int cb = half * hc; cb < half * hc + hc; cb += 8) {
                    float v[8];
                    tc::tmem_ld8(tmem + tlane + L.d1 + c0 + cb, v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int c = c0 + cb + j;
                        float h = 0.f;
                        if (c < p.Ch) {
                            h = v[j] + vb1[c];
                            if (p.act1) h = gelu_erf(h);
                        }
                        v[j] = h;
                    }
                    store_a4(hh, hl, pt, cb, v);
                    store_a4(hh, hl, pt, cb + 4, v + 4);
                }
                sync_for_mma();
                if (tid == 0)
                    gemm(s_hh, s_hl, s_w2h + c0 * L.N2 * 4, s_w2l + c0 * L.N2 * 4, L.N2, L.chunk / 8, L.d2, L.idesc2,
                         ch == 0);
                if (!commit_wait()) break;
            }
            if (!ok) break;
        } else {
            if (tid == 0) gemm(s_ah, s_al, s_w2h, s_w2l, L.N2, L.K1 / 8, L.d2, L.idesc2, true);
            if (!commit_wait()) break;
        }

        // ---- epilogue 2: y = act2(D2 + b2 + gb + g * r); store, and write back as layer 3's A ----
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");  // this tile's residual
        __syncthreads();
        const int n2h = L.N2 / 2;
        for (int cb = half * n2h; cb < half * n2h + n2h; cb += 8) {
            float v[8];
            tc::tmem_ld8(tmem + tlane + L.d2 + cb, v);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = cb + j;
                float y = 0.f;
                if (c < p.Cy) {
                    y = v[j] + vb2[c];
                    if (p.r) y = fmaf(vg[c], *reinterpret_cast<const float*>(rstg + c * SROW + 4 * pt), y);
                    if (p.act2) y = gelu_erf(y);
                    p.y[(b * p.Cy + c) * p.P + pix0 + pt] = y;
                }
                v[j] = y;
            }
            if (L.N3) {
                store_a4(ah, al, pt, cb, v);
                store_a4(ah, al, pt, cb + 4, v + 4);
            }
        }

        // ---- layer 3: z = W3 y ----
        if (L.N3) {
            sync_for_mma();
            stage_r(p, L, sm, nt);  // every thread is past its residual reads
            if (tid == 0) gemm(s_ah, s_al, s_w3h, s_w3l, L.N3, L.K3 / 8, L.d3, L.idesc3, true);
            if (!commit_wait()) break;
            const int n3h = L.N3 / 2;
            for (int cb = half * n3h; cb < half * n3h + n3h; cb += 8) {
                float v[8];
                tc::tmem_ld8(tmem + tlane + L.d3 + cb, v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int c = cb + j;
                    if (c < p.Cz) p.z[(b * p.Cz + c) * p.P + pix0 + pt] = v[j];
                }
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();  // the A tiles, h and the accumulators are reused by the next tile
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (!L.N3) stage_r(p, L, sm, nt);
    }
    // leave no copy in flight; after an expired wait, let issued MMAs drain (bounded) before the tensor
    // memory is freed
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    if (!ok && tid == 0) {  // drain: a last commit, waited for without the abort shortcut (bounded)
        tc::mma_commit(bar);
        tc::mbar_wait(bar, phase & 1, nullptr);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
}

}  // namespace pwtc
}  // namespace nop

// Per-mode complex contraction on tcgen05 with TMA operand loads (sm_100a).
//
//   Y[q][b][o][j] = sum_i X[q][b][i][j] W_q[i][o][j]        (complex, mode 8 q + j)
//
// The MMA formulation of tc::k_mix_tc (mix_tc.cuh: per mode one real GEMM, M = 128 = [Xr;Xi] of 64
// batch rows, N = 2 CO = [Wr|Wi], K = input channels; three-pass TF32 or one bf16 pass; the re / im
// combination with lane shuffles in the epilogue) on tiles of TWO modes (a quarter mode block), so a
// tile's accumulators take 2 x 2 CO <= 256 tensor-memory columns and two tiles' accumulators
// alternate: the epilogue of one tile runs under the MMAs of the next.  Operands reach shared memory
// by tensor copies:
//
//   TMA warp 13 (lane 0) : per K step two cp.async.bulk.tensor loads into a landing slot (ring of RS),
//                          completing on `land_full[slot]` (transaction bytes):
//                            X box {2 modes (4 floats), 64 batch rows, KS channels} of the
//                              mode-blocked spectrum [Q][B][Ci][8 modes]  -> landing [i][b][4 floats]
//                            W box {CO float4 (output channels), 1 mode pair, KS channels} of the
//                              packed weights W_q[i][p][o]                -> landing [i][CO float4]
//                          rows past B, channels past Ci / Co are zero-filled by the copy itself
//   producer warps 4..11 : wait `land_full`, read their values (X: one batch row and a K half per thread,
//                          consecutive threads on consecutive 16-byte rows; W: one output channel and a
//                          K half), release the slot (`land_empty`), split into tf32 hi / lo (or round to
//                          bf16) and store the canonical K-major stage (ring of NS) for the MMA warp
//   MMA warp 12 (lane 0) : wait `full[s]`, issue the step's MMAs for the two modes, commit to `empty[s]`;
//                          after a tile's last step commit to `acc_full[a]` (a = tile parity)
//   epilogue warps 0..3  : wait `acc_full[a]`, tcgen05.ld their lane quadrant (the next column group's
//                          loads in flight while the current one is combined), release `acc_empty[a]`,
//                          combine re / im with shuffles into a staging tile and write it with
//                          one tensor store per 16 rows x 8 channels (a per-thread store would touch 32
//                          spectrum rows per warp instruction and hold the load/store unit that the
//                          producers need)
//
// Measured on B200 (C2 shapes, clock64 trace per role): with four-mode tiles the single accumulator
// made every tile's epilogue (~12k cycles) stall the MMA and, through the full stages, the producers.
// No multicast: every copy is a plain tiled load of this GPU's memory.  Every wait is bounded
// (kWaitCycles); on expiry the kernel records the status word, the roles leave their loops, the
// copies in flight and the issued MMAs are drained (bounded) and the tensor memory is freed.
#pragma once

#include <cuda.h>

#include "mix_tc.cuh"

namespace nop {
namespace tma_mix {

using tc::BT;
using tc::EPI_WARPS;
using tc::M;
using tc::MMA_WARP;
using tc::PROD_THREADS;
using tc::PROD_WARPS;
constexpr int TMA_WARP = MMA_WARP + 1;
constexpr int THREADS = 32 * (TMA_WARP + 1);  // 448
constexpr int TM = 2;                         // modes per tile

template <int CO, bool BF16>
struct Cfg {
    static constexpr int N = 2 * CO;
    static constexpr int KS = BF16 ? 16 : 8;           // K per MMA instruction (32 bytes of K)
    static constexpr int SPLITS = BF16 ? 1 : 2;         // hi / lo operand copies
    static constexpr int A_TILE = M * 32;               // bytes of one mode's A for one K step
    static constexpr int B_TILE = N * 32;
    static constexpr int STAGE = TM * SPLITS * (A_TILE + B_TILE);
    static constexpr int XBYTES = KS * BT * 16;         // [KS][64][4 floats]
    static constexpr int WBYTES = KS * CO * 16;         // [KS][CO float4]
    static constexpr int RAW = XBYTES + WBYTES;         // one landing slot
    static constexpr int RS = 4;
    // epilogue staging: per epilogue warp two 2 KB tiles [8 channels][16 rows][16 B]
    static constexpr int EPI_TILE = 2048;
    static constexpr int EPI_BYTES = EPI_WARPS * 2 * EPI_TILE;
    static constexpr int NS0 = (226 * 1024 - RS * RAW - EPI_BYTES) / STAGE;
    static constexpr int NS = NS0 > 8 ? 8 : NS0;
    static constexpr int ACC_COLS = TM * N;             // tensor-memory columns of one tile
    static constexpr int NACC = 2;
    static constexpr int TMEM_COLS = 512;
    static constexpr int EPI_OFF = NS * STAGE;
    static constexpr int RAW_OFF = EPI_OFF + EPI_BYTES;
    static constexpr int BODY = RAW_OFF + RS * RAW;
    // after the body: full[NS], empty[NS], land_full[RS], land_empty[RS], acc_full[2], acc_empty[2], drain,
    // then the tensor-memory address and the abort flag
    static constexpr int TAIL = (2 * NS + 2 * RS + 5) * 8 + 8;
    static constexpr int SMEM = BODY + 256;
    static_assert(TAIL <= 256, "barrier area overflows its reservation");
    static_assert(NS >= 2, "at least two stages");
    static_assert(RAW_OFF % 128 == 0 && RAW % 128 == 0, "landing slots 128-byte aligned");
    static_assert(EPI_OFF % 128 == 0, "epilogue tiles 128-byte aligned");
    static_assert(BODY + 256 <= 227 * 1024, "shared memory per CTA");
    static_assert(NACC * ACC_COLS <= TMEM_COLS, "accumulators exceed tensor memory");
    static_assert(SMEM > 116 * 1024, "one CTA per SM: the whole tensor memory is allocated");
    // instruction descriptor: D f32, A/B tf32 (2) or bf16 (1), both K-major, N >> 3, M >> 4
    static constexpr uint32_t IDESC = (1u << 4) | ((BF16 ? 1u : 2u) << 7) | ((BF16 ? 1u : 2u) << 10) |
                                      ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
};

// one K step of a producer thread: per channel c of its K half, the two modes (re0, im0, re1, im1)
template <bool BF16>
struct Step {
    static constexpr int KH = BF16 ? 8 : 4;
    float4 v[KH];
};

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(tc::smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(tc::smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(tc::smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(tc::smem_u32(bar)), "l"(pol)
        : "memory");
}

// tensor store of a shared-memory tile (bulk async group of the issuing thread)
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3,
                                             uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4, %5}], [%1], %6;" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(tc::smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(pol)
        : "memory");
}

// tile t: mode quarter h (fastest), output tile, local mode block q, batch tile -- the tiles that read
// the same X rows run on neighbouring CTAs at the same time, so X comes from L2 after its first read
struct TileIdx {
    int h, o0, q, qw, b0;
};

__device__ __forceinline__ TileIdx tile_idx(int t, int ot, int local, int qpl, int qtot, int qbeg, int co_tile) {
    TileIdx r;
    r.h = t & 3;
    int rest = t >> 2;
    r.o0 = (rest % ot) * co_tile;
    rest /= ot;
    r.q = rest % local;
    r.b0 = (rest / local) * BT;
    r.qw = (r.q / qpl) * qtot + qbeg + r.q % qpl;  // local mode block -> weight block
    return r;
}

// producer thread p's values of one K step from a landing slot.  X threads p < 128: batch row
// b = p % 64, K half p / 64 (consecutive threads read consecutive 16-byte rows); W threads: output
// channel u % CO, K half u / CO (consecutive threads read consecutive float4).
template <int CO, bool BF16>
__device__ __forceinline__ void read_landed(const char* slot, int p, Step<BF16>& st) {
    using C = Cfg<CO, BF16>;
    constexpr int KH = Step<BF16>::KH;
    if (p < 128) {
        const int b = p & 63, kh = p >> 6;
        const float4* x = reinterpret_cast<const float4*>(slot);
#pragma unroll
        for (int c = 0; c < KH; ++c) st.v[c] = x[(kh * KH + c) * BT + b];
    } else if (p < 128 + 2 * CO) {
        const int u = p - 128;
        const int o = u % CO, kh = u / CO;
        const float4* w = reinterpret_cast<const float4*>(slot + C::XBYTES);
#pragma unroll
        for (int c = 0; c < KH; ++c) st.v[c] = w[(kh * KH + c) * CO + o];
    }
}

// the canonical K-major stage of one K step: 8-row x 16-byte core matrices (tc::tile_off), A rows
// [Xr; Xi] in 16-row halves of every 32-row quadrant (tc::a_row), B rows [Wr | Wi]
template <int CO, bool BF16>
__device__ __forceinline__ void store_landed(const Step<BF16>& st, char* stage, int p) {
    using C = Cfg<CO, BF16>;
    constexpr int KH = Step<BF16>::KH;
    int rows[2], kh, tile_bytes;
    char* base;
    if (p < 128) {
        rows[0] = tc::a_row(p & 63, 0);
        rows[1] = tc::a_row(p & 63, 1);
        kh = p >> 6;
        base = stage;
        tile_bytes = C::A_TILE;
    } else if (p < 128 + 2 * CO) {
        const int u = p - 128;
        rows[0] = u % CO;       // columns of Wr
        rows[1] = u % CO + CO;  // columns of Wi
        kh = u / CO;
        base = stage + TM * C::SPLITS * C::A_TILE;
        tile_bytes = C::B_TILE;
    } else {
        return;
    }
#pragma unroll
    for (int jl = 0; jl < TM; ++jl) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const uint32_t off = tc::tile_off(rows[e], kh);
            float x[KH];
#pragma unroll
            for (int c = 0; c < KH; ++c) {
                const float4 v = st.v[c];
                x[c] = jl ? (e ? v.w : v.z) : (e ? v.y : v.x);
            }
            if constexpr (BF16) {
                uint4 w;
                w.x = tc::pack_bf16(x[0], x[1]);
                w.y = tc::pack_bf16(x[2], x[3]);
                w.z = tc::pack_bf16(x[4], x[5]);
                w.w = tc::pack_bf16(x[6], x[7]);
                *reinterpret_cast<uint4*>(base + jl * tile_bytes + off) = w;
            } else {
                float hi[4], lo[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    hi[c] = tc::tf32_round(x[c]);
                    lo[c] = tc::tf32_round(x[c] - hi[c]);
                }
                *reinterpret_cast<float4*>(base + (jl * 2 + 0) * tile_bytes + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<float4*>(base + (jl * 2 + 1) * tile_bytes + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
    }
}

// one column group (8 columns of Re-weight and Im-weight products for both modes) of this warp's lane
// quadrant of a tile's accumulators
template <int CO, bool BF16>
__device__ __forceinline__ void load_group_t(uint32_t tbase, int cb, float (&P)[TM][8], float (&Q)[TM][8]) {
    using C = Cfg<CO, BF16>;
#pragma unroll
    for (int jl = 0; jl < TM; ++jl) {
        tc::tmem_ld8(tbase + jl * C::N + cb, P[jl]);
        tc::tmem_ld8(tbase + jl * C::N + CO + cb, Q[jl]);
    }
}

// wait for this thread's tensor-memory loads; the loaded registers are operands of the wait, so no use
// of them is scheduled before it
__device__ __forceinline__ void wait_regs(float (&v)[TM][8]) {
    static_assert(TM == 2, "operand list written for two modes");
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(v[0][0]), "+f"(v[0][1]), "+f"(v[0][2]), "+f"(v[0][3]), "+f"(v[0][4]), "+f"(v[0][5]),
                   "+f"(v[0][6]), "+f"(v[0][7]), "+f"(v[1][0]), "+f"(v[1][1]), "+f"(v[1][2]), "+f"(v[1][3]),
                   "+f"(v[1][4]), "+f"(v[1][5]), "+f"(v[1][6]), "+f"(v[1][7])
                 :
                 : "memory");
}

// Persistent: CTA c takes tiles c, c + gridDim.x, ...  `w_rank` 4: weights per mode block (map dims
// {4 Co floats, 4, Ci, blocks}); 3: one weight matrix for every block (a Tucker factor).
template <int CO, bool BF16>
__global__ void __maxnreg__(128)
k_mix_tma(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
          const __grid_constant__ CUtensorMap tmy, int w_rank, int B, int Ci, int Co, int local, int qpl, int qtot,
          int qbeg, int* __restrict__ status) {
    using C = Cfg<CO, BF16>;
    constexpr int NS = C::NS, NACC = C::NACC, RS = C::RS;
    extern __shared__ __align__(1024) char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BODY);
    uint64_t* empty = full + NS;
    uint64_t* land_full = empty + NS;
    uint64_t* land_empty = land_full + RS;
    uint64_t* acc_full = land_empty + RS;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int bt = (B + BT - 1) / BT, ot = (Co + CO - 1) / CO;
    const int tiles = 4 * local * bt * ot;
    const int my_tiles = tiles > (int)blockIdx.x ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nk = (Ci + C::KS - 1) / C::KS;
    auto tile_k = [&](int k) { return tile_idx((int)blockIdx.x + k * (int)gridDim.x, ot, local, qpl, qtot, qbeg, CO); };

    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            tc::mbar_init(&full[i], PROD_WARPS);  // one arrival per producer warp
            tc::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < RS; ++i) {
            tc::mbar_init(&land_full[i], 1);  // the TMA thread's expect_tx arrival + the copies' bytes
            tc::mbar_init(&land_empty[i], PROD_WARPS);
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
    const int steps = my_tiles * nk;

    if (warp == TMA_WARP) {
        // ------------------------------ tensor copies ------------------------------
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmx)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmw)) : "memory");
            const uint64_t pol = l2::evict_first();  // spectrum and weights are read once
            int issued = 0;
            TileIdx tl{};
            for (int g = 0; g < steps; ++g) {
                const int slot = g % RS, use = g / RS;
                if (use > 0 && !tc::mbar_wait(&land_empty[slot], (uint32_t)((use - 1) & 1), abort_flag)) {
                    give_up();
                    break;
                }
                const int kc = g % nk;
                if (kc == 0) tl = tile_k(g / nk);
                char* dst = smem + C::RAW_OFF + slot * C::RAW;
                mbar_expect_tx(&land_full[slot], C::RAW);
                tma_load_4d(dst, &tmx, 4 * tl.h, tl.b0, kc * C::KS, tl.q, &land_full[slot], pol);
                if (w_rank == 4)
                    tma_load_4d(dst + C::XBYTES, &tmw, 4 * tl.o0, tl.h, kc * C::KS, tl.qw, &land_full[slot], pol);
                else
                    tma_load_3d(dst + C::XBYTES, &tmw, 4 * tl.o0, tl.h, kc * C::KS, &land_full[slot], pol);
                issued = g + 1;
            }
            // the copies still in flight land before the CTA can exit (bounded; they depend on no
            // other role)
            for (int g = issued - RS > 0 ? issued - RS : 0; g < issued; ++g)
                if (!tc::mbar_wait(&land_full[g % RS], (uint32_t)((g / RS) & 1), nullptr)) give_up();
        }
    } else if (warp >= EPI_WARPS && warp < MMA_WARP) {
        // ------------------------------ producers ------------------------------
        const int p = tid - 32 * EPI_WARPS;
        Step<BF16> cur;
        int s = 0;
        uint32_t upar = 0;   // parity of the current use of stage s
        bool reuse = false;  // stage s held an earlier step
        for (int g = 0; g < steps; ++g) {
            const int slot = g % RS;
            if (!tc::mbar_wait(&land_full[slot], (uint32_t)((g / RS) & 1), abort_flag)) {
                give_up();
                break;
            }
            read_landed<CO, BF16>(smem + C::RAW_OFF + slot * C::RAW, p, cur);
            // the slot's next contents arrive through the async proxy: order these generic-proxy reads
            // before that write
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&land_empty[slot]);
            if (reuse && !tc::mbar_wait(&empty[s], upar ^ 1, abort_flag)) {
                give_up();
                break;
            }
            store_landed<CO, BF16>(cur, smem + s * C::STAGE, p);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&full[s]);
            if (++s == NS) {
                s = 0;
                upar ^= 1;
                reuse = true;
            }
        }
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
                    const uint32_t bq = a0 + TM * C::SPLITS * C::A_TILE;
#pragma unroll
                    for (int jl = 0; jl < TM; ++jl) {
                        const uint32_t d = dacc + jl * C::N;
                        if constexpr (BF16) {
                            tc::mma_bf16(d, tc::smem_desc(a0 + jl * C::A_TILE), tc::smem_desc(bq + jl * C::B_TILE),
                                         C::IDESC, kc > 0);
                        } else {
                            const uint64_t ahi = tc::smem_desc(a0 + (jl * 2) * C::A_TILE);
                            const uint64_t alo = tc::smem_desc(a0 + (jl * 2 + 1) * C::A_TILE);
                            const uint64_t bhi = tc::smem_desc(bq + (jl * 2) * C::B_TILE);
                            const uint64_t blo = tc::smem_desc(bq + (jl * 2 + 1) * C::B_TILE);
                            tc::mma_tf32(d, ahi, bhi, C::IDESC, kc > 0);
                            tc::mma_tf32(d, ahi, blo, C::IDESC, 1);
                            tc::mma_tf32(d, alo, bhi, C::IDESC, 1);
                        }
                    }
                    tc::mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
                    if (++s == NS) {
                        s = 0;
                        upar ^= 1;
                    }
                }
                if (!ok) break;
                tc::mma_commit(&acc_full[a]);  // the tile's accumulators are complete
            }
            // drain: every MMA issued so far has finished once this commit lands (also after an
            // abort, so the tensor memory is never freed under a running MMA)
            tc::mma_commit(drain);
            if (!tc::mbar_wait(drain, 0, nullptr)) give_up();
        }
    } else if (warp < EPI_WARPS) {
        // ------------------------------ epilogue (warps 0..3) ------------------------------
        // Each warp owns 16 batch rows (its tensor-memory lane quadrant holds their Xr and Xi rows).  Per
        // group of 8 output channels it writes the combined values into a staging tile
        // [8 channels][16 rows][2 modes] (per store instruction the 16 re lanes fill one channel's 256
        // contiguous bytes and the 16 im lanes another: no bank conflicts) and lane 0 stores the tile
        // with one tensor store; the copy clips rows past B and channels past Co.
        const int qd = warp;                   // tensor-memory lane quadrant
        const bool im = lane >= 16;            // this lane holds the Xi row of its batch entry
        const int rl = lane & 15;              // batch row within the warp's 16
        const uint64_t pol_out = l2::evict_last();  // the output spectrum is read back by the inverse
        char* epi = smem + C::EPI_OFF + qd * 2 * C::EPI_TILE;
        auto load_group = [](uint32_t tb, int cb, float (&P)[TM][8], float (&Q)[TM][8]) {
            load_group_t<CO, BF16>(tb, cb, P, Q);
        };
        auto wait_group = [](float (&P)[TM][8], float (&Q)[TM][8]) {
            wait_regs(P);
            wait_regs(Q);
        };
        int stores = 0;  // tensor stores issued by this warp (lane 0)
        for (int k = 0; k < my_tiles; ++k) {
            const int a = k % NACC;
            if (!tc::mbar_wait(&acc_full[a], (uint32_t)((k / NACC) & 1), abort_flag)) {
                give_up();
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const TileIdx tl = tile_k(k);
            const uint32_t tbase = tmem + ((uint32_t)(qd * 32) << 16) + a * C::ACC_COLS;
            // column groups of 8: the next group's tensor-memory loads are in flight while the current
            // group is combined and stored
            float P[2][TM][8], Qv[2][TM][8];
            load_group(tbase, 0, P[0], Qv[0]);
            wait_group(P[0], Qv[0]);
#pragma unroll
            for (int g = 0; g < CO / 8; ++g) {
                const int cb = 8 * g, cur = g & 1;
                if (g + 1 < CO / 8) {
                    load_group(tbase, cb + 8, P[cur ^ 1], Qv[cur ^ 1]);
                } else {
                    // every load of this tile has completed: the next tile using this buffer may start
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&acc_empty[a]);
                }
                // re lanes finish channels 0..3 of this group, im lanes channels 4..7
                float out[4][2 * TM];
#pragma unroll
                for (int jl = 0; jl < TM; ++jl) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float* Pc = P[cur][jl];
                        const float* Qc = Qv[cur][jl];
                        const float sp = im ? Pc[c] : Pc[4 + c];
                        const float sq = im ? Qc[c] : Qc[4 + c];
                        const float rp = __shfl_xor_sync(0xffffffffu, sp, 16);
                        const float rq = __shfl_xor_sync(0xffffffffu, sq, 16);
                        if (!im) {  // own Xr row: P = Xr Wr, Q = Xr Wi; partner: Xi Wr, Xi Wi
                            out[c][2 * jl] = Pc[c] - rq;
                            out[c][2 * jl + 1] = Qc[c] + rp;
                        } else {    // own Xi row; partner: Xr Wr, Xr Wi of channels 4..7
                            out[c][2 * jl] = rp - Qc[4 + c];
                            out[c][2 * jl + 1] = rq + Pc[4 + c];
                        }
                    }
                }
                // the staging tile written two groups ago has been read by its tensor store
                char* tile = epi + (stores & 1) * C::EPI_TILE;
                if (lane == 0 && stores >= 2) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                __syncwarp();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int ch = (im ? 4 : 0) + c;
                    *reinterpret_cast<float4*>(tile + (ch * 16 + rl) * 16) =
                        make_float4(out[c][0], out[c][1], out[c][2], out[c][3]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor store
                __syncwarp();
                if (lane == 0) {
                    tma_store_4d(&tmy, tile, 4 * tl.h, tl.b0 + qd * 16, tl.o0 + cb, tl.q, pol_out);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
                ++stores;
                if (g + 1 < CO / 8) wait_group(P[cur ^ 1], Qv[cur ^ 1]);
            }
        }
        // the staging tiles stay allocated until the tensor stores have completed
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
}

}  // namespace tma_mix
}  // namespace nop

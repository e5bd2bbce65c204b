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
//   TMA warp 13 (lane 0) : per K step
//                            - one cp.async.bulk.tensor load of the X box {2 modes (4 floats), 64 batch
//                              rows, KS channels} of the mode-blocked spectrum [Q][B][Ci][8 modes] into a
//                              landing slot [i][b][4 floats] (ring of RS, `land_full[slot]`; rows past B
//                              and channels past Ci zero-filled by the copy);
//                            - once the MMAs have released stage s (`empty[s]`), one cp.async.bulk copy of
//                              the step's weight tiles, packed ahead of time in the MMA's own layout (tf32
//                              hi / lo or bf16, zero past Ci / Co; see k_pack_tc), straight into the B half
//                              of stage s (transaction bytes on `full[s]`)
//   producer warps 4..11 : wait `land_full`, read their X values (thread = one batch row, one K half, one
//                          mode; a warp = one mode of 32 consecutive rows), release the slot
//                          (`land_empty`), split into tf32 hi / lo (or round to bf16) and store the A half
//                          of stage s in the canonical K-major layout (`full[s]`: 8 producer arrivals plus
//                          the weight copy's bytes)
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
// made every tile's epilogue (~12k cycles) stall the MMA and, through the full stages, the producers;
// with the weights converted by the producers too, shared-memory traffic (~112 KB per K step) bounded
// the producers, which the pre-split weight tiles cut to ~96 KB and half the producer work.
// Every copy is a plain (single-CTA) tiled copy of this GPU's own memory.  Every wait is bounded
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
    static constexpr int RAW = XBYTES;                  // one landing slot
    static constexpr int A_BYTES = TM * SPLITS * A_TILE;  // the producers' half of a stage
    static constexpr int W_STEP = TM * SPLITS * B_TILE;   // the weight copy's half (bytes per K step)
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

// one K step of a producer thread: per channel c of its K half, its mode's (re, im)
template <bool BF16>
struct Step {
    static constexpr int KH = BF16 ? 8 : 4;
    float2 v[KH];
};

// Pre-split weight tiles (written by k_pack_tc, read by one bulk copy per K step).  Tile id
//   T = (((qw * H + h) * ot + otile) * nk + k) * TM + jl
// for weight block qw (0 for a matrix shared by every block, with H = 1 and h taken as 0), mode pair
// h, output tile otile (CO channels), K step k and mode jl of the pair; per tile SPLITS B images of
// 2 CO rows ([Wr | Wi] of the CO channels) x KS channels in the canonical K-major layout.
__host__ __device__ __forceinline__ int64_t tc_tile(int64_t qw, int H, int h, int ot, int otile, int nk, int k, int jl) {
    return (((qw * H + h) * ot + otile) * nk + k) * TM + jl;
}

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

// contiguous global -> shared copy completing on an mbarrier (transaction bytes)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            tc::smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(tc::smem_u32(bar)), "l"(pol)
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

// producer thread p's values of one K step from a landing slot: batch row b = p % 64, mode
// jl = (p / 64) % 2, K half p / 128.  A warp holds one mode of 32 consecutive rows, so its stores
// of the A half hit distinct bank groups (measured: lanes of both modes in one warp stored to tiles a
// multiple of 128 bytes apart, 1.7 M extra shared-memory wavefronts on C2)
template <int CO, bool BF16>
__device__ __forceinline__ void read_landed(const char* slot, int p, Step<BF16>& st) {
    constexpr int KH = Step<BF16>::KH;
    const int b = p & 63, jl = (p >> 6) & 1, kh = p >> 7;
    const float2* x = reinterpret_cast<const float2*>(slot);
#pragma unroll
    for (int c = 0; c < KH; ++c) st.v[c] = x[((kh * KH + c) * BT + b) * 2 + jl];
}

// the A half of a stage: the thread's mode jl, rows (Xr, Xi) of its batch entry, its K half, in the
// canonical K-major layout (8-row x 16-byte core matrices, tc::tile_off; rows tc::a_row)
template <int CO, bool BF16>
__device__ __forceinline__ void store_landed(const Step<BF16>& st, char* stage, int p) {
    using C = Cfg<CO, BF16>;
    constexpr int KH = Step<BF16>::KH;
    const int b = p & 63, jl = (p >> 6) & 1, kh = p >> 7;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const uint32_t off = tc::tile_off(tc::a_row(b, e), kh);
        float x[KH];
#pragma unroll
        for (int c = 0; c < KH; ++c) x[c] = e ? st.v[c].y : st.v[c].x;
        if constexpr (BF16) {
            uint4 w;
            w.x = tc::pack_bf16(x[0], x[1]);
            w.y = tc::pack_bf16(x[2], x[3]);
            w.z = tc::pack_bf16(x[4], x[5]);
            w.w = tc::pack_bf16(x[6], x[7]);
            *reinterpret_cast<uint4*>(stage + jl * C::A_TILE + off) = w;
        } else {
            float hi[4], lo[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                hi[c] = tc::tf32_round(x[c]);
                lo[c] = tc::tf32_round(x[c] - hi[c]);
            }
            *reinterpret_cast<float4*>(stage + (jl * 2 + 0) * C::A_TILE + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<float4*>(stage + (jl * 2 + 1) * C::A_TILE + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
        }
    }
}

// Weight packing for this kernel: element (i, o, m) of the weight at W[i * s_i + o * s_o + m * s_m]
// (s_m = 0: one matrix for every block) into the tiles described at tc_tile, conjugated when `conj`.
// One thread per 16-byte piece: B row r (r < CO: Re of channel otile * CO + r, else Im of channel
// otile * CO + r - CO), K half kh; tf32 hi / lo pieces (the split of the producers, so the MMA
// operands equal a per-launch split bit for bit) or 8 bf16.
template <int CO, bool BF16>
__global__ void k_pack_tc(const float2* __restrict__ W, char* __restrict__ out, int I, int O, int64_t Mt, int64_t Qw,
                          int H, int ot, int nk, int64_t s_i, int64_t s_o, int64_t s_m, int conj) {
    using C = Cfg<CO, BF16>;
    constexpr int HALF = C::KS / 2;  // channels per 16-byte piece
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t tiles = Qw * H * ot * nk * TM;
    if (idx >= tiles * 2 * CO * 2) return;
    const int kh = (int)(idx & 1);
    const int r = (int)((idx >> 1) % (2 * CO));
    int64_t t = (idx >> 1) / (2 * CO);
    const int jl = (int)(t % TM);
    int64_t u = t / TM;
    const int k = (int)(u % nk);
    u /= nk;
    const int otile = (int)(u % ot);
    u /= ot;
    const int h = (int)(u % H);
    const int64_t qw = u / H;
    const int o = otile * CO + (r < CO ? r : r - CO);
    const int64_t m = 8 * qw + 2 * h + jl;
    const bool ok = o < O && (s_m == 0 || m < Mt);
    float v[HALF];
#pragma unroll
    for (int c = 0; c < HALF; ++c) {
        const int i = k * C::KS + kh * HALF + c;
        float2 w = make_float2(0.f, 0.f);
        if (ok && i < I) w = W[i * s_i + o * s_o + (s_m ? m * s_m : 0)];
        v[c] = r < CO ? w.x : (conj ? -w.y : w.y);
    }
    char* tile = out + t * C::SPLITS * C::B_TILE;
    const uint32_t off = tc::tile_off(r, kh);
    if constexpr (BF16) {
        uint4 w;
        w.x = tc::pack_bf16(v[0], v[1]);
        w.y = tc::pack_bf16(v[2], v[3]);
        w.z = tc::pack_bf16(v[4], v[5]);
        w.w = tc::pack_bf16(v[6], v[7]);
        *reinterpret_cast<uint4*>(tile + off) = w;
    } else {
        float hi[4], lo[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            hi[c] = tc::tf32_round(v[c]);
            lo[c] = tc::tf32_round(v[c] - hi[c]);
        }
        *reinterpret_cast<float4*>(tile + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<float4*>(tile + C::B_TILE + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// The same tiles for weights per mode block with contiguous modes (s_m = 1: dense weights, their
// adjoint, the expanded Tucker core), one CTA per (weight block qw, output tile, K step): for every
// (channel, output) pair of the step the block's 8 modes are one 64-byte run, read into shared
// memory ([channel][mode][output], conflict-free both ways) a K half at a time, then written as the
// 16-byte pieces of the 4 mode pairs x 2 modes (values identical to k_pack_tc's).
template <int CO, bool BF16>
__global__ void __launch_bounds__(256) k_pack_tc_block(const float2* __restrict__ W, char* __restrict__ out, int I,
                                                       int O, int64_t Mt, int ot, int nk, int64_t s_i, int64_t s_o,
                                                       int conj) {
    using C = Cfg<CO, BF16>;
    constexpr int HALF = C::KS / 2;  // channels per 16-byte piece
    __shared__ float2 S[HALF][8][CO];
    const int k = (int)(blockIdx.x % nk);
    const int otile = (int)((blockIdx.x / nk) % ot);
    const int64_t qw = blockIdx.x / ((int64_t)nk * ot);
    for (int kh = 0; kh < 2; ++kh) {
        for (int e = threadIdx.x; e < HALF * CO; e += blockDim.x) {
            const int ol = e % CO, c = e / CO;
            const int o = otile * CO + ol, i = k * C::KS + kh * HALF + c;
            const bool ok = o < O && i < I;
            const float2* src = W + (ok ? i * s_i + o * s_o + 8 * qw : 0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float2 w = make_float2(0.f, 0.f);
                if (ok && 8 * qw + j < Mt) w = src[j];
                S[c][j][ol] = conj ? make_float2(w.x, -w.y) : w;
            }
        }
        __syncthreads();
        for (int f = threadIdx.x; f < 4 * TM * 2 * CO; f += blockDim.x) {
            const int r = f % (2 * CO);
            const int jl = (f / (2 * CO)) % TM;
            const int h = f / (2 * CO * TM);
            const int ol = r < CO ? r : r - CO;
            float v[HALF];
#pragma unroll
            for (int c = 0; c < HALF; ++c) {
                const float2 w = S[c][2 * h + jl][ol];
                v[c] = r < CO ? w.x : w.y;
            }
            char* tile = out + tc_tile(qw, 4, h, ot, otile, nk, k, jl) * C::SPLITS * C::B_TILE;
            const uint32_t off = tc::tile_off(r, kh);
            if constexpr (BF16) {
                uint4 w;
                w.x = tc::pack_bf16(v[0], v[1]);
                w.y = tc::pack_bf16(v[2], v[3]);
                w.z = tc::pack_bf16(v[4], v[5]);
                w.w = tc::pack_bf16(v[6], v[7]);
                *reinterpret_cast<uint4*>(tile + off) = w;
            } else {
                float hi[4], lo[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    hi[c] = tc::tf32_round(v[c]);
                    lo[c] = tc::tf32_round(v[c] - hi[c]);
                }
                *reinterpret_cast<float4*>(tile + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<float4*>(tile + C::B_TILE + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
        __syncthreads();
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

// Persistent: CTA c takes tiles c, c + gridDim.x, ...  Wtc: weight tiles from k_pack_tc; H = 4 for
// weights per mode block, H = 1 for one matrix shared by every block (a Tucker factor).
template <int CO, bool BF16>
__global__ void __maxnreg__(128)
k_mix_tma(const __grid_constant__ CUtensorMap tmx, const char* __restrict__ Wtc,
          const __grid_constant__ CUtensorMap tmy, int H, int B, int Ci, int Co, int local, int qpl, int qtot,
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
            tc::mbar_init(&full[i], PROD_WARPS + 1);  // one arrival per producer warp + the weight copy
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
            const uint64_t pol = l2::evict_first();  // spectrum and weights are read once
            int issued = 0, issued_w = 0;
            bool ok = true;
            TileIdx tl{};
            for (int g = 0; g < steps && ok; ++g) {
                const int kc = g % nk;
                if (kc == 0) tl = tile_k(g / nk);
                // X box -> landing slot
                const int slot = g % RS, use = g / RS;
                if (use > 0 && !tc::mbar_wait(&land_empty[slot], (uint32_t)((use - 1) & 1), abort_flag)) {
                    ok = false;
                    break;
                }
                char* dst = smem + C::RAW_OFF + slot * C::RAW;
                mbar_expect_tx(&land_full[slot], C::RAW);
                tma_load_4d(dst, &tmx, 4 * tl.h, tl.b0, kc * C::KS, tl.q, &land_full[slot], pol);
                issued = g + 1;
                // weight tiles -> the B half of stage s once the MMAs have released it
                const int st = g % NS, suse = g / NS;
                if (suse > 0 && !tc::mbar_wait(&empty[st], (uint32_t)((suse - 1) & 1), abort_flag)) {
                    ok = false;
                    break;
                }
                const int64_t tile = tc_tile(H == 1 ? 0 : tl.qw, H, H == 1 ? 0 : tl.h, ot, tl.o0 / CO, nk, kc, 0);
                mbar_expect_tx(&full[st], C::W_STEP);
                bulk_load(smem + st * C::STAGE + C::A_BYTES, Wtc + tile * C::SPLITS * C::B_TILE, C::W_STEP,
                          &full[st], pol);
                issued_w = g + 1;
            }
            if (!ok) give_up();
            // the copies still in flight land before the CTA can exit (bounded)
            for (int g = issued - RS > 0 ? issued - RS : 0; g < issued; ++g)
                if (!tc::mbar_wait(&land_full[g % RS], (uint32_t)((g / RS) & 1), nullptr)) give_up();
            for (int g = issued_w - NS > 0 ? issued_w - NS : 0; g < issued_w; ++g)
                if (!tc::mbar_wait(&full[g % NS], (uint32_t)((g / NS) & 1), nullptr)) give_up();
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
                    const uint32_t bq = a0 + C::A_BYTES;
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

// Per-mode complex contraction on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   Y[q][b][o][j] = sum_i X[q][b][i][j] W_q[i][o][j]        (complex, mode 8 q + j)
//
// on the mode-blocked spectrum [Q][B][C][8] with weights packed as W_q[i][p][o] = float4(mode 8q+2p,
// mode 8q+2p+1).  A tile is four modes (half a mode block), 64 batch entries and CO output channels.
// For each mode the complex product is ONE real GEMM with M = 128, N = 2 CO, K = input channels:
//
//   A rows: in every 32-row quadrant, 16 batch rows of Xr followed by the same 16 rows of Xi
//   B = [Wr | Wi]  (columns 0..CO-1: real parts, CO..2CO-1: imaginary parts)
//   D row (Xr of b) = [Xr Wr, Xr Wi],  D row (Xi of b) = [Xi Wr, Xi Wi], 16 lanes apart in one warp's
//   tensor-memory quadrant, so Yr = Xr Wr - Xi Wi and Yi = Xr Wi + Xi Wr combine with lane shuffles.
//
// fp32 accuracy from tf32 operands (three-pass split): every operand x = hi + lo with
// hi = tf32(x), lo = tf32(x - hi), and D = A_hi B_hi + A_hi B_lo + A_lo B_hi (the dropped lo*lo term
// is below 2^-22 relative), accumulated in fp32 in tensor memory.  With the bf16 contraction the
// operands are rounded to bf16 and one kind::f16 MMA per K step replaces the three tf32 ones.
//
// Warp-specialised persistent CTAs (one per SM), connected by mbarriers:
//   producer warps 4..11 : global X / W -> raw ring (cp.async, RS - 1 steps ahead) -> registers -> tf32 hi/lo or bf16 ->
//                          shared-memory stage (ring of NS) in the canonical no-swizzle K-major layout
//                          (8-row x 16-byte core matrices) -> arrive `full[s]`
//   MMA warp 12 (lane 0) : wait `full[s]`, issue the step's MMAs for the four modes, commit to
//                          `empty[s]`; after a tile's last step commit to `acc_full[a]`
//   epilogue warps 0..3  : wait `acc_full[a]`, tcgen05.ld their lane quadrant, release the
//                          accumulator (`acc_empty[a]`), combine re / im with shuffles, store 32
//                          contiguous bytes (four modes) per (b, o)
// Accumulators: 4 modes x 2 CO fp32 columns per tile; with CO = 32 two tiles' accumulators alternate.
// Every wait is bounded (about one second of clock cycles): on expiry the kernel records a status
// word (nop_device_status), all roles leave their loops, the issued MMAs are drained (bounded) and
// the tensor memory is freed.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "l2_hints.cuh"
#include "nop_internal.cuh"

namespace nop {
namespace tc {

constexpr int EPI_WARPS = 4;                 // warps 0..3
constexpr int PROD_WARPS = 8;                // warps 4..11
constexpr int MMA_WARP = EPI_WARPS + PROD_WARPS;
constexpr int THREADS = 32 * (MMA_WARP + 1); // 416
constexpr int PROD_THREADS = 32 * PROD_WARPS;
constexpr int MODES = 4;   // modes per tile
constexpr int BT = 64;     // batch rows per tile (A has 2 BT = 128 rows)
constexpr int M = 128;
constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz

// status word written when a bounded wait expires (read by nop_device_status)
constexpr int kStatusMmaTimeout = 1;

template <int CO, bool BF16>
struct Cfg {
    static constexpr int N = 2 * CO;
    static constexpr int KS = BF16 ? 16 : 8;           // K per MMA instruction (32 bytes of K)
    static constexpr int SPLITS = BF16 ? 1 : 2;         // hi / lo operand copies
    static constexpr int A_TILE = M * 32;               // bytes of one mode's A for one K step
    static constexpr int B_TILE = N * 32;
    static constexpr int STAGE = MODES * SPLITS * (A_TILE + B_TILE);
    // raw ring: every producer thread's X / W values of one K step (cp.async, RS steps deep)
    static constexpr int RAWF4 = BF16 ? 16 : 8;          // float4 per producer thread per step
    static constexpr int RAW = PROD_THREADS * RAWF4 * 16;
    static constexpr int RS = BF16 ? 2 : 3;
    static constexpr int NS0 = (226 * 1024 - RS * RAW) / STAGE;
    static constexpr int NS = NS0 > 6 ? 6 : NS0;         // operand stages in the ring
    static constexpr int ACC_COLS = MODES * N;          // tensor-memory columns of one tile
    static constexpr int NACC = ACC_COLS <= 256 ? 2 : 1;
    static constexpr int TMEM_COLS = 512;
    static constexpr int RAW_OFF = NS * STAGE;
    static constexpr int BODY = NS * STAGE + RS * RAW;
    // after the stages: full[NS], empty[NS], acc_full[2], acc_empty[2], drain (8 bytes each), then the
    // tensor-memory address and the abort flag (4 bytes each)
    static constexpr int TAIL = (2 * NS + 5) * 8 + 8;
    static constexpr int SMEM = BODY + 256;
    static_assert(TAIL <= 256, "barrier area overflows its reservation");
    static_assert(NS >= 2, "at least two stages");
    static_assert(ACC_COLS * NACC <= TMEM_COLS, "accumulators exceed tensor memory");
    static_assert(SMEM > 116 * 1024, "one CTA per SM: the whole tensor memory is allocated");
    // instruction descriptor: D f32, A/B tf32 (2) or bf16 (1), both K-major, N >> 3, M >> 4
    static constexpr uint32_t IDESC = (1u << 4) | ((BF16 ? 1u : 2u) << 7) | ((BF16 ? 1u : 2u) << 10) |
                                      ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
};

// byte offset of the 16-byte group (row r, K half kh) inside one operand tile: core matrices of
// 8 rows x 16 bytes stored contiguously; K-adjacent core matrices 128 B apart (LBO), 8-row groups
// 256 B apart (SBO)
__device__ __forceinline__ uint32_t tile_off(int r, int kh) { return (r >> 3) * 256 + kh * 128 + (r & 7) * 16; }

// A row of batch entry b (0..63), real (e = 0) or imaginary (e = 1) part
__device__ __forceinline__ int a_row(int b, int e) { return (b >> 4) * 32 + e * 16 + (b & 15); }

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
           (1ull << 46);
}

__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

// bounded wait for the completion of the phase with parity `parity`; gives up early when `abort`
// (if given) is set.  Each try_wait may suspend the thread until the phase completes, for at most
// kSuspendNs, so a waiting thread costs a few instructions per wake-up rather than a spin loop, and
// the time limit and the abort flag are still checked at least every kSuspendNs.
constexpr uint32_t kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const uint32_t addr = smem_u32(bar);
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity), "r"(kSuspendNs)
            : "memory");
        if (done) return true;
        if ((abort && *abort) || clock64() - t0 > kWaitCycles) return false;
    }
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        :
        : "r"(tmem), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        :
        : "r"(tmem), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 32-byte global load / store (one sector per request)
__device__ __forceinline__ void ldg32B(const void* p, float4& a, float4& b) {
    asm volatile("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=f"(a.x), "=f"(a.y), "=f"(a.z), "=f"(a.w), "=f"(b.x), "=f"(b.y), "=f"(b.z), "=f"(b.w)
                 : "l"(p));
}

__device__ __forceinline__ void stg32B(void* p, const float4& a, const float4& b) {
    asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(a.x), "f"(a.y), "f"(a.z),
                 "f"(a.w), "f"(b.x), "f"(b.y), "f"(b.z), "f"(b.w)
                 : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Tile of the contraction: mode half h of local mode block q, batch rows b0.., output channels o0..
struct Tile {
    int h, b0, o0;
    const float2* Xq;
    const float4* Wq;
    float2* Yq;
};

struct Problem {
    const float2* X;
    const float4* Wp;
    int64_t wq;
    float2* Y;
    int B, Ci, Co;
    int local;  // local mode blocks (< 2^31; the host checks the tile count fits an int)
    int qpl, qtot, qbeg;
    int bt, ot;  // batch tiles, output tiles
};

// decode of tile t (done once per tile; 32-bit divisions).  Order: mode half fastest, then output
// tile, local mode block, batch tile -- the tiles that read the same X run on neighbouring CTAs at
// the same time, so X comes from L2 after its first read.
__device__ __forceinline__ Tile tile_at(const Problem& pr, int t, int co_tile) {
    Tile r;
    r.h = t & 1;
    int rest = t >> 1;
    r.o0 = (rest % pr.ot) * co_tile;
    rest /= pr.ot;
    const int q = rest % pr.local;
    r.b0 = (rest / pr.local) * BT;
    r.Xq = pr.X + (int64_t)q * pr.B * pr.Ci * 8;
    // local mode block q -> weight block (identity unless plane-mode blocks are split across ranks)
    r.Wq = pr.Wp + (int64_t)((q / pr.qpl) * pr.qtot + pr.qbeg + q % pr.qpl) * pr.wq;
    r.Yq = pr.Y + (int64_t)q * pr.B * pr.Co * 8;
    return r;
}

// Producer unit for one K step.  X unit (p < 128): batch row b = p / 2, K half kh = p % 2, all four
// modes.  W unit (128 <= p < 128 + 2 CO): output channel o = u % CO, K half u / CO (u = p - 128).
// A K half is 16 bytes of K: 4 tf32 or 8 bf16 channels; per channel two float4 (four modes, complex).
template <bool BF16>
struct Step {
    static constexpr int KH = BF16 ? 8 : 4;
    float4 v[2 * KH];
};

__device__ __forceinline__ void cp_async16z(void* smem, const void* gmem, bool valid) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem), "r"(valid ? 16 : 0)
                 : "memory");
}

// issue the copies of producer thread p's raw values for one K step into a raw-ring slot
// (layout [value c][thread p] float4, so the threads' later reads are conflict-free); values out of
// range are zero-filled
template <int CO, bool BF16>
__device__ __forceinline__ void issue_step(float4* slot, const Problem& pr, const Tile& tl, int k0, int p,
                                           uint64_t pol) {
    constexpr int KH = Step<BF16>::KH;
    if (p < 128) {
        const int b = p >> 1, kh = p & 1;
        const bool bok = tl.b0 + b < pr.B;
        const float2* src = tl.Xq + ((int64_t)(tl.b0 + b) * pr.Ci + k0 + kh * KH) * 8 + 4 * tl.h;
#pragma unroll
        for (int c = 0; c < KH; ++c) {
            const bool ok = bok && k0 + kh * KH + c < pr.Ci;
            const float2* sc = ok ? src + c * 8 : pr.X;
            l2::cp_async16(slot + (2 * c) * PROD_THREADS + p, sc, ok, pol);
            l2::cp_async16(slot + (2 * c + 1) * PROD_THREADS + p, ok ? sc + 2 : pr.X, ok, pol);
        }
    } else if (p < 128 + 2 * CO) {
        const int u = p - 128;
        const int o = u % CO, kh = u / CO;
        const bool ook = tl.o0 + o < pr.Co;
#pragma unroll
        for (int c = 0; c < KH; ++c) {
            const int i = k0 + kh * KH + c;
            const bool ok = ook && i < pr.Ci;
            const float4* s4 = ok ? tl.Wq + ((int64_t)i * 4 + 2 * tl.h) * pr.Co + tl.o0 + o : pr.Wp;
            l2::cp_async16(slot + (2 * c) * PROD_THREADS + p, s4, ok, pol);
            l2::cp_async16(slot + (2 * c + 1) * PROD_THREADS + p, ok ? s4 + pr.Co : pr.Wp, ok, pol);
        }
    }
}

template <int CO, bool BF16>
__device__ __forceinline__ void store_step(const Step<BF16>& st, char* stage, int p) {
    using C = Cfg<CO, BF16>;
    constexpr int KH = Step<BF16>::KH;
    int rows[2], kh, tile_bytes;
    char* base;
    if (p < 128) {
        rows[0] = a_row(p >> 1, 0);
        rows[1] = a_row(p >> 1, 1);
        kh = p & 1;
        base = stage;
        tile_bytes = C::A_TILE;
    } else if (p < 128 + 2 * CO) {
        const int u = p - 128;
        rows[0] = u % CO;       // columns of Wr
        rows[1] = u % CO + CO;  // columns of Wi
        kh = u / CO;
        base = stage + MODES * C::SPLITS * C::A_TILE;
        tile_bytes = C::B_TILE;
    } else {
        return;
    }
#pragma unroll
    for (int jl = 0; jl < MODES; ++jl) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const uint32_t off = tile_off(rows[e], kh);
            float x[KH];
#pragma unroll
            for (int c = 0; c < KH; ++c) {
                const float4 v = st.v[2 * c + (jl >> 1)];
                x[c] = (jl & 1) ? (e ? v.w : v.z) : (e ? v.y : v.x);
            }
            if constexpr (BF16) {
                uint4 w;
                w.x = pack_bf16(x[0], x[1]);
                w.y = pack_bf16(x[2], x[3]);
                w.z = pack_bf16(x[4], x[5]);
                w.w = pack_bf16(x[6], x[7]);
                *reinterpret_cast<uint4*>(base + jl * tile_bytes + off) = w;
            } else {
                float hi[4], lo[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    hi[c] = tf32_round(x[c]);
                    lo[c] = tf32_round(x[c] - hi[c]);
                }
                *reinterpret_cast<float4*>(base + (jl * 2 + 0) * tile_bytes + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<float4*>(base + (jl * 2 + 1) * tile_bytes + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
    }
}

// Persistent: CTA c takes tiles c, c + gridDim.x, ...; tiles ordered mode half fastest, then local
// mode block, batch tile, output tile.  Global K step g of the CTA = (its tile g / nk, step g % nk).
template <int CO, bool BF16>
// 13 warps: the SM's four register banks hold at most 4 warps each at 128 registers per thread
__global__ void __maxnreg__(128)
k_mix_tc(const float2* __restrict__ X, const float4* __restrict__ Wp, int64_t wq, float2* __restrict__ Y, int B,
         int Ci, int Co, int local, int qpl, int qtot, int qbeg, int* __restrict__ status) {
    using C = Cfg<CO, BF16>;
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

    Problem pr{X, Wp, wq, Y, B, Ci, Co, local, qpl, qtot, qbeg, (B + BT - 1) / BT, (Co + CO - 1) / CO};
    const int tiles = 2 * local * pr.bt * pr.ot;
    const int my_tiles = tiles > (int)blockIdx.x ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nk = (Ci + C::KS - 1) / C::KS;
    auto tile_k = [&](int k) { return tile_at(pr, (int)blockIdx.x + k * (int)gridDim.x, CO); };

    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], PROD_WARPS);  // one arrival per producer warp
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], EPI_WARPS);
        }
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort_flag = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
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
        atomicExch(status, kStatusMmaTimeout);
    };

    if (warp >= EPI_WARPS && warp < MMA_WARP) {
        // ------------------------------ producers ------------------------------
        const int p = tid - 32 * EPI_WARPS;
        const uint64_t pol_in = l2::evict_first();  // spectrum and weights are read once
        // raw ring: the copies of the next RS - 1 steps are in flight (cp.async, no registers held)
        // while this thread converts the current step; each thread reads back only what it copied
        constexpr int RS = C::RS;
        float4* raw = reinterpret_cast<float4*>(smem + C::RAW_OFF);
        constexpr int SLOT_F4 = PROD_THREADS * C::RAWF4;
        int lk = 0, lkc = 0;              // tile and K step of the next copy
        Tile ltile;
        if (my_tiles > 0) ltile = tile_k(0);
        int slot_in = 0, slot_out = 0;
        auto issue_next = [&]() {
            if (lk < my_tiles) {
                issue_step<CO, BF16>(raw + slot_in * SLOT_F4, pr, ltile, lkc * C::KS, p, pol_in);
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
        Step<BF16> cur;
        int s = 0;
        uint32_t upar = 0;                // parity of the current use of stage s
        bool reuse = false;               // stage s held an earlier step
        for (int k = 0; k < my_tiles; ++k) {
            for (int kc = 0; kc < nk; ++kc) {
                issue_next();
                asm volatile("cp.async.wait_group %0;\n" ::"n"(RS - 1) : "memory");
                const float4* mine = raw + slot_out * SLOT_F4 + p;
#pragma unroll
                for (int c = 0; c < C::RAWF4; ++c) cur.v[c] = mine[c * PROD_THREADS];
                if (++slot_out == RS) slot_out = 0;
                if (reuse && !mbar_wait(&empty[s], upar ^ 1, abort_flag)) {
                    give_up();
                    k = my_tiles;
                    break;
                }
                store_step<CO, BF16>(cur, smem + s * C::STAGE, p);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
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
                if (v > 0 && !mbar_wait(&acc_empty[a], (uint32_t)((v - 1) & 1), abort_flag)) {
                    give_up();
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dacc = tmem + a * C::ACC_COLS;
                for (int kc = 0; kc < nk; ++kc) {
                    if (!mbar_wait(&full[s], upar, abort_flag)) {
                        give_up();
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a0 = smem_u32(smem + s * C::STAGE);
                    const uint32_t bq = a0 + MODES * C::SPLITS * C::A_TILE;
#pragma unroll
                    for (int jl = 0; jl < MODES; ++jl) {
                        const uint32_t d = dacc + jl * C::N;
                        if constexpr (BF16) {
                            mma_bf16(d, smem_desc(a0 + jl * C::A_TILE), smem_desc(bq + jl * C::B_TILE), C::IDESC,
                                     kc > 0);
                        } else {
                            const uint64_t ahi = smem_desc(a0 + (jl * 2) * C::A_TILE);
                            const uint64_t alo = smem_desc(a0 + (jl * 2 + 1) * C::A_TILE);
                            const uint64_t bhi = smem_desc(bq + (jl * 2) * C::B_TILE);
                            const uint64_t blo = smem_desc(bq + (jl * 2 + 1) * C::B_TILE);
                            mma_tf32(d, ahi, bhi, C::IDESC, kc > 0);
                            mma_tf32(d, ahi, blo, C::IDESC, 1);
                            mma_tf32(d, alo, bhi, C::IDESC, 1);
                        }
                    }
                    mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
                    if (++s == NS) {
                        s = 0;
                        upar ^= 1;
                    }
                }
                if (!ok) break;
                mma_commit(&acc_full[a]);   // the tile's accumulators are complete
            }
            // drain: every MMA issued so far has finished once this commit lands (also after an
            // abort, so the tensor memory is never freed under a running MMA)
            mma_commit(drain);
            if (!mbar_wait(drain, 0, nullptr)) give_up();
        }
    } else {
        // ------------------------------ epilogue (warps 0..3) ------------------------------
        const int qd = warp;                   // tensor-memory lane quadrant
        const bool im = lane >= 16;            // this lane holds the Xi row of its batch entry
        const int bl = qd * 16 + (lane & 15);  // batch entry within the tile
        const uint64_t pol_out = l2::evict_last();  // the output spectrum is read back by the inverse
        for (int k = 0; k < my_tiles; ++k) {
            const int a = k % NACC;
            if (!mbar_wait(&acc_full[a], (uint32_t)((k / NACC) & 1), abort_flag)) {
                give_up();
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const Tile tl = tile_k(k);
            const uint32_t tbase = tmem + ((uint32_t)(qd * 32) << 16) + a * C::ACC_COLS;
            const bool bok = tl.b0 + bl < B;
            for (int cb = 0; cb < CO; cb += 8) {
                float P[MODES][8], Qv[MODES][8];
#pragma unroll
                for (int jl = 0; jl < MODES; ++jl) {
                    tmem_ld8(tbase + jl * C::N + cb, P[jl]);
                    tmem_ld8(tbase + jl * C::N + CO + cb, Qv[jl]);
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (cb + 8 >= CO) {
                    // accumulators read: the next tile using this buffer may start
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[a]);
                }
                // re lanes finish columns 0..3 of this group, im lanes columns 4..7
                float out[4][2 * MODES];
#pragma unroll
                for (int jl = 0; jl < MODES; ++jl) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float sp = im ? P[jl][c] : P[jl][4 + c];
                        const float sq = im ? Qv[jl][c] : Qv[jl][4 + c];
                        const float rp = __shfl_xor_sync(0xffffffffu, sp, 16);
                        const float rq = __shfl_xor_sync(0xffffffffu, sq, 16);
                        if (!im) {  // own Xr row: P = Xr Wr, Q = Xr Wi; partner: Xi Wr, Xi Wi
                            out[c][2 * jl] = P[jl][c] - rq;
                            out[c][2 * jl + 1] = Qv[jl][c] + rp;
                        } else {    // own Xi row; partner: Xr Wr, Xr Wi of columns 4..7
                            out[c][2 * jl] = rp - Qv[jl][4 + c];
                            out[c][2 * jl + 1] = rq + P[jl][4 + c];
                        }
                    }
                }
                if (bok) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int o = tl.o0 + cb + (im ? 4 : 0) + c;
                        if (o >= Co) continue;
                        l2::st8(tl.Yq + ((int64_t)(tl.b0 + bl) * Co + o) * 8 + 4 * tl.h,
                                make_float4(out[c][0], out[c][1], out[c][2], out[c][3]),
                                make_float4(out[c][4], out[c][5], out[c][6], out[c][7]), pol_out);
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

}  // namespace tc
}  // namespace nop

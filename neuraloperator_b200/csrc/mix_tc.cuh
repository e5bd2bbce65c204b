// Per-mode complex contraction on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   Y[q][b][o][j] = sum_i X[q][b][i][j] W_q[i][o][j]        (complex, mode 8 q + j)
//
// on the mode-blocked spectrum [Q][B][C][8] with weights packed as W_q[i][p][o] = float4(mode 8q+2p,
// mode 8q+2p+1).  One CTA takes four modes (half a mode block), 64 batch entries and CO output
// channels.  For each mode the complex product becomes ONE real GEMM with M = 128, N = 2 CO:
//
//   A = [Xr ; Xi]  (rows 0..63: real parts of the 64 batch rows, rows 64..127: imaginary parts)
//   B = [Wr | Wi]  (columns 0..CO-1: real parts, CO..2CO-1: imaginary parts),  K = input channels
//   D = A B = [[Xr Wr, Xr Wi], [Xi Wr, Xi Wi]]   ->   Yr = D[b][o] - D[64+b][CO+o],
//                                                      Yi = D[b][CO+o] + D[64+b][o].
//
// fp32 accuracy from tf32 operands (three-pass split): every operand x = hi + lo with
// hi = tf32(x), lo = tf32(x - hi), and D = A_hi B_hi + A_hi B_lo + A_lo B_hi (the dropped lo*lo term
// is below 2^-22 relative), accumulated in fp32 in tensor memory.  With the bf16 contraction the
// operands are rounded to bf16 and one kind::f16 MMA per K step replaces the three tf32 ones.
//
// Pipeline per CTA (256 threads, one CTA per SM): the K loop runs over 8 input channels (tf32) or
// 16 (bf16) at a time.  All threads load the next step's X and W into registers while the current
// step is converted and stored into a shared-memory stage in the canonical no-swizzle K-major layout
// (8-row x 16-byte core matrices); thread 0 issues the MMAs for the four modes and commits them to
// the stage's mbarrier, which the threads wait on before they overwrite that stage two steps later.
// The four modes' accumulators (4 x 2 CO fp32 columns) live in tensor memory for the whole K loop.
// Epilogue: tensor memory -> registers (tcgen05.ld) -> padded shared memory -> combined complex
// outputs, 32 contiguous bytes (four modes) per (b, o).
//
// Every wait is bounded (about one second of clock cycles): on expiry the kernel records a status
// word (nop_device_status), stops issuing, waits (bounded) for its MMAs and frees its tensor memory.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "nop_internal.cuh"

namespace nop {
namespace tc {

constexpr int THREADS = 256;
constexpr int MODES = 4;   // modes per CTA
constexpr int BT = 64;     // batch rows per CTA (A has 2 BT = 128 rows)
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
    static constexpr int DUMP_PITCH = 33;               // floats per dumped row (32 columns + pad)
    static constexpr int DUMP = MODES * M * DUMP_PITCH * 4;
    static constexpr int TMEM_COLS = MODES * N;         // 256 or 512
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "tensor-memory allocation must be a power of 2");
    // a CTA holding all 512 columns must be alone on its SM (more than half the shared memory), so
    // that no second CTA blocks in tcgen05.alloc; two 256-column CTAs share an SM
    static constexpr int MIN_BODY = TMEM_COLS == 512 ? 117 * 1024 : 0;
    static constexpr int BODY0 = 2 * STAGE > DUMP ? 2 * STAGE : DUMP;
    static constexpr int BODY = BODY0 > MIN_BODY ? BODY0 : MIN_BODY;
    static constexpr int SMEM = BODY + 64;              // + two mbarriers + tensor-memory address
    // instruction descriptor: D f32, A/B tf32 (2) or bf16 (1), both K-major, N >> 3, M >> 4
    static constexpr uint32_t IDESC = (1u << 4) | ((BF16 ? 1u : 2u) << 7) | ((BF16 ? 1u : 2u) << 10) |
                                      ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
};

// byte offset of the 16-byte group (row r, K half kh) inside one operand tile: core matrices of
// 8 rows x 16 bytes stored contiguously; K-adjacent core matrices 128 B apart (LBO), 8-row groups
// 256 B apart (SBO)
__device__ __forceinline__ uint32_t tile_off(int r, int kh) { return (r >> 3) * 256 + kh * 128 + (r & 7) * 16; }

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

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if (clock64() - t0 > kWaitCycles) return false;
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Operand staging for one K step.  X unit (thread t < 128): batch row b = t / 2, K quarter kq = t % 2
// (tf32: 4 channels = 16 bytes; bf16: 8 channels = 16 bytes), all four modes.  W unit
// (128 <= t < 128 + 2 CO): output channel o = (t - 128) % CO, K quarter (t - 128) / CO.
template <int CO, bool BF16>
struct Step {
    static constexpr int KQ = BF16 ? 8 : 4;  // channels per unit
    float4 v[BF16 ? 16 : 8];                 // [channel][mode pair] raw complex values
};

template <int CO, bool BF16>
__device__ __forceinline__ void load_step(Step<CO, BF16>& st, const float2* __restrict__ Xq,
                                          const float4* __restrict__ Wq, int B, int Ci, int Co, int b0, int o0, int h,
                                          int k0) {
    constexpr int KQ = Step<CO, BF16>::KQ;
    const int t = threadIdx.x;
    if (t < 128) {
        const int b = t >> 1, kq = t & 1;
        const bool bok = b0 + b < B;
#pragma unroll
        for (int c = 0; c < KQ; ++c) {
            const int i = k0 + kq * KQ + c;
            const bool ok = bok && i < Ci;
            const float4* src = reinterpret_cast<const float4*>(Xq + ((int64_t)(b0 + b) * Ci + i) * 8 + 4 * h);
            st.v[2 * c] = ok ? __ldg(src) : make_float4(0.f, 0.f, 0.f, 0.f);
            st.v[2 * c + 1] = ok ? __ldg(src + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    } else if (t < 128 + 2 * CO) {
        const int o = (t - 128) % CO, kq = (t - 128) / CO;
        const bool ook = o0 + o < Co;
#pragma unroll
        for (int c = 0; c < KQ; ++c) {
            const int i = k0 + kq * KQ + c;
            const bool ok = ook && i < Ci;
#pragma unroll
            for (int pp = 0; pp < 2; ++pp) {
                const float4* src = Wq + ((int64_t)i * 4 + 2 * h + pp) * Co + o0 + o;
                st.v[2 * c + pp] = ok ? __ldg(src) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
}

// component e (0: re, 1: im) of local mode jl from a unit's raw values for channel c
template <int CO, bool BF16>
__device__ __forceinline__ float comp(const Step<CO, BF16>& st, int c, int jl, int e) {
    const float4 v = st.v[2 * c + (jl >> 1)];
    return (jl & 1) ? (e ? v.w : v.z) : (e ? v.y : v.x);
}

template <int CO, bool BF16>
__device__ __forceinline__ void store_step(const Step<CO, BF16>& st, char* stage) {
    using C = Cfg<CO, BF16>;
    const int t = threadIdx.x;
    char* a_base = stage;                                          // [mode][split] A tiles
    char* b_base = stage + MODES * C::SPLITS * C::A_TILE;          // [mode][split] B tiles
    int row[2], kq;
    char* base;
    int tile_bytes;
    if (t < 128) {
        row[0] = t >> 1;          // real parts
        row[1] = (t >> 1) + BT;   // imaginary parts
        kq = t & 1;
        base = a_base;
        tile_bytes = C::A_TILE;
    } else if (t < 128 + 2 * CO) {
        row[0] = (t - 128) % CO;        // columns of Wr
        row[1] = (t - 128) % CO + CO;   // columns of Wi
        kq = (t - 128) / CO;
        base = b_base;
        tile_bytes = C::B_TILE;
    } else {
        return;
    }
#pragma unroll
    for (int jl = 0; jl < MODES; ++jl) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const uint32_t off = tile_off(row[e], kq);
            if constexpr (BF16) {
                uint4 w;
                w.x = pack_bf16(comp(st, 0, jl, e), comp(st, 1, jl, e));
                w.y = pack_bf16(comp(st, 2, jl, e), comp(st, 3, jl, e));
                w.z = pack_bf16(comp(st, 4, jl, e), comp(st, 5, jl, e));
                w.w = pack_bf16(comp(st, 6, jl, e), comp(st, 7, jl, e));
                *reinterpret_cast<uint4*>(base + jl * tile_bytes + off) = w;
            } else {
                float hi[4], lo[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float x = comp(st, c, jl, e);
                    hi[c] = tf32_round(x);
                    lo[c] = tf32_round(x - hi[c]);
                }
                *reinterpret_cast<float4*>(base + (jl * 2 + 0) * tile_bytes + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<float4*>(base + (jl * 2 + 1) * tile_bytes + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
    }
}

// grid: x = 2 * local mode blocks (mode half fastest), y = batch tiles of 64, z = output tiles of CO
template <int CO, bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
k_mix_tc(const float2* __restrict__ X, const float4* __restrict__ Wp, int64_t wq, float2* __restrict__ Y, int B,
         int Ci, int Co, int qpl, int qtot, int qbeg, int* __restrict__ status) {
    using C = Cfg<CO, BF16>;
    extern __shared__ __align__(1024) char smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BODY);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::BODY + 16);
    int* abort_flag = reinterpret_cast<int*>(smem + C::BODY + 20);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int h = blockIdx.x & 1;
    const int64_t q = blockIdx.x >> 1;
    const int b0 = blockIdx.y * BT;
    const int o0 = blockIdx.z * CO;
    const float2* Xq = X + q * (int64_t)B * Ci * 8;
    const float4* Wq = Wp + ((q / qpl) * qtot + qbeg + q % qpl) * wq;
    const int nk = (Ci + C::KS - 1) / C::KS;

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[0])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[1])) : "memory");
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

    Step<CO, BF16> cur, nxt;
    load_step<CO, BF16>(cur, Xq, Wq, B, Ci, Co, b0, o0, h, 0);
    bool aborted = false;
    int issued = 0;  // K steps whose MMAs were committed
    for (int kc = 0; kc < nk; ++kc) {
        if (kc + 1 < nk) load_step<CO, BF16>(nxt, Xq, Wq, B, Ci, Co, b0, o0, h, (kc + 1) * C::KS);
        const int s = kc & 1;
        char* stage = smem + s * C::STAGE;
        if (kc >= 2 && !mbar_wait(smem_u32(&bars[s]), ((kc >> 1) - 1) & 1)) *abort_flag = 1;
        store_step<CO, BF16>(cur, stage);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (*abort_flag) {
            aborted = true;
            break;
        }
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = smem_u32(stage);
            const uint32_t bq = a0 + MODES * C::SPLITS * C::A_TILE;
#pragma unroll
            for (int jl = 0; jl < MODES; ++jl) {
                const uint32_t d = tmem + jl * C::N;
                if constexpr (BF16) {
                    mma_bf16(d, smem_desc(a0 + jl * C::A_TILE), smem_desc(bq + jl * C::B_TILE), C::IDESC, kc > 0);
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
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&bars[s]))
                         : "memory");
        }
        issued = kc + 1;
        if (kc + 1 < nk) cur = nxt;
    }
    // every committed MMA has finished once the last commit's phase completes
    bool ok = true;
    if (issued > 0) {
        const int kl = issued - 1;
        ok = mbar_wait(smem_u32(&bars[kl & 1]), (kl >> 1) & 1);
    }
    const int bad = __syncthreads_or(!ok || aborted);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (bad && tid == 0) atomicExch(status, kStatusMmaTimeout);

    if (!bad) {
        // ---- epilogue: 16 output channels per pass; warpgroup g dumps modes 2g, 2g+1 ----
        float* dump = reinterpret_cast<float*>(smem);
        const int lane_base = (warp & 3) * 32;
        const int row = lane_base + (tid & 31);
        const int g = warp >> 2;
        float2* Yq = Y + q * (int64_t)B * Co * 8;
        for (int ob = 0; ob < CO; ob += 16) {
#pragma unroll
            for (int mm = 0; mm < 2; ++mm) {
                const int jl = 2 * g + mm;
                float pv[16], qv[16];
                const uint32_t ta = tmem + ((uint32_t)lane_base << 16) + jl * C::N + ob;
                tmem_ld16(ta, pv);
                tmem_ld16(ta + CO, qv);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                float* drow = dump + ((size_t)jl * M + row) * C::DUMP_PITCH;
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    drow[c] = pv[c];
                    drow[16 + c] = qv[c];
                }
            }
            __syncthreads();
            for (int e = tid; e < BT * 16; e += THREADS) {
                const int b = e >> 4, oo = e & 15;
                const int o = o0 + ob + oo;
                if (b0 + b >= B || o >= Co) continue;
                float out[8];
#pragma unroll
                for (int jl = 0; jl < MODES; ++jl) {
                    const float* top = dump + ((size_t)jl * M + b) * C::DUMP_PITCH;
                    const float* bot = dump + ((size_t)jl * M + BT + b) * C::DUMP_PITCH;
                    out[2 * jl] = top[oo] - bot[16 + oo];      // Xr Wr - Xi Wi
                    out[2 * jl + 1] = top[16 + oo] + bot[oo];  // Xr Wi + Xi Wr
                }
                float4* dst = reinterpret_cast<float4*>(Yq + ((int64_t)(b0 + b) * Co + o) * 8 + 4 * h);
                dst[0] = make_float4(out[0], out[1], out[2], out[3]);
                dst[1] = make_float4(out[4], out[5], out[6], out[7]);
            }
            __syncthreads();
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
}

}  // namespace tc
}  // namespace nop

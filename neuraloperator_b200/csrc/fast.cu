// Fused FFT engine.
//
// 2D (square N x N grids, N in {128, 256, 512}), real data, n_out == n_in:
//   k_plane_fwd  : one CTA per (batch, channel) plane.  Row transforms (two real rows packed as one
//                  complex line) keep rFFT bins 0..Kx-1 in a shared-memory column store; column
//                  transforms keep the My bins (m - off) mod N.  Only the kept modes reach HBM.
//   k_mix        : per-mode complex contraction on the mode-blocked spectrum [Q][B][C][8]
//                  (modes in blocks of 8), weights pre-packed once per weight version; Tucker
//                  weights run as three such contractions (input factor, core, output factor).
//   k_plane_inv  : column inverses of the kept modes, then row inverses (two real rows per complex
//                  line) with the epilogue bias (+ skip) (+ GELU) fused into the final pass.
// Other shapes fall back to the generic engine (plan-time decision).
#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "fft_core.cuh"
#include "nop_internal.cuh"
#include "axis.cuh"
#include "plane256.cuh"
#include "plane512.cuh"
#include "row1d.cuh"
#include "mix_tc.cuh"
#include "mix_tma.cuh"

namespace nop {
namespace {

using fft::LineShape;
using fft::pad;

template <int N>
struct PlaneCfg {
    static constexpr int THREADS = N >= 512 ? 512 : 256;
    static constexpr int G = LineShape<N>::G;
    static constexpr int GROUPS = THREADS / G;
    static constexpr int LINE = LineShape<N>::BUF;
    static constexpr int TPITCH = LINE + 1;  // odd pitch (in float2) for the column store
    static constexpr int MIN_BLOCKS = N >= 512 ? 1 : 2;
};

template <int N>
size_t plane_smem_bytes(int Kx, int My) {
    using C = PlaneCfg<N>;
    size_t x = (size_t)C::GROUPS * C::LINE;
    size_t stage = (size_t)My * Kx;
    return sizeof(float2) * ((size_t)N + (size_t)Kx * C::TPITCH + (x > stage ? x : stage));
}

// ------------------------------------------------------------------------------------------
// forward plane transform: x [L, N, N] real  ->  out [L, My, Kx] complex (kept modes only)
// ------------------------------------------------------------------------------------------
template <int N>
__global__ void __launch_bounds__(PlaneCfg<N>::THREADS, PlaneCfg<N>::MIN_BLOCKS)
k_plane_fwd(const float* __restrict__ x, float2* __restrict__ out, const float2* __restrict__ twg, int Kx, int My,
            int off_y, float scale, int64_t blk_stride) {
    using C = PlaneCfg<N>;
    extern __shared__ float2 smem[];
    float2* tw = smem;
    float2* T = tw + N;                    // column store: T[c * TPITCH + pad(row)]
    float2* X = T + (size_t)Kx * C::TPITCH;  // per-group line buffers, later the output stage
    const int64_t plane = blockIdx.x;
    const int g = threadIdx.x / C::G;
    const int t = threadIdx.x % C::G;
    const float* xp = x + plane * (int64_t)N * N;
    float2* buf = X + g * C::LINE;
    // ---- rows: pair (2p, 2p+1) -> z = a + i b, keep bins k < Kx and their mirrors ----
    // The next pair's loads are issued before the current pair is transformed (the first pair's
    // before the twiddle table is staged).
    float2 nxt[16];
    auto load_pair = [&](int pr) {
        const float* ra = xp + (int64_t)(2 * pr) * N + t;
#pragma unroll
        for (int r = 0; r < 16; ++r) nxt[r] = make_float2(__ldg(ra + r * C::G), __ldg(ra + N + r * C::G));
    };
    if (g < N / 2) load_pair(g);
    for (int i = threadIdx.x; i < N; i += C::THREADS) tw[i] = twg[i];
    __syncthreads();
    for (int base = 0; base < N / 2; base += C::GROUPS) {
        const int pr = base + g;
        const bool active = pr < N / 2;
        float2 v[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) v[r] = active ? nxt[r] : make_float2(0.f, 0.f);
        if (pr + C::GROUPS < N / 2) load_pair(pr + C::GROUPS);
        fft::line_fft_regs<N, false>(v, buf, tw, t, active, [&](int k, float2 w) {
            if (k < Kx || k > N - Kx) buf[pad(k)] = w;
        });
        __syncwarp();
        if (active) {
            for (int k = t; k < Kx; k += C::G) {
                float2 zk = buf[pad(k)];
                float2 zn = buf[pad((N - k) & (N - 1))];
                float2 A = make_float2(0.5f * (zk.x + zn.x), 0.5f * (zk.y - zn.y));
                float2 B = make_float2(0.5f * (zk.y + zn.y), 0.5f * (zn.x - zk.x));
                T[k * C::TPITCH + pad(2 * pr)] = A;
                T[k * C::TPITCH + pad(2 * pr + 1)] = B;
            }
        }
        __syncwarp();
    }
    __syncthreads();
    // ---- columns: complex transform along y, keep My bins (m - off_y) mod N ----
    float2* stage = X;
    const int warp_first_group = (threadIdx.x & ~31) / C::G;
    for (int base = 0; base < Kx; base += C::GROUPS) {
        if (base + warp_first_group >= Kx) break;  // warp-uniform: no column left for this warp
        const int c = base + g;
        const bool active = c < Kx;
        float2* col = T + (active ? c : 0) * C::TPITCH;
        fft::line_fft<N, false>(
            col, tw, t, active,
            [&](int i) { return active ? col[pad(i)] : make_float2(0.f, 0.f); },
            [&](int k, float2 v) {
                const int m = (k + off_y) & (N - 1);
                if (active && m < My) stage[m * Kx + c] = fft::cscale(v, scale);
            });
    }
    __syncthreads();
    // kept modes -> mode-blocked spectrum [Q][L][8] (zero padding beyond Mt)
    const int Mt = My * Kx;
    const int Q = (Mt + 7) >> 3;
    float2* op = out + plane * 8;
    for (int e = threadIdx.x; e < Q * 4; e += C::THREADS) {
        const int q = e >> 2, m = 8 * q + 2 * (e & 3);
        const float2 a = m < Mt ? stage[m] : make_float2(0.f, 0.f);
        const float2 b = m + 1 < Mt ? stage[m + 1] : make_float2(0.f, 0.f);
        *reinterpret_cast<float4*>(op + q * blk_stride + 2 * (e & 3)) = make_float4(a.x, a.y, b.x, b.y);
    }
}

// ------------------------------------------------------------------------------------------
// inverse plane transform: in [L, My, Kx] complex -> y [L, N, N] real, with epilogue
// ------------------------------------------------------------------------------------------
struct Epilogue {
    const float* bias;    // [C] or null
    const float* addend;  // [L, N, N] or null
    int apply_gelu;
    int C;                // channels
    int64_t chan_div;     // planes per channel index step (1 for 2D; Nx for 3D planes)
    int z0, z1, z2;       // last-axis bins read as real
};

template <int N>
__global__ void __launch_bounds__(PlaneCfg<N>::THREADS, PlaneCfg<N>::MIN_BLOCKS)
k_plane_inv(const float2* __restrict__ in, float* __restrict__ y, const float2* __restrict__ twg, int Kx, int My,
            int off_y, float scale, int64_t blk_stride, Epilogue ep) {
    using C = PlaneCfg<N>;
    extern __shared__ float2 smem[];
    float2* tw = smem;
    float2* T = tw + N;
    float2* X = T + (size_t)Kx * C::TPITCH;
    const int64_t plane = blockIdx.x;
    const int g = threadIdx.x / C::G;
    const int t = threadIdx.x % C::G;
    for (int i = threadIdx.x; i < N; i += C::THREADS) tw[i] = twg[i];
    float2* stage = X;
    {  // mode-blocked spectrum [Q][L][8] -> kept modes of this plane
        const int Mt = My * Kx;
        const int Q = (Mt + 7) >> 3;
        const float2* ip = in + plane * 8;
        for (int e = threadIdx.x; e < Q * 4; e += C::THREADS) {
            const int q = e >> 2, m = 8 * q + 2 * (e & 3);
            const float4 v = __ldg(reinterpret_cast<const float4*>(ip + q * blk_stride + 2 * (e & 3)));
            if (m < Mt) stage[m] = make_float2(v.x, v.y);
            if (m + 1 < Mt) stage[m + 1] = make_float2(v.z, v.w);
        }
    }
    __syncthreads();
    // ---- columns: kept bins -> full y lines in the column store ----
    const int warp_first_group = (threadIdx.x & ~31) / C::G;
    for (int base = 0; base < Kx; base += C::GROUPS) {
        if (base + warp_first_group >= Kx) break;  // warp-uniform: no column left for this warp
        const int c = base + g;
        const bool active = c < Kx;
        float2* col = T + (active ? c : 0) * C::TPITCH;
        fft::line_fft<N, true>(
            col, tw, t, active,
            [&](int i) {
                const int m = (i + off_y) & (N - 1);
                return (active && m < My) ? stage[m * Kx + c] : make_float2(0.f, 0.f);
            },
            [&](int k, float2 v) {
                if (active) col[pad(k)] = v;
            });
    }
    __syncthreads();
    // ---- rows: Z = A + iB (bins < Kx), mirrors conj(A) + i conj(B); inverse; epilogue ----
    const float bias = ep.bias ? ep.bias[(plane / ep.chan_div) % ep.C] : 0.f;
    float* yp = y + plane * (int64_t)N * N;
    const float* ap = ep.addend ? ep.addend + plane * (int64_t)N * N : nullptr;
    float2* buf = X + g * C::LINE;
    for (int base = 0; base < N / 2; base += C::GROUPS) {
        const int pr = base + g;
        const bool active = pr < N / 2;
        const int na = 2 * pr, nb = 2 * pr + 1;
        fft::line_fft<N, true>(
            buf, tw, t, active,
            [&](int i) -> float2 {
                if (!active) return make_float2(0.f, 0.f);
                int k;
                bool mirror;
                if (i < Kx) {
                    k = i;
                    mirror = false;
                } else if (N - i < Kx && 2 * i > N) {
                    k = N - i;
                    mirror = true;
                } else {
                    return make_float2(0.f, 0.f);
                }
                float2 A = T[k * C::TPITCH + pad(na)];
                float2 B = T[k * C::TPITCH + pad(nb)];
                if (k == ep.z0 || k == ep.z1 || k == ep.z2) {
                    A.y = 0.f;
                    B.y = 0.f;
                }
                return mirror ? make_float2(A.x + B.y, B.x - A.y) : make_float2(A.x - B.y, A.y + B.x);
            },
            [&](int n, float2 v) {
                if (!active) return;
                float va = v.x * scale + bias;
                float vb = v.y * scale + bias;
                if (ap) {
                    va += __ldg(ap + (int64_t)na * N + n);
                    vb += __ldg(ap + (int64_t)nb * N + n);
                }
                if (ep.apply_gelu) {
                    va = gelu_erf(va);
                    vb = gelu_erf(vb);
                }
                yp[(int64_t)na * N + n] = va;
                yp[(int64_t)nb * N + n] = vb;
            });
    }
}

// ------------------------------------------------------------------------------------------
// per-mode contraction on the mode-blocked spectrum
//   Y[q][b][o][j] = sum_i X[q][b][i][j] W_q[i][o][8 q + j]      (j < 8: mode 8 q + j)
// Packed weights: W_q[i][p][o] = float4(mode 8q+2p, mode 8q+2p+1), q stride `wq` float4 (0 when
// the weight is the same for every mode).  CTA tile: one mode block x 16 batch x 64 out; the Ci
// loop runs in chunks of 8 with cp.async double buffering.  Thread (og, mp, bg): o = o0 + og + 16 j,
// modes 2 mp, 2 mp + 1, batch b0 + 4 bg + {0..3}.
// ------------------------------------------------------------------------------------------
constexpr int kMixThreads = 256;
constexpr int kMixKC = 8;
constexpr int kMixXs = kMixKC * 16 * 8;   // float2 per X stage
constexpr int kMixWs = kMixKC * 4 * 64;   // float4 per W stage
constexpr size_t kMixSmem = 2 * (kMixXs * sizeof(float2) + kMixWs * sizeof(float4));

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ float4 bf16x4(float4 v) {
    return make_float4(round_bf16(v.x), round_bf16(v.y), round_bf16(v.z), round_bf16(v.w));
}

template <bool BF16>
__global__ void __launch_bounds__(kMixThreads, 2)
k_mix(const float2* __restrict__ X, const float4* __restrict__ Wp, int64_t wq, float2* __restrict__ Y, int B, int Ci,
      int Co, int qpl, int qtot, int qbeg) {
    extern __shared__ float4 mix_smem[];
    float4* Ws = mix_smem;                                          // [2][KC][4][64]
    float2* Xs = reinterpret_cast<float2*>(mix_smem + 2 * kMixWs);  // [2][KC][16][8]
    const int tid = threadIdx.x;
    const int og = tid & 15, mp = (tid >> 4) & 3, bg = tid >> 6;
    const int64_t q = blockIdx.x;
    const int b0 = blockIdx.y * 16;
    const int o0 = blockIdx.z * 64;
    const float2* Xq = X + q * (int64_t)B * Ci * 8;
    // local mode block q -> weight block: (q / qpl) * qtot + qbeg + q mod qpl (identity unless the
    // plane-mode blocks are split across ranks)
    const float4* Wq = Wp + ((q / qpl) * qtot + qbeg + q % qpl) * wq;
    const int nchunks = (Ci + kMixKC - 1) / kMixKC;

    auto load_chunk = [&](int c, int buf) {
        const int i0 = c * kMixKC;
        float2* xs = Xs + buf * kMixXs;
        for (int e = tid; e < kMixKC * 16 * 4; e += kMixThreads) {  // 16-byte pieces of X
            const int piece = e & 3, i = (e >> 2) % kMixKC, b = (e >> 2) / kMixKC;
            const bool ok = b0 + b < B && i0 + i < Ci;
            const float2* src = ok ? Xq + ((int64_t)(b0 + b) * Ci + i0 + i) * 8 + 2 * piece : Xq;
            cp_async16(xs + (i * 16 + b) * 8 + 2 * piece, src, ok);
        }
        float4* ws = Ws + buf * kMixWs;
        for (int e = tid; e < kMixWs; e += kMixThreads) {
            const int o = e & 63, p = (e >> 6) & 3, i = e >> 8;
            const bool ok = i0 + i < Ci && o0 + o < Co;
            const float4* src = ok ? Wq + ((int64_t)(i0 + i) * 4 + p) * Co + o0 + o : Wq;
            cp_async16(ws + (i * 4 + p) * 64 + o, src, ok);
        }
        cp_async_commit();
    };

    float2 acc[4][4][2];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[a][j][0] = acc[a][j][1] = make_float2(0.f, 0.f);

    load_chunk(0, 0);
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) {
            load_chunk(c + 1, (c + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float2* xs = Xs + (c & 1) * kMixXs;
        const float4* ws = Ws + (c & 1) * kMixWs;
#pragma unroll 2
        for (int i = 0; i < kMixKC; ++i) {
            float4 xv[4], wv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) xv[a] = *reinterpret_cast<const float4*>(xs + (i * 16 + 4 * bg + a) * 8 + 2 * mp);
#pragma unroll
            for (int j = 0; j < 4; ++j) wv[j] = ws[(i * 4 + mp) * 64 + og + 16 * j];
            if constexpr (BF16) {
#pragma unroll
                for (int a = 0; a < 4; ++a) xv[a] = bf16x4(xv[a]);
#pragma unroll
                for (int j = 0; j < 4; ++j) wv[j] = bf16x4(wv[j]);
            }
#pragma unroll
            for (int a = 0; a < 4; ++a) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2& c0 = acc[a][j][0];
                    c0.x = fmaf(xv[a].x, wv[j].x, c0.x);
                    c0.x = fmaf(-xv[a].y, wv[j].y, c0.x);
                    c0.y = fmaf(xv[a].x, wv[j].y, c0.y);
                    c0.y = fmaf(xv[a].y, wv[j].x, c0.y);
                    float2& c1 = acc[a][j][1];
                    c1.x = fmaf(xv[a].z, wv[j].z, c1.x);
                    c1.x = fmaf(-xv[a].w, wv[j].w, c1.x);
                    c1.y = fmaf(xv[a].z, wv[j].w, c1.y);
                    c1.y = fmaf(xv[a].w, wv[j].z, c1.y);
                }
            }
        }
        __syncthreads();
    }
    float2* Yq = Y + q * (int64_t)B * Co * 8;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int b = b0 + 4 * bg + a;
        if (b >= B) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int o = o0 + og + 16 * j;
            if (o >= Co) continue;
            *reinterpret_cast<float4*>(Yq + ((int64_t)b * Co + o) * 8 + 2 * mp) =
                make_float4(acc[a][j][0].x, acc[a][j][0].y, acc[a][j][1].x, acc[a][j][1].y);
        }
    }
}

// ------------------------------------------------------------------------------------------
// weight packing (weight-only work, redone when the weights change)
// ------------------------------------------------------------------------------------------
// per-mode weight, element (i, o, m) at W[i * s_i + o * s_o + m]  ->  [Q][I][4][O] float4
__global__ void k_pack_modes(const float2* __restrict__ W, float4* __restrict__ Wp, int I, int O, int64_t Mt,
                             int64_t Q, int64_t s_i, int64_t s_o, int conj = 0) {
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= Q * I * 4 * O) return;
    const int o = (int)(idx % O);
    const int p = (int)((idx / O) & 3);
    const int i = (int)((idx / (4 * (int64_t)O)) % I);
    const int64_t q = idx / (4 * (int64_t)O * I);
    const int64_t m = 8 * q + 2 * p;
    const float2* src = W + i * s_i + o * s_o;
    const float2 a = m < Mt ? src[m] : make_float2(0.f, 0.f);
    const float2 b = m + 1 < Mt ? src[m + 1] : make_float2(0.f, 0.f);
    Wp[idx] = conj ? make_float4(a.x, -a.y, b.x, -b.y) : make_float4(a.x, a.y, b.x, b.y);
}

// mode-independent weight, element (i, o) at U[i * s_i + o * s_o]  ->  [I][4][O] float4
__global__ void k_pack_broadcast(const float2* __restrict__ U, float4* __restrict__ Up, int I, int O, int64_t s_i,
                                 int64_t s_o) {
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= (int64_t)I * 4 * O) return;
    const int o = (int)(idx % O);
    const int i = (int)(idx / (4 * (int64_t)O));
    const float2 v = U[i * s_i + o * s_o];
    Up[idx] = make_float4(v.x, v.y, v.x, v.y);
}

constexpr size_t kSmemLimit = 227 * 1024;

// per-device "dynamic shared memory limit raised" bits, one word per kernel instantiation
std::atomic<uint64_t> g_attr_done[32];

template <class K>
cudaError_t ensure_smem_attr(K kernel, int slot, int device, size_t bytes = kSmemLimit) {
    const uint64_t bit = uint64_t(1) << (device & 63);
    if (g_attr_done[slot].load() & bit) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) g_attr_done[slot].fetch_or(bit);
    return e;
}

inline size_t up256(size_t v) { return (v + 255) / 256 * 256; }
inline int64_t mode_blocks(const Plan& p) { return (p.modes_total + 7) / 8; }

// mode blocks this rank contracts and their position in the packed weights
struct BlockMap {
    int64_t local;   // mode blocks in the local spectrum
    int qpl, qtot, qbeg;
};

BlockMap block_map(const Plan& p) {
    const int64_t Q = mode_blocks(p);
    if (p.fast_kind != FastKind::Vol3DSlab) return {Q, (int)Q, (int)Q, 0};
    const int mx = (int)p.d.kept[0];
    const int qtot = (int)(Q / mx);
    return {(int64_t)mx * p.slab_qcount[p.slab_rank], (int)p.slab_qcount[p.slab_rank], qtot,
            (int)p.slab_qbegin[p.slab_rank]};
}

// status word of the tensor-core kernels (bounded waits that expired), per device
__device__ int g_device_status;

int* device_status_ptr(int device) {
    static std::atomic<int*> ptrs[64];
    int* ptr = ptrs[device & 63].load();
    if (!ptr) {
        void* addr = nullptr;
        if (cudaGetSymbolAddress(&addr, g_device_status) != cudaSuccess) return nullptr;
        ptr = static_cast<int*>(addr);
        ptrs[device & 63].store(ptr);
    }
    return ptr;
}

template <int CO, bool BF16>
cudaError_t launch_mix_tc(const Plan& p, const BlockMap& bm, const float2* X, const float4* W, int64_t wq, float2* Y,
                          int Ci, int Co, int slot, cudaStream_t s) {
    using C = tc::Cfg<CO, BF16>;
    cudaError_t err = ensure_smem_attr(tc::k_mix_tc<CO, BF16>, slot, p.device, C::SMEM);
    if (err != cudaSuccess) return err;
    int* status = device_status_ptr(p.device);
    if (!status) return cudaErrorInvalidSymbol;
    const int64_t tiles = 2 * bm.local * ceil_div(p.d.batch, tc::BT) * ceil_div(Co, CO);  // 2 mode halves per block
    if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;  // tile indices are 32-bit
    const unsigned grid = (unsigned)(tiles < p.sm_count ? tiles : p.sm_count);  // persistent, one CTA per SM
    tc::k_mix_tc<CO, BF16><<<grid, tc::THREADS, C::SMEM, s>>>(X, W, wq, Y, (int)p.d.batch, Ci, Co, (int)bm.local,
                                                              bm.qpl, bm.qtot, bm.qbeg, status);
    return cudaGetLastError();
}

// cuTensorMapEncodeTiled, looked up once through the runtime (no link against the driver library)
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled() {
    static const EncodeTiled fn = []() -> EncodeTiled {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<EncodeTiled>(f);
    }();
    return fn;
}

// Geometry of the pre-split weight tiles of one contraction (I input, O output channels; Qw weight
// blocks and H = 4 mode pairs each, or Qw = H = 1 for a matrix shared by every block): see
// tma_mix::tc_tile.  Output tiles of 64 channels unless the channels fit 32.
struct TcGeom {
    int co, ot, nk;
    bool bf16;
    int64_t bytes;
};

TcGeom tc_geom(const Plan& p, int64_t I, int64_t O, int64_t Qw, int H) {
    TcGeom g;
    g.co = O > 32 ? 64 : 32;
    g.bf16 = p.d.precision == NOP_PRECISION_BF16;
    g.ot = (int)ceil_div(O, g.co);
    g.nk = (int)ceil_div(I, g.bf16 ? 16 : 8);
    g.bytes = Qw * H * g.ot * g.nk * tma_mix::TM * (g.bf16 ? 1 : 2) * (2 * g.co * 32);
    return g;
}

// weight element (i, o, m) at W[i * s_i + o * s_o + m * s_m] (s_m = 0: shared by every block)
cudaError_t pack_tc(const Plan& p, const float2* W, char* out, int64_t I, int64_t O, int64_t Qw, int H, int64_t s_i,
                    int64_t s_o, int64_t s_m, int conj, cudaStream_t s) {
    const TcGeom g = tc_geom(p, I, O, Qw, H);
    const int64_t n = Qw * H * g.ot * g.nk * tma_mix::TM * 2 * g.co * 2;
    const unsigned grid = (unsigned)ceil_div(n, 256);
    const int64_t Mt = p.modes_total;
    if (H == 4 && s_m == 1) {  // per-block weights with contiguous modes: coalesced 64-byte reads
        const unsigned blocks = (unsigned)(Qw * g.ot * g.nk);
        if (g.co == 64) {
            if (g.bf16)
                tma_mix::k_pack_tc_block<64, true><<<blocks, 256, 0, s>>>(W, out, (int)I, (int)O, Mt, g.ot, g.nk, s_i,
                                                                          s_o, conj);
            else
                tma_mix::k_pack_tc_block<64, false><<<blocks, 256, 0, s>>>(W, out, (int)I, (int)O, Mt, g.ot, g.nk,
                                                                           s_i, s_o, conj);
        } else {
            if (g.bf16)
                tma_mix::k_pack_tc_block<32, true><<<blocks, 256, 0, s>>>(W, out, (int)I, (int)O, Mt, g.ot, g.nk, s_i,
                                                                          s_o, conj);
            else
                tma_mix::k_pack_tc_block<32, false><<<blocks, 256, 0, s>>>(W, out, (int)I, (int)O, Mt, g.ot, g.nk,
                                                                           s_i, s_o, conj);
        }
        return cudaGetLastError();
    }
    if (g.co == 64) {
        if (g.bf16)
            tma_mix::k_pack_tc<64, true><<<grid, 256, 0, s>>>(W, out, (int)I, (int)O, Mt, Qw, H, g.ot, g.nk, s_i, s_o,
                                                              s_m, conj);
        else
            tma_mix::k_pack_tc<64, false><<<grid, 256, 0, s>>>(W, out, (int)I, (int)O, Mt, Qw, H, g.ot, g.nk, s_i,
                                                               s_o, s_m, conj);
    } else {
        if (g.bf16)
            tma_mix::k_pack_tc<32, true><<<grid, 256, 0, s>>>(W, out, (int)I, (int)O, Mt, Qw, H, g.ot, g.nk, s_i, s_o,
                                                              s_m, conj);
        else
            tma_mix::k_pack_tc<32, false><<<grid, 256, 0, s>>>(W, out, (int)I, (int)O, Mt, Qw, H, g.ot, g.nk, s_i,
                                                               s_o, s_m, conj);
    }
    return cudaGetLastError();
}

// The contraction with TMA operand loads and result stores (mix_tma.cuh) on weight tiles from
// pack_tc.  Tensor maps, innermost dimension first:
//   X  {16 floats (a mode block of one (q, b, i)), B, Ci, local blocks}, box {4, 64, KS, 1} (two modes)
//      at {4 h, b0, k0, q}: strides Ci * 64 B, 64 B, B Ci 64 B (all multiples of 16 B; x = 4 h floats)
//   Y  {16 floats, B, Co, local blocks} (stores), box {4, 16, 8, 1} (two modes of 16 rows of 8 channels,
//      one epilogue warp's group; shared-memory image [channel][row][4 floats]) at {4 h, b0 + 16 w,
//      o0 + 8 g, q}: strides Co * 64 B, 64 B, B Co 64 B
template <int CO, bool BF16>
cudaError_t launch_mix_tma_t(const Plan& p, const BlockMap& bm, const float2* X, const char* Wtc, int H, float2* Y,
                             int Ci, int Co, int slot, cudaStream_t s) {
    using C = tma_mix::Cfg<CO, BF16>;
    const EncodeTiled enc = encode_tiled();
    if (!enc) return cudaErrorNotSupported;
    cudaError_t err = ensure_smem_attr(tma_mix::k_mix_tma<CO, BF16>, slot, p.device, C::SMEM);
    if (err != cudaSuccess) return err;
    int* status = device_status_ptr(p.device);
    if (!status) return cudaErrorInvalidSymbol;
    const int64_t B = p.d.batch;
    const int64_t tiles = 4 * bm.local * ceil_div(B, tc::BT) * ceil_div(Co, CO);  // 4 mode pairs per block
    if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;  // tile indices are 32-bit
    CUtensorMap tmx, tmy;
    const cuuint32_t ones[4] = {1, 1, 1, 1};
    const cuuint64_t xd[4] = {16, (cuuint64_t)B, (cuuint64_t)Ci, (cuuint64_t)bm.local};
    const cuuint64_t xs[3] = {(cuuint64_t)Ci * 64, 64, (cuuint64_t)(B * Ci * 64)};
    const cuuint32_t xb[4] = {4, (cuuint32_t)tc::BT, (cuuint32_t)C::KS, 1};
    if (enc(&tmx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float2*>(X), xd, xs, xb, ones,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    const cuuint64_t yd[4] = {16, (cuuint64_t)B, (cuuint64_t)Co, (cuuint64_t)bm.local};
    const cuuint64_t ys[3] = {(cuuint64_t)Co * 64, 64, (cuuint64_t)(B * Co * 64)};
    const cuuint32_t yb[4] = {4, 16, 8, 1};
    if (enc(&tmy, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Y, yd, ys, yb, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    const unsigned grid = (unsigned)(tiles < p.sm_count ? tiles : p.sm_count);  // persistent, one CTA per SM
    tma_mix::k_mix_tma<CO, BF16><<<grid, tma_mix::THREADS, C::SMEM, s>>>(
        tmx, Wtc, tmy, H, (int)B, Ci, Co, (int)bm.local, bm.qpl, bm.qtot, bm.qbeg, status);
    return cudaGetLastError();
}

cudaError_t launch_mix_tma(const Plan& p, const float2* X, const char* Wtc, int H, float2* Y, int Ci, int Co,
                           cudaStream_t s) {
    const BlockMap bm = block_map(p);
    if (bm.local == 0) return cudaSuccess;
    const bool bf16 = p.d.precision == NOP_PRECISION_BF16;
    cudaError_t err;
    if (Co > 32)
        err = bf16 ? launch_mix_tma_t<64, true>(p, bm, X, Wtc, H, Y, Ci, Co, 24, s)
                   : launch_mix_tma_t<64, false>(p, bm, X, Wtc, H, Y, Ci, Co, 25, s);
    else
        err = bf16 ? launch_mix_tma_t<32, true>(p, bm, X, Wtc, H, Y, Ci, Co, 26, s)
                   : launch_mix_tma_t<32, false>(p, bm, X, Wtc, H, Y, Ci, Co, 27, s);
    if (err == cudaSuccess) launch_mark(s);
    return err;
}

cudaError_t launch_mix(const Plan& p, const float2* X, const float4* W, int64_t wq, float2* Y, int Ci, int Co,
                       cudaStream_t s) {
    const BlockMap bm = block_map(p);
    if (bm.local == 0) return cudaSuccess;
    cudaError_t err;
    const bool bf16 = p.d.precision == NOP_PRECISION_BF16;
    if (p.mix_tc) {
        // 64-wide output tiles (N = 128) unless the channels fit a 32-wide tile
        // 64-wide output tiles (N = 128) unless the channels fit a 32-wide tile
        if (Co > 32)
            err = bf16 ? launch_mix_tc<64, true>(p, bm, X, W, wq, Y, Ci, Co, 16, s)
                       : launch_mix_tc<64, false>(p, bm, X, W, wq, Y, Ci, Co, 17, s);
        else
            err = bf16 ? launch_mix_tc<32, true>(p, bm, X, W, wq, Y, Ci, Co, 18, s)
                       : launch_mix_tc<32, false>(p, bm, X, W, wq, Y, Ci, Co, 19, s);
    } else {
        err = ensure_smem_attr(bf16 ? k_mix<true> : k_mix<false>, bf16 ? 14 : 15, p.device, kMixSmem);
        if (err != cudaSuccess) return err;
        dim3 grid((unsigned)bm.local, (unsigned)ceil_div(p.d.batch, 16), (unsigned)ceil_div(Co, 64));
        if (bf16)
            k_mix<true><<<grid, kMixThreads, kMixSmem, s>>>(X, W, wq, Y, (int)p.d.batch, Ci, Co, bm.qpl, bm.qtot,
                                                             bm.qbeg);
        else
            k_mix<false><<<grid, kMixThreads, kMixSmem, s>>>(X, W, wq, Y, (int)p.d.batch, Ci, Co, bm.qpl, bm.qtot,
                                                              bm.qbeg);
        err = cudaGetLastError();
    }
    if (err == cudaSuccess) launch_mark(s);
    return err;
}

// contraction on the mode-blocked spectrum with packed weights
int32_t mix_stage(const Plan& p, const float2* Xh, const char* packed, float2* Yh, char* ws, cudaStream_t s) {
    const nop_spectral_desc& d = p.d;
    const int Ci = (int)d.in_channels, Co = (int)d.out_channels;
    cudaError_t err;
    if (p.mix_tma) {
        // weight tiles from pack_tc: per mode block (H = 4) or one matrix for every block (H = 1)
        if (d.weight_kind == NOP_WEIGHT_DENSE) {
            err = launch_mix_tma(p, Xh, packed + p.pk_w, 4, Yh, Ci, Co, s);
            return err == cudaSuccess ? NOP_OK : cuda_fail(err, "mix launch");
        }
        const int rin = (int)d.ranks[0], rout = (int)d.ranks[1];
        float2* xf = reinterpret_cast<float2*>(ws + p.ws.xf);
        float2* z = reinterpret_cast<float2*>(ws + p.ws.z);
        if ((err = launch_mix_tma(p, Xh, packed + p.pk_uin, 1, xf, Ci, rin, s)) != cudaSuccess)
            return cuda_fail(err, "mix launch (input factor)");
        if ((err = launch_mix_tma(p, xf, packed + p.pk_w, 4, z, rin, rout, s)) != cudaSuccess)
            return cuda_fail(err, "mix launch (core)");
        if ((err = launch_mix_tma(p, z, packed + p.pk_uout, 1, Yh, rout, Co, s)) != cudaSuccess)
            return cuda_fail(err, "mix launch (output factor)");
        return NOP_OK;
    }
    if (d.weight_kind == NOP_WEIGHT_DENSE) {
        const float4* W = reinterpret_cast<const float4*>(packed + p.pk_w);
        err = launch_mix(p, Xh, W, (int64_t)Ci * 4 * Co, Yh, Ci, Co, s);
        return err == cudaSuccess ? NOP_OK : cuda_fail(err, "mix launch");
    }
    // Tucker: xf = X . U_in, z = xf . G (per mode), Y = z . U_out^T
    const int rin = (int)d.ranks[0], rout = (int)d.ranks[1];
    float2* xf = reinterpret_cast<float2*>(ws + p.ws.xf);
    float2* z = reinterpret_cast<float2*>(ws + p.ws.z);
    if ((err = launch_mix(p, Xh, reinterpret_cast<const float4*>(packed + p.pk_uin), 0, xf, Ci, rin, s)) !=
        cudaSuccess)
        return cuda_fail(err, "mix launch (input factor)");
    if ((err = launch_mix(p, xf, reinterpret_cast<const float4*>(packed + p.pk_w), (int64_t)rin * 4 * rout, z, rin,
                          rout, s)) != cudaSuccess)
        return cuda_fail(err, "mix launch (core)");
    if ((err = launch_mix(p, z, reinterpret_cast<const float4*>(packed + p.pk_uout), 0, Yh, rout, Co, s)) !=
        cudaSuccess)
        return cuda_fail(err, "mix launch (output factor)");
    return NOP_OK;
}

// planes per CTA of the 256 x 256 inverse plane kernel: two, so each CTA prefetches one plane's
// spectrum across planes, once the grid still fills the 2 CTAs x SMs slots several times over
// (measured on B200 with 4096 planes: 1 -> 307 us, 2 -> 301 us, 3 -> 322 us, 4 -> 302 us)
// planes per CTA of the 256 x 256 inverse: two from 8 planes per SM; persistent (two CTAs per SM, every
// CTA the same number of planes, the twiddle tables built once per CTA) from 64 planes per SM.  Measured
// on B200: the C5 layer's inverse (65536 planes) 3.69 -> 3.56 ms persistent, while the C2 layer's
// (4096 planes, 14 per CTA persistent) ran 261 -> 275 us, so it keeps two per CTA.
inline int planes_per_cta(const Plan& p, int64_t planes) {
    const int64_t sms = p.sm_count;
    if (planes >= 64 * sms) return (int)((planes + 2 * sms - 1) / (2 * sms));
    return planes >= 8 * sms ? 2 : 1;
}

inline unsigned plane_ctas(const Plan& p, int64_t planes) {
    const int ppc = planes_per_cta(p, planes);
    return (unsigned)((planes + ppc - 1) / ppc);
}

// kept-mode specialisations of the 256 x 256 plane kernels (see plane256.cuh)
template <int KX, int MY>
bool p256_applies(const nop_spectral_desc& d) {
    if (d.n_in[0] != 256 || d.kept[1] != KX || d.kept[0] != MY || d.fwd_off[0] != MY / 2 || d.inv_off[0] != MY / 2)
        return false;
    // the inverse forces only bin 0 real; every other forced bin must lie outside the kept range
    bool has0 = false;
    for (int i = 0; i < d.n_zero_imag; ++i) {
        if (d.zero_imag_bins[i] == 0) has0 = true;
        else if (d.zero_imag_bins[i] < KX) return false;
    }
    return has0;
}

template <int KX, int MY>
int32_t run_p256(const Plan& p, const void* x, const char* packed, const float* bias, const float* addend,
                 int apply_gelu, void* y, char* ws, cudaStream_t s, int slot, float2* xs) {
    const nop_spectral_desc& d = p.d;
    const int64_t Lin = d.batch * d.in_channels, Lout = d.batch * d.out_channels;
    constexpr size_t smem = p256::smem_bytes<KX, MY>();
    const TwiddleTable* tt = p.table(256);
    float2* Xh = xs ? xs : reinterpret_cast<float2*>(ws + p.ws.buf_a);
    float2* Yh = reinterpret_cast<float2*>(ws + p.ws.buf_b);
    cudaError_t err;
    if ((err = ensure_smem_attr(p256::k_fwd<KX, MY>, slot, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(p256 fwd)");
    if ((err = ensure_smem_attr(p256::k_inv<KX, MY>, slot + 1, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(p256 inv)");
    p256::k_fwd<KX, MY><<<(unsigned)Lin, p256::THREADS, smem, s>>>(static_cast<const float*>(x), Xh, tt->f_table,
                                                                     (float)d.fwd_scale, Lin * 8);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "p256 fwd launch");
    launch_mark(s);
    int32_t rc = mix_stage(p, Xh, packed, Yh, ws, s);
    if (rc != NOP_OK) return rc;
    p256::Epi ep{bias, addend, apply_gelu, (int)d.out_channels, 1};
    p256::k_inv<KX, MY><<<plane_ctas(p, Lout), p256::THREADS, smem, s>>>(Yh, static_cast<float*>(y), tt->f_table,
                                                                           (float)d.inv_scale, Lout * 8, ep, Lout,
                                                                           planes_per_cta(p, Lout));
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "p256 inv launch");
    launch_mark(s);
    return NOP_OK;
}

// 512 x 512 planes through the 256-point machinery (see plane512.cuh); same kept-mode rule as p256
template <int KX, int MY>
bool p512_applies(const nop_spectral_desc& d) {
    nop_spectral_desc h = d;
    if (d.n_in[0] != 512 || d.n_in[1] != 512) return false;
    h.n_in[0] = h.n_in[1] = 256;  // the kept-mode / forced-real checks do not depend on the length
    return p256_applies<KX, MY>(h);
}

template <int KX, int MY>
int32_t run_p512(const Plan& p, const void* x, const char* packed, const float* bias, const float* addend,
                 int apply_gelu, void* y, char* ws, cudaStream_t s, int slot, float2* xs) {
    const nop_spectral_desc& d = p.d;
    const int64_t Lin = d.batch * d.in_channels, Lout = d.batch * d.out_channels;
    constexpr size_t smem = p512::smem_bytes<KX, MY>();
    const TwiddleTable* tt = p.table(512);
    float2* Xh = xs ? xs : reinterpret_cast<float2*>(ws + p.ws.buf_a);
    float2* Yh = reinterpret_cast<float2*>(ws + p.ws.buf_b);
    cudaError_t err;
    if ((err = ensure_smem_attr(p512::k_fwd<KX, MY>, slot, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(p512 fwd)");
    if ((err = ensure_smem_attr(p512::k_inv<KX, MY>, slot + 1, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(p512 inv)");
    p512::k_fwd<KX, MY><<<(unsigned)Lin, p512::THREADS, smem, s>>>(static_cast<const float*>(x), Xh, tt->f_table,
                                                                     (float)d.fwd_scale, Lin * 8);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "p512 fwd launch");
    launch_mark(s);
    int32_t rc = mix_stage(p, Xh, packed, Yh, ws, s);
    if (rc != NOP_OK) return rc;
    p256::Epi ep{bias, addend, apply_gelu, (int)d.out_channels, 1};
    p512::k_inv<KX, MY><<<(unsigned)Lout, p512::THREADS, smem, s>>>(Yh, static_cast<float*>(y), tt->f_table,
                                                                      (float)d.inv_scale, Lout * 8, ep);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "p512 inv launch");
    launch_mark(s);
    return NOP_OK;
}

template <int N>
int32_t run_plane_2d(const Plan& p, const void* x, const char* packed, const float* bias, const float* addend,
                     int apply_gelu, void* y, char* ws, cudaStream_t s, float2* xs) {
    const nop_spectral_desc& d = p.d;
    if constexpr (N == 256) {
        if (p256_applies<33, 64>(d)) return run_p256<33, 64>(p, x, packed, bias, addend, apply_gelu, y, ws, s, 6, xs);
        if (p256_applies<17, 32>(d)) return run_p256<17, 32>(p, x, packed, bias, addend, apply_gelu, y, ws, s, 8, xs);
    }
    if constexpr (N == 512) {
        if (p512_applies<33, 64>(d)) return run_p512<33, 64>(p, x, packed, bias, addend, apply_gelu, y, ws, s, 20, xs);
        if (p512_applies<17, 32>(d)) return run_p512<17, 32>(p, x, packed, bias, addend, apply_gelu, y, ws, s, 22, xs);
    }
    const int Kx = (int)d.kept[1], My = (int)d.kept[0];
    const int64_t Lin = d.batch * d.in_channels, Lout = d.batch * d.out_channels;
    const size_t smem = plane_smem_bytes<N>(Kx, My);
    const TwiddleTable* tt = p.table(N);
    float2* Xh = xs ? xs : reinterpret_cast<float2*>(ws + p.ws.buf_a);
    float2* Yh = reinterpret_cast<float2*>(ws + p.ws.buf_b);
    cudaError_t err;
    constexpr int slot = fft::ilog2(N) - 7;  // 0, 1, 2 for N = 128, 256, 512
    if ((err = ensure_smem_attr(k_plane_fwd<N>, 2 * slot, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(plane_fwd)");
    if ((err = ensure_smem_attr(k_plane_inv<N>, 2 * slot + 1, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(plane_inv)");
    k_plane_fwd<N><<<(unsigned)Lin, PlaneCfg<N>::THREADS, smem, s>>>(
        static_cast<const float*>(x), Xh, tt->f_table, Kx, My, (int)d.fwd_off[0], (float)d.fwd_scale, Lin * 8);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "plane_fwd launch");
    launch_mark(s);
    int32_t rc = mix_stage(p, Xh, packed, Yh, ws, s);
    if (rc != NOP_OK) return rc;
    Epilogue ep{};
    ep.bias = bias;
    ep.addend = addend;
    ep.apply_gelu = apply_gelu;
    ep.C = (int)d.out_channels;
    ep.chan_div = 1;
    ep.z0 = ep.z1 = ep.z2 = -1;
    if (d.n_zero_imag > 0) ep.z0 = (int)d.zero_imag_bins[0];
    if (d.n_zero_imag > 1) ep.z1 = (int)d.zero_imag_bins[1];
    if (d.n_zero_imag > 2) ep.z2 = (int)d.zero_imag_bins[2];
    k_plane_inv<N><<<(unsigned)Lout, PlaneCfg<N>::THREADS, smem, s>>>(Yh, static_cast<float*>(y), tt->f_table, Kx,
                                                                       My, (int)d.inv_off[0], (float)d.inv_scale,
                                                                       Lout * 8, ep);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "plane_inv launch");
    launch_mark(s);
    return NOP_OK;
}

// ---- 1D: long lines, few kept bins ----
template <int N, int K>
int32_t run_row1d(const Plan& p, const void* x, const char* packed, const float* bias, const float* addend,
                  int apply_gelu, void* y, char* ws, cudaStream_t s, float2* xs) {
    const nop_spectral_desc& d = p.d;
    const int64_t Lin = d.batch * d.in_channels, Lout = d.batch * d.out_channels;
    const TwiddleTable* tt = p.table(N);
    float2* Xh = xs ? xs : reinterpret_cast<float2*>(ws + p.ws.buf_a);
    float2* Yh = reinterpret_cast<float2*>(ws + p.ws.buf_b);
    cudaError_t err;
    r1d::k_fwd<N, K><<<(unsigned)ceil_div(Lin, r1d::LINES), r1d::THREADS, 0, s>>>(
        static_cast<const float*>(x), Xh, tt->f_table, Lin, (float)d.fwd_scale, Lin * 8);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "row1d fwd launch");
    launch_mark(s);
    int32_t rc = mix_stage(p, Xh, packed, Yh, ws, s);
    if (rc != NOP_OK) return rc;
    r1d::Epi1 ep{bias, addend, apply_gelu, (int)d.out_channels};
    r1d::k_inv<N, K><<<(unsigned)ceil_div(Lout, r1d::LINES), r1d::THREADS, 0, s>>>(
        Yh, static_cast<float*>(y), tt->f_table, Lout, (float)d.inv_scale, Lout * 8, ep);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "row1d inv launch");
    launch_mark(s);
    return NOP_OK;
}

template <int N>
int32_t run_row1d_k(const Plan& p, const void* x, const char* packed, const float* bias, const float* addend,
                    int apply_gelu, void* y, char* ws, cudaStream_t s, float2* xs) {
    switch (p.d.kept[0]) {
        case 9: return run_row1d<N, 9>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
        case 17: return run_row1d<N, 17>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
        default: return fail(NOP_E_UNSUPPORTED, "fused 1D engine: unsupported kept-bin count");
    }
}

// ---- 3D: (y, z) plane kernels, outer-axis transforms along x, contraction ----
template <int KZ, int MY, int MX>
int32_t run_vol3d(const Plan& p, const void* x, const char* packed, const float* bias, const float* addend,
                  int apply_gelu, void* y, char* ws, cudaStream_t s, int slot, float2* xs) {
    const nop_spectral_desc& d = p.d;
    const int64_t Nx = d.n_in[0];
    const int64_t BCi = d.batch * d.in_channels, BCo = d.batch * d.out_channels;
    const int64_t Lin = BCi * Nx, Lout = BCo * Nx;
    constexpr int QP = MY * KZ / 8;
    constexpr size_t smem = p256::smem_bytes<KZ, MY>();
    float2* Pa = reinterpret_cast<float2*>(ws + p.ws.pl_a);
    float2* Pb = reinterpret_cast<float2*>(ws + p.ws.pl_b);
    float2* Xh = xs ? xs : reinterpret_cast<float2*>(ws + p.ws.buf_a);
    float2* Yh = reinterpret_cast<float2*>(ws + p.ws.buf_b);
    const float2* tw256 = p.table(256)->f_table;
    cudaError_t err;
    if ((err = ensure_smem_attr(p256::k_fwd<KZ, MY>, slot, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(p256 fwd)");
    if ((err = ensure_smem_attr(p256::k_inv<KZ, MY>, slot + 1, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(p256 inv)");
    p256::k_fwd<KZ, MY><<<(unsigned)Lin, p256::THREADS, smem, s>>>(static_cast<const float*>(x), Pa, tw256,
                                                                     (float)d.fwd_scale, Lin * 8);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "vol3d plane fwd launch");
    launch_mark(s);
    axis::k_fwd<MX><<<(unsigned)(QP * BCi), axis::THREADS, 0, s>>>(Pa, Xh, tw256, QP, BCi, (int)Nx, 0);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "vol3d axis fwd launch");
    launch_mark(s);
    int32_t rc = mix_stage(p, Xh, packed, Yh, ws, s);
    if (rc != NOP_OK) return rc;
    axis::k_inv<MX><<<(unsigned)(QP * BCo), axis::THREADS, 0, s>>>(Yh, Pb, tw256, QP, BCo, (int)Nx, 0);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "vol3d axis inv launch");
    launch_mark(s);
    p256::Epi ep{bias, addend, apply_gelu, (int)d.out_channels, Nx};
    p256::k_inv<KZ, MY><<<plane_ctas(p, Lout), p256::THREADS, smem, s>>>(Pb, static_cast<float*>(y), tw256,
                                                                           (float)d.inv_scale, Lout * 8, ep, Lout,
                                                                           planes_per_cta(p, Lout));
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "vol3d plane inv launch");
    launch_mark(s);
    return NOP_OK;
}

// ---- 3D slab stages (first axis split across ranks; exchanges run between the stages) ----
template <int KZ, int MY>
int32_t slab_planes_fwd_t(const Plan& p, const float* x, float2* send1, cudaStream_t s, int slot) {
    const nop_spectral_desc& d = p.d;
    const int64_t L = d.batch * d.in_channels * p.slab_nx;
    if (L == 0) return NOP_OK;
    cudaError_t err;
    if ((err = ensure_smem_attr(p256::k_fwd<KZ, MY>, slot, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(p256 fwd)");
    p256::k_fwd<KZ, MY><<<(unsigned)L, p256::THREADS, p256::smem_bytes<KZ, MY>(), s>>>(
        x, send1, p.table(256)->f_table, (float)d.fwd_scale, L * 8);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "slab plane fwd launch");
    launch_mark(s);
    return NOP_OK;
}

template <int MX>
int32_t slab_modes_t(const Plan& p, const float2* recv1, const char* packed, float2* send2, char* ws,
                     cudaStream_t s) {
    const nop_spectral_desc& d = p.d;
    const int64_t qc = p.slab_qcount[p.slab_rank], nx = p.slab_nx;
    if (qc == 0) return NOP_OK;
    const int64_t BCi = d.batch * d.in_channels, BCo = d.batch * d.out_channels;
    float2* Xh = reinterpret_cast<float2*>(ws + p.ws.buf_a);
    float2* Yh = reinterpret_cast<float2*>(ws + p.ws.buf_b);
    const float2* tw256 = p.table(256)->f_table;
    cudaError_t err;
    axis::k_fwd<MX><<<(unsigned)(qc * BCi), axis::THREADS, 0, s>>>(recv1, Xh, tw256, (int)qc, BCi, (int)nx,
                                                                    qc * BCi * nx * 8);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "slab axis fwd launch");
    launch_mark(s);
    int32_t rc = mix_stage(p, Xh, packed, Yh, ws, s);
    if (rc != NOP_OK) return rc;
    axis::k_inv<MX><<<(unsigned)(qc * BCo), axis::THREADS, 0, s>>>(Yh, send2, tw256, (int)qc, BCo, (int)nx,
                                                                    qc * BCo * nx * 8);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "slab axis inv launch");
    launch_mark(s);
    return NOP_OK;
}

template <int KZ, int MY>
int32_t slab_planes_inv_t(const Plan& p, const float2* recv2, const float* bias, const float* addend,
                          int apply_gelu, float* y, cudaStream_t s, int slot) {
    const nop_spectral_desc& d = p.d;
    const int64_t L = d.batch * d.out_channels * p.slab_nx;
    if (L == 0) return NOP_OK;
    cudaError_t err;
    if ((err = ensure_smem_attr(p256::k_inv<KZ, MY>, slot, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(p256 inv)");
    p256::Epi ep{bias, addend, apply_gelu, (int)d.out_channels, p.slab_nx};
    p256::k_inv<KZ, MY><<<plane_ctas(p, L), p256::THREADS, p256::smem_bytes<KZ, MY>(), s>>>(
        recv2, y, p.table(256)->f_table, (float)d.inv_scale, L * 8, ep, L, planes_per_cta(p, L));
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "slab plane inv launch");
    launch_mark(s);
    return NOP_OK;
}

bool vol3d_shape(const nop_spectral_desc& d, int* which) {
    // x-axis 256 with MX centred bins; (y, z) planes 256 x 256 specialised on (kept y, kept z)
    if (d.ndim != 3 || d.n_in[0] != 256 || d.n_in[1] != 256 || d.n_in[2] != 256) return false;
    if (d.fwd_off[0] != d.kept[0] / 2 || d.inv_off[0] != d.kept[0] / 2) return false;
    nop_spectral_desc plane = d;  // view the last two axes as a 2D plane for the p256 check
    plane.n_in[0] = 256;
    plane.kept[0] = d.kept[1];
    plane.kept[1] = d.kept[2];
    plane.fwd_off[0] = d.fwd_off[1];
    plane.inv_off[0] = d.inv_off[1];
    if (d.kept[0] == 32 && p256_applies<17, 32>(plane)) {
        *which = 0;
        return true;
    }
    if (d.kept[0] == 64 && p256_applies<33, 64>(plane)) {
        *which = 1;
        return true;
    }
    return false;
}

size_t plane_smem_for(int64_t N, int Kx, int My) {
    switch (N) {
        case 128: return plane_smem_bytes<128>(Kx, My);
        case 256: return plane_smem_bytes<256>(Kx, My);
        case 512: return plane_smem_bytes<512>(Kx, My);
        default: return 0;
    }
}

}  // namespace

bool fast_supported(const nop_spectral_desc& d, FastKind* kind, std::string* why) {
    *kind = FastKind::None;
    if (d.complex_data) return *why = "complex data", false;
    for (int j = 0; j < d.ndim; ++j)
        if (d.n_out[j] != d.n_in[j]) return *why = "output resampling", false;
    if (d.separable) return *why = "separable contraction", false;
    if (d.weight_kind != NOP_WEIGHT_DENSE && d.weight_kind != NOP_WEIGHT_TUCKER)
        return *why = "weight kind other than dense / Tucker", false;
    if (d.batch * d.in_channels > 0x7fffffffLL || d.batch * d.out_channels > 0x7fffffffLL ||
        (d.batch + 15) / 16 > 65535)
        return *why = "too many lines for one launch", false;
    bool forced_ok = true;  // only bin 0 may be forced real inside the kept range of the last axis
    for (int i = 0; i < d.n_zero_imag; ++i)
        if (d.zero_imag_bins[i] != 0 && d.zero_imag_bins[i] < d.kept[d.ndim - 1]) forced_ok = false;
    if (d.ndim == 1) {
        const int64_t N = d.n_in[0];
        if (N != 2048 && N != 4096 && N != 8192 && N != 16384) return *why = "1D length not in {2048..16384}", false;
        if (d.kept[0] != 9 && d.kept[0] != 17) return *why = "1D kept bins not in {9, 17}", false;
        if (!forced_ok) return *why = "forced-real bins inside the kept range", false;
        *kind = FastKind::Row1D;
        return true;
    }
    if (d.ndim == 3) {
        int which;
        if (!vol3d_shape(d, &which)) return *why = "3D shape not covered (256^3 with (32,32,17) or (64,64,33) modes)", false;
        if (d.batch * d.in_channels * 256 > 0x7fffffffLL || d.batch * d.out_channels * 256 > 0x7fffffffLL)
            return *why = "too many planes for one launch", false;
        *kind = FastKind::Vol3D;
        return true;
    }
    if (d.ndim != 2) return *why = "4D is not fused", false;
    const int64_t N = d.n_in[0];
    if (d.n_in[1] != N) return *why = "non-square plane", false;
    if (N != 128 && N != 256 && N != 512) return *why = "plane size not in {128, 256, 512}", false;
    if (d.batch * d.in_channels > 0x7fffffffLL || d.batch * d.out_channels > 0x7fffffffLL ||
        (d.batch + 15) / 16 > 65535)
        return *why = "too many planes for one launch", false;
    const size_t smem = plane_smem_for(N, (int)d.kept[1], (int)d.kept[0]);
    if (smem > kSmemLimit) return *why = "kept modes need more shared memory than a CTA has", false;
    *kind = FastKind::Plane2D;
    return true;
}

// Workspace: mode-blocked X^ and Y^, Tucker intermediates, packing temporaries, packed weights
// (the latter only used by the unpacked forward).  Also fixes the packed-weight layout.
size_t fast_workspace_bytes(Plan& p, WorkspaceLayout* ws) {
    const nop_spectral_desc& d = p.d;
    const int64_t Q = mode_blocks(p), B = d.batch, Ci = d.in_channels, Co = d.out_channels;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t at = off;
        off += up256(bytes);
        return at;
    };
    ws->buf_a = take((size_t)Q * 8 * B * Ci * sizeof(float2));
    ws->buf_b = take((size_t)Q * 8 * B * Co * sizeof(float2));
    if (p.fast_kind == FastKind::Vol3D) {  // (slab plans keep their plane spectra in caller buffers)
        const size_t plane_modes = (size_t)d.kept[1] * d.kept[2];
        ws->pl_a = take(plane_modes * B * Ci * d.n_in[0] * sizeof(float2));
        ws->pl_b = take(plane_modes * B * Co * d.n_in[0] * sizeof(float2));
    }
    ws->buf_elems = 0;
    size_t pk = 0;
    auto pk_take = [&](size_t bytes) {
        size_t at = pk;
        pk += up256(bytes);
        return at;
    };
    // packed weights: tiles for the TMA contraction (pack_tc) or [Q][I][4][O] float4 (k_pack_modes)
    if (d.weight_kind == NOP_WEIGHT_DENSE) {
        p.pk_w = pk_take(p.mix_tma ? (size_t)tc_geom(p, Ci, Co, Q, 4).bytes : (size_t)Q * Ci * 4 * Co * sizeof(float4));
        ws->xf = ws->z = ws->g = ws->g_tmp = 0;
    } else {
        const int64_t rin = d.ranks[0], rout = d.ranks[1];
        p.pk_w = pk_take(p.mix_tma ? (size_t)tc_geom(p, rin, rout, Q, 4).bytes
                                   : (size_t)Q * rin * 4 * rout * sizeof(float4));
        p.pk_uin = pk_take(p.mix_tma ? (size_t)tc_geom(p, Ci, rin, 1, 1).bytes : (size_t)Ci * 4 * rin * sizeof(float4));
        p.pk_uout = pk_take(p.mix_tma ? (size_t)tc_geom(p, rout, Co, 1, 1).bytes
                                      : (size_t)rout * 4 * Co * sizeof(float4));
        ws->xf = take((size_t)Q * 8 * B * rin * sizeof(float2));
        ws->z = take((size_t)Q * 8 * B * rout * sizeof(float2));
        int64_t g = 0;
        for (int j = 0; j < d.ndim; ++j) {
            int64_t e = rin * rout;
            for (int i = 0; i <= j; ++i) e *= d.kept[i];
            for (int i = j + 1; i < d.ndim; ++i) e *= d.ranks[2 + i];
            if (e > g) g = e;
        }
        ws->g = take((size_t)g * sizeof(float2));
        ws->g_tmp = take((size_t)g * sizeof(float2));
    }
    p.packed_bytes = pk;
    ws->packed = take(pk);
    return off;
}

int* status_word(int device) { return device_status_ptr(device); }

void* tensor_map_encoder() { return reinterpret_cast<void*>(encode_tiled()); }

int32_t fast_device_status(int* status, bool clear) {
    int v = 0;
    cudaError_t err = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
    if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyFromSymbol(status)");
    if (clear && v != 0) {
        const int zero = 0;
        if ((err = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int))) != cudaSuccess)
            return cuda_fail(err, "cudaMemcpyToSymbol(status)");
    }
    *status = v;
    return NOP_OK;
}

int32_t fast_launches(const Plan& p) {
    // 3D (whole or slab): plane transforms and outer-axis transforms in both directions
    const bool vol = p.fast_kind == FastKind::Vol3D || p.fast_kind == FastKind::Vol3DSlab;
    const int transforms = vol ? 4 : 2;
    return transforms + (p.d.weight_kind == NOP_WEIGHT_DENSE ? 1 : 3);
}

int32_t fast_pack_adjoint(const Plan& p, const void* W, char* packed, cudaStream_t s) {
    // p is the adjoint plan (Ci' = Co, Co' = Ci); W the forward's dense weight [Co'][Ci'][Mt]:
    // W'[i'][o'][m] = conj(W[o'][i'][m]) is element i' * Mt + o' * (Ci' * Mt) of W
    const nop_spectral_desc& d = p.d;
    if (d.weight_kind != NOP_WEIGHT_DENSE)
        return fail(NOP_E_UNSUPPORTED, "adjoint packing from the forward weight needs dense weights");
    const int64_t Q = mode_blocks(p), Mt = p.modes_total, Ci = d.in_channels, Co = d.out_channels;
    if (p.mix_tma) {
        const cudaError_t e = pack_tc(p, static_cast<const float2*>(W), packed + p.pk_w, Ci, Co, Q, 4, Mt, Ci * Mt, 1,
                                      1, s);
        return e == cudaSuccess ? NOP_OK : cuda_fail(e, "adjoint pack launch");
    }
    const int64_t n = Q * Ci * 4 * Co;
    k_pack_modes<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(static_cast<const float2*>(W),
                                                            reinterpret_cast<float4*>(packed + p.pk_w), (int)Ci,
                                                            (int)Co, Mt, Q, Mt, Ci * Mt, 1);
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? NOP_OK : cuda_fail(err, "adjoint pack launch");
}

int32_t fast_pack(const Plan& p, const void* const* weights, char* packed, char* ws, cudaStream_t s) {
    const nop_spectral_desc& d = p.d;
    const int64_t Q = mode_blocks(p), Mt = p.modes_total, Ci = d.in_channels, Co = d.out_channels;
    cudaError_t err;
    if (p.mix_tma) {
        if (d.weight_kind == NOP_WEIGHT_DENSE) {
            err = pack_tc(p, static_cast<const float2*>(weights[0]), packed + p.pk_w, Ci, Co, Q, 4, Co * Mt, Mt, 1, 0, s);
            return err == cudaSuccess ? NOP_OK : cuda_fail(err, "pack launch");
        }
        const int64_t rin = d.ranks[0], rout = d.ranks[1];
        float2* G = expand_tucker_core(p, static_cast<const float2*>(weights[0]), weights, 3, rin * rout, ws, &err, s);
        if (!G) return cuda_fail(err, "tucker core expansion");
        if ((err = pack_tc(p, G, packed + p.pk_w, rin, rout, Q, 4, rout * Mt, Mt, 1, 0, s)) != cudaSuccess)
            return cuda_fail(err, "pack launch (core)");
        launch_mark(s);
        // U_in [Ci][r_in]: xf[f] = sum_i x[i] U_in[i][f]
        if ((err = pack_tc(p, static_cast<const float2*>(weights[1]), packed + p.pk_uin, Ci, rin, 1, 1, rin, 1, 0, 0,
                           s)) != cudaSuccess)
            return cuda_fail(err, "pack launch (input factor)");
        launch_mark(s);
        // U_out [Co][r_out]: y[o] = sum_g z[g] U_out[o][g]
        err = pack_tc(p, static_cast<const float2*>(weights[2]), packed + p.pk_uout, rout, Co, 1, 1, 1, rout, 0, 0, s);
        return err == cudaSuccess ? NOP_OK : cuda_fail(err, "pack launch (output factor)");
    }
    if (d.weight_kind == NOP_WEIGHT_DENSE) {
        const int64_t n = Q * Ci * 4 * Co;
        k_pack_modes<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(static_cast<const float2*>(weights[0]),
                                                                reinterpret_cast<float4*>(packed + p.pk_w), (int)Ci,
                                                                (int)Co, Mt, Q, Co * Mt, Mt);
        return (err = cudaGetLastError()) == cudaSuccess ? NOP_OK : cuda_fail(err, "pack launch");
    }
    const int64_t rin = d.ranks[0], rout = d.ranks[1];
    // G[f][g][m] = core x_2 U_1 x_3 U_2 ... (per-mode r_in x r_out matrices)
    float2* G = expand_tucker_core(p, static_cast<const float2*>(weights[0]), weights, 3, rin * rout, ws, &err, s);
    if (!G) return cuda_fail(err, "tucker core expansion");
    int64_t n = Q * rin * 4 * rout;
    k_pack_modes<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(G, reinterpret_cast<float4*>(packed + p.pk_w), (int)rin,
                                                            (int)rout, Mt, Q, rout * Mt, Mt);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "pack launch (core)");
    launch_mark(s);
    // U_in [Ci][r_in]: xf[f] = sum_i x[i] U_in[i][f]
    n = Ci * 4 * rin;
    k_pack_broadcast<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(static_cast<const float2*>(weights[1]),
                                                                reinterpret_cast<float4*>(packed + p.pk_uin), (int)Ci,
                                                                (int)rin, rin, 1);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "pack launch (input factor)");
    launch_mark(s);
    // U_out [Co][r_out]: y[o] = sum_g z[g] U_out[o][g]
    n = rout * 4 * Co;
    k_pack_broadcast<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(static_cast<const float2*>(weights[2]),
                                                                reinterpret_cast<float4*>(packed + p.pk_uout),
                                                                (int)rout, (int)Co, 1, rout);
    return (err = cudaGetLastError()) == cudaSuccess ? NOP_OK : cuda_fail(err, "pack launch (output factor)");
}

int32_t fast_forward_packed(const Plan& p, const void* x, const char* packed, const float* bias,
                            const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s, float2* xs) {
    if (p.fast_kind == FastKind::Row1D) {
        switch (p.d.n_in[0]) {
            case 2048: return run_row1d_k<2048>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
            case 4096: return run_row1d_k<4096>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
            case 8192: return run_row1d_k<8192>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
            case 16384: return run_row1d_k<16384>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
            default: return fail(NOP_E_UNSUPPORTED, "fused 1D engine: unsupported length");
        }
    }
    if (p.fast_kind == FastKind::Vol3DSlab)
        return fail(NOP_E_UNSUPPORTED, "slab plans run through the nop_spectral_slab_* stage calls");
    if (p.fast_kind == FastKind::Vol3D) {
        int which = -1;
        vol3d_shape(p.d, &which);
        if (which == 0) return run_vol3d<17, 32, 32>(p, x, packed, bias, addend, apply_gelu, y, ws, s, 10, xs);
        return run_vol3d<33, 64, 64>(p, x, packed, bias, addend, apply_gelu, y, ws, s, 12, xs);
    }
    switch (p.d.n_in[0]) {
        case 128: return run_plane_2d<128>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
        case 256: return run_plane_2d<256>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
        case 512: return run_plane_2d<512>(p, x, packed, bias, addend, apply_gelu, y, ws, s, xs);
        default: return fail(NOP_E_UNSUPPORTED, "fused engine: unsupported plane size");
    }
}

int32_t fast_slab_planes_fwd(const Plan& p, const float* x, void* send1, cudaStream_t s) {
    int which = -1;
    vol3d_shape(p.d, &which);
    if (which == 0) return slab_planes_fwd_t<17, 32>(p, x, static_cast<float2*>(send1), s, 10);
    return slab_planes_fwd_t<33, 64>(p, x, static_cast<float2*>(send1), s, 12);
}

int32_t fast_slab_modes(const Plan& p, const void* recv1, const char* packed, void* send2, char* ws,
                        cudaStream_t s) {
    int which = -1;
    vol3d_shape(p.d, &which);
    if (which == 0) return slab_modes_t<32>(p, static_cast<const float2*>(recv1), packed, static_cast<float2*>(send2), ws, s);
    return slab_modes_t<64>(p, static_cast<const float2*>(recv1), packed, static_cast<float2*>(send2), ws, s);
}

int32_t fast_slab_planes_inv(const Plan& p, const void* recv2, const float* bias, const float* addend,
                             int apply_gelu, float* y, cudaStream_t s) {
    int which = -1;
    vol3d_shape(p.d, &which);
    if (which == 0)
        return slab_planes_inv_t<17, 32>(p, static_cast<const float2*>(recv2), bias, addend, apply_gelu, y, s, 11);
    return slab_planes_inv_t<33, 64>(p, static_cast<const float2*>(recv2), bias, addend, apply_gelu, y, s, 13);
}

int32_t fast_forward(const Plan& p, const void* x, const void* const* weights, const float* bias,
                     const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s, float2* xs) {
    int32_t rc = fast_pack(p, weights, ws + p.ws.packed, ws, s);
    if (rc != NOP_OK) return rc;
    return fast_forward_packed(p, x, ws + p.ws.packed, bias, addend, apply_gelu, y, ws, s, xs);
}

}  // namespace nop

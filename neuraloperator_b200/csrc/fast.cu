// Fused FFT engine.
//
// 2D (square N x N grids, N in {128, 256, 512}), real data, n_out == n_in:
//   k_plane_fwd  : one CTA per (batch, channel) plane.  Row transforms (two real rows packed as one
//                  complex line) keep rFFT bins 0..Kx-1 in a shared-memory column store; column
//                  transforms keep the My bins (m - off) mod N.  Only the kept modes reach HBM.
//   k_mix_dense  : per-mode complex Cin x Cout contraction, 8-mode x 16-batch x 64-out tiles (fp32 FMA).
//   k_plane_inv  : column inverses of the kept modes, then row inverses (two real rows per complex
//                  line) with the epilogue bias (+ skip) (+ GELU) fused into the final pass.
// Other shapes fall back to the generic engine (plan-time decision).
#include <atomic>

#include "fft_core.cuh"
#include "nop_internal.cuh"

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
            int off_y, float scale) {
    using C = PlaneCfg<N>;
    extern __shared__ float2 smem[];
    float2* tw = smem;
    float2* T = tw + N;                    // column store: T[c * TPITCH + pad(row)]
    float2* X = T + (size_t)Kx * C::TPITCH;  // per-group line buffers, later the output stage
    const int64_t plane = blockIdx.x;
    const int g = threadIdx.x / C::G;
    const int t = threadIdx.x % C::G;
    for (int i = threadIdx.x; i < N; i += C::THREADS) tw[i] = twg[i];
    __syncthreads();

    const float* xp = x + plane * (int64_t)N * N;
    float2* buf = X + g * C::LINE;
    // ---- rows: pair (2p, 2p+1) -> z = a + i b, keep bins k < Kx and their mirrors ----
    for (int base = 0; base < N / 2; base += C::GROUPS) {
        const int pr = base + g;
        const bool active = pr < N / 2;
        const float* ra = xp + (int64_t)(2 * pr) * N;
        const float* rb = ra + N;
        fft::line_fft<N, false>(
            buf, tw, t, active,
            [&](int i) { return active ? make_float2(__ldg(ra + i), __ldg(rb + i)) : make_float2(0.f, 0.f); },
            [&](int k, float2 v) {
                if (k < Kx || k > N - Kx) buf[pad(k)] = v;
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
    for (int base = 0; base < Kx; base += C::GROUPS) {
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
    float2* op = out + plane * (int64_t)My * Kx;
    for (int i = threadIdx.x; i < My * Kx; i += C::THREADS) op[i] = stage[i];
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
            int off_y, float scale, Epilogue ep) {
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
    const float2* ip = in + plane * (int64_t)My * Kx;
    for (int i = threadIdx.x; i < My * Kx; i += C::THREADS) stage[i] = ip[i];
    __syncthreads();
    // ---- columns: kept bins -> full y lines in the column store ----
    for (int base = 0; base < Kx; base += C::GROUPS) {
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
// dense contraction  Y[b, o, m] = sum_i X[b, i, m] W[i, o, m]   (fp32 FMA, optional bf16 operands)
// CTA tile: 8 modes x 16 batch x 64 out; K loop over Ci in chunks of 16.
// Thread (og, mp, bg): o = o0 + og + 16 j (j < 4), modes m0 + 2 mp + {0,1}, b = b0 + 4 bg + {0..3}.
// ------------------------------------------------------------------------------------------
constexpr int kMixThreads = 256;
constexpr int kMixKC = 8;  // Ci chunk

template <bool BF16>
__global__ void __launch_bounds__(kMixThreads, 2)
k_mix_dense(const float2* __restrict__ X, const float2* __restrict__ W, float2* __restrict__ Y, int B, int Ci,
            int Co, int64_t Mt) {
    __shared__ __align__(16) float2 Xs[kMixKC][16][8];  // [i][b][m]
    __shared__ __align__(16) float4 Ws[kMixKC][4][64];  // [i][m pair][o] -> (m even, m odd)
    const int tid = threadIdx.x;
    const int og = tid & 15, mp = (tid >> 4) & 3, bg = tid >> 6;
    const int64_t m0 = (int64_t)blockIdx.x * 8;
    const int b0 = blockIdx.y * 16;
    const int o0 = blockIdx.z * 64;
    float2 acc[4][4][2];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[a][j][0] = acc[a][j][1] = make_float2(0.f, 0.f);

    for (int i0 = 0; i0 < Ci; i0 += kMixKC) {
        // X chunk: 16 i x 16 b x 8 m  (m fastest in global memory)
        for (int e = tid; e < kMixKC * 16 * 8; e += kMixThreads) {
            const int m = e & 7, i = (e >> 3) % kMixKC, b = (e >> 3) / kMixKC;
            float2 v = make_float2(0.f, 0.f);
            if (b0 + b < B && i0 + i < Ci && m0 + m < Mt) v = __ldg(X + ((int64_t)(b0 + b) * Ci + i0 + i) * Mt + m0 + m);
            if constexpr (BF16) v = make_float2(round_bf16(v.x), round_bf16(v.y));
            Xs[i][b][m] = v;
        }
        // W chunk: 16 i x 64 o x 8 m
        for (int e = tid; e < kMixKC * 64 * 4; e += kMixThreads) {
            const int p = e & 3, o = (e >> 2) & 63, i = e >> 8;  // i < kMixKC
            float2 v0 = make_float2(0.f, 0.f), v1 = v0;
            if (i0 + i < Ci && o0 + o < Co) {
                const float2* src = W + ((int64_t)(i0 + i) * Co + o0 + o) * Mt + m0 + 2 * p;
                if (m0 + 2 * p < Mt) v0 = __ldg(src);
                if (m0 + 2 * p + 1 < Mt) v1 = __ldg(src + 1);
            }
            if constexpr (BF16) {
                v0 = make_float2(round_bf16(v0.x), round_bf16(v0.y));
                v1 = make_float2(round_bf16(v1.x), round_bf16(v1.y));
            }
            Ws[i][p][o] = make_float4(v0.x, v0.y, v1.x, v1.y);
        }
        __syncthreads();
#pragma unroll 2
        for (int i = 0; i < kMixKC; ++i) {
            float4 xv[4], wv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) xv[a] = *reinterpret_cast<const float4*>(&Xs[i][4 * bg + a][2 * mp]);
#pragma unroll
            for (int j = 0; j < 4; ++j) wv[j] = Ws[i][mp][og + 16 * j];
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
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int b = b0 + 4 * bg + a;
        if (b >= B) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int o = o0 + og + 16 * j;
            if (o >= Co) continue;
            float2* dst = Y + ((int64_t)b * Co + o) * Mt + m0 + 2 * mp;
            if (m0 + 2 * mp < Mt) dst[0] = acc[a][j][0];
            if (m0 + 2 * mp + 1 < Mt) dst[1] = acc[a][j][1];
        }
    }
}

constexpr size_t kSmemLimit = 227 * 1024;

// per-device "dynamic shared memory limit raised" bits, one word per kernel instantiation
std::atomic<uint64_t> g_attr_done[8];

template <class K>
cudaError_t ensure_smem_attr(K kernel, int slot, int device) {
    const uint64_t bit = uint64_t(1) << (device & 63);
    if (g_attr_done[slot].load() & bit) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit);
    if (e == cudaSuccess) g_attr_done[slot].fetch_or(bit);
    return e;
}

template <int N>
int32_t run_plane_2d(const Plan& p, const void* x, const void* const* weights, const float* bias,
                     const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s) {
    const nop_spectral_desc& d = p.d;
    const int Kx = (int)d.kept[1], My = (int)d.kept[0];
    const int64_t Lin = d.batch * d.in_channels, Lout = d.batch * d.out_channels;
    const size_t smem = plane_smem_bytes<N>(Kx, My);
    const TwiddleTable* tt = p.table(N);
    float2* Xh = reinterpret_cast<float2*>(ws + p.ws.buf_a);
    float2* Yh = reinterpret_cast<float2*>(ws + p.ws.buf_b);
    cudaError_t err;
    constexpr int slot = fft::ilog2(N) - 7;  // 0, 1, 2 for N = 128, 256, 512
    if ((err = ensure_smem_attr(k_plane_fwd<N>, 2 * slot, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(plane_fwd)");
    if ((err = ensure_smem_attr(k_plane_inv<N>, 2 * slot + 1, p.device)) != cudaSuccess)
        return cuda_fail(err, "cudaFuncSetAttribute(plane_inv)");
    k_plane_fwd<N><<<(unsigned)Lin, PlaneCfg<N>::THREADS, smem, s>>>(
        static_cast<const float*>(x), Xh, tt->f_table, Kx, My, (int)d.fwd_off[0], (float)d.fwd_scale);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "plane_fwd launch");
    if (d.weight_kind == NOP_WEIGHT_DENSE && !d.separable) {
        dim3 grid((unsigned)ceil_div(p.modes_total, 8), (unsigned)ceil_div(d.batch, 16),
                  (unsigned)ceil_div(d.out_channels, 64));
        if (d.precision == NOP_PRECISION_BF16)
            k_mix_dense<true><<<grid, kMixThreads, 0, s>>>(Xh, static_cast<const float2*>(weights[0]), Yh,
                                                           (int)d.batch, (int)d.in_channels, (int)d.out_channels,
                                                           p.modes_total);
        else
            k_mix_dense<false><<<grid, kMixThreads, 0, s>>>(Xh, static_cast<const float2*>(weights[0]), Yh,
                                                            (int)d.batch, (int)d.in_channels, (int)d.out_channels,
                                                            p.modes_total);
        if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "mix_dense launch");
    } else {
        int32_t rc = contract_stage(p, Xh, weights, Yh, ws, s);
        if (rc != NOP_OK) return rc;
    }
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
                                                                       ep);
    if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "plane_inv launch");
    return NOP_OK;
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
    if (d.ndim != 2) return *why = "only 2D planes are fused so far", false;
    const int64_t N = d.n_in[0];
    if (d.n_in[1] != N) return *why = "non-square plane", false;
    if (N != 128 && N != 256 && N != 512) return *why = "plane size not in {128, 256, 512}", false;
    if (d.batch * d.in_channels > 0x7fffffffLL || d.batch * d.out_channels > 0x7fffffffLL)
        return *why = "too many planes for one launch", false;
    const size_t smem = plane_smem_for(N, (int)d.kept[1], (int)d.kept[0]);
    if (smem > kSmemLimit) return *why = "kept modes need more shared memory than a CTA has", false;
    *kind = FastKind::Plane2D;
    return true;
}

size_t fast_workspace_bytes(const Plan& p, WorkspaceLayout* ws) {
    const size_t a = (size_t)p.d.batch * p.d.in_channels * p.modes_total * sizeof(float2);
    const size_t b = (size_t)p.d.batch * p.d.out_channels * p.modes_total * sizeof(float2);
    auto up = [](size_t v) { return (v + 255) / 256 * 256; };
    ws->buf_a = 0;
    ws->buf_b = up(a);
    ws->buf_elems = 0;
    return up(a) + up(b);
}

int32_t fast_launches(const Plan& p) {
    const bool dense = p.d.weight_kind == NOP_WEIGHT_DENSE && !p.d.separable;
    return 2 + (dense ? 1 : contract_launches(p));
}

int32_t fast_forward(const Plan& p, const void* x, const void* const* weights, const float* bias,
                     const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s) {
    switch (p.d.n_in[0]) {
        case 128: return run_plane_2d<128>(p, x, weights, bias, addend, apply_gelu, y, ws, s);
        case 256: return run_plane_2d<256>(p, x, weights, bias, addend, apply_gelu, y, ws, s);
        case 512: return run_plane_2d<512>(p, x, weights, bias, addend, apply_gelu, y, ws, s);
        default: return fail(NOP_E_UNSUPPORTED, "fused engine: unsupported plane size");
    }
}

}  // namespace nop

// Backward of the spectral block: weight and bias gradients from kept spectra.
//
// For y = SpectralConv(x) (neuralop/layers/spectral_convolution.py:417-570) and a real loss L
// with g = dL/dy, torch autograd through rfftn / slicing / the contraction einsum
// (:21-46, separable :49-52) / ifftn + irfft / bias (:567-568) gives
//
//   dL/dW[i, o, t] = d_t * sum_b conj(Xh[b, i, t]) * Gh[b, o, t]        (separable: o = i)
//   dL/dbias[o]    = sum_{b, n} g[b, o, n]
//
// where Xh is the kept spectrum of x as the forward computed it (fwd_scale applied), and
// Gh = inv_scale * (unnormalised DFT of g at the inverse's bins) is the kept spectrum the
// ADJOINT plan's forward computes from g.  d_t = 2 for real data on last-axis bins that the
// inverse real FFT counts twice (0 < bin < n_out/2), else 1: the c2r backward of torch
// (an r2c of g, interior bins doubled).  The bias sum is the DC mode of Gh over inv_scale.
//
// Spectra are read through (q_stride, b_stride, c_stride): element (b, c, t = 8 q + l) at
// q * q_stride + b * b_stride + c * c_stride + l complex elements from the base.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "nop_internal.cuh"
#include "wgrad_tc.cuh"

namespace nop {

static std::atomic<uint64_t> g_wg_attr{0};
static std::atomic<uint64_t> g_wgtc_attr[2];
namespace wg {

constexpr int TI = 32;       // input channels per CTA
constexpr int TO = 32;       // output channels per CTA
constexpr int BK = 8;        // batch rows per pipeline stage
constexpr int THREADS = 256; // thread (l, ot, it): l = tid & 7 mode lane, ot = (tid >> 3) & 3, it = warp
constexpr int GROW = 72;     // float2 per 8 output channels of one lane set (64 + 8 pad: conflict-free reads)
constexpr int XS = BK * TI * 8;   // float2 per X stage
constexpr int GS = BK * 4 * GROW; // float2 per G stage
constexpr size_t SMEM = 2 * (XS + GS) * sizeof(float2);

struct Spec {
    const float2* p;
    int64_t sq, sb, sc;
};

// 8-byte async copy; when !valid nothing is read (src-size 0 zero-fills) and `base`, a valid global
// address, stands in for the out-of-range source
__device__ __forceinline__ void cp_async8(float2* dst, const float2* src, const float2* base, bool valid) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    const int n = valid ? 8 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(valid ? src : base), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// per-mode factor d_t (see the file comment); kl = kept modes of the last axis, nyq = the output's
// Nyquist bin of the last axis (-1 if odd or complex data), dbl = 0 for complex data
__device__ __forceinline__ float mode_factor(int64_t t, int kl, int nyq, int dbl) {
    if (!dbl) return 1.f;
    const int m = (int)(t % kl);
    return (m == 0 || m == nyq) ? 1.f : 2.f;
}

// grid: (mode blocks Q x batch splits S, ceil(Ci / TI), ceil(Co / TO)).  Split s sums batch rows
// [s * bsplit, min(B, (s + 1) * bsplit)).  S == 1: gw = [Ci][Co][Mt] complex64 with the factor d_t;
// S > 1: gw = partial sums [S][Ci][Co][Mt] without it (k_reduce_splits finishes).
__global__ void __launch_bounds__(THREADS, 2)
k_weight_grad(Spec X, Spec G, float2* __restrict__ gw, int B, int Ci, int Co, int64_t Mt, int kl, int nyq, int dbl,
              int64_t Q, int bsplit) {
    extern __shared__ __align__(16) float2 sm[];
    const int tid = threadIdx.x;
    const int l = tid & 7, ot = (tid >> 3) & 3, it = tid >> 5;
    const int64_t q = blockIdx.x % Q;
    const int split = (int)(blockIdx.x / Q);
    const bool partial = gridDim.x > Q;
    const int bbeg = split * bsplit, bend = min(B, bbeg + bsplit);
    const int i0 = blockIdx.y * TI, o0 = blockIdx.z * TO;
    const int64_t t_tid = 8 * q + l;

    // stage loader: X rows (b, i) and G rows (b, o), 8 lanes each; element e of 2048 per operand
    auto load = [&](int stage, int b0) {
        float2* xs = sm + stage * (XS + GS);
        float2* gs = xs + XS;
#pragma unroll
        for (int k = 0; k < XS / THREADS; ++k) {
            const int e = k * THREADS + tid;
            const int ll = e & 7, i = (e >> 3) % TI, b = e / (8 * TI);
            const int64_t t = 8 * q + ll;
            const bool v = b0 + b < bend && i0 + i < Ci && t < Mt;
            cp_async8(xs + e, X.p + q * X.sq + (int64_t)(b0 + b) * X.sb + (int64_t)(i0 + i) * X.sc + ll, X.p, v);
        }
#pragma unroll
        for (int k = 0; k < (BK * TO * 8) / THREADS; ++k) {
            const int e = k * THREADS + tid;
            const int ll = e & 7, o = (e >> 3) % TO, b = e / (8 * TO);
            const int64_t t = 8 * q + ll;
            const bool v = b0 + b < bend && o0 + o < Co && t < Mt;
            cp_async8(gs + b * (4 * GROW) + (o >> 3) * GROW + (o & 7) * 8 + ll,
                      G.p + q * G.sq + (int64_t)(b0 + b) * G.sb + (int64_t)(o0 + o) * G.sc + ll, G.p, v);
        }
        cp_commit();
    };

    float2 acc[4][8];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int s = 0; s < 8; ++s) acc[r][s] = make_float2(0.f, 0.f);

    const int nchunks = (bend - bbeg + BK - 1) / BK;
    if (nchunks > 0) load(0, bbeg);
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) {
            load((c + 1) & 1, bbeg + (c + 1) * BK);
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        const float2* xs = sm + (c & 1) * (XS + GS);
        const float2* gs = xs + XS;
#pragma unroll
        for (int b = 0; b < BK; ++b) {
            float2 xv[4], gv[8];
#pragma unroll
            for (int r = 0; r < 4; ++r) xv[r] = xs[(b * TI + it * 4 + r) * 8 + l];
#pragma unroll
            for (int s = 0; s < 8; ++s) gv[s] = gs[b * (4 * GROW) + ot * GROW + s * 8 + l];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int s = 0; s < 8; ++s) {  // conj(x) * g
                    acc[r][s].x = fmaf(xv[r].x, gv[s].x, fmaf(xv[r].y, gv[s].y, acc[r][s].x));
                    acc[r][s].y = fmaf(xv[r].x, gv[s].y, fmaf(-xv[r].y, gv[s].x, acc[r][s].y));
                }
        }
        __syncthreads();  // the next iteration's load overwrites this stage
    }

    if (t_tid >= Mt) return;
    const float f = partial ? 1.f : mode_factor(t_tid, kl, nyq, dbl);
    float2* out = gw + (partial ? (int64_t)split * Ci * Co * Mt : 0);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int i = i0 + it * 4 + r;
        if (i >= Ci) continue;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int o = o0 + ot * 8 + s;
            if (o < Co) out[((int64_t)i * Co + o) * Mt + t_tid] = make_float2(f * acc[r][s].x, f * acc[r][s].y);
        }
    }
}

// gw[e] = d_t * sum_s part[s][e] over the S batch splits, in split order (deterministic)
__global__ void k_reduce_splits(const float2* __restrict__ part, float2* __restrict__ gw, int64_t n, int S,
                                int64_t Mt, int kl, int nyq, int dbl) {
    const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (e >= n) return;
    float2 a = part[e];
    for (int s = 1; s < S; ++s) {
        const float2 v = part[(int64_t)s * n + e];
        a.x += v.x;
        a.y += v.y;
    }
    const float f = mode_factor(e % Mt, kl, nyq, dbl);
    gw[e] = make_float2(f * a.x, f * a.y);
}

// separable weights: gw = [C][Mt]; one thread per (c, t)
__global__ void k_weight_grad_sep(Spec X, Spec G, float2* __restrict__ gw, int B, int C, int64_t Mt, int kl, int nyq,
                                  int dbl) {
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= (int64_t)C * Mt) return;
    const int64_t t = idx % Mt;
    const int c = (int)(idx / Mt);
    const int64_t q = t >> 3;
    const int l = (int)(t & 7);
    float2 a = make_float2(0.f, 0.f);
    for (int b = 0; b < B; ++b) {
        const float2 xv = X.p[q * X.sq + (int64_t)b * X.sb + (int64_t)c * X.sc + l];
        const float2 gv = G.p[q * G.sq + (int64_t)b * G.sb + (int64_t)c * G.sc + l];
        a.x = fmaf(xv.x, gv.x, fmaf(xv.y, gv.y, a.x));
        a.y = fmaf(xv.x, gv.y, fmaf(-xv.y, gv.x, a.y));
    }
    const float f = mode_factor(t, kl, nyq, dbl);
    gw[idx] = make_float2(f * a.x, f * a.y);
}

// dbias[o] = sum_b Re Gh[b, o, t_dc] / inv_scale (Gh's DC mode is inv_scale * sum_n g)
__global__ void k_bias_grad(Spec G, float* __restrict__ gb, int B, int Co, int64_t t_dc, float inv) {
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= Co) return;
    const int64_t q = t_dc >> 3;
    const int l = (int)(t_dc & 7);
    float a = 0.f;
    for (int b = 0; b < B; ++b) a += G.p[q * G.sq + (int64_t)b * G.sb + (int64_t)o * G.sc + l].x;
    gb[o] = a * inv;
}

}  // namespace wg

int32_t spectrum_layout(const Plan& p, int64_t* q_stride, int64_t* b_stride, int64_t* c_stride, size_t* bytes) {
    const nop_spectral_desc& d = p.d;
    const int64_t C = d.in_channels, Mt = p.modes_total, Q = (Mt + 7) / 8;
    if (p.fast_kind == FastKind::Vol3DSlab) return fail(NOP_E_UNSUPPORTED, "slab plans keep no whole spectrum");
    if (p.fast) {  // mode-blocked [Q][B * C][8]
        *q_stride = d.batch * C * 8;
        *b_stride = C * 8;
        *c_stride = 8;
        *bytes = (size_t)Q * 8 * d.batch * C * sizeof(float2);
    } else {       // generic engine: [B][C][Mt]
        *q_stride = 8;
        *b_stride = C * Mt;
        *c_stride = Mt;
        *bytes = (size_t)d.batch * C * Mt * sizeof(float2);
    }
    return NOP_OK;
}

// batch splits of the dense weight-gradient kernel: enough CTAs for about two waves of 2 CTAs per SM,
// each split at least one pipeline stage of batch rows
static void wg_splits(const Plan& p, int* S, int* bsplit) {
    const nop_spectral_desc& d = p.d;
    const int64_t base = ((p.modes_total + 7) / 8) * ceil_div(d.in_channels, wg::TI) * ceil_div(d.out_channels, wg::TO);
    const int64_t chunks = ceil_div(d.batch, wg::BK);
    const int64_t want = 4 * (int64_t)p.sm_count;
    int64_t s = base >= want ? 1 : std::min<int64_t>(chunks, ceil_div(want, std::max<int64_t>(base, 1)));
    s = std::max<int64_t>(1, std::min<int64_t>(s, 64));
    const int64_t per = ceil_div(chunks, s) * wg::BK;  // batch rows per split, whole stages
    *bsplit = (int)per;
    *S = (int)ceil_div(d.batch, per);
}

size_t weight_grad_workspace(const Plan& p) {
    if (p.d.separable || p.d.batch == 0) return 0;
    int S, bs;
    wg_splits(p, &S, &bs);
    return S > 1 ? (size_t)S * p.d.in_channels * p.d.out_channels * p.modes_total * sizeof(float2) : 0;
}

int32_t weight_grad(const Plan& p, const void* x_spec, const Plan& a, const void* g_spec, void* grad_w,
                    float* grad_bias, void* workspace, size_t workspace_bytes, cudaStream_t s) {
    const nop_spectral_desc& d = p.d;
    const nop_spectral_desc& e = a.d;
    if (e.ndim != d.ndim || e.batch != d.batch || e.in_channels != d.out_channels ||
        e.out_channels != d.in_channels || e.separable != d.separable || e.complex_data != d.complex_data)
        return fail(NOP_E_INVALID, "adjoint plan does not match the forward plan (batch, channels, ndim, kinds)");
    for (int j = 0; j < d.ndim; ++j)
        if (e.kept[j] != d.kept[j] || e.n_in[j] != d.n_out[j] || e.n_out[j] != d.n_in[j] ||
            e.fwd_off[j] != d.inv_off[j] || e.inv_off[j] != d.fwd_off[j])
            return fail(NOP_E_INVALID, "adjoint plan geometry is not the transpose of the forward plan's");
    if (d.batch == 0 || (!grad_w && !grad_bias)) return NOP_OK;
    int64_t xq, xb, xc, gq, gb, gc;
    size_t bytes;
    int32_t rc = spectrum_layout(p, &xq, &xb, &xc, &bytes);
    if (rc != NOP_OK) return rc;
    if ((rc = spectrum_layout(a, &gq, &gb, &gc, &bytes)) != NOP_OK) return rc;
    const wg::Spec X{static_cast<const float2*>(x_spec), xq, xb, xc};
    const wg::Spec G{static_cast<const float2*>(g_spec), gq, gb, gc};
    const int nd = d.ndim;
    const int kl = (int)d.kept[nd - 1];
    const int dbl = d.complex_data ? 0 : 1;
    const int nyq = (!d.complex_data && d.n_out[nd - 1] % 2 == 0) ? (int)(d.n_out[nd - 1] / 2) : -1;
    const int64_t Mt = p.modes_total;
    const int B = (int)d.batch, Ci = (int)d.in_channels, Co = (int)d.out_channels;
    cudaError_t err;
    // tensor cores: both spectra mode-blocked (fused engine), dense weights, contractions on tcgen05, and a
    // shape that keeps them busy -- at least 4 K steps of 8 batch entries and a tile per SM (measured on
    // B200: C2 139.6 -> 82.4 us, C4 78.2 -> 57.9 us; with batch 8 (C5) or few mode blocks (C1, C3) the
    // CUDA-core kernel, which can split the batch, is faster)
    const int64_t tc_tiles = 2 * ((Mt + 7) / 8) * ceil_div(Ci, wgtc::BT) * ceil_div(Co, Co > 32 ? 64 : 32);
    const bool tc_path = grad_w && !d.separable && p.fast && a.fast && p.mix_tc && B >= 32 &&
                         tc_tiles >= p.sm_count;
    if (tc_path) {
        if (!x_spec || !g_spec) return fail(NOP_E_INVALID, "spectra must be non-NULL");
        const int CO = Co > 32 ? 64 : 32;
        wgtc::Problem pr{static_cast<const float2*>(x_spec), static_cast<const float2*>(g_spec),
                         static_cast<float2*>(grad_w), B, Ci, Co, (int)((Mt + 7) / 8), Mt,
                         (int)ceil_div(Ci, wgtc::BT), (int)ceil_div(Co, CO), kl, nyq, dbl};
        const int64_t tiles = 2 * (int64_t)pr.Q * pr.it * pr.ot;
        if (tiles > 0x7fffffffLL) return fail(NOP_E_UNSUPPORTED, "weight gradient tile count exceeds 2^31");
        int* status = status_word(p.device);
        if (!status) return fail(NOP_E_CUDA, "status word of the tensor-core kernels is not available");
        const unsigned grid = (unsigned)(tiles < p.sm_count ? tiles : p.sm_count);
        const uint64_t bit = uint64_t(1) << (p.device & 63);
        auto launch = [&](auto kernel, size_t smem, int slot) -> cudaError_t {
            if (!(g_wgtc_attr[slot].load() & bit)) {
                cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                if (e != cudaSuccess) return e;
                g_wgtc_attr[slot].fetch_or(bit);
            }
            kernel<<<grid, wgtc::THREADS, smem, s>>>(pr, status);
            return cudaGetLastError();
        };
        err = CO == 64 ? launch(wgtc::k_wgrad_tc<64>, tc::Cfg<64, false>::SMEM, 0)
                       : launch(wgtc::k_wgrad_tc<32>, tc::Cfg<32, false>::SMEM, 1);
        if (err != cudaSuccess) return cuda_fail(err, "tensor-core weight gradient launch");
        launch_mark(s);
    } else if (grad_w) {
        if (!x_spec || !g_spec) return fail(NOP_E_INVALID, "spectra must be non-NULL");
        if (d.separable) {
            const int64_t n = (int64_t)Ci * Mt;
            wg::k_weight_grad_sep<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(X, G, static_cast<float2*>(grad_w), B,
                                                                             Ci, Mt, kl, nyq, dbl);
        } else {
            const uint64_t bit = uint64_t(1) << (p.device & 63);
            if (!(g_wg_attr.load() & bit)) {  // dynamic shared memory above 48 KB, once per device
                if ((err = cudaFuncSetAttribute(wg::k_weight_grad, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)wg::SMEM)) != cudaSuccess)
                    return cuda_fail(err, "cudaFuncSetAttribute(weight_grad)");
                g_wg_attr.fetch_or(bit);
            }
            int S, bsplit;
            wg_splits(p, &S, &bsplit);
            const size_t need = weight_grad_workspace(p);
            if (need > 0 && (!workspace || workspace_bytes < need))
                return fail(NOP_E_WORKSPACE, "weight-gradient workspace missing or smaller than "
                                             "nop_spectral_weight_grad_workspace_size");
            const int64_t Q = (Mt + 7) / 8;
            const dim3 grid((unsigned)(Q * S), (unsigned)ceil_div(Ci, wg::TI), (unsigned)ceil_div(Co, wg::TO));
            if (Q * S > 0x7fffffff || grid.y > 65535u || grid.z > 65535u)
                return fail(NOP_E_UNSUPPORTED, "weight gradient grid too large");
            float2* dst = S > 1 ? static_cast<float2*>(workspace) : static_cast<float2*>(grad_w);
            wg::k_weight_grad<<<grid, wg::THREADS, wg::SMEM, s>>>(X, G, dst, B, Ci, Co, Mt, kl, nyq, dbl, Q, bsplit);
            if (S > 1 && (err = cudaGetLastError()) == cudaSuccess) {
                launch_mark(s);
                const int64_t n = (int64_t)Ci * Co * Mt;
                wg::k_reduce_splits<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(dst, static_cast<float2*>(grad_w), n, S,
                                                                              Mt, kl, nyq, dbl);
            }
        }
        if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "weight gradient launch");
        launch_mark(s);
    }
    if (grad_bias) {
        if (!g_spec) return fail(NOP_E_INVALID, "gradient spectrum must be non-NULL");
        // DC mode of the adjoint forward: bin 0 of every axis is kept mode fwd_off (row-major flattening)
        int64_t t_dc = 0;
        for (int j = 0; j < nd; ++j) t_dc = t_dc * e.kept[j] + e.fwd_off[j];
        if (e.fwd_scale == 0.0) return fail(NOP_E_INVALID, "adjoint plan has fwd_scale 0");
        wg::k_bias_grad<<<(unsigned)ceil_div(Co, 128), 128, 0, s>>>(G, grad_bias, B, Co, t_dc,
                                                                     (float)(1.0 / e.fwd_scale));
        if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "bias gradient launch");
        launch_mark(s);
    }
    return NOP_OK;
}

}  // namespace nop

// Generic direct-DFT engine: any transform lengths, 1..4 spatial dims, dense / separable /
// Tucker / CP weights, real or complex data, output resampling.  Each axis transform is a
// truncated DFT evaluated directly (double accumulation, twiddles from a double table), with
// the intermediate spectra in the caller's workspace.  It is the correctness backbone for
// shapes the fused kernels do not cover; the math is the one of SpectralConv.forward
// (neuralop/layers/spectral_convolution.py:417-570) in per-axis form.
#include "nop_internal.cuh"

namespace nop {
namespace {

constexpr int kThreads = 256;

inline unsigned grid_for(int64_t n) { return (unsigned)ceil_div(n, kThreads); }

// forward, real last axis:  out[l, k] = scale * sum_n x[l, n] e^{-2 pi i k n / N},  k < K
__global__ void __launch_bounds__(kThreads)
g_fwd_last_real(const float* __restrict__ x, float2* __restrict__ out, int64_t L, int N, int K,
                const double2* __restrict__ tw, double scale) {
    int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= L * K) return;
    int64_t l = idx / K;
    int k = (int)(idx - l * K);
    const float* row = x + l * (int64_t)N;
    double re = 0.0, im = 0.0;
    int ph = 0;
    for (int n = 0; n < N; ++n) {
        double v = row[n];
        double2 w = tw[ph];
        re += v * w.x;
        im -= v * w.y;
        ph += k;
        if (ph >= N) ph -= N;
    }
    out[idx] = make_float2((float)(re * scale), (float)(im * scale));
}

// forward, complex axis:  in [A, N, R] -> out [A, M, R]
//   out[a, m, r] = scale * sum_n in[a, n, r] e^{-2 pi i u n / N},  u = (m - off) mod N
__global__ void __launch_bounds__(kThreads)
g_axis_fwd(const float2* __restrict__ in, float2* __restrict__ out, int64_t A, int N, int M, int64_t R,
           int off, const double2* __restrict__ tw, double scale) {
    int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= A * M * R) return;
    int64_t r = idx % R;
    int64_t t = idx / R;
    int m = (int)(t % M);
    int64_t a = t / M;
    int u = ((m - off) % N + N) % N;
    const float2* src = in + a * (int64_t)N * R + r;
    double re = 0.0, im = 0.0;
    int ph = 0;
    for (int n = 0; n < N; ++n) {
        float2 v = src[(int64_t)n * R];
        double2 w = tw[ph];  // e^{-i theta} = (c, -s)
        re += (double)v.x * w.x + (double)v.y * w.y;
        im += (double)v.y * w.x - (double)v.x * w.y;
        ph += u;
        if (ph >= N) ph -= N;
    }
    out[idx] = make_float2((float)(re * scale), (float)(im * scale));
}

// inverse, complex axis:  in [A, M, R] -> out [A, Nout, R]
//   out[a, n, r] = scale * sum_m [u < Nout] in[a, m, r] e^{+2 pi i u n / Nout},  u = (m - off) mod Nin
// Optional epilogue (complex data, last axis): real part += bias[channel], channel = (a / chan_div) % C
__global__ void __launch_bounds__(kThreads)
g_axis_inv(const float2* __restrict__ in, float2* __restrict__ out, int64_t A, int M, int Nin, int Nout,
           int64_t R, int off, const double2* __restrict__ tw, double scale, const float* __restrict__ bias,
           int64_t chan_div, int64_t C) {
    int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= A * Nout * R) return;
    int64_t r = idx % R;
    int64_t t = idx / R;
    int n = (int)(t % Nout);
    int64_t a = t / Nout;
    const float2* src = in + a * (int64_t)M * R + r;
    double re = 0.0, im = 0.0;
    for (int m = 0; m < M; ++m) {
        int u = ((m - off) % Nin + Nin) % Nin;
        if (u >= Nout) continue;
        int ph = (int)(((int64_t)u * n) % Nout);
        float2 v = src[(int64_t)m * R];
        double2 w = tw[ph];  // e^{+i theta} = (c, s)
        re += (double)v.x * w.x - (double)v.y * w.y;
        im += (double)v.x * w.y + (double)v.y * w.x;
    }
    float2 o = make_float2((float)(re * scale), (float)(im * scale));
    if (bias) o.x += bias[(a / chan_div) % C];
    out[idx] = o;
}

// inverse, real last axis (Hermitian c2r):  in [L, K] -> y [L, Nout]
//   y[l, n] = scale * sum_{k < Ku} w_k (Re Z_k cos(2 pi k n / Nout) - Im' Z_k sin(2 pi k n / Nout))
//   Ku = min(K, Nout/2 + 1); w_k = 1 for k = 0 and k = Nout/2 (even Nout), else 2;
//   Im' = 0 for the bins in zero_imag.
// Epilogue: v = y + bias[o]; v += addend; v = gelu(v)   (o = (l / rows_per_chan) % C)
__global__ void __launch_bounds__(kThreads)
g_inv_last_real(const float2* __restrict__ in, float* __restrict__ y, int64_t L, int K, int Nout,
                const double2* __restrict__ tw, double scale, int z0, int z1, int z2,
                const float* __restrict__ bias, const float* __restrict__ addend, int apply_gelu,
                int64_t rows_per_chan, int64_t C) {
    int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= L * Nout) return;
    int64_t l = idx / Nout;
    int n = (int)(idx - l * Nout);
    int Ku = K < Nout / 2 + 1 ? K : Nout / 2 + 1;
    const float2* z = in + l * (int64_t)K;
    double acc = 0.0;
    int ph = 0;
    for (int k = 0; k < Ku; ++k) {
        float2 v = z[k];
        double im = (k == z0 || k == z1 || k == z2) ? 0.0 : (double)v.y;
        double wk = (k == 0 || (2 * k == Nout)) ? 1.0 : 2.0;
        double2 w = tw[ph];
        acc += wk * ((double)v.x * w.x - im * w.y);
        ph += n;
        if (ph >= Nout) ph -= Nout;
    }
    float v = (float)(acc * scale);
    if (bias) v += bias[(l / rows_per_chan) % C];
    if (addend) v += addend[idx];
    if (apply_gelu) v = gelu_erf(v);
    y[idx] = v;
}

// ------------------------------------------------------------------------------------------
// contraction kernels (also used by the fused engine for weight kinds it does not fuse)
// ------------------------------------------------------------------------------------------

// dense:      Y[b, o, m] = sum_i X[b, i, m] W[i, o, m]
// separable:  Y[b, c, m] = X[b, c, m] W[c, m]
__global__ void __launch_bounds__(kThreads)
g_mix(const float2* __restrict__ X, const float2* __restrict__ W, float2* __restrict__ Y, int64_t B, int Ci,
      int Co, int64_t Mt, int separable, int bf16) {
    int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= B * Co * Mt) return;
    int64_t m = idx % Mt;
    int64_t t = idx / Mt;
    int o = (int)(t % Co);
    int64_t b = t / Co;
    double re = 0.0, im = 0.0;
    if (separable) {
        float2 xv = X[idx], wv = W[(int64_t)o * Mt + m];
        if (bf16) {
            xv = make_float2(round_bf16(xv.x), round_bf16(xv.y));
            wv = make_float2(round_bf16(wv.x), round_bf16(wv.y));
        }
        re = (double)xv.x * wv.x - (double)xv.y * wv.y;
        im = (double)xv.x * wv.y + (double)xv.y * wv.x;
    } else {
        const float2* xr = X + b * (int64_t)Ci * Mt + m;
        const float2* wr = W + (int64_t)o * Mt + m;
        for (int i = 0; i < Ci; ++i) {
            float2 xv = xr[(int64_t)i * Mt];
            float2 wv = wr[(int64_t)i * Co * Mt];
            if (bf16) {
                xv = make_float2(round_bf16(xv.x), round_bf16(xv.y));
                wv = make_float2(round_bf16(wv.x), round_bf16(wv.y));
            }
            re += (double)xv.x * wv.x - (double)xv.y * wv.y;
            im += (double)xv.x * wv.y + (double)xv.y * wv.x;
        }
    }
    Y[idx] = make_float2((float)re, (float)im);
}

// mode product:  O[p, e, q] = sum_d T[p, d, q] U[e * su_e + d * su_d]
__global__ void __launch_bounds__(kThreads)
g_mode_product(const float2* __restrict__ T, const float2* __restrict__ U, float2* __restrict__ O, int64_t P,
               int D, int E, int64_t Q, int64_t su_e, int64_t su_d) {
    int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= P * E * Q) return;
    int64_t q = idx % Q;
    int64_t t = idx / Q;
    int e = (int)(t % E);
    int64_t p = t / E;
    const float2* tr = T + p * (int64_t)D * Q + q;
    const float2* ur = U + (int64_t)e * su_e;
    double re = 0.0, im = 0.0;
    for (int d = 0; d < D; ++d) {
        float2 a = tr[(int64_t)d * Q];
        float2 b = ur[(int64_t)d * su_d];
        re += (double)a.x * b.x - (double)a.y * b.y;
        im += (double)a.x * b.y + (double)a.y * b.x;
    }
    O[idx] = make_float2((float)re, (float)im);
}

struct CPArgs {
    const float2* lam;                 // [R]
    const float2* uc;                  // [C, R] or null
    const float2* u[NOP_MAX_DIMS];     // [kept_j, R]
    int64_t kept[NOP_MAX_DIMS];
    int ndim;
    int R;
    int64_t rows;                      // C (with uc) or R (without)
    int64_t Mt;
};

// without uc:  out[e, mode] = lam_e prod_j U_j[m_j, e]
// with uc:     out[c, mode] = sum_e lam_e Uc[c, e] prod_j U_j[m_j, e]
__global__ void __launch_bounds__(kThreads) g_cp_weight(CPArgs a, float2* __restrict__ out) {
    int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= a.rows * a.Mt) return;
    int64_t mode = idx % a.Mt;
    int64_t row = idx / a.Mt;
    int64_t mj[NOP_MAX_DIMS];
    int64_t rem = mode;
    for (int j = a.ndim - 1; j >= 0; --j) {
        mj[j] = rem % a.kept[j];
        rem /= a.kept[j];
    }
    int e0 = a.uc ? 0 : (int)row;
    int e1 = a.uc ? a.R : (int)row + 1;
    double re = 0.0, im = 0.0;
    for (int e = e0; e < e1; ++e) {
        double2 acc = make_double2(a.lam[e].x, a.lam[e].y);
        if (a.uc) {
            float2 c = a.uc[row * a.R + e];
            acc = make_double2(acc.x * c.x - acc.y * c.y, acc.x * c.y + acc.y * c.x);
        }
        for (int j = 0; j < a.ndim; ++j) {
            float2 c = a.u[j][mj[j] * a.R + e];
            acc = make_double2(acc.x * c.x - acc.y * c.y, acc.x * c.y + acc.y * c.x);
        }
        re += acc.x;
        im += acc.y;
    }
    out[idx] = make_float2((float)re, (float)im);
}

inline cudaError_t launch_mode_product(const float2* T, const float2* U, float2* O, int64_t P, int64_t D,
                                       int64_t E, int64_t Q, int64_t su_e, int64_t su_d, cudaStream_t s) {
    int64_t n = P * E * Q;
    if (n == 0) return cudaSuccess;
    g_mode_product<<<grid_for(n), kThreads, 0, s>>>(T, U, O, P, (int)D, (int)E, Q, su_e, su_d);
    return cudaGetLastError();
}

inline cudaError_t launch_mix(const float2* X, const float2* W, float2* Y, int64_t B, int64_t Ci, int64_t Co,
                              int64_t Mt, int separable, int bf16, cudaStream_t s) {
    int64_t n = B * Co * Mt;
    if (n == 0) return cudaSuccess;
    g_mix<<<grid_for(n), kThreads, 0, s>>>(X, W, Y, B, (int)Ci, (int)Co, Mt, separable, bf16);
    return cudaGetLastError();
}

}  // namespace

// Tucker core expanded along the spatial modes: core [lead..., r_1..r_d] -> [lead..., kept_1..kept_d]
// (lead = r_in*r_out, or C for the separable layout), by successive mode products that alternate
// between the g and g_tmp workspace regions.
float2* expand_tucker_core(const Plan& p, const float2* core, const void* const* weights, int first_spatial_w,
                           int64_t lead, char* ws, cudaError_t* err, cudaStream_t s) {
    const nop_spectral_desc& d = p.d;
    const int nd = d.ndim;
    const int r0 = d.separable ? 1 : 2;  // index in ranks[] of r_1
    const float2* cur = core;
    float2* bufs[2] = {reinterpret_cast<float2*>(ws + p.ws.g), reinterpret_cast<float2*>(ws + p.ws.g_tmp)};
    int which = 0;
    for (int j = 0; j < nd; ++j) {
        int64_t P = lead;
        for (int i = 0; i < j; ++i) P *= d.kept[i];
        int64_t Q = 1;
        for (int i = j + 1; i < nd; ++i) Q *= d.ranks[r0 + i];
        int64_t rj = d.ranks[r0 + j];
        const float2* U = static_cast<const float2*>(weights[first_spatial_w + j]);
        float2* out = bufs[which];
        *err = launch_mode_product(cur, U, out, P, rj, d.kept[j], Q, rj, 1, s);
        if (*err != cudaSuccess) return nullptr;
        cur = out;
        which ^= 1;
    }
    return const_cast<float2*>(cur);
}

int32_t contract_stage(const Plan& p, const float2* X, const void* const* weights, float2* Y, char* ws,
                       cudaStream_t s) {
    const nop_spectral_desc& d = p.d;
    const int64_t B = d.batch, Ci = d.in_channels, Co = d.out_channels, Mt = p.modes_total;
    const int bf16 = d.precision == NOP_PRECISION_BF16;
    cudaError_t err = cudaSuccess;
    if (d.weight_kind == NOP_WEIGHT_DENSE) {
        err = launch_mix(X, static_cast<const float2*>(weights[0]), Y, B, Ci, Co, Mt, d.separable, bf16, s);
        return err == cudaSuccess ? NOP_OK : cuda_fail(err, "dense contraction launch");
    }
    if (d.weight_kind == NOP_WEIGHT_TUCKER) {
        const float2* core = static_cast<const float2*>(weights[0]);
        if (d.separable) {
            // W = core x_0 U_c x_1 U_1 ... (elementwise weight), then Y = X * W
            const int64_t rc = d.ranks[0];
            int64_t Q = 1;
            for (int j = 0; j < d.ndim; ++j) Q *= d.ranks[1 + j];
            float2* t0 = reinterpret_cast<float2*>(ws + p.ws.xf);
            err = launch_mode_product(core, static_cast<const float2*>(weights[1]), t0, 1, rc, Ci, Q, rc, 1, s);
            if (err != cudaSuccess) return cuda_fail(err, "tucker channel factor");
            float2* W = expand_tucker_core(p, t0, weights, 2, Ci, ws, &err, s);
            if (!W) return cuda_fail(err, "tucker spatial factors");
            err = launch_mix(X, W, Y, B, Ci, Co, Mt, 1, bf16, s);
            return err == cudaSuccess ? NOP_OK : cuda_fail(err, "separable contraction launch");
        }
        // factorized: G = core x_2 U_1 ... (per-mode r_in x r_out), xf = X x_1 U_in^T, z = xf . G, Y = z x_1 U_out
        const int64_t rin = d.ranks[0], rout = d.ranks[1];
        float2* G = expand_tucker_core(p, core, weights, 3, rin * rout, ws, &err, s);
        if (!G) return cuda_fail(err, "tucker spatial factors");
        float2* xf = reinterpret_cast<float2*>(ws + p.ws.xf);
        float2* z = reinterpret_cast<float2*>(ws + p.ws.z);
        err = launch_mode_product(X, static_cast<const float2*>(weights[1]), xf, B, Ci, rin, Mt, 1, rin, s);
        if (err != cudaSuccess) return cuda_fail(err, "tucker input factor");
        err = launch_mix(xf, G, z, B, rin, rout, Mt, 0, bf16, s);
        if (err != cudaSuccess) return cuda_fail(err, "tucker core contraction");
        err = launch_mode_product(z, static_cast<const float2*>(weights[2]), Y, B, rout, Co, Mt, rout, 1, s);
        return err == cudaSuccess ? NOP_OK : cuda_fail(err, "tucker output factor");
    }
    if (d.weight_kind == NOP_WEIGHT_CP) {
        CPArgs a{};
        a.lam = static_cast<const float2*>(weights[0]);
        a.ndim = d.ndim;
        a.R = (int)d.ranks[0];
        a.Mt = Mt;
        const int first_spatial = d.separable ? 2 : 3;
        for (int j = 0; j < d.ndim; ++j) {
            a.u[j] = static_cast<const float2*>(weights[first_spatial + j]);
            a.kept[j] = d.kept[j];
        }
        float2* wd = reinterpret_cast<float2*>(ws + p.ws.g);
        if (d.separable) {
            a.uc = static_cast<const float2*>(weights[1]);
            a.rows = Ci;
            g_cp_weight<<<grid_for(a.rows * Mt), kThreads, 0, s>>>(a, wd);
            if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "cp weight");
            err = launch_mix(X, wd, Y, B, Ci, Co, Mt, 1, bf16, s);
            return err == cudaSuccess ? NOP_OK : cuda_fail(err, "separable contraction launch");
        }
        a.uc = nullptr;
        a.rows = a.R;
        g_cp_weight<<<grid_for(a.rows * Mt), kThreads, 0, s>>>(a, wd);
        if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "cp weight");
        float2* xf = reinterpret_cast<float2*>(ws + p.ws.xf);
        float2* z = reinterpret_cast<float2*>(ws + p.ws.z);
        err = launch_mode_product(X, static_cast<const float2*>(weights[1]), xf, B, Ci, a.R, Mt, 1, a.R, s);
        if (err != cudaSuccess) return cuda_fail(err, "cp input factor");
        err = launch_mix(xf, wd, z, B, a.R, a.R, Mt, 1, bf16, s);
        if (err != cudaSuccess) return cuda_fail(err, "cp diagonal");
        err = launch_mode_product(z, static_cast<const float2*>(weights[2]), Y, B, a.R, Co, Mt, a.R, 1, s);
        return err == cudaSuccess ? NOP_OK : cuda_fail(err, "cp output factor");
    }
    return fail(NOP_E_UNSUPPORTED, "unknown weight kind");
}

int32_t contract_launches(const Plan& p) {
    const nop_spectral_desc& d = p.d;
    if (d.weight_kind == NOP_WEIGHT_DENSE) return 1;
    if (d.weight_kind == NOP_WEIGHT_TUCKER) return d.separable ? d.ndim + 2 : d.ndim + 3;
    return d.separable ? 2 : 4;
}

int32_t generic_launches(const Plan& p) { return 2 * p.d.ndim + contract_launches(p); }

// ------------------------------------------------------------------------------------------
// generic forward
// ------------------------------------------------------------------------------------------
int64_t generic_buffer_elems(const nop_spectral_desc& d) {
    const int nd = d.ndim;
    int64_t best = 0;
    // forward: after transforming axes j..nd-1 (last first): B*Ci*prod_{i<j} n_in_i * prod_{i>=j} kept_i
    for (int j = nd - 1; j >= 0; --j) {
        int64_t e = d.batch * d.in_channels;
        for (int i = 0; i < j; ++i) e *= d.n_in[i];
        for (int i = j; i < nd; ++i) e *= d.kept[i];
        if (e > best) best = e;
    }
    // inverse: after inverting axes 0..j: B*Co*prod_{i<=j} n_out_i * prod_{i>j} kept_i
    for (int j = 0; j < nd; ++j) {
        int64_t e = d.batch * d.out_channels;
        for (int i = 0; i <= j; ++i) e *= d.n_out[i];
        for (int i = j + 1; i < nd; ++i) e *= d.kept[i];
        if (e > best) best = e;
    }
    return best;
}

int32_t generic_forward(const Plan& p, const void* x, const void* const* weights, const float* bias,
                        const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s, float2* xs) {
    const nop_spectral_desc& d = p.d;
    const int nd = d.ndim;
    const int64_t B = d.batch, Ci = d.in_channels, Co = d.out_channels;
    float2* bufs[2] = {reinterpret_cast<float2*>(ws + p.ws.buf_a), reinterpret_cast<float2*>(ws + p.ws.buf_b)};
    int cur = 0;
    cudaError_t err;

    // ---- forward transforms: last axis first ----
    {
        const int j = nd - 1;
        int64_t L = B * Ci;
        for (int i = 0; i < j; ++i) L *= d.n_in[i];
        const TwiddleTable* t = p.table(d.n_in[j]);
        int64_t n = L * d.kept[j];
        if (!d.complex_data) {
            g_fwd_last_real<<<grid_for(n), kThreads, 0, s>>>(static_cast<const float*>(x), bufs[cur], L,
                                                             (int)d.n_in[j], (int)d.kept[j], t->d_table,
                                                             d.fwd_scale);
        } else {
            g_axis_fwd<<<grid_for(n), kThreads, 0, s>>>(static_cast<const float2*>(x), bufs[cur], L,
                                                        (int)d.n_in[j], (int)d.kept[j], 1, (int)d.fwd_off[j],
                                                        t->d_table, d.fwd_scale);
        }
        if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "forward last-axis launch");
    }
    for (int j = nd - 2; j >= 0; --j) {
        int64_t A = B * Ci;
        for (int i = 0; i < j; ++i) A *= d.n_in[i];
        int64_t R = 1;
        for (int i = j + 1; i < nd; ++i) R *= d.kept[i];
        const TwiddleTable* t = p.table(d.n_in[j]);
        int64_t n = A * d.kept[j] * R;
        g_axis_fwd<<<grid_for(n), kThreads, 0, s>>>(bufs[cur], bufs[cur ^ 1], A, (int)d.n_in[j], (int)d.kept[j],
                                                    R, (int)d.fwd_off[j], t->d_table, 1.0);
        if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "forward axis launch");
        cur ^= 1;
    }

    if (xs) {  // keep the kept input spectrum [B][Ci][Mt] for the caller (the buffers are reused below)
        const size_t bytes = (size_t)B * Ci * p.modes_total * sizeof(float2);
        if ((err = cudaMemcpyAsync(xs, bufs[cur], bytes, cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
            return cuda_fail(err, "spectrum copy");
    }

    // ---- contraction ----
    int32_t rc = contract_stage(p, bufs[cur], weights, bufs[cur ^ 1], ws, s);
    if (rc != NOP_OK) return rc;
    cur ^= 1;

    // ---- inverse transforms: first axis first ----
    const int n_complex_inv = d.complex_data ? nd : nd - 1;
    for (int j = 0; j < n_complex_inv; ++j) {
        int64_t A = B * Co;
        for (int i = 0; i < j; ++i) A *= d.n_out[i];
        int64_t R = 1;
        for (int i = j + 1; i < nd; ++i) R *= d.kept[i];
        const TwiddleTable* t = p.table(d.n_out[j]);
        const bool final_pass = d.complex_data && j == nd - 1;
        float2* dst = final_pass ? static_cast<float2*>(y) : bufs[cur ^ 1];
        int64_t chan_div = 1;
        for (int i = 0; i < nd - 1; ++i) chan_div *= d.n_out[i];
        int64_t n = A * d.n_out[j] * R;
        g_axis_inv<<<grid_for(n), kThreads, 0, s>>>(bufs[cur], dst, A, (int)d.kept[j], (int)d.n_in[j],
                                                    (int)d.n_out[j], R, (int)d.inv_off[j], t->d_table,
                                                    j == 0 ? d.inv_scale : 1.0, final_pass ? bias : nullptr,
                                                    chan_div, Co);
        if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "inverse axis launch");
        cur ^= 1;
    }
    if (!d.complex_data) {
        const int j = nd - 1;
        int64_t rows_per_chan = 1;
        for (int i = 0; i < j; ++i) rows_per_chan *= d.n_out[i];
        int64_t L = B * Co * rows_per_chan;
        const TwiddleTable* t = p.table(d.n_out[j]);
        int zb[3] = {-1, -1, -1};
        for (int i = 0; i < d.n_zero_imag; ++i) zb[i] = (int)d.zero_imag_bins[i];
        int64_t n = L * d.n_out[j];
        g_inv_last_real<<<grid_for(n), kThreads, 0, s>>>(bufs[cur], static_cast<float*>(y), L, (int)d.kept[j],
                                                         (int)d.n_out[j], t->d_table, nd == 1 ? d.inv_scale : 1.0,
                                                         zb[0], zb[1], zb[2], bias, addend, apply_gelu,
                                                         rows_per_chan, Co);
        if ((err = cudaGetLastError()) != cudaSuccess) return cuda_fail(err, "inverse last-axis launch");
    }
    return NOP_OK;
}

}  // namespace nop

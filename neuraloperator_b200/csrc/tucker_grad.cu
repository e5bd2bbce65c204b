// Gradients of the factors of a Tucker-factorized spectral weight (TFNO training).
//
// The reference's TFNO weight is W = core x_0 U_0 x_1 U_1 ... x_{n-1} U_{n-1} (complex; U_0 = U_in,
// U_1 = U_out, then one factor per spatial mode), contracted by `_contract_tucker`
// (neuralop/layers/spectral_convolution.py:76-103); its backward is torch autograd through that einsum.
// Given dL/dW = gw (from nop_spectral_weight_grad), autograd's values are the adjoint products
//
//   dL/dcore = gw x_0 conj(U_0) x_1 conj(U_1) ... x_{n-1} conj(U_{n-1})
//   dL/dU_k  = sum over every mode but k of T_k * conj(core),  T_k = gw x_j conj(U_j) for every j != k
//
// (torch's convention for complex leaves: dL/dRe + i dL/dIm).  The projections of the two halves of the
// modes are shared: A_right = gw projected on the right half of the modes, A_left on the left half, the
// core gradient is A_right projected on the left half, and factor k's T_k is A_right (k in the left
// half) or A_left (k in the right half) projected on the remaining modes of its half.  Two kernels:
//   k_mode_dot   out[p][r][q] = sum_n t[p][n][q] conj(u[n][r])        (one mode at rank size)
//   k_mode_gram  g[x][a]     = sum_{p,q} t[p][x][q] c[p][a][q]         (c = conj(core), two stages: the
//                                                                     reduction order is fixed)
// Every product runs in fp32 with fp32 accumulation on CUDA cores (the tensors are small: the C4
// gradient is 69 MB, the projections a few MB).
#include <cuda_runtime.h>

#include <string>

#include "nop_internal.cuh"

namespace nop {
namespace tg {

constexpr int RB = 16;           // ranks per pass of k_mode_dot
constexpr int THREADS = 256;
constexpr int GA = 16;           // columns a per block of k_mode_gram
constexpr int MAX_MODES = NOP_MAX_DIMS + 2;

__device__ __forceinline__ float2 cfma(float2 a, float2 b, float2 acc) {  // acc + a b
    acc.x = fmaf(a.x, b.x, fmaf(-a.y, b.y, acc.x));
    acc.y = fmaf(a.x, b.y, fmaf(a.y, b.x, acc.y));
    return acc;
}

// out[p][r][q] = sum_n t[p][n][q] conj(u[n][r]); thread = (p, q), ranks r0 .. r0 + RB (grid.y); conj(u) is
// staged in shared memory NC rows at a time
constexpr int NC = 256;
__global__ void __launch_bounds__(THREADS, 2) k_mode_dot(const float2* __restrict__ t, const float2* __restrict__ u,
                                                      float2* __restrict__ out, int64_t P, int N, int64_t Q, int R) {
    __shared__ float2 us[NC * RB];
    const int r0 = blockIdx.y * RB;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = idx < P * Q;
    const int64_t p = live ? idx / Q : 0, q = live ? idx - p * Q : 0;
    float2 acc[RB];
#pragma unroll
    for (int j = 0; j < RB; ++j) acc[j] = make_float2(0.f, 0.f);
    const float2* tp = t + p * N * Q + q;
    for (int n0 = 0; n0 < N; n0 += NC) {
        const int nc = N - n0 < NC ? N - n0 : NC;
        __syncthreads();
        for (int e = threadIdx.x; e < nc * RB; e += blockDim.x) {
            const int n = e / RB, j = e % RB;
            const float2 v = r0 + j < R ? u[(int64_t)(n0 + n) * R + r0 + j] : make_float2(0.f, 0.f);
            us[e] = make_float2(v.x, -v.y);
        }
        __syncthreads();
        if (live)
            for (int n = 0; n < nc; ++n) {
                const float2 tv = tp[(int64_t)(n0 + n) * Q];
#pragma unroll
                for (int j = 0; j < RB; ++j) acc[j] = cfma(tv, us[n * RB + j], acc[j]);
            }
    }
    if (!live) return;
    float2* op = out + (p * R + r0) * Q + q;
#pragma unroll
    for (int j = 0; j < RB; ++j)
        if (r0 + j < R) op[(int64_t)j * Q] = acc[j];
}

// stage 1 of g[x][a] = sum_{p,q} t[p][x][q] c[p][a][q]: block (split s, x, column group) sums the index
// range [s * chunk, (s + 1) * chunk) of the flattened (p, q) space; part[s][x][a] holds the sums
__global__ void __launch_bounds__(THREADS) k_mode_gram(const float2* __restrict__ t, const float2* __restrict__ c,
                                                       float2* __restrict__ part, int64_t P, int X, int A, int64_t Q,
                                                       int64_t chunk) {
    __shared__ float2 red[THREADS][GA + 1];
    const int s = blockIdx.x, x = blockIdx.y, a0 = blockIdx.z * GA;
    const int64_t PQ = P * Q, lo = (int64_t)s * chunk, hi = lo + chunk < PQ ? lo + chunk : PQ;
    float2 acc[GA];
#pragma unroll
    for (int j = 0; j < GA; ++j) acc[j] = make_float2(0.f, 0.f);
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int64_t p = i / Q, q = i - p * Q;
        const float2 tv = t[(p * X + x) * Q + q];
        const float2* cp = c + (p * A + a0) * Q + q;
#pragma unroll
        for (int j = 0; j < GA; ++j)
            if (a0 + j < A) acc[j] = cfma(tv, cp[(int64_t)j * Q], acc[j]);
    }
#pragma unroll
    for (int j = 0; j < GA; ++j) red[threadIdx.x][j] = acc[j];
    __syncthreads();
    for (int w = THREADS / 2; w > 0; w >>= 1) {  // fixed-order tree
        if (threadIdx.x < w)
#pragma unroll
            for (int j = 0; j < GA; ++j) {
                red[threadIdx.x][j].x += red[threadIdx.x + w][j].x;
                red[threadIdx.x][j].y += red[threadIdx.x + w][j].y;
            }
        __syncthreads();
    }
    if (threadIdx.x < GA && a0 + threadIdx.x < A) part[((int64_t)s * X + x) * A + a0 + threadIdx.x] = red[0][threadIdx.x];
}

// stage 2: g[x][a] = sum over splits in order
__global__ void k_gram_sum(const float2* __restrict__ part, float2* __restrict__ g, int S, int XA) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= XA) return;
    float2 acc = make_float2(0.f, 0.f);
    for (int s = 0; s < S; ++s) {
        const float2 v = part[(int64_t)s * XA + i];
        acc.x += v.x;
        acc.y += v.y;
    }
    g[i] = acc;
}

// dims of a tensor: mode sizes; every mode k is either full (d_k) or projected (r_k)
struct Shape {
    int n;
    int64_t s[MAX_MODES];
    int64_t numel() const {
        int64_t v = 1;
        for (int k = 0; k < n; ++k) v *= s[k];
        return v;
    }
};

constexpr int kGramSplits = 64;

struct Plan {
    int n;
    int64_t d[MAX_MODES], r[MAX_MODES];
};

// the order in which a set of modes is projected: the largest reduction (d - r) first, so the tensor
// shrinks as early as possible
int order(const Plan& pl, const int* modes, int m, int* out) {
    for (int i = 0; i < m; ++i) out[i] = modes[i];
    for (int i = 0; i < m; ++i)
        for (int j = i + 1; j < m; ++j)
            if (pl.d[out[j]] - pl.r[out[j]] > pl.d[out[i]] - pl.r[out[i]]) {
                const int tmp = out[i];
                out[i] = out[j];
                out[j] = tmp;
            }
    return m;
}

// project `src` (shape sh) on the modes listed; intermediates ping-pong through b0 / b1, the result lands
// in `dst`; sh becomes the result's shape and *peak the largest intermediate (elements).  Without `run`
// only the shapes are followed (workspace sizing).
int32_t project(const Plan& pl, const float2* const* U, const float2* src, Shape* sh, const int* modes, int m,
                float2* b0, float2* b1, float2* dst, int64_t* peak, cudaStream_t s, bool run) {
    int ord[MAX_MODES];
    order(pl, modes, m, ord);
    const float2* cur = src;
    for (int i = 0; i < m; ++i) {
        const int k = ord[i];
        int64_t P = 1, Q = 1;
        for (int j = 0; j < k; ++j) P *= sh->s[j];
        for (int j = k + 1; j < sh->n; ++j) Q *= sh->s[j];
        const int N = (int)sh->s[k], R = (int)pl.r[k];
        float2* out = i == m - 1 ? dst : ((i & 1) ? b1 : b0);
        if (P * R * Q > *peak) *peak = P * R * Q;
        if (run) {
            const dim3 grid((unsigned)ceil_div(P * Q, THREADS), (unsigned)ceil_div(R, RB));
            k_mode_dot<<<grid, THREADS, 0, s>>>(cur, U[k], out, P, N, Q, R);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return cuda_fail(e, "tucker mode product launch");
        }
        sh->s[k] = R;
        cur = out;
    }
    return NOP_OK;
}

int32_t gram(const float2* t, const Shape& sh, const float2* cc, int k, int A, float2* part, float2* g,
             cudaStream_t s) {
    int64_t P = 1, Q = 1;
    for (int j = 0; j < k; ++j) P *= sh.s[j];
    for (int j = k + 1; j < sh.n; ++j) Q *= sh.s[j];
    const int X = (int)sh.s[k];
    const int64_t chunk = ceil_div(P * Q, kGramSplits);
    const dim3 grid(kGramSplits, X, (unsigned)ceil_div(A, GA));
    k_mode_gram<<<grid, THREADS, 0, s>>>(t, cc, part, P, X, A, Q, chunk);
    k_gram_sum<<<(unsigned)ceil_div((int64_t)X * A, 256), 256, 0, s>>>(part, g, kGramSplits, X * A);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NOP_OK : cuda_fail(e, "tucker mode gram launch");
}

__global__ void k_conj(const float2* __restrict__ a, float2* __restrict__ b, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) b[i] = make_float2(a[i].x, -a[i].y);
}

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

struct Io {
    const float2* U[MAX_MODES];
    const float2 *core, *gw;
    float2 *g_core, *g_fac[MAX_MODES];
    float2 *b[4], *cc, *part;  // workspace: 4 projection buffers, conj(core), gram partials
};

// the whole computation (run) or its shapes only (!run: *peak = largest intermediate in elements)
int32_t orchestrate(const Plan& pl, const Io& io, int64_t* peak, cudaStream_t s, bool run) {
    const int n = pl.n;
    int left[MAX_MODES], right[MAX_MODES], nl = n / 2, nr = n - n / 2;
    for (int k = 0; k < nl; ++k) left[k] = k;
    for (int k = 0; k < nr; ++k) right[k] = nl + k;
    Shape full{n, {}};
    for (int k = 0; k < n; ++k) full.s[k] = pl.d[k];
    int32_t rc;
    float2* const* b = io.b;
    // A_right -> b[2], A_left -> b[3] (scratch b[0], b[1])
    Shape sr = full, sl = full;
    if ((rc = project(pl, io.U, io.gw, &sr, right, nr, b[0], b[1], b[2], peak, s, run)) != NOP_OK) return rc;
    if ((rc = project(pl, io.U, io.gw, &sl, left, nl, b[0], b[1], b[3], peak, s, run)) != NOP_OK) return rc;
    // dL/dcore = A_right projected on the left modes
    Shape sc = sr;
    if ((rc = project(pl, io.U, b[2], &sc, left, nl, b[0], b[1], io.g_core, peak, s, run)) != NOP_OK) return rc;
    if (run) {
        const int64_t rprod = sc.numel();
        k_conj<<<(unsigned)ceil_div(rprod, 256), 256, 0, s>>>(io.core, io.cc, rprod);
    }
    // dL/dU_k: T_k (the other modes of k's half projected) against conj(core) over every mode but k
    for (int k = 0; k < n; ++k) {
        const bool in_left = k < nl;
        const int* half = in_left ? left : right;
        const int hn = in_left ? nl : nr;
        int rest[MAX_MODES], m = 0;
        for (int i = 0; i < hn; ++i)
            if (half[i] != k) rest[m++] = half[i];
        Shape st = in_left ? sr : sl;
        const float2* tk = in_left ? b[2] : b[3];
        if (m > 0) {
            float2* dst = b[(m - 1) & 1];  // not the buffer the last step reads
            if ((rc = project(pl, io.U, tk, &st, rest, m, b[0], b[1], dst, peak, s, run)) != NOP_OK) return rc;
            tk = dst;
        }
        if (run && (rc = gram(tk, st, io.cc, k, (int)pl.r[k], io.part, io.g_fac[k], s)) != NOP_OK) return rc;
    }
    return NOP_OK;
}

struct Ws {
    size_t buf, cc, part, bytes;
};

Ws workspace(const Plan& pl) {
    int64_t peak = 0, amax = 0, xmax = 0, rprod = 1;
    Io none{};
    orchestrate(pl, none, &peak, nullptr, false);
    for (int k = 0; k < pl.n; ++k) {
        amax = pl.r[k] > amax ? pl.r[k] : amax;
        xmax = pl.d[k] > xmax ? pl.d[k] : xmax;
        rprod *= pl.r[k];
    }
    Ws w{};
    w.buf = up256((size_t)peak * sizeof(float2));
    w.cc = up256((size_t)rprod * sizeof(float2));
    w.part = up256((size_t)kGramSplits * xmax * amax * sizeof(float2));
    w.bytes = 4 * w.buf + w.cc + w.part;
    return w;
}

int32_t check(int32_t n, const int64_t* dims, const int64_t* ranks, Plan* pl) {
    if (n < 2 || n > MAX_MODES) return fail(NOP_E_INVALID, "a Tucker weight has 2 to 6 modes");
    if (!dims || !ranks) return fail(NOP_E_INVALID, "dims and ranks must be non-NULL");
    pl->n = n;
    int64_t total = 1;
    for (int k = 0; k < n; ++k) {
        if (dims[k] < 1 || ranks[k] < 1) return fail(NOP_E_INVALID, "mode sizes and ranks must be positive");
        if (dims[k] > 65536 || ranks[k] > 65536)
            return fail(NOP_E_UNSUPPORTED, "mode sizes and ranks above 65536 are not supported");
        total *= dims[k] > ranks[k] ? dims[k] : ranks[k];
        if (total > (int64_t(1) << 40)) return fail(NOP_E_UNSUPPORTED, "the weight is too large");
        pl->d[k] = dims[k];
        pl->r[k] = ranks[k];
    }
    return NOP_OK;
}

}  // namespace tg
}  // namespace nop

using namespace nop;

extern "C" {

int32_t nop_tucker_grads_workspace_size(int32_t n, const int64_t* dims, const int64_t* ranks, size_t* bytes) {
    if (!bytes) return fail(NOP_E_INVALID, "bytes is NULL");
    tg::Plan pl;
    int32_t rc = tg::check(n, dims, ranks, &pl);
    if (rc != NOP_OK) return rc;
    *bytes = tg::workspace(pl).bytes;
    return NOP_OK;
}

int32_t nop_tucker_grads(int32_t n, const int64_t* dims, const int64_t* ranks, const void* core,
                         const void* const* factors, const void* grad_w, void* grad_core, void* const* grad_factors,
                         void* workspace, size_t workspace_bytes, void* stream) {
    tg::Plan pl;
    int32_t rc = tg::check(n, dims, ranks, &pl);
    if (rc != NOP_OK) return rc;
    if (!core || !factors || !grad_w || !grad_core || !grad_factors)
        return fail(NOP_E_INVALID, "core, factors, grad_w and the gradient outputs must be non-NULL");
    for (int k = 0; k < n; ++k)
        if (!factors[k] || !grad_factors[k]) return fail(NOP_E_INVALID, "a factor or factor gradient is NULL");
    const tg::Ws w = tg::workspace(pl);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(NOP_E_WORKSPACE, "workspace missing or smaller than nop_tucker_grads_workspace_size");
    if ((uintptr_t)workspace % 256) return fail(NOP_E_ALIGNMENT, "workspace must be 256-byte aligned");
    char* base = static_cast<char*>(workspace);
    tg::Io io{};
    for (int i = 0; i < 4; ++i) io.b[i] = reinterpret_cast<float2*>(base + i * w.buf);
    io.cc = reinterpret_cast<float2*>(base + 4 * w.buf);
    io.part = reinterpret_cast<float2*>(base + 4 * w.buf + w.cc);
    for (int k = 0; k < n; ++k) {
        io.U[k] = static_cast<const float2*>(factors[k]);
        io.g_fac[k] = static_cast<float2*>(grad_factors[k]);
    }
    io.core = static_cast<const float2*>(core);
    io.gw = static_cast<const float2*>(grad_w);
    io.g_core = static_cast<float2*>(grad_core);
    int64_t peak = 0;
    return tg::orchestrate(pl, io, &peak, static_cast<cudaStream_t>(stream), true);
}

}  // extern "C"

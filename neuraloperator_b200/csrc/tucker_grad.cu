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
//   k_mode_gram  g[x][a]     = sum_{p,q} t[p][x][q] c[p][a][q]         (c = conj(core))
// Every product runs in fp32 with fp32 accumulation on CUDA cores, every sum in a fixed order (the
// results do not depend on scheduling).  The tensors are small -- the C4 gradient is 69 MB, the
// projections a few MB -- so the two passes over gw bound the time.
#include <cuda_runtime.h>

#include <string>

#include "nop_internal.cuh"

namespace nop {
namespace tg {

constexpr int THREADS = 256;
constexpr int MD_THREADS = 256;  // k_mode_dot block
constexpr int NCH = 128;    // rows of conj(u) staged per pass of k_mode_dot
constexpr int MAX_RB = 16;  // ranks per pass of k_mode_dot
constexpr int GX = 64;      // k_gram_part output tile: GX rows x by 16 JA columns a
constexpr int LC = 32;      // summation indices staged per step of k_gram_part
constexpr int MAX_MODES = NOP_MAX_DIMS + 2;

// acc + a b for complex a, b with b given as (b.re, b.im, -b.im, b.re): two packed FMAs
__device__ __forceinline__ float2 cmac(float2 a, float4 b, float2 acc) {
    acc = __ffma2_rn(make_float2(a.x, a.x), make_float2(b.x, b.y), acc);
    return __ffma2_rn(make_float2(a.y, a.y), make_float2(b.z, b.w), acc);
}

__device__ __forceinline__ float4 cexpand(float2 b) { return make_float4(b.x, b.y, -b.y, b.x); }

// out[p][r][q] = sum_n t[p][n][q] conj(u[n][r]).  Thread = one (p, q) column over the whole n sum, RB ranks
// per block, so loads and stores run along q and every output has one owner (fixed summation order).
// Block b takes rank pass b % passes of column tile b / passes: the passes over one tile run side by
// side and read t from L2 after the first.  conj(u) is staged in shared memory NCH rows at a time in the
// expanded form cmac takes; four rows of t are loaded ahead.
template <int RB>
__global__ void __launch_bounds__(MD_THREADS) k_mode_dot(const float2* __restrict__ t, const float2* __restrict__ u,
                                                      float2* __restrict__ out, int64_t P, int N, int64_t Q, int R,
                                                      int passes) {
    __shared__ float4 us[NCH * RB];
    const int r0 = (int)(blockIdx.x % passes) * RB;
    const int64_t PQ = P * Q;
    const int64_t c = (int64_t)(blockIdx.x / passes) * MD_THREADS + threadIdx.x;
    const bool live = c < PQ;
    const int64_t p = live ? c / Q : 0, q = live ? c - p * Q : 0;
    const float2* tp = t + p * N * Q + q;
    float2 acc[RB];
#pragma unroll
    for (int j = 0; j < RB; ++j) acc[j] = make_float2(0.f, 0.f);
    for (int n0 = 0; n0 < N; n0 += NCH) {
        const int nc = N - n0 < NCH ? N - n0 : NCH;
        __syncthreads();
#pragma unroll 4  // several loads in flight before their shared-memory stores
        for (int e = threadIdx.x; e < nc * RB; e += MD_THREADS) {
            const int n = e / RB, j = e % RB;
            const float2 v = r0 + j < R ? u[(int64_t)(n0 + n) * R + r0 + j] : make_float2(0.f, 0.f);
            us[e] = cexpand(make_float2(v.x, -v.y));
        }
        __syncthreads();
        if (!live) continue;
        const float2* tc = tp + (int64_t)n0 * Q;
        int n = 0;
        for (; n + 4 <= nc; n += 4) {
            float2 v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = tc[(int64_t)(n + i) * Q];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < RB; ++j) acc[j] = cmac(v[i], us[(n + i) * RB + j], acc[j]);
        }
        for (; n < nc; ++n) {
            const float2 x = tc[(int64_t)n * Q];
#pragma unroll
            for (int j = 0; j < RB; ++j) acc[j] = cmac(x, us[n * RB + j], acc[j]);
        }
    }
    if (!live) return;
    float2* op = out + (p * R + r0) * Q + q;
#pragma unroll
    for (int j = 0; j < RB; ++j)
        if (r0 + j < R) op[(int64_t)j * Q] = acc[j];
}

// one tile of g[x][a] = sum_l t[p][x][q] c[p][a][q], l = (p, q) flattened, over the index range of split
// blockIdx.x ([s * lper, (s + 1) * lper)); rows x0 .. x0 + GX (blockIdx.y), columns a0 .. a0 + 16 JA
// (blockIdx.z).  Thread (tx, ta) owns x = x0 + tx + 16 i (i < 4), a = a0 + ta + 16 j (j < JA); the partial
// sums go to part[x][a][s] and k_gram_sum adds the splits in order.  The element offsets of each staged
// l are computed once per step (one division per l).
template <int JA>
__global__ void __launch_bounds__(THREADS) k_gram_part(const float2* __restrict__ t, const float2* __restrict__ c,
                                                       float2* __restrict__ part, int64_t P, int X, int A, int64_t Q,
                                                       int64_t lper, int S) {
    constexpr int AT = 16 * JA;
    __shared__ float2 ts[LC][GX + 1];  // padded: the staging stores along l hit distinct banks
    __shared__ float2 cs[LC][AT + 1];
    __shared__ int64_t off_t[LC], off_c[LC];
    const int tx = threadIdx.x & 15, ta = threadIdx.x >> 4;
    const int x0 = blockIdx.y * GX, a0 = blockIdx.z * AT;
    const int64_t L = P * Q, lb = (int64_t)blockIdx.x * lper;
    const int64_t le = lb + lper < L ? lb + lper : L;
    const bool lfast = Q >= 8;  // load order: along l when q runs contiguous, else along x / a
    float2 acc[4][JA];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < JA; ++j) acc[i][j] = make_float2(0.f, 0.f);
    for (int64_t l0 = lb; l0 < le; l0 += LC) {
        __syncthreads();
        if (threadIdx.x < LC) {
            const int64_t l = l0 + threadIdx.x;
            const int64_t pp = l / Q, qq = l - pp * Q;
            off_t[threadIdx.x] = l < le ? pp * X * Q + qq : -1;
            off_c[threadIdx.x] = l < le ? pp * A * Q + qq : -1;
        }
        __syncthreads();
#pragma unroll 4  // several loads in flight before their shared-memory stores
        for (int e = threadIdx.x; e < LC * GX; e += THREADS) {
            const int li = lfast ? e % LC : e / GX, xi = lfast ? e / LC : e % GX;
            const int64_t o = off_t[li];
            ts[li][xi] = o >= 0 && x0 + xi < X ? t[o + (int64_t)(x0 + xi) * Q] : make_float2(0.f, 0.f);
        }
#pragma unroll 4
        for (int e = threadIdx.x; e < LC * AT; e += THREADS) {
            const int li = lfast ? e % LC : e / AT, ai = lfast ? e / LC : e % AT;
            const int64_t o = off_c[li];
            cs[li][ai] = o >= 0 && a0 + ai < A ? c[o + (int64_t)(a0 + ai) * Q] : make_float2(0.f, 0.f);
        }
        __syncthreads();
#pragma unroll 4
        for (int li = 0; li < LC; ++li) {
            float2 tv[4];
            float4 cv[JA];
#pragma unroll
            for (int i = 0; i < 4; ++i) tv[i] = ts[li][tx + 16 * i];
#pragma unroll
            for (int j = 0; j < JA; ++j) cv[j] = cexpand(cs[li][ta + 16 * j]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < JA; ++j) acc[i][j] = cmac(tv[i], cv[j], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < JA; ++j) {
            const int x = x0 + tx + 16 * i, a = a0 + ta + 16 * j;
            if (x < X && a < A) part[((int64_t)x * A + a) * S + blockIdx.x] = acc[i][j];
        }
}

// g[i] = sum over the S splits of part[i][s]: one warp per output, lane k adding splits k, k + 32, ...
// in order, then a fixed butterfly across the lanes
__global__ void k_gram_sum(const float2* __restrict__ part, float2* __restrict__ g, int S, int64_t XA) {
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (i >= XA) return;
    float2 acc = make_float2(0.f, 0.f);
    for (int s = lane; s < S; s += 32) {
        const float2 v = part[i * S + s];
        acc.x += v.x;
        acc.y += v.y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
    }
    if (lane == 0) g[i] = acc;
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
        if (ceil_div(P * Q, MD_THREADS) * ceil_div(R, 4) > INT32_MAX)
            return fail(NOP_E_UNSUPPORTED, "the weight is too large for the mode-product grid");
        if (run) {
            const int64_t passes = ceil_div(R, MAX_RB), per = ceil_div(R, passes);
            const int rb = per <= 4 ? 4 : per <= 8 ? 8 : per <= 12 ? 12 : MAX_RB;
            const int np = (int)ceil_div(R, rb);
            const unsigned grid = (unsigned)(ceil_div(P * Q, MD_THREADS) * np);
            if (rb == 4)
                k_mode_dot<4><<<grid, MD_THREADS, 0, s>>>(cur, U[k], out, P, N, Q, R, np);
            else if (rb == 8)
                k_mode_dot<8><<<grid, MD_THREADS, 0, s>>>(cur, U[k], out, P, N, Q, R, np);
            else if (rb == 12)
                k_mode_dot<12><<<grid, MD_THREADS, 0, s>>>(cur, U[k], out, P, N, Q, R, np);
            else
                k_mode_dot<MAX_RB><<<grid, MD_THREADS, 0, s>>>(cur, U[k], out, P, N, Q, R, np);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return cuda_fail(e, "tucker mode product launch");
        }
        sh->s[k] = R;
        cur = out;
    }
    return NOP_OK;
}

int gram_ja(int A) { return A <= 32 ? 2 : A <= 48 ? 3 : 4; }

// splits of a gram's summation range: about two blocks per SM over all output tiles, LC-aligned ranges
void gram_split(int X, int A, int64_t L, int* S, int64_t* lper) {
    const int64_t tiles = ceil_div(X, GX) * ceil_div(A, 16 * gram_ja(A));
    int64_t splits = ceil_div(296, tiles), most = ceil_div(L, LC);
    splits = splits < most ? splits : most;
    splits = splits < 1 ? 1 : splits;
    *lper = ceil_div(ceil_div(L, splits), LC) * LC;
    *S = (int)ceil_div(L, *lper);
}

// factor k's gradient g[x][a] from T_k (shape sh, mode k full) and conj(core); part: the split sums
// (*part_peak: their element count, for workspace sizing)
int32_t gram(const float2* t, const Shape& sh, const float2* cc, int k, int A, float2* part, float2* g,
             int64_t* part_peak, cudaStream_t s, bool run) {
    int64_t P = 1, Q = 1;
    for (int j = 0; j < k; ++j) P *= sh.s[j];
    for (int j = k + 1; j < sh.n; ++j) Q *= sh.s[j];
    const int X = (int)sh.s[k];
    int S;
    int64_t lper;
    gram_split(X, A, P * Q, &S, &lper);
    if ((int64_t)S * X * A > *part_peak) *part_peak = (int64_t)S * X * A;
    if (!run) return NOP_OK;
    const int ja = gram_ja(A);
    const dim3 grid(S, (unsigned)ceil_div(X, GX), (unsigned)ceil_div(A, 16 * ja));
    if (ja == 2)
        k_gram_part<2><<<grid, THREADS, 0, s>>>(t, cc, part, P, X, A, Q, lper, S);
    else if (ja == 3)
        k_gram_part<3><<<grid, THREADS, 0, s>>>(t, cc, part, P, X, A, Q, lper, S);
    else
        k_gram_part<4><<<grid, THREADS, 0, s>>>(t, cc, part, P, X, A, Q, lper, S);
    k_gram_sum<<<(unsigned)ceil_div((int64_t)X * A * 32, 256), 256, 0, s>>>(part, g, S, (int64_t)X * A);
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
    float2 *b[4], *cc, *part;  // workspace: 4 projection buffers, conj(core), gram split sums
};

// the whole computation (run) or its shapes only (!run: *peak = largest intermediate, *part_peak = largest
// set of gram split sums, in elements)
int32_t orchestrate(const Plan& pl, const Io& io, int64_t* peak, int64_t* part_peak, cudaStream_t s, bool run) {
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
        if ((rc = gram(tk, st, io.cc, k, (int)pl.r[k], io.part, io.g_fac[k], part_peak, s, run)) != NOP_OK) return rc;
    }
    return NOP_OK;
}

struct Ws {
    size_t buf, cc, part, bytes;
};

int32_t workspace(const Plan& pl, Ws* w) {
    int64_t peak = 0, part_peak = 0, rprod = 1;
    Io none{};
    const int32_t rc = orchestrate(pl, none, &peak, &part_peak, nullptr, false);
    if (rc != NOP_OK) return rc;
    for (int k = 0; k < pl.n; ++k) rprod *= pl.r[k];
    w->buf = up256((size_t)peak * sizeof(float2));
    w->cc = up256((size_t)rprod * sizeof(float2));
    w->part = up256((size_t)part_peak * sizeof(float2));
    w->bytes = 4 * w->buf + w->cc + w->part;
    return NOP_OK;
}

int32_t check(int32_t n, const int64_t* dims, const int64_t* ranks, Plan* pl) {
    if (n < 2 || n > MAX_MODES) return fail(NOP_E_INVALID, "a Tucker weight has 2 to 6 modes");
    if (!dims || !ranks) return fail(NOP_E_INVALID, "dims and ranks must be non-NULL");
    pl->n = n;
    int64_t total = 1;
    for (int k = 0; k < n; ++k) {
        if (dims[k] < 1 || ranks[k] < 1) return fail(NOP_E_INVALID, "mode sizes and ranks must be positive");
        if (dims[k] > 65535 || ranks[k] > 65535)
            return fail(NOP_E_UNSUPPORTED, "mode sizes and ranks above 65535 are not supported");
        total *= dims[k] > ranks[k] ? dims[k] : ranks[k];
        if (total > (int64_t(1) << 35)) return fail(NOP_E_UNSUPPORTED, "the weight is too large");
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
    tg::Ws w{};
    if ((rc = tg::workspace(pl, &w)) != NOP_OK) return rc;
    *bytes = w.bytes;
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
    tg::Ws w{};
    if ((rc = tg::workspace(pl, &w)) != NOP_OK) return rc;
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
    int64_t peak = 0, part_peak = 0;
    return tg::orchestrate(pl, io, &peak, &part_peak, static_cast<cudaStream_t>(stream), true);
}

}  // extern "C"

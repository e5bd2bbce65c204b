// Backward of the per-pixel layer chain (training): the gradients torch autograd computes through the
// reference modules of one FNO block after its spectral convolution (linear skip
// neuralop/layers/skip_connections.py:96-127, ChannelMLP neuralop/layers/channel_mlp.py:82-119 with exact
// GELU, SoftGating skip_connections.py:53-94, the GELUs of fno_block.py:339-381), of the lifting with
// GridEmbeddingND's channels (neuralop/models/fno.py:387-396, neuralop/layers/embeddings.py:147-164) and
// of the projection (fno.py:404-406).  Forward (per point, as in chain.cu):
//
//   z0 = W0 x + s,  u = act0(z0)           (skip stage; without it u = [x ; grid])
//   z1 = W1 u + b1, h = GELU(z1)
//   z2 = W2 h + b2 + g x + gb,  y = act2(z2)
//
// Backward, given dy:  dz2 = dy act2'(z2);  dz1 = (W2^T dz2) GELU'(z1);  du = W1^T dz1;
//   dz0 = du act0'(z0) = ds;  dx = W0^T dz0 + g dz2  (without the skip stage dx = du[:Cx] + g dz2);
//   dW2 = sum dz2 h^T, db2 = dgb = sum dz2, dg = sum dz2 x, dW1 = sum dz1 u^T, db1 = sum dz1,
//   dW0 = sum dz0 x^T   (sums over every point of the batch).
//
// A CTA (256 threads, persistent) takes tiles of TP points of one sample.  Everything of a tile lives in
// shared memory as [channel][point] rows (stride TP + 4): x, u, act0'(z0) then dz0, h, GELU'(z1) then dz1,
// dy then dz2; the forward is recomputed from x and s.  Every layer is a tile GEMM on CUDA cores
// (fp32, packed FMAs, 4 x 4 outputs per thread: weights x activation rows for the per-point layers,
// activation rows x activation rows over the tile's points for the weight gradients).  Weight and bias
// gradients accumulate in shared memory over the CTA's tiles (each entry owned by one thread, so the
// order is fixed), are written per CTA, and a second kernel adds the CTAs' sums in CTA order: the
// result does not depend on scheduling.
#include <cuda_runtime.h>

#include <cstdlib>
#include <string>

#include "nop_internal.cuh"

namespace nop {
namespace cbwd {

constexpr int THREADS = 512;
constexpr int MAX_KB = 3;   // 4 x 4 weight-gradient blocks per thread (registers)
constexpr int MAX_C = 128;  // channel counts per slot the backward takes
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr int SMEM_HALF = 113 * 1024;  // two CTAs per SM (228 KB, 1 KB reserved per CTA)

__host__ __device__ constexpr int up4(int v) { return (v + 3) & ~3; }

// sizes, flags and shared-memory offsets (floats) of one backward call
struct Dims {
    int Cx, Cs, nd, K1, Ch, Cy;        // real channel counts (K1 = Cs, or Cx + nd without the skip stage)
    int pX, pS, pK1, pH, pY;           // padded to multiples of 4
    int act0, act2, gate, gbias, skip;
    int TP, ld;                        // points per tile, row stride (TP + 4)
    int nt;                            // threads per CTA (256: two CTAs per SM; 512)
    int oW0, oW1, oW2, oB1, oB2, oG, oGB;        // weights (padded, row-major [out][in]) and vectors
    int nAcc;                                    // per-CTA sums: dW0, dW1, dW2, db1, db2, dg
    int aW0, aW1, aW2, aB1, aB2, aG;             // their offsets inside the accumulator block
    int oX, oU, oA0, oH, oG1, oDZ2;              // tiles ([rows][ld]); oU == oX when u is x itself
    int smem;                                    // bytes
};

struct Ptrs {
    const float *x, *s, *w0, *w1, *b1, *w2, *b2, *g, *gb, *dy;
    float *dx, *ds;
    float* part;  // [CTAs][nAcc] per-CTA sums
    int64_t P, tps, tiles;
    int64_t sp[NOP_MAX_DIMS], goff[NOP_MAX_DIMS];
    float glo[NOP_MAX_DIMS], gstep[NOP_MAX_DIMS];
};

// GELU(z) and GELU'(z) = Phi(z) + z phi(z), with erf from Abramowitz & Stegun eq. 7.1.26 (|error| <=
// 1.5e-7) on x = |z| / sqrt 2, whose exp(-x^2) = exp(-z^2 / 2) also gives phi(z) = exp(-z^2 / 2) / sqrt(2 pi)
__device__ __forceinline__ void gelu_and_slope(float z, float& gv, float& slope) {
    const float ax = fabsf(z) * 0.70710678118654752f;
    float t, e;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, ax, 1.0f)));
    float q = fmaf(t, 1.061405429f, -1.453152027f);
    q = fmaf(t, q, 1.421413741f);
    q = fmaf(t, q, -0.284496736f);
    q = fmaf(t, q, 0.254829592f);
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-(ax * ax) * 1.4426950408889634f));
    const float erf_ax = fmaf(-(q * t), e, 1.0f);
    const float cdf = 0.5f + copysignf(0.5f * erf_ax, z);  // Phi(z)
    gv = z * cdf;
    slope = fmaf(z * 0.3989422804014327f, e, cdf);          // Phi(z) + z phi(z)
}

// C (M x TP) = A (M x K) * B (K x TP): A = weights in shared memory, element (m, k) at a[m * am + k * ak]
// (am / ak select W or W^T); B = an activation tile ([k][point], row stride ld).  4 x 4 outputs per thread
// (4 rows m, 4 consecutive points), tiles dealt round-robin; epi(m0, n0, c) gets c[i] = rows m0 + i as
// float4 over points n0 .. n0 + 3.
template <class Epi>
__device__ __forceinline__ void act_gemm(const float* a, int am, int ak, const float* b, int ld, int M, int K, int TP,
                                         Epi epi) {
    const int tn = TP / 4, tiles = (M / 4) * tn;
    for (int q = threadIdx.x; q < tiles; q += blockDim.x) {
        const int m0 = (q / tn) * 4, n0 = (q % tn) * 4;
        float2 c[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i][0] = c[i][1] = make_float2(0.f, 0.f);
        const float* bp = b + n0;
        const float* ap = a + m0 * am;
        for (int k = 0; k < K; k += 4) {  // K is a multiple of 4: 4 x 4 blocks of A and B per step
            float av[4][4];  // av[kk][i] = A(m0 + i, k + kk)
            if (am == 1) {   // W^T: rows m0 .. m0 + 3 are consecutive for each k
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float4 v = *reinterpret_cast<const float4*>(ap + (k + kk) * ak);
                    av[kk][0] = v.x, av[kk][1] = v.y, av[kk][2] = v.z, av[kk][3] = v.w;
                }
            } else {         // W: k .. k + 3 are consecutive in each row
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 v = *reinterpret_cast<const float4*>(ap + i * am + k);
                    av[0][i] = v.x, av[1][i] = v.y, av[2][i] = v.z, av[3][i] = v.w;
                }
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float4 bv = *reinterpret_cast<const float4*>(bp + (k + kk) * ld);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    c[i][0] = __ffma2_rn(make_float2(av[kk][i], av[kk][i]), make_float2(bv.x, bv.y), c[i][0]);
                    c[i][1] = __ffma2_rn(make_float2(av[kk][i], av[kk][i]), make_float2(bv.z, bv.w), c[i][1]);
                }
            }
        }
        float4 r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = make_float4(c[i][0].x, c[i][0].y, c[i][1].x, c[i][1].y);
        epi(m0, n0, r);
    }
}

// a[i][j] += sum over the tile's points p of d[m0 + i][p] v[nb + j nstep][p] (d, v activation tiles of row
// stride ld): one 4 x 4 block of a weight gradient.  The four columns are nstep apart so that the threads
// of a warp (consecutive nb) read consecutive rows of v: with ld / 4 odd those fall in distinct banks.
__device__ __forceinline__ void wgrad_block(const float* d, const float* v, int ld, int TP, int m0, int nb, int nstep,
                                            float (&a)[16]) {
    float2 c[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) c[i][j] = make_float2(0.f, 0.f);
    for (int p = 0; p < TP; p += 4) {
        float4 dv[4], vv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) dv[i] = *reinterpret_cast<const float4*>(d + (m0 + i) * ld + p);
#pragma unroll
        for (int j = 0; j < 4; ++j) vv[j] = *reinterpret_cast<const float4*>(v + (nb + j * nstep) * ld + p);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                c[i][j] = __ffma2_rn(make_float2(dv[i].x, dv[i].y), make_float2(vv[j].x, vv[j].y), c[i][j]);
                c[i][j] = __ffma2_rn(make_float2(dv[i].z, dv[i].w), make_float2(vv[j].z, vv[j].w), c[i][j]);
            }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) a[i * 4 + j] += c[i][j].x + c[i][j].y;
}

// which weight gradient block q (of all three, dW0's first) is: the operand tiles, its rows m0 .. m0 + 3,
// its columns nb + j N / 4 (j < 4), and its first accumulator index (row stride N)
struct WBlock {
    int which, m0, nb, base, N;
};

__device__ __forceinline__ WBlock wblock(const Dims& D, int q) {
    const int n0b = D.skip ? (D.pS / 4) * (D.pX / 4) : 0, n1b = (D.pH / 4) * (D.pK1 / 4);
    WBlock w{};
    int N, base;
    if (q < n0b) {
        w.which = 0, N = D.pX, base = D.aW0;
    } else if ((q -= n0b) < n1b) {
        w.which = 1, N = D.pK1, base = D.aW1;
    } else {
        q -= n1b;
        w.which = 2, N = D.pH, base = D.aW2;
    }
    w.m0 = (q / (N / 4)) * 4;
    w.nb = q % (N / 4);
    w.base = base;
    w.N = N;
    return w;
}

// sum over the tile's points of d[m][p] (and of d[m][p] v[m][p] when v is given)
__device__ __forceinline__ float row_sum(const float* d, const float* v, int ld, int TP, int m) {
    float2 s = make_float2(0.f, 0.f);
    for (int p = 0; p < TP; p += 4) {
        const float4 a = *reinterpret_cast<const float4*>(d + m * ld + p);
        if (v) {
            const float4 b = *reinterpret_cast<const float4*>(v + m * ld + p);
            s = __ffma2_rn(make_float2(a.x, a.y), make_float2(b.x, b.y), s);
            s = __ffma2_rn(make_float2(a.z, a.w), make_float2(b.z, b.w), s);
        } else {
            s = __fadd2_rn(s, make_float2(a.x + a.z, a.y + a.w));
        }
    }
    return s.x + s.y;
}

__device__ __forceinline__ float4 ld4_or0(const float* p, bool ok) {
    return ok ? __ldg(reinterpret_cast<const float4*>(p)) : make_float4(0.f, 0.f, 0.f, 0.f);
}

__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__device__ __forceinline__ float comp(const float4& v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

// padded row-major copy of W [rows x cols] into [R][C] (zeros outside)
__device__ void load_padded(float* dst, const float* w, int rows, int cols, int R, int C) {
    for (int e = threadIdx.x; e < R * C; e += blockDim.x) {
        const int r = e / C, c = e % C;
        dst[e] = (w && r < rows && c < cols) ? __ldg(w + (int64_t)r * cols + c) : 0.f;
    }
}

// NT threads per CTA: 256 with tiles small enough for two CTAs per SM (one CTA's tile loads and
// barrier waits then overlap the other's arithmetic), 512 where the channels need the larger CTA
template <int KB, int NT>
__global__ void __launch_bounds__(NT, NT == 256 ? 2 : 1) k_chain_bwd(Ptrs P, Dims D) {
    extern __shared__ __align__(16) float sm[];
    const int tid = threadIdx.x, TP = D.TP, ld = D.ld;
    float* W0 = sm + D.oW0;
    float* W1 = sm + D.oW1;
    float* W2 = sm + D.oW2;
    float* vb1 = sm + D.oB1;
    float* vb2 = sm + D.oB2;
    float* vg = sm + D.oG;
    float* vgb = sm + D.oGB;
    float* X = sm + D.oX;
    float* U = sm + D.oU;
    float* A0 = sm + D.oA0;
    float* H = sm + D.oH;
    float* G1 = sm + D.oG1;
    float* DZ2 = sm + D.oDZ2;
    if (D.skip) load_padded(W0, P.w0, D.Cs, D.Cx, D.pS, D.pX);
    load_padded(W1, P.w1, D.Ch, D.K1, D.pH, D.pK1);
    load_padded(W2, P.w2, D.Cy, D.Ch, D.pY, D.pH);
    load_padded(vb1, P.b1, 1, D.Ch, 1, D.pH);
    load_padded(vb2, P.b2, 1, D.Cy, 1, D.pY);
    load_padded(vg, D.gate ? P.g : nullptr, 1, D.Cy, 1, D.pY);
    load_padded(vgb, D.gbias ? P.gb : nullptr, 1, D.Cy, 1, D.pY);
    float accw[KB][16];  // this thread's weight-gradient blocks tid, tid + NT, ...
#pragma unroll
    for (int k = 0; k < KB; ++k)
#pragma unroll
        for (int i = 0; i < 16; ++i) accw[k][i] = 0.f;
    float accv = 0.f;    // and its bias / gate entry (vector item tid)
    for (int i = D.oX + tid; i < D.smem / 4; i += NT) sm[i] = 0.f;  // tiles: padding rows stay zero
    __syncthreads();

    const int nq = TP / 4;
    const int nblk = (D.skip ? (D.pS / 4) * (D.pX / 4) : 0) + (D.pH / 4) * (D.pK1 / 4) + (D.pY / 4) * (D.pH / 4);
    const int nvec = D.pH + D.pY + (D.gate ? D.pY : 0);
    for (int64_t t = blockIdx.x; t < P.tiles; t += gridDim.x) {
        const int64_t b = t / P.tps;
        const int64_t p0 = (t - b * P.tps) * TP;
        const int np = (int)(P.P - p0 < TP ? P.P - p0 : TP);  // valid points (a multiple of 4)

        // ---- 0. x, dy (and the grid channels of the lifting) -> tiles; points past np read as zero.  The
        // copy loops are unrolled so that several 16-byte loads per thread are in flight before their
        // shared-memory stores (the stores cannot alias the global loads) ----
#pragma unroll 4
        for (int e = tid; e < D.Cx * nq; e += NT) {
            const int c = e / nq, n = (e % nq) * 4;
            st4(X + c * ld + n, ld4_or0(P.x + ((int64_t)b * D.Cx + c) * P.P + p0 + n, n < np));
        }
#pragma unroll 4
        for (int e = tid; e < D.Cy * nq; e += NT) {
            const int c = e / nq, n = (e % nq) * 4;
            st4(DZ2 + c * ld + n, ld4_or0(P.dy + ((int64_t)b * D.Cy + c) * P.P + p0 + n, n < np));
        }
        if (D.skip) {  // s into the act0' rows (the skip stage's epilogue reads it and writes act0' in place)
#pragma unroll 4
            for (int e = tid; e < D.Cs * nq; e += NT) {
                const int c = e / nq, n = (e % nq) * 4;
                st4(A0 + c * ld + n, ld4_or0(P.s + ((int64_t)b * D.Cs + c) * P.P + p0 + n, n < np));
            }
        }
        if (!D.skip && D.nd) {
#pragma unroll 4
            for (int e = tid; e < D.Cx * nq; e += NT) {
                const int c = e / nq, n = (e % nq) * 4;
                st4(U + c * ld + n, ld4_or0(P.x + ((int64_t)b * D.Cx + c) * P.P + p0 + n, n < np));
            }
            for (int n = tid; n < TP; n += NT) {
                float crd[NOP_MAX_DIMS] = {0.f, 0.f, 0.f, 0.f};
                if (n < np) {
                    int64_t idx = p0 + n;
                    for (int a = D.nd - 1; a >= 0; --a) {
                        const int64_t q = idx / P.sp[a];
                        crd[a] = P.glo[a] + (float)(idx - q * P.sp[a] + P.goff[a]) * P.gstep[a];
                        idx = q;
                    }
                }
                for (int a = 0; a < D.nd; ++a) U[(D.Cx + a) * ld + n] = crd[a];
            }
        }
        __syncthreads();

        // ---- 1. skip stage: z0 = W0 x + s -> u = act0(z0), act0'(z0) ----
        if (D.skip) {
            act_gemm(W0, D.pX, 1, X, ld, D.pS, D.pX, TP, [&](int m0, int n0, float4 (&r)[4]) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = m0 + i;
                    const float4 sv = ld4(A0 + m * ld + n0);  // s (zero in padding rows and past np)
                    float u[4], sl[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float z = comp(r[i], j) + comp(sv, j);
                        if (D.act0) gelu_and_slope(z, u[j], sl[j]);
                        else u[j] = z, sl[j] = 1.f;
                    }
                    st4(U + m * ld + n0, make_float4(u[0], u[1], u[2], u[3]));
                    st4(A0 + m * ld + n0, make_float4(sl[0], sl[1], sl[2], sl[3]));
                }
            });
            __syncthreads();
        }

        // ---- 2. z1 = W1 u + b1 -> h = GELU(z1), GELU'(z1) ----
        act_gemm(W1, D.pK1, 1, U, ld, D.pH, D.pK1, TP, [&](int m0, int n0, float4 (&r)[4]) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int m = m0 + i;
                float h[4], sl[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) gelu_and_slope(comp(r[i], j) + vb1[m], h[j], sl[j]);
                st4(H + m * ld + n0, make_float4(h[0], h[1], h[2], h[3]));
                st4(G1 + m * ld + n0, make_float4(sl[0], sl[1], sl[2], sl[3]));
            }
        });
        __syncthreads();

        // ---- 3. dz2 = dy act2'(z2), z2 = W2 h + b2 + g x + gb (only with act2) ----
        if (D.act2) {
            act_gemm(W2, D.pH, 1, H, ld, D.pY, D.pH, TP, [&](int m0, int n0, float4 (&r)[4]) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = m0 + i;
                    const float4 xv = D.gate ? ld4(X + m * ld + n0) : make_float4(0.f, 0.f, 0.f, 0.f);
                    float4 dz = ld4(DZ2 + m * ld + n0);
                    float o[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float z = comp(r[i], j) + vb2[m] + vg[m] * comp(xv, j) + vgb[m];
                        float gv, sl;
                        gelu_and_slope(z, gv, sl);
                        o[j] = comp(dz, j) * sl;
                    }
                    st4(DZ2 + m * ld + n0, make_float4(o[0], o[1], o[2], o[3]));
                }
            });
            __syncthreads();
        }

        // ---- 4. dz1 = (W2^T dz2) GELU'(z1), in place of GELU'(z1) ----
        act_gemm(W2, 1, D.pH, DZ2, ld, D.pH, D.pY, TP, [&](int m0, int n0, float4 (&r)[4]) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float* g1 = G1 + (m0 + i) * ld + n0;
                const float4 sl = ld4(g1);
                st4(g1, make_float4(r[i].x * sl.x, r[i].y * sl.y, r[i].z * sl.z, r[i].w * sl.w));
            }
        });
        __syncthreads();

        // ---- 5. du = W1^T dz1: skip stage -> dz0 = du act0'(z0) (= ds); else dx = du[:Cx] + g dz2 ----
        act_gemm(W1, 1, D.pK1, G1, ld, D.pK1, D.pH, TP, [&](int m0, int n0, float4 (&r)[4]) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int m = m0 + i;
                if (D.skip) {
                    float* a0 = A0 + m * ld + n0;
                    const float4 sl = ld4(a0);
                    const float4 dz = make_float4(r[i].x * sl.x, r[i].y * sl.y, r[i].z * sl.z, r[i].w * sl.w);
                    st4(a0, dz);
                    if (P.ds && m < D.Cs && n0 < np) st4(P.ds + ((int64_t)b * D.Cs + m) * P.P + p0 + n0, dz);
                } else if (P.dx && m < D.Cx && n0 < np) {
                    float4 v = r[i];
                    if (D.gate) {
                        const float4 d2 = ld4(DZ2 + m * ld + n0);
                        v = make_float4(fmaf(vg[m], d2.x, v.x), fmaf(vg[m], d2.y, v.y), fmaf(vg[m], d2.z, v.z),
                                        fmaf(vg[m], d2.w, v.w));
                    }
                    st4(P.dx + ((int64_t)b * D.Cx + m) * P.P + p0 + n0, v);
                }
            }
        });
        __syncthreads();

        // ---- 6. dx = W0^T dz0 + g dz2 (skip stage) ----
        if (D.skip && P.dx) {
            act_gemm(W0, 1, D.pX, A0, ld, D.pX, D.pS, TP, [&](int m0, int n0, float4 (&r)[4]) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = m0 + i;
                    if (m >= D.Cx || n0 >= np) continue;
                    float4 v = r[i];
                    if (D.gate) {
                        const float4 d2 = ld4(DZ2 + m * ld + n0);
                        v = make_float4(fmaf(vg[m], d2.x, v.x), fmaf(vg[m], d2.y, v.y), fmaf(vg[m], d2.z, v.z),
                                        fmaf(vg[m], d2.w, v.w));
                    }
                    st4(P.dx + ((int64_t)b * D.Cx + m) * P.P + p0 + n0, v);
                }
            });
        }

        // ---- 7. weight and bias gradients over the tile's points (tiles only read from here on) ----
#pragma unroll
        for (int k = 0; k < KB; ++k) {
            const int q = tid + k * NT;
            if (q >= nblk) break;
            const WBlock w = wblock(D, q);
            const float* dd = w.which == 0 ? A0 : w.which == 1 ? G1 : DZ2;
            const float* vv = w.which == 0 ? X : w.which == 1 ? U : H;
            wgrad_block(dd, vv, ld, TP, w.m0, w.nb, w.N / 4, accw[k]);
        }
        // the vector entries on the last threads, idle in the weight-gradient blocks above when nblk + nvec
        // <= NT (entry r on thread NT - nvec + r)
        if (tid >= NT - nvec) {
            int r = tid - (NT - nvec);
            if (r < D.pH) accv += row_sum(G1, nullptr, ld, TP, r);
            else if ((r -= D.pH) < D.pY) accv += row_sum(DZ2, nullptr, ld, TP, r);
            else accv += row_sum(DZ2, X, ld, TP, r - D.pY);
        }
        __syncthreads();  // the next tile overwrites the tiles
    }
    float* part = P.part + (int64_t)blockIdx.x * D.nAcc;
#pragma unroll
    for (int k = 0; k < KB; ++k) {
        const int q = tid + k * NT;
        if (q >= nblk) break;
        const WBlock w = wblock(D, q);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) part[w.base + (w.m0 + i) * w.N + w.nb + j * (w.N / 4)] = accw[k][i * 4 + j];
    }
    if (tid >= NT - nvec)
        part[D.aB1 + tid - (NT - nvec)] = accv;  // db1, db2, dg are consecutive in the accumulator layout
}

// the gradients: per-CTA sums added in CTA order, unpadded into the callers' arrays
struct Outs {
    float *dw0, *dw1, *db1, *dw2, *db2, *dg, *dgb;
};

__global__ void k_chain_bwd_reduce(const float* __restrict__ part, int ctas, Dims D, Outs o) {
    const int n0 = D.skip ? D.Cs * D.Cx : 0, n1 = D.Ch * D.K1, n2 = D.Cy * D.Ch;
    const int total = n0 + n1 + n2 + D.Ch + 3 * D.Cy;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    int r = i, src;
    float* dst;
    if (r < n0) {
        src = D.aW0 + (r / D.Cx) * D.pX + r % D.Cx;
        dst = o.dw0 ? o.dw0 + r : nullptr;
    } else if ((r -= n0) < n1) {
        src = D.aW1 + (r / D.K1) * D.pK1 + r % D.K1;
        dst = o.dw1 ? o.dw1 + r : nullptr;
    } else if ((r -= n1) < n2) {
        src = D.aW2 + (r / D.Ch) * D.pH + r % D.Ch;
        dst = o.dw2 ? o.dw2 + r : nullptr;
    } else if ((r -= n2) < D.Ch) {
        src = D.aB1 + r;
        dst = o.db1 ? o.db1 + r : nullptr;
    } else if ((r -= D.Ch) < D.Cy) {
        src = D.aB2 + r;
        dst = o.db2 ? o.db2 + r : nullptr;
    } else if ((r -= D.Cy) < D.Cy) {
        src = D.aB2 + r;  // dL/dgb = dL/db2
        dst = (o.dgb && D.gbias) ? o.dgb + r : nullptr;
    } else {
        r -= D.Cy;
        src = D.aG + r;
        dst = (o.dg && D.gate) ? o.dg + r : nullptr;
    }
    if (!dst) return;
    float s = 0.f;
    for (int c = 0; c < ctas; ++c) s += part[(int64_t)c * D.nAcc + src];
    *dst = s;
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
constexpr int MAX_CTAS = 148 * 4;  // per-CTA partial sums in the workspace (grid capped at this)

int32_t check(const nop_chain_desc* d, int64_t* P) {
    if (!d) return fail(NOP_E_INVALID, "descriptor is NULL");
    if (d->abi_version != NOP_ABI_VERSION) return fail(NOP_E_INVALID, "ABI version mismatch");
    if (d->ndim < 1 || d->ndim > NOP_MAX_DIMS) return fail(NOP_E_INVALID, "ndim must be in 1..4");
    if (d->batch < 0) return fail(NOP_E_INVALID, "batch must be >= 0");
    if (d->grid_dims != 0 && d->grid_dims != d->ndim) return fail(NOP_E_INVALID, "grid_dims must be 0 or ndim");
    if (d->x_channels < 1 || d->hidden_channels < 1 || d->out_channels < 1 || d->skip_channels < 0)
        return fail(NOP_E_INVALID, "x_channels, hidden_channels and out_channels must be positive");
    if (d->skip_channels && d->grid_dims)
        return fail(NOP_E_INVALID, "grid channels are appended only without the skip stage");
    if (d->gate && d->x_channels != d->out_channels)
        return fail(NOP_E_INVALID, "the soft-gating skip needs x_channels == out_channels");
    if (d->proj_hidden) return fail(NOP_E_UNSUPPORTED, "the backward takes chains without the projection");
    if (d->x_channels + d->grid_dims > MAX_C || d->skip_channels > MAX_C || d->hidden_channels > MAX_C ||
        d->out_channels > MAX_C)
        return fail(NOP_E_UNSUPPORTED, "the backward takes channel counts up to 128");
    int64_t n = 1;
    for (int j = 0; j < d->ndim; ++j) {
        if (d->spatial[j] < 1) return fail(NOP_E_INVALID, "spatial sizes must be >= 1");
        n *= d->spatial[j];
    }
    if (n % 4) return fail(NOP_E_UNSUPPORTED, "points per sample must be a multiple of 4 (16-byte rows)");
    if (n > 0x7fffff80LL) return fail(NOP_E_UNSUPPORTED, "more than 2^31 points per sample");
    *P = n;
    return NOP_OK;
}

// the layout with the largest tile (256, 128, 64 or 32 points) that fits a CTA's shared memory
bool plan(const nop_chain_desc* d, Dims* out) {
    Dims D{};
    D.Cx = d->x_channels;
    D.Cs = d->skip_channels;
    D.nd = d->grid_dims;
    D.skip = D.Cs > 0;
    D.K1 = D.skip ? D.Cs : D.Cx + D.nd;
    D.Ch = d->hidden_channels;
    D.Cy = d->out_channels;
    D.pX = up4(D.Cx);
    D.pS = up4(D.Cs);
    D.pK1 = up4(D.K1);
    D.pH = up4(D.Ch);
    D.pY = up4(D.Cy);
    D.act0 = d->act_skip ? 1 : 0;
    D.act2 = d->act_out ? 1 : 0;
    D.gate = d->gate ? 1 : 0;
    D.gbias = 0;  // set per call (whether gb is given)
    int off = 0;
    D.oW0 = off;
    off += D.skip ? D.pS * D.pX : 0;
    D.oW1 = off;
    off += D.pH * D.pK1;
    D.oW2 = off;
    off += D.pY * D.pH;
    D.oB1 = off;
    off += D.pH;
    D.oB2 = off;
    off += D.pY;
    D.oG = off;
    off += D.pY;
    D.oGB = off;
    off += D.pY;
    D.aW0 = 0;
    D.aW1 = D.aW0 + (D.skip ? D.pS * D.pX : 0);
    D.aW2 = D.aW1 + D.pH * D.pK1;
    D.aB1 = D.aW2 + D.pY * D.pH;
    D.aB2 = D.aB1 + D.pH;
    D.aG = D.aB2 + D.pY;
    D.nAcc = D.aG + D.pY;  // the per-CTA sums' layout (held in registers in the kernel)
    const int nblk = (D.skip ? (D.pS / 4) * (D.pX / 4) : 0) + (D.pH / 4) * (D.pK1 / 4) + (D.pY / 4) * (D.pH / 4);
    const int nvec = D.pH + 2 * D.pY;
    if (nblk > MAX_KB * THREADS || nvec > THREADS) return false;
    const bool own_u = D.skip || D.nd > 0;
    const int rows = D.pX + (own_u ? D.pK1 : 0) + (D.skip ? D.pS : 0) + 2 * D.pH + D.pY;
    // two CTAs of 256 threads per SM when the weight-gradient blocks and vector entries fit 256 threads
    // and a tile of at least 64 points fits half the SM's shared memory (measured on B200, C5 training:
    // one CTA of 512 threads spent its time in barrier and global-load stalls, issue 34-42% active);
    // else one CTA of 512 threads with the largest tile.  NOP_CHAIN_BWD_NT=512 forces the latter (read
    // at every call, for A/B timing).
    const char* e = std::getenv("NOP_CHAIN_BWD_NT");
    const bool small_ok = nblk <= MAX_KB * 256 && nvec <= 256 && !(e && std::atoi(e) == 512);
    for (int pass = small_ok ? 0 : 1; pass < 2; ++pass)
    for (int tp = 256; tp >= (pass == 0 ? 64 : 32); tp /= 2) {
        const int ld = tp + 4;
        const int bytes = 4 * (off + rows * ld);
        if (bytes > (pass == 0 ? SMEM_HALF : SMEM_LIMIT)) continue;
        D.nt = pass == 0 ? 256 : THREADS;
        D.TP = tp;
        D.ld = ld;
        int o = off;
        D.oX = o;
        o += D.pX * ld;
        if (own_u) {
            D.oU = o;
            o += D.pK1 * ld;
        } else {
            D.oU = D.oX;
        }
        D.oA0 = o;
        o += D.skip ? D.pS * ld : 0;
        D.oH = o;
        o += D.pH * ld;
        D.oG1 = o;
        o += D.pH * ld;
        D.oDZ2 = o;
        o += D.pY * ld;
        D.smem = 4 * o;
        *out = D;
        return true;
    }
    return false;
}

}  // namespace cbwd
}  // namespace nop

using namespace nop;

extern "C" {

int32_t nop_chain_backward_query(const nop_chain_desc* d, size_t* workspace_bytes) {
    int64_t P = 0;
    int32_t rc = cbwd::check(d, &P);
    if (rc != NOP_OK) return rc;
    cbwd::Dims D;
    if (!cbwd::plan(d, &D)) return fail(NOP_E_UNSUPPORTED, "the backward's tiles exceed a CTA's shared memory");
    if (workspace_bytes) *workspace_bytes = (size_t)cbwd::MAX_CTAS * D.nAcc * sizeof(float);
    return NOP_OK;
}

int32_t nop_chain_backward(const nop_chain_desc* d, const nop_chain_operands* o, const nop_chain_grads* g,
                           void* workspace, size_t workspace_bytes, void* stream) {
    int64_t P = 0;
    int32_t rc = cbwd::check(d, &P);
    if (rc != NOP_OK) return rc;
    cbwd::Dims D;
    if (!cbwd::plan(d, &D)) return fail(NOP_E_UNSUPPORTED, "the backward's tiles exceed a CTA's shared memory");
    if (!o || !g) return fail(NOP_E_INVALID, "operands and grads must be non-NULL");
    if (!o->x || !o->w1 || !o->w2 || !g->dy) return fail(NOP_E_INVALID, "x, w1, w2 and dy must be non-NULL");
    if (D.skip && (!o->s || !o->w0)) return fail(NOP_E_INVALID, "s and w0 are needed with skip_channels > 0");
    if (D.gate && !o->g) return fail(NOP_E_INVALID, "g is needed when gate is set");
    for (const void* p : {(const void*)o->x, (const void*)o->s, (const void*)g->dy, (const void*)g->dx,
                          (const void*)g->ds})
        if ((uintptr_t)p % 16) return fail(NOP_E_ALIGNMENT, "x, s, dy, dx and ds must be 16-byte aligned");
    const size_t need = (size_t)cbwd::MAX_CTAS * D.nAcc * sizeof(float);
    if (!workspace || workspace_bytes < need)
        return fail(NOP_E_WORKSPACE, "workspace missing or smaller than nop_chain_backward_query's size");
    if ((uintptr_t)workspace % 256) return fail(NOP_E_ALIGNMENT, "workspace must be 256-byte aligned");
    D.gbias = (D.gate && o->gb) ? 1 : 0;
    cbwd::Ptrs p{};
    p.x = o->x;
    p.s = o->s;
    p.w0 = o->w0;
    p.w1 = o->w1;
    p.b1 = o->b1;
    p.w2 = o->w2;
    p.b2 = o->b2;
    p.g = o->g;
    p.gb = o->gb;
    p.dy = g->dy;
    p.dx = g->dx;
    p.ds = g->ds;
    p.part = static_cast<float*>(workspace);
    p.P = P;
    p.tps = ceil_div(P, D.TP);
    p.tiles = d->batch * p.tps;
    for (int j = 0; j < NOP_MAX_DIMS; ++j) {
        p.sp[j] = j < d->ndim ? d->spatial[j] : 1;
        p.goff[j] = j < d->ndim ? d->grid_offset[j] : 0;
        p.glo[j] = d->grid_lo[j];
        p.gstep[j] = d->grid_step[j];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int dev = 0, sms = 148, per_sm = 1;
    NOP_CUDA_TRY(cudaGetDevice(&dev));
    NOP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int nblk = (D.skip ? (D.pS / 4) * (D.pX / 4) : 0) + (D.pH / 4) * (D.pK1 / 4) + (D.pY / 4) * (D.pH / 4);
    const int kb = (int)ceil_div(nblk, D.nt);
    void (*kernel)(cbwd::Ptrs, cbwd::Dims) =
        D.nt == 256 ? (kb <= 1 ? cbwd::k_chain_bwd<1, 256> : kb == 2 ? cbwd::k_chain_bwd<2, 256> : cbwd::k_chain_bwd<3, 256>)
                    : (kb <= 1 ? cbwd::k_chain_bwd<1, 512> : kb == 2 ? cbwd::k_chain_bwd<2, 512> : cbwd::k_chain_bwd<3, 512>);
    NOP_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, D.smem));
    NOP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, D.nt, D.smem));
    int64_t ctas = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
    if (ctas > cbwd::MAX_CTAS) ctas = cbwd::MAX_CTAS;
    if (ctas > p.tiles) ctas = p.tiles;
    const cbwd::Outs outs{g->dw0, g->dw1, g->db1, g->dw2, g->db2, g->dg, g->dgb};
    const int total = (D.skip ? D.Cs * D.Cx : 0) + D.Ch * D.K1 + D.Cy * D.Ch + D.Ch + 3 * D.Cy;
    if (ctas == 0) {  // empty batch: zero weight gradients
        NOP_CUDA_TRY(cudaMemsetAsync(workspace, 0, (size_t)D.nAcc * sizeof(float), s));
        ctas = 1;
    } else {
        kernel<<<(unsigned)ctas, D.nt, D.smem, s>>>(p, D);
        NOP_CUDA_TRY(cudaGetLastError());
    }
    cbwd::k_chain_bwd_reduce<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(p.part, (int)ctas, D, outs);
    NOP_CUDA_TRY(cudaGetLastError());
    return NOP_OK;
}

}  // extern "C"

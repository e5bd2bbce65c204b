// Per-pixel layer chain of the FNO on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// At every spatial point of x [B, Cx, P] (P = points per sample; s [B, Cs, P] when the skip stage is on):
//
//   u = Cs ? act_skip(W0 x + s) : [x ; grid]        the block's linear skip added to the spectral output
//   h = GELU(W1 u + b1)                              ChannelMLP, first layer
//   y = act_out(W2 h + b2 + g * x + gb)              second layer + soft-gating skip of x (gate)
//   p = GELU(W3 y + b3),  out = W4 p + b4            the projection ChannelMLP (when proj_hidden > 0)
//
// One FNO block after its spectral convolution is a single pass over HBM: read x and s, write y.  The
// last block also evaluates the projection, and the lifting is the chain without the skip stage.
//
// Each layer is a GEMM per tile of 128 points:  D[p][n] = sum_k A[p][k] W[n][k]  (M = 128 points,
// N = output channels padded to 16, K = input channels).  The A operand (activations, one row per
// point) lives in TENSOR MEMORY, written by the thread that owns the point with tcgen05.st (lane p =
// point p, column k = channel k): every epilogue writes the next layer's operand in place, so no
// activation ever passes through shared memory in the MMA's layout.  W (K-major hi / lo images in the
// canonical no-swizzle layout) sits in shared memory for the whole kernel.  fp32 accuracy from tf32
// MMAs by the three-pass split: each operand value v = hi + lo (hi = tf32(v), lo = tf32(v - hi)) and
// D = A_hi W_hi + A_hi W_lo + A_lo W_hi in fp32 (the dropped terms are below 2^-20 relative; the
// activations' hi is v truncated to tf32, st_split16).
//
// Work split: a CTA (one per SM, persistent) holds up to five independent groups of 128 threads; group
// g walks its own tiles and issues its own MMAs (one elected thread), so the epilogue arithmetic of one
// group runs while the MMAs and loads of the others are in flight.  Per tile a group:
//   1. waits for its x tile (TMA box {128 points, Cx channels} -> stash [c][p]) and writes A = x
//      (+ grid coordinates) and, for the gate, the raw x into tensor memory -- or keeps the tile's x in
//      its stash buffer (two buffers per group) or re-reads it from L2 when tensor memory is short; the
//      next tile's x load is issued (into the other buffer);
//   2. skip stage: MMA, wait; u = act(acc + s) -> A (the s stash is free: the next tile's s load);
//   3. fc1 / fc2: MMA(s), wait; h = GELU(acc + b1) -> A; MMA, wait.  A wide hidden layer runs in chunks
//      of NC channels: chunk c's fc2 MMA and chunk c + 1's fc1 MMA are issued together;
//   4. y = act(acc + b2 + g x + gb): stored (coalesced: a warp writes 32 consecutive points of a
//      channel), or written as A of the projection, which repeats step 3 and stores its output.
// Tensor memory per group: the raw-x region (gate), the chunk regions, A (hi | lo) and the accumulator
// (twice as wide in the wide MMA form, layer_mma); the host planner (constexpr, so the FNO
// configurations' layouts are also compiled as constants: FixedLayout) picks the group count, the MMA
// form and the chunk widths that fit 512 columns and 227 KB of shared memory.  Every wait is bounded: on expiry the kernel records NOP_DEVICE_MMA_TIMEOUT in the status
// word, every group leaves its loop at the next group barrier, issued MMAs and loads are drained
// (bounded) and the tensor memory is freed.
#include <cuda.h>

#include <cstdlib>
#include <cstring>
#include <string>

#include "l2_hints.cuh"
#include "mix_tc.cuh"

namespace nop {
namespace chain {

constexpr int TP = 128;          // points per tile (MMA M)
constexpr int GT = 128;          // threads per group: one per point / tensor-memory lane
constexpr int MAX_GROUPS = 5;
constexpr int TMEM_COLS = 512;
constexpr int SMEM_LIMIT = 227 * 1024;

__host__ __device__ constexpr int up8(int v) { return (v + 7) & ~7; }
__host__ __device__ constexpr int up16(int v) { return (v + 15) & ~15; }
__host__ __device__ constexpr int up1k(int v) { return (v + 1023) & ~1023; }

struct Params {
    int64_t P, tiles, tps;          // points per sample, tiles, tiles per sample
    int64_t sp[NOP_MAX_DIMS];       // spatial sizes of this call (row-major point index)
    int64_t goff[NOP_MAX_DIMS];     // index offset of the first point per axis (slabs)
    float glo[NOP_MAX_DIMS], gstep[NOP_MAX_DIMS];
    const float *w0, *w1, *b1, *w2, *b2, *g, *gb, *w3, *b3, *w4, *b4;
    const float* x;  // the block input, re-read for the gate when it is not kept in tensor memory
    float* y;
};

constexpr int kW0 = 1, kW1 = 2, kW2 = 4, kW3 = 8, kW4 = 16, kWAll = 31;  // Layout::wide bits

struct Layout {
    int Kx;                          // A columns written from x (+ grid channels)
    int RX;                          // raw-x columns (gate) or 0
    int gx;                          // 1: the gate re-reads x from L2 instead of keeping it in tensor memory
    int N0, K1, N1, N2, N3, N4;      // padded GEMM sizes (0: stage absent)
    int NC1, NC3;                    // chunk widths (== N1 / N3 when the layer runs whole)
    int tail;                        // 1: the final layer (<= 4 outputs) runs on CUDA cores in the last epilogue
    int Kt;                          // its input width (N1 without, N3 with the projection)
    int KA;                          // columns of each half (hi, lo) of the A region
    int cX, cC1, cH1, cC3, cH3, cA, cD, cols;  // tensor-memory columns relative to the group's base
    int groups;
    int o_w0, o_w1, o_w2, o_w3, o_w4;          // weight images (hi, then lo), shared-memory bytes
    int o_wt;                                  // the CUDA-core final layer's weights, fp32 [4][Kt] (zero padded)
    int o_vec;                                 // b1 [N1], b2 + gb [N2], g [N2], b3 [N3], b4 [N4]
    int o_stash, stash_bytes;                  // per group: x stash (Cx rows), then s stash (Cs rows)
    int o_bar;
    int smem;
    int Cx, Cs, nd, Ch, Cy, Cp, Co;  // real channel counts (Co: rows of W4)
    int act0, act2, gate;            // activation after the skip stage / after fc2, soft-gating skip
    int wide;                        // layers in the wide MMA form (two MMAs per K step instead of three,
                                     // layer_mma): bit k for W_k (kW0 .. kW4)
    int gs;                          // 1: two x stash buffers per group, and the gate reads x from the stash
};

__host__ __device__ inline uint32_t idesc_tf32(int N) {
    // D f32, A and B tf32, both K-major, N >> 3, M >> 4
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TP >> 4) << 24);
}

// byte offset of element (row n, column k) of an N-row K-major operand image (core matrices of 8 rows x
// 16 bytes; K halves of a 32-byte K step 128 B apart, 8-row groups 256 B apart, K steps N * 32 B apart)
__host__ __device__ inline uint32_t kmaj_off(int n, int k, int N) {
    return (k >> 3) * (N * 32) + (n >> 3) * 256 + ((k >> 2) & 1) * 128 + (n & 7) * 16 + (k & 3) * 4;
}

// ------------------------------------------------------------------------------------------------
// device helpers
// ------------------------------------------------------------------------------------------------
// the hi part of an activation's split: v truncated to tf32 (the 13 low mantissa bits cleared, one
// integer operation); lo = v - hi is then exact in fp32 with |lo| < 2^-10 |v|
__device__ __forceinline__ float tf32_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }
__device__ __forceinline__ void group_bar(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(GT) : "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// wait for this thread's tensor-memory loads; the registers are operands so no use moves above it
__device__ __forceinline__ void tmem_wait_ld(float (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                   "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]),
                   "+f"(v[15])
                 :
                 : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

// The CUDA-core final layer: acc[j] += sum_i wt[j][k0 + i] v[i] for the 4 (zero-padded) outputs, as
// pairs of partial sums (even / odd i) with packed FMAs; wt is fp32 [4][Kt] in shared memory (broadcast
// reads, 16-byte aligned: Kt and k0 are multiples of 16)
__device__ __forceinline__ void tail_acc16(float2 (&acc)[4], const float* __restrict__ wt, int Kt, int k0,
                                           const float (&v)[16]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float* w = wt + j * Kt + k0;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            const float4 q = *reinterpret_cast<const float4*>(w + i);
            acc[j] = __ffma2_rn(make_float2(q.x, q.y), make_float2(v[i], v[i + 1]), acc[j]);
            acc[j] = __ffma2_rn(make_float2(q.z, q.w), make_float2(v[i + 2], v[i + 3]), acc[j]);
        }
    }
}

// hi / lo split of 16 values written to two column groups (the A operand's halves).  lo = v - hi is
// exact in fp32; the tensor core reads its top 19 bits (tf32), so lo is not rounded first: its dropped
// low bits are below 2^-20 of v, the order of the lo * lo term the split omits anyway.  Rounding hi to
// nearest instead halves that bound for one more integer operation per value (80-112 values per point):
// measured on B200, the truncating split ran the C5 forward 1.4% faster, and the chain's relative L2
// error against float64 went from 2.4e-7 .. 1.1e-6 to 4.8e-7 .. 1.4e-6 over the parity cases.
__device__ __forceinline__ void st_split16(uint32_t t_hi, uint32_t t_lo, const float (&v)[16]) {
    uint32_t h[16], l[16];
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        const float2 hv = make_float2(tf32_hi(v[j]), tf32_hi(v[j + 1]));
        const float2 lv = __ffma2_rn(hv, make_float2(-1.0f, -1.0f), make_float2(v[j], v[j + 1]));  // exact
        h[j] = __float_as_uint(hv.x);
        h[j + 1] = __float_as_uint(hv.y);
        l[j] = __float_as_uint(lv.x);
        l[j + 1] = __float_as_uint(lv.y);
    }
    tmem_st16(t_hi, h);
    tmem_st16(t_lo, l);
}

// D (tensor memory) += A (tensor memory) * B (shared-memory descriptor), tf32
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        :
        : "r"(d), "r"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

// D (tensor memory) += A (tensor memory) * B, always accumulating (no predicate to evaluate)
__device__ __forceinline__ void mma_ts_acc(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
    asm volatile("tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%4, %5, %6, %7}, 1;" ::"r"(d), "r"(a),
                 "l"(b), "r"(idesc), "r"(0), "r"(0), "r"(0), "r"(0)
                 : "memory");
}

// One layer (or one chunk of one) as three-pass tf32 MMAs: A columns a .. a + K (hi) and a + lo_off ..
// (lo) of the group's tensor memory; W rows row0 .. row0 + N of an Nfull-row image whose K steps start
// at ks0; D columns d .. d + N.  `acc` = 0 clears D first.  Each MMA costs the issuing thread about 55
// cycles whatever N (measured on B200 for N <= 64), so the loop keeps everything else out of the way:
// both weight descriptors are built once and stepped through the K steps by adding to their address
// field (shared-memory byte address / 16 in the low 14 bits; the images stay below 256 KB, so the add
// never carries out of the field).
// `wide`: the weight image holds, per chunk of N rows, the N hi rows followed by the N lo rows (2 Nfull
// rows in all), and each K step is two MMAs instead of three: A_hi [W_hi | W_lo] into D columns
// d .. d + 2N, then A_lo W_hi accumulated into d .. d + N.  The layer's result is then the sum of the two
// column halves (ld_acc16), the same three products for two thirds of the MMA issue cost.
__device__ __forceinline__ void layer_mma(uint32_t tb, int a, int lo_off, int K, uint32_t w_hi, uint32_t w_lo,
                                          int Nfull, int row0, int ks0, int d, int N, bool acc, bool wide) {
    const uint32_t td = tb + (uint32_t)d;
    uint32_t ta = tb + (uint32_t)a;
    const int nk = K / 8;
    if (wide) {
        const uint32_t id2 = idesc_tf32(2 * N), id1 = idesc_tf32(N);
        const uint32_t boff = (uint32_t)(ks0 * 2 * Nfull * 32 + ((2 * row0) >> 3) * 256);
        uint64_t b = tc::smem_desc(w_hi + boff);
        const uint64_t step = (uint64_t)((2 * Nfull * 32) >> 4);
        if (acc) mma_ts_acc(td, ta, b, id2);
        else mma_ts(td, ta, b, id2, 0u);
        mma_ts_acc(td, ta + (uint32_t)lo_off, b, id1);
        for (int ks = 1; ks < nk; ++ks) {
            b += step;
            ta += 8;
            mma_ts_acc(td, ta, b, id2);
            mma_ts_acc(td, ta + (uint32_t)lo_off, b, id1);
        }
        return;
    }
    const uint32_t idesc = idesc_tf32(N);
    const uint32_t boff = (uint32_t)(ks0 * Nfull * 32 + (row0 >> 3) * 256);
    uint64_t bh = tc::smem_desc(w_hi + boff), bl = tc::smem_desc(w_lo + boff);
    const uint64_t step = (uint64_t)((Nfull * 32) >> 4);
    if (acc) mma_ts_acc(td, ta, bh, idesc);
    else mma_ts(td, ta, bh, idesc, 0u);
    mma_ts_acc(td, ta, bl, idesc);
    mma_ts_acc(td, ta + (uint32_t)lo_off, bh, idesc);
    for (int ks = 1; ks < nk; ++ks) {
        bh += step;
        bl += step;
        ta += 8;
        mma_ts_acc(td, ta, bh, idesc);
        mma_ts_acc(td, ta, bl, idesc);
        mma_ts_acc(td, ta + (uint32_t)lo_off, bh, idesc);
    }
}

// 16 accumulator columns col + c0 .. of a layer's result: with `half` > 0 (wide layers) the sum of the
// two column halves, half columns apart
__device__ __forceinline__ void ld_acc16(uint32_t col, int half, int c0, float (&v)[16]) {
    tmem_ld16(col + (uint32_t)c0, v);
    if (half) {
        float w[16];
        tmem_ld16(col + (uint32_t)(half + c0), w);
        tmem_wait_ld(v);
        tmem_wait_ld(w);
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const float2 q = __fadd2_rn(make_float2(v[j], v[j + 1]), make_float2(w[j], w[j + 1]));
            v[j] = q.x;
            v[j + 1] = q.y;
        }
    } else {
        tmem_wait_ld(v);
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(tc::smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(tc::smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// K-major hi / lo images of W [rows x cols] (row-major, out x in) padded with zeros to N x K: two N-row
// images (hi, then lo), or with `wide` one 2N-row image whose chunks of C rows are hi rows followed by
// the same rows' lo parts (layer_mma); the weights are multiplied by `scale` (1, or 0.5 for a layer whose
// input is a GELU computed without its final halving)
__device__ void load_weight(char* sm, int off, const float* w, int rows, int cols, int N, int K, int C, bool wide,
                            float scale) {
    if (N == 0) return;
    float* hi = reinterpret_cast<float*>(sm + off);
    float* lo = reinterpret_cast<float*>(sm + off + 4 * N * K);
    for (int e = threadIdx.x; e < N * K; e += blockDim.x) {
        const int n = e / K, k = e % K;
        const float v = (n < rows && k < cols) ? scale * __ldg(w + (int64_t)n * cols + k) : 0.f;
        const float h = tc::tf32_round(v);
        if (wide) {
            const int r = (n / C) * 2 * C + n % C;
            float* img = reinterpret_cast<float*>(sm + off);
            img[kmaj_off(r, k, 2 * N) / 4] = h;
            img[kmaj_off(r + C, k, 2 * N) / 4] = tc::tf32_round(v - h);
        } else {
            const uint32_t o = kmaj_off(n, k, N) / 4;
            hi[o] = h;
            lo[o] = tc::tf32_round(v - h);
        }
    }
}

__device__ __forceinline__ float vec_or0(const float* v, int i, int n) { return (v && i < n) ? __ldg(v + i) : 0.f; }


// Exact-form GELU, 0.5 v (1 + erf(v / sqrt 2)) = 0.5 (v + |v| erf(|v| / sqrt 2)) (erf is odd), with erf
// from the rational approximation of Abramowitz & Stegun, Handbook of Mathematical Functions (1964),
// eq. 7.1.26 (after Hastings):
//     erf(x) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-x^2),  t = 1 / (1 + p x),  x >= 0,
// |error| <= 1.5e-7; the published p and a1..a5 below.  It is evaluated on y = x sqrt(log2 e), so that
// exp(-x^2) = exp2(-y^2) and t = 1 / (1 + (p / sqrt(log2 e)) y): one reciprocal and one exp2 on the
// special-function unit, the rest FMAs; the odd extension needs no sign manipulation in this form.
// Measured 1.57x the throughput of the erff form on B200 (80 GELUs per point make it the kernel's
// largest instruction cost); against the exact GELU on N(0, 1) inputs the relative L2 error is ~1e-7.
constexpr float kGeluY = 0.849321800288019f;    // sqrt(log2 e) / sqrt 2
constexpr float kGeluP = 0.2727374808792225f;   // p / sqrt(log2 e), p = 0.3275911
constexpr float kA1 = 0.254829592f, kA2 = -0.284496736f, kA3 = 1.421413741f, kA4 = -1.453152027f,
                kA5 = 1.061405429f;

__device__ __forceinline__ float gelu_fast(float v) {
    const float av = fabsf(v);
    const float y = av * kGeluY;
    float t, e;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(y, kGeluP, 1.0f)));
    float ns = fmaf(t, -kA5, -kA4);  // -(a4 + t a5), ... : the negated polynomial
    ns = fmaf(t, ns, -kA3);
    ns = fmaf(t, ns, -kA2);
    ns = fmaf(t, ns, -kA1);
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-(y * y)));
    const float erf_x = fmaf(t * e, ns, 1.0f);
    return 0.5f * fmaf(av, erf_x, v);
}

// gelu_fast of two values with packed fp32x2 arithmetic (the same operations and roundings per lane).
// kHalf = false returns 2 GELU(v) (the final halving left out): where the GELU feeds a layer of the
// chain, its weights are halved instead (exact, and exact through the tf32 split: the results are
// bit-identical), saving a multiply per pair.
template <bool kHalf = true>
__device__ __forceinline__ float2 gelu_fast2(float2 v) {
    const float2 av = make_float2(fabsf(v.x), fabsf(v.y));
    const float2 y = __fmul2_rn(av, make_float2(kGeluY, kGeluY));
    const float2 d = __ffma2_rn(y, make_float2(kGeluP, kGeluP), make_float2(1.0f, 1.0f));
    float2 t, e;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.x) : "f"(d.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.y) : "f"(d.y));
    float2 ns = __ffma2_rn(t, make_float2(-kA5, -kA5), make_float2(-kA4, -kA4));
    ns = __ffma2_rn(t, ns, make_float2(-kA3, -kA3));
    ns = __ffma2_rn(t, ns, make_float2(-kA2, -kA2));
    ns = __ffma2_rn(t, ns, make_float2(-kA1, -kA1));
    const float2 sq = __fmul2_rn(y, y);
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(-sq.x));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(-sq.y));
    const float2 erf_x = __ffma2_rn(__fmul2_rn(t, e), ns, make_float2(1.0f, 1.0f));
    const float2 g2 = __ffma2_rn(av, erf_x, v);
    return kHalf ? __fmul2_rn(g2, make_float2(0.5f, 0.5f)) : g2;
}

// GELU of 16 values in place (pairs); kHalf = false: 2 GELU (gelu_fast2)
template <bool kHalf = true>
__device__ __forceinline__ void gelu16(float (&v)[16]) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        const float2 g = gelu_fast2<kHalf>(make_float2(v[j], v[j + 1]));
        v[j] = g.x;
        v[j + 1] = g.y;
    }
}

// v[j] += a[j] for 16 values (pairs)
__device__ __forceinline__ void add16(float (&v)[16], const float* __restrict__ a) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
        const float4 q = *reinterpret_cast<const float4*>(a + j);
        const float2 s0 = __fadd2_rn(make_float2(v[j], v[j + 1]), make_float2(q.x, q.y));
        const float2 s1 = __fadd2_rn(make_float2(v[j + 2], v[j + 3]), make_float2(q.z, q.w));
        v[j] = s0.x;
        v[j + 1] = s0.y;
        v[j + 2] = s1.x;
        v[j + 3] = s1.y;
    }
}

// ------------------------------------------------------------------------------------------------
// the kernel
// ------------------------------------------------------------------------------------------------
// Instantiated per group count G so each launch gets the registers its thread count allows (4 groups:
// 128 per thread; 3: 168; 2 and 1: 255), which sets how many independent GELU chains the compiler keeps
// in flight per thread.
template <int G, class LT>
__global__ void __launch_bounds__(G * GT, 1)
k_chain(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tms, Params p, Layout Lp,
        int* __restrict__ status) {
    const auto L = LT::get(Lp);  // FixedLayout: every field a compile-time constant
    extern __shared__ __align__(1024) char sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = warp >> 2;                 // group
    const int quad = warp & 3;                 // tensor-memory lane quadrant of this warp
    const int pt = quad * 32 + lane;           // this thread's point in the tile (= its lane)
    // the thread that waits on the group's barriers and issues its copies and MMAs: lane 0 of the group's
    // warp grp % 4, so the groups' leaders sit on different SM sub-partitions (an MMA costs its issuing
    // warp tens of cycles; with every leader on sub-partition 0, one scheduler carried all of them and the
    // C5 lifting took 10.9 ms instead of 9.7, the block chain 11.4 instead of 11.0)
    const bool leader = (tid & (GT - 1)) == 32 * (grp & 3);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.o_bar);
    uint64_t* mbar = bars + 3 * grp;           // MMA completion of this group
    uint64_t* xfull = mbar + 1;                // x stash landed
    uint64_t* sfull = mbar + 2;                // s stash landed
    uint64_t* drain = bars + 3 * L.groups;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* gflag = abort_flag + 1 + grp;  // this group gives up (read after a group barrier)

    if (tid == 0) {
        for (int i = 0; i < 3 * L.groups; ++i) tc::mbar_init(&bars[i], 1);
        tc::mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort_flag = 0;
        for (int i = 0; i < MAX_GROUPS; ++i) abort_flag[1 + i] = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // weights and vectors, once per CTA
    const int K1r = L.Cs ? L.Cs : L.Cx + L.nd;
    // a layer fed by a GELU takes half weights (the GELU is evaluated without its final halving)
    load_weight(sm, L.o_w0, p.w0, L.Cs, L.Cx, L.N0, L.Kx, L.N0, L.wide & kW0, 1.f);
    load_weight(sm, L.o_w1, p.w1, L.Ch, K1r, L.N1, L.K1, L.NC1, L.wide & kW1, (L.Cs && L.act0) ? 0.5f : 1.f);
    if (!(L.tail && !L.Cp)) load_weight(sm, L.o_w2, p.w2, L.Cy, L.Ch, L.N2, L.N1, L.N2, L.wide & kW2, 0.5f);
    load_weight(sm, L.o_w3, p.w3, L.Cp, L.Cy, L.N3, L.N2, L.NC3, L.wide & kW3, L.act2 ? 0.5f : 1.f);
    if (!L.tail) load_weight(sm, L.o_w4, p.w4, L.Co, L.Cp, L.N4, L.N3, L.N4, L.wide & kW4, 0.5f);
    if (L.tail) {  // fp32 [4][Kt], rows past the outputs and columns past the hidden width zero
        float* wt = reinterpret_cast<float*>(sm + L.o_wt);
        const float* src = L.Cp ? p.w4 : p.w2;
        const int rows = L.Cp ? L.Co : L.Cy, cols = L.Cp ? L.Cp : L.Ch;
        const int kt = L.Kt > 0 ? L.Kt : 1;  // (Kt > 0 whenever tail is set)
        for (int e = threadIdx.x; e < 4 * kt; e += blockDim.x) {
            const int r = e / kt, k = e % kt;
            wt[e] = (r < rows && k < cols) ? 0.5f * __ldg(src + (int64_t)r * cols + k) : 0.f;  // GELU-fed
        }
    }
    float* vb1 = reinterpret_cast<float*>(sm + L.o_vec);
    float* vb2 = vb1 + L.N1;
    float* vg = vb2 + L.N2;
    float* vb3 = vg + L.N2;
    float* vb4 = vb3 + L.N3;
    for (int c = tid; c < L.N1; c += blockDim.x) vb1[c] = vec_or0(p.b1, c, L.Ch);
    for (int c = tid; c < L.N2; c += blockDim.x) {
        vb2[c] = vec_or0(p.b2, c, L.Cy) + (L.gate ? vec_or0(p.gb, c, L.Cy) : 0.f);
        vg[c] = L.gate ? vec_or0(p.g, c, L.Cy) : 0.f;
    }
    for (int c = tid; c < L.N3; c += blockDim.x) vb3[c] = vec_or0(p.b3, c, L.Cp);
    for (int c = tid; c < L.N4; c += blockDim.x) vb4[c] = vec_or0(p.b4, c, L.Co);
    {  // zero the stash padding rows of every group (the tensor copies fill only the first Cx / Cs rows)
        const int xr = L.Kx > L.RX ? L.Kx : L.RX;
        const int xpad = (xr - L.Cx) * TP, spad = (L.N0 - L.Cs) * TP;
        for (int g = 0; g < L.groups; ++g) {
            float* xs = reinterpret_cast<float*>(sm + L.o_stash + g * L.stash_bytes);
            float* ss = xs + (L.gs ? 2 : 1) * up1k(xr * TP * 4) / 4;
            for (int e = tid; e < xpad; e += blockDim.x) xs[L.Cx * TP + e] = 0.f;
            if (L.gs)
                for (int e = tid; e < xpad; e += blockDim.x) xs[up1k(xr * TP * 4) / 4 + L.Cx * TP + e] = 0.f;
            for (int e = tid; e < spad; e += blockDim.x) ss[L.Cs * TP + e] = 0.f;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // weight images -> tensor-core reads
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    const uint32_t tb = *tmem_slot + (uint32_t)(grp * L.cols);   // this group's columns, lane 0
    const uint32_t tl = tb + ((uint32_t)(quad * 32) << 16);      // this warp's lane quadrant
    const uint32_t s_w0 = tc::smem_u32(sm + L.o_w0), s_w1 = tc::smem_u32(sm + L.o_w1);
    const uint32_t s_w2 = tc::smem_u32(sm + L.o_w2), s_w3 = tc::smem_u32(sm + L.o_w3);
    const uint32_t s_w4 = tc::smem_u32(sm + L.o_w4);
    const uint32_t lo0 = 4u * L.N0 * L.Kx, lo1 = 4u * L.N1 * L.K1, lo2 = 4u * L.N2 * L.N1;
    const uint32_t lo3 = 4u * L.N3 * L.N2, lo4 = 4u * L.N4 * L.N3;
    const float* xst0 = reinterpret_cast<const float*>(sm + L.o_stash + grp * L.stash_bytes);
    const int xrows = L.Kx > L.RX ? L.Kx : L.RX;       // stash rows read in stage 1 (>= Cx)
    const int xbuf = up1k(xrows * TP * 4) / 4;          // floats per x buffer (1 KB aligned)
    const float* sst = xst0 + (L.gs ? 2 : 1) * xbuf;    // 1 KB aligned (tensor-copy destination)
    const bool ch1 = L.NC1 < L.N1, ch3 = L.N3 > 0 && L.NC3 < L.N3;
    const int nch1 = L.N1 / L.NC1, nch3 = L.N3 ? L.N3 / L.NC3 : 0;
    const uint32_t xbytes = (uint32_t)L.Cx * TP * 4, sbytes = (uint32_t)L.Cs * TP * 4;
    const uint64_t pol = l2::evict_first();
    // x must survive in L2 until the gate reads it, unless the gate reads the stash
    const uint64_t pol_x = (L.gx && !L.gs) ? l2::evict_normal() : pol;
    const int bar_id = 1 + grp;

    auto give_up = [&]() {
        *gflag = 1;
        *abort_flag = 1;
        atomicExch(status, tc::kStatusMmaTimeout);
    };
    // bounded wait of the group's leader (the other threads sleep in the group barrier that follows); an
    // expired wait flags the group, which every thread sees after the next group barrier
    auto wait_bar = [&](uint64_t* b, uint32_t ph) {
        if (leader && !tc::mbar_wait(b, ph, abort_flag)) give_up();
    };
    const int64_t stride = (int64_t)gridDim.x * L.groups;
    int64_t t = (int64_t)blockIdx.x * L.groups + grp;
    const uint32_t tps = (uint32_t)p.tps;
    // the group's tiles alternate between the x buffers (one buffer without gs)
    auto xbuf_of = [&](int it) { return xst0 + ((L.gs && (it & 1)) ? xbuf : 0); };
    auto issue_x = [&](int64_t tt, int it) {
        const uint32_t b = (uint32_t)tt / tps;
        expect_tx(xfull, xbytes);
        tma_load_2d(const_cast<float*>(xbuf_of(it)), &tmx, (int)(((uint32_t)tt - b * tps) * TP), (int)(b * L.Cx),
                    xfull, pol_x);
    };
    auto issue_s = [&](int64_t tt) {
        const uint32_t b = (uint32_t)tt / tps;
        expect_tx(sfull, sbytes);
        tma_load_2d(const_cast<float*>(sst), &tms, (int)(((uint32_t)tt - b * tps) * TP), (int)(b * L.Cs), sfull, pol);
    };
    int x_pending = 0, s_pending = 0;  // loads issued and not yet waited for (leader's count)
    int it = 0;  // this group's tile count (selects the x buffer)
    if (leader && t < p.tiles) {
        issue_x(t, 0);
        ++x_pending;
        if (L.Cs) {
            issue_s(t);
            ++s_pending;
        }
    }
    uint32_t mph = 0, xph = 0, sph = 0;
    bool stop = false;
    // group barrier; false when the group has given up (every thread of the group sees the same flag)
    auto barrier_ok = [&]() -> bool {
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        group_bar(bar_id);
        if (*gflag) {
            stop = true;
            return false;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        return true;
    };
    // the MMAs just issued complete (and, with `s_too`, this tile's s stash has landed); then the group
    // meets, so every thread may read the accumulators
    auto commit_wait = [&](bool s_too) {
        if (leader) tc::mma_commit(mbar);
        wait_bar(mbar, mph);
        mph ^= 1;
        if (s_too) {
            wait_bar(sfull, sph);
            sph ^= 1;
            if (leader) --s_pending;
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        group_bar(bar_id);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    };

    for (; t < p.tiles && !stop; t += stride, ++it) {
        const float* xst = xbuf_of(it);
        const uint32_t b = (uint32_t)t / tps;
        const uint32_t pnt = ((uint32_t)t - b * tps) * TP + pt;  // point index within the sample
        const bool valid = pnt < (uint32_t)p.P;
        const int64_t nt = t + stride;

        // ---- 1. x tile -> A (hi | lo) [+ grid coordinates], raw x for the gate ----
        wait_bar(xfull, xph);
        xph ^= 1;
        if (leader) --x_pending;
        group_bar(bar_id);  // the stash has landed (the leader waited)
        float crd[NOP_MAX_DIMS] = {0.f, 0.f, 0.f, 0.f};
        if (L.nd) {
            uint32_t idx = pnt;
#pragma unroll
            for (int a = NOP_MAX_DIMS - 1; a >= 0; --a) {
                if (a < L.nd) {
                    const uint32_t n = (uint32_t)p.sp[a];
                    const uint32_t q = idx / n;
                    crd[a] = p.glo[a] + (float)((int64_t)(idx - q * n) + p.goff[a]) * p.gstep[a];
                    idx = q;
                }
            }
        }
        for (int c0 = 0; c0 < xrows; c0 += 8) {
            float v[8];
            const float* xc = xst + c0 * TP + pt;
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = xc[j * TP];  // rows past Cx read the zeroed padding
            if (L.nd) {  // grid channels Cx .. Cx + nd - 1 (lifting only)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int a = c0 + j - L.Cx;
                    if (a >= 0 && a < L.nd) v[j] = a == 0 ? crd[0] : a == 1 ? crd[1] : a == 2 ? crd[2] : crd[3];
                }
            }
            if (c0 < L.Kx) {
                uint32_t h[8], l[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {  // scalar: pairing these stash values costs more moves than it saves
                    const float hv = tf32_hi(v[j]);
                    h[j] = __float_as_uint(hv);
                    l[j] = __float_as_uint(v[j] - hv);
                }
                tmem_st8(tl + L.cA + c0, h);
                tmem_st8(tl + L.cA + L.KA + c0, l);
            }
            if (c0 < L.RX) {
                uint32_t r[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) r[j] = __float_as_uint(v[j]);
                tmem_st8(tl + L.cX + c0, r);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // stash reads before the next TMA write
        if (!barrier_ok()) break;
        if (leader) {
            if (nt < p.tiles) {
                issue_x(nt, it + 1);
                ++x_pending;
            }
            if (L.N0)
                layer_mma(tb, L.cA, L.KA, L.Kx, s_w0, s_w0 + lo0, L.N0, 0, 0, L.cD, L.N0, false, L.wide & kW0);
            else
                layer_mma(tb, L.cA, L.KA, L.K1, s_w1, s_w1 + lo1, L.N1, 0, 0, ch1 ? L.cC1 : L.cD, L.NC1, false, L.wide & kW1);
        }
        commit_wait(L.N0 > 0);

        // ---- 2. skip stage: u = act(W0 x + s) -> A ----
        if (L.N0) {
            for (int c0 = 0; c0 < L.N0; c0 += 16) {
                float v[16];
                ld_acc16(tl + L.cD, (L.wide & kW0) ? L.N0 : 0, c0, v);
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                    const int c = c0 + j;  // channels past Cs (padding) add 0
                    const float s0 = sst[c * TP + pt];  // rows past Cs read the zeroed padding
                    const float s1 = sst[(c + 1) * TP + pt];
                    const float2 u = __fadd2_rn(make_float2(v[j], v[j + 1]), make_float2(s0, s1));
                    v[j] = u.x;
                    v[j + 1] = u.y;
                }
                if (L.act0) gelu16<false>(v);
                st_split16(tl + L.cA + c0, tl + L.cA + L.KA + c0, v);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (!barrier_ok()) break;
            if (leader) {
                if (nt < p.tiles) {
                    issue_s(nt);
                    ++s_pending;
                }
                layer_mma(tb, L.cA, L.KA, L.K1, s_w1, s_w1 + lo1, L.N1, 0, 0, ch1 ? L.cC1 : L.cD, L.NC1, false, L.wide & kW1);
            }
            commit_wait(false);
        }

        // ---- 3'. fc1 -> GELU -> fc2 with fc2 (<= 4 outputs) on CUDA cores: one epilogue, no round trip ----
        float* const yb = p.y + ((int64_t)b * (L.N3 ? L.Co : L.Cy) * p.P + pnt);  // channel c at yb + c P
        const float* wt = reinterpret_cast<const float*>(sm + L.o_wt);
        if (L.tail && !L.N3) {
            float2 acc[4] = {};
            for (int c0 = 0; c0 < L.N1; c0 += 16) {
                float v[16];
                ld_acc16(tl + L.cD, (L.wide & kW1) ? L.N1 : 0, c0, v);
                add16(v, vb1 + c0);
                gelu16<false>(v);
                tail_acc16(acc, wt, L.Kt, c0, v);
            }
            if (valid) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < L.Cy) {
                        const float o = acc[j].x + acc[j].y + vb2[j];
                        __stcs(yb + (int64_t)j * p.P, L.act2 ? gelu_fast(o) : o);
                    }
                }
            }
            continue;
        }

        // ---- 3. fc1 (chunks) -> GELU -> fc2 ----
        bool broke = false;
        for (int c = 0; c < nch1; ++c) {
            const int src = ch1 ? L.cC1 : L.cD;
            const int dst = ch1 ? L.cH1 : L.cA;
            const int dlo = ch1 ? L.NC1 : L.KA;
            for (int c0 = 0; c0 < L.NC1; c0 += 16) {
                float v[16];
                ld_acc16(tl + src, (L.wide & kW1) ? L.NC1 : 0, c0, v);
                add16(v, vb1 + c * L.NC1 + c0);
                gelu16<false>(v);
                st_split16(tl + dst + c0, tl + dst + dlo + c0, v);
            }
            if (!barrier_ok()) {
                broke = true;
                break;
            }
            if (leader) {
                layer_mma(tb, dst, dlo, L.NC1, s_w2, s_w2 + lo2, L.N2, 0, c * L.NC1 / 8, L.cD, L.N2, c > 0, L.wide & kW2);
                if (c + 1 < nch1)
                    layer_mma(tb, L.cA, L.KA, L.K1, s_w1, s_w1 + lo1, L.N1, (c + 1) * L.NC1, 0, L.cC1, L.NC1, false, L.wide & kW1);
            }
            commit_wait(false);
        }
        if (broke) break;

        // ---- 4. y = act(fc2 + b2 + g x + gb): store, or A of the projection ----
        for (int c0 = 0; c0 < L.N2; c0 += 16) {
            float v[16], xr[16];
            if (L.gs) {  // x from this tile's stash buffer
#pragma unroll
                for (int j = 0; j < 16; ++j) xr[j] = c0 + j < L.Cx ? xst[(c0 + j) * TP + pt] : 0.f;
            } else if (L.gx) {  // x from L2 (coalesced: a warp reads 32 consecutive points of a channel)
                const float* xg = p.x + ((int64_t)b * L.Cx + c0) * p.P + pnt;
#pragma unroll
                for (int j = 0; j < 16; ++j) xr[j] = (valid && c0 + j < L.Cx) ? l2::ld(xg + (int64_t)j * p.P, pol) : 0.f;
            }
            if (L.gate && !L.gx) tmem_ld16(tl + L.cX + c0, xr);
            ld_acc16(tl + L.cD, (L.wide & kW2) ? L.N2 : 0, c0, v);
            if (L.gate && !L.gx) tmem_wait_ld(xr);
            add16(v, vb2 + c0);
            if (L.gate) {
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                    const float4 gq = *reinterpret_cast<const float4*>(vg + c0 + j);
                    const float2 o0 = __ffma2_rn(make_float2(gq.x, gq.y), make_float2(xr[j], xr[j + 1]),
                                                 make_float2(v[j], v[j + 1]));
                    const float2 o1 = __ffma2_rn(make_float2(gq.z, gq.w), make_float2(xr[j + 2], xr[j + 3]),
                                                 make_float2(v[j + 2], v[j + 3]));
                    v[j] = o0.x;
                    v[j + 1] = o0.y;
                    v[j + 2] = o1.x;
                    v[j + 3] = o1.y;
                }
            }
            if (L.act2) {
                gelu16<false>(v);
                if (!L.N3) {  // stored: halve here (with the projection, W3 takes half weights)
#pragma unroll
                    for (int j = 0; j < 16; j += 2) {
                        const float2 h = __fmul2_rn(make_float2(v[j], v[j + 1]), make_float2(0.5f, 0.5f));
                        v[j] = h.x;
                        v[j + 1] = h.y;
                    }
                }
            }
            if (L.N3) {
                st_split16(tl + L.cA + c0, tl + L.cA + L.KA + c0, v);
            } else if (valid) {
                float* yc = yb + (int64_t)c0 * p.P;
                if (c0 + 16 <= L.Cy) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) __stcs(yc + (int64_t)j * p.P, v[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (c0 + j < L.Cy) __stcs(yc + (int64_t)j * p.P, v[j]);
                }
            }
        }
        if (!L.N3) continue;

        // ---- 5. projection: p = GELU(W3 y + b3) (chunks), out = W4 p + b4 ----
        if (!barrier_ok()) break;
        if (leader) layer_mma(tb, L.cA, L.KA, L.N2, s_w3, s_w3 + lo3, L.N3, 0, 0, ch3 ? L.cC3 : L.cD, L.NC3, false, L.wide & kW3);
        commit_wait(false);
        if (L.tail) {  // out = W4 GELU(W3 y + b3) + b4 with W4 (<= 4 outputs) on CUDA cores
            float2 acc[4] = {};
            for (int c0 = 0; c0 < L.N3; c0 += 16) {
                float v[16];
                ld_acc16(tl + L.cD, (L.wide & kW3) ? L.N3 : 0, c0, v);
                add16(v, vb3 + c0);
                gelu16<false>(v);
                tail_acc16(acc, wt, L.Kt, c0, v);
            }
            if (valid) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < L.Co) __stcs(yb + (int64_t)j * p.P, acc[j].x + acc[j].y + vb4[j]);
            }
            continue;
        }
        for (int c = 0; c < nch3; ++c) {
            const int src = ch3 ? L.cC3 : L.cD;
            const int dst = ch3 ? L.cH3 : L.cA;
            const int dlo = ch3 ? L.NC3 : L.KA;
            for (int c0 = 0; c0 < L.NC3; c0 += 16) {
                float v[16];
                ld_acc16(tl + src, (L.wide & kW3) ? L.NC3 : 0, c0, v);
                add16(v, vb3 + c * L.NC3 + c0);
                gelu16<false>(v);
                st_split16(tl + dst + c0, tl + dst + dlo + c0, v);
            }
            if (!barrier_ok()) {
                broke = true;
                break;
            }
            if (leader) {
                layer_mma(tb, dst, dlo, L.NC3, s_w4, s_w4 + lo4, L.N4, 0, c * L.NC3 / 8, L.cD, L.N4, c > 0, L.wide & kW4);
                if (c + 1 < nch3)
                    layer_mma(tb, L.cA, L.KA, L.N2, s_w3, s_w3 + lo3, L.N3, (c + 1) * L.NC3, 0, L.cC3, L.NC3, false, L.wide & kW3);
            }
            commit_wait(false);
        }
        if (broke) break;
        for (int c0 = 0; c0 < L.N4; c0 += 16) {
            float v[16];
            ld_acc16(tl + L.cD, (L.wide & kW4) ? L.N4 : 0, c0, v);
            if (valid) {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (c0 + j < L.Co) __stcs(yb + (int64_t)(c0 + j) * p.P, v[j] + vb4[c0 + j]);
            }
        }
    }

    // drain: loads still in flight land, and after an expired wait the issued MMAs finish, before the
    // shared and tensor memory are released (all bounded)
    if (leader) {
        for (; x_pending > 0; --x_pending, xph ^= 1)
            if (!tc::mbar_wait(xfull, xph, nullptr)) atomicExch(status, tc::kStatusMmaTimeout);
        for (; s_pending > 0; --s_pending, sph ^= 1)
            if (!tc::mbar_wait(sfull, sph, nullptr)) atomicExch(status, tc::kStatusMmaTimeout);
    }
    if (leader && *gflag) {  // a wait expired: let the issued MMAs finish before the memory is freed
        tc::mma_commit(mbar);
        tc::mbar_wait(mbar, mph, nullptr);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(*tmem_slot), "r"(TMEM_COLS) : "memory");
}

// ------------------------------------------------------------------------------------------------
// host planner
// ------------------------------------------------------------------------------------------------
struct Sizes {
    int Cx, Cs, nd, Ch, Cy, Cp, Co, gate, act0, act2;
};

constexpr int cmax(int a, int b) { return a > b ? a : b; }

// The layout of one chain for `groups` groups and chunk widths nc1 / nc3 (false when it does not fit).
// constexpr: the layouts of the FNO configurations' chains are also computed at compile time, and a
// kernel instantiated on one of them (FixedLayout) takes every size and offset as a constant.
// `wide`: the layers in the wide MMA form (Layout::wide bits).
constexpr bool layout_for(const Sizes& z, int groups, int nc1, int nc3, bool gate_global, int wide, Layout* out) {
    Layout L{};
    L.groups = groups;
    L.Cx = z.Cx;
    L.Cs = z.Cs;
    L.nd = z.nd;
    L.Ch = z.Ch;
    L.Cy = z.Cy;
    L.Cp = z.Cp;
    L.Co = z.Co;
    L.gate = z.gate;
    L.act0 = z.act0;
    L.act2 = z.act2;
    L.Kx = up8(z.Cx + (z.Cs ? 0 : z.nd));
    L.gx = (z.gate && gate_global) ? 1 : 0;
    L.RX = (z.gate && !gate_global) ? up16(z.Cx) : 0;
    L.N0 = z.Cs ? up16(z.Cs) : 0;
    L.K1 = z.Cs ? L.N0 : L.Kx;
    L.N1 = up16(z.Ch);
    L.N2 = up16(z.Cy);
    L.N3 = z.Cp ? up16(z.Cp) : 0;
    L.N4 = z.Cp ? up16(z.Co) : 0;
    // the final layer runs on CUDA cores when it has at most 4 outputs (the FNO projection to 1 or 3
    // channels): its hidden input is then consumed in the epilogue that produces it, so it needs no MMA
    // round trip and the layer before it runs unchunked
    L.tail = (z.Cp ? z.Co <= 4 : (z.Cy <= 4 && !z.gate)) ? 1 : 0;
    if (L.tail) {
        if (z.Cp) nc3 = L.N3;
        else nc1 = L.N1;
    }
    L.Kt = L.tail ? (z.Cp ? L.N3 : L.N1) : 0;
    L.NC1 = nc1;
    L.NC3 = L.N3 ? nc3 : 0;
    const bool ch1 = L.NC1 < L.N1, ch3 = L.N3 && L.NC3 < L.N3;
    const bool fc2_mma = !(L.tail && !z.Cp), fc4_mma = !L.tail;
    // only the layers present are wide; each wide MMA of 2 N columns stays within N <= 256
    if (!L.N0) wide &= ~kW0;
    if (!fc2_mma) wide &= ~kW2;
    if (!L.N3) wide &= ~kW3;
    if (!L.N4 || !fc4_mma) wide &= ~kW4;
    L.wide = wide;
    // accumulator columns per output channel of each layer
    const int dw0 = (wide & kW0) ? 2 : 1, dw1 = (wide & kW1) ? 2 : 1, dw2 = (wide & kW2) ? 2 : 1,
              dw3 = (wide & kW3) ? 2 : 1, dw4 = (wide & kW4) ? 2 : 1;
    if (dw0 * L.N0 > 256 || dw1 * L.NC1 > 256 || dw2 * L.N2 > 256 || dw3 * L.NC3 > 256 || dw4 * L.N4 > 256)
        return false;
    int ka = cmax(L.Kx, L.N0);
    if (!ch1 && !(L.tail && !z.Cp)) ka = cmax(ka, L.N1);  // h written as A (not when fc2 runs on CUDA cores)
    if (L.N3) ka = cmax(ka, L.N2);
    if (L.N3 && !ch3 && !L.tail) ka = cmax(ka, L.N3);
    L.KA = up8(ka);
    int nd = dw0 * L.N0;
    if (fc2_mma) nd = cmax(nd, dw2 * L.N2);
    if (fc4_mma) nd = cmax(nd, dw4 * L.N4);
    if (!ch1) nd = cmax(nd, dw1 * L.N1);
    if (L.N3 && !ch3) nd = cmax(nd, dw3 * L.N3);
    // temporary region: raw x (live until the gate) next to fc1's chunk regions (the chunk's accumulator,
    // then its h as A hi | lo); the projection's chunk regions reuse it once the gate is done
    const int t1 = L.RX + (ch1 ? (dw1 + 2) * L.NC1 : 0);
    const int t3 = ch3 ? (dw3 + 2) * L.NC3 : 0;
    const int tw = up16(cmax(t1, t3));
    L.cX = 0;
    L.cC1 = L.RX;
    L.cH1 = L.RX + dw1 * L.NC1;
    L.cC3 = 0;
    L.cH3 = dw3 * L.NC3;
    L.cA = tw;
    L.cD = L.cA + 2 * L.KA;
    L.cols = up16(L.cD + nd);
    if (L.cols * groups > TMEM_COLS) return false;
    int off = 0;
    L.o_w0 = off;
    off += up1k(8 * L.N0 * L.Kx);
    L.o_w1 = off;
    off += up1k(8 * L.N1 * L.K1);
    L.o_w2 = off;
    off += up1k((L.tail && !z.Cp) ? 0 : 8 * L.N2 * L.N1);
    L.o_w3 = off;
    off += up1k(8 * L.N3 * L.N2);
    L.o_w4 = off;
    off += up1k(L.tail ? 0 : 8 * L.N4 * L.N3);
    L.o_wt = off;
    off += up1k(L.tail ? 16 * L.Kt : 0);
    L.o_vec = off;
    off += up1k(4 * (L.N1 + 2 * L.N2 + L.N3 + L.N4));
    // per group: x stash padded to the rows stage 1 reads, s stash padded to N0 rows; the copies fill the
    // first Cx / Cs rows, the padding rows are zeroed once so the reads need no per-channel guard
    // with the gate's x read back (gx), a second x buffer per group keeps the tile's x in shared memory
    // until the gate while the next tile's x lands in the other one, when shared memory allows
    const int xb = up1k(cmax(L.Kx, L.RX) * TP * 4), sb = up1k(L.N0 * TP * 4);
    const int tail_bytes = 8 * (3 * groups + 1) + 8 + 4 * (1 + MAX_GROUPS);
    L.gs = (L.gx && off + groups * (2 * xb + sb) + tail_bytes <= SMEM_LIMIT) ? 1 : 0;
    L.stash_bytes = (L.gs ? 2 : 1) * xb + sb;
    L.o_stash = off;
    off += groups * L.stash_bytes;
    L.o_bar = off;
    off += tail_bytes;
    L.smem = off;
    if (L.smem > SMEM_LIMIT) return false;
    // more than half an SM's shared memory: one CTA per SM, so a second CTA never waits in
    // tcgen05.alloc for the first one's tensor memory
    if (L.smem < 120 * 1024) L.smem = 120 * 1024;
    *out = L;
    return true;
}

// the layout with the most groups (at most max_groups), then the widest chunks (fewest MMA round trips);
// the gate's x stays in tensor memory unless dropping it buys another group (it is then re-read from
// L2, where the tile's copy left it)
constexpr bool plan_layout_upto(const Sizes& z, int max_groups, int wide, Layout* out) {
    const int N1 = up16(z.Ch), N3 = z.Cp ? up16(z.Cp) : 16;
    const int cand[3] = {64, 32, 16};
    int opts1[4] = {N1, 0, 0, 0}, n1 = 1, opts3[4] = {N3, 0, 0, 0}, n3 = 1;
    for (int i = 0; i < 3; ++i) {
        if (cand[i] < N1 && N1 % cand[i] == 0) opts1[n1++] = cand[i];
        if (cand[i] < N3 && N3 % cand[i] == 0) opts3[n3++] = cand[i];
    }
    for (int groups = max_groups; groups >= 1; --groups)
        for (int gg = 0; gg < (z.gate ? 2 : 1); ++gg)
            for (int i = 0; i < n1; ++i)
                for (int j = 0; j < (z.Cp ? n3 : 1); ++j)
                    if (layout_for(z, groups, opts1[i], z.Cp ? opts3[j] : 0, gg == 1, wide, out)) return true;
    return false;
}

// The MMA form.  Wide (two MMAs per K step, layer_mma) doubles the accumulator columns, so it usually
// costs tiles in flight; it is chosen for large problems when it keeps at least 4 groups and loses at
// most one.  Measured on B200: the C5 block chain (1M tiles) ran 4% faster wide with 4 groups than narrow
// with 5, while the C1 block chain (2048 tiles, 14 per SM) ran 54% slower wide (fewer tiles per round
// leave a larger last round); the lifting (3 groups against 5) and the last block with the projection
// (2 against 4) ran 23% and 28% slower wide, and the width-64 chains (2 groups either way) 8-12% slower.
// With a projection, a third form keeps the projection's layers narrow and makes the block's layers
// (skip, fc1, fc2) wide: the projection's 64-column accumulator bounds the tensor memory either way, so
// it costs no group; it is taken whenever it keeps the narrow form's group count (the C5 last block with
// the projection: 42 -> 32 MMAs per tile, 14.7 -> 14.0 ms on a box held at 1750 MHz).
// NOP_CHAIN_WIDE=0 / 1 / 2 forces the narrow / wide / block-wide form (read at every call, for A/B timing;
// 2 only where a projection is fused, other chains keep the choice above).
constexpr int64_t kWideMinTiles = 148 * 64;
constexpr int kWBlock = kW0 | kW1 | kW2;

constexpr bool plan_choice(const Sizes& z, int max_groups, int force_wide, int64_t tiles, Layout* out) {
    Layout narrow{}, wide{}, mixed{};
    const bool has_n = plan_layout_upto(z, max_groups, 0, &narrow);
    const bool has_w = plan_layout_upto(z, max_groups, kWAll, &wide);
    const bool has_m = z.Cp && plan_layout_upto(z, max_groups, kWBlock, &mixed);
    bool use_w = has_w && (!has_n || (tiles >= kWideMinTiles && wide.groups >= 4 && wide.groups + 1 >= narrow.groups));
    bool use_m = !use_w && has_m && (!has_n || mixed.groups >= narrow.groups);
    if (force_wide == 0) use_w = use_m = false;
    if (force_wide == 1 && has_w) use_w = true, use_m = false;
    if (force_wide == 2 && has_m) use_m = true, use_w = false;
    if (!use_w && !use_m && !has_n) return false;
    *out = use_w ? wide : use_m ? mixed : narrow;
    return true;
}

// plan_choice with MAX_GROUPS, or the cap in NOP_CHAIN_MAX_GROUPS (1..5, read at every call) for A/B
// timing of fewer tiles in flight with wider chunks against more tiles in flight with narrower ones
bool plan_layout(const Sizes& z, int64_t tiles, Layout* out) {
    int max_groups = MAX_GROUPS;
    if (const char* e = std::getenv("NOP_CHAIN_MAX_GROUPS")) {
        const int v = std::atoi(e);
        if (v >= 1 && v <= MAX_GROUPS) max_groups = v;
    }
    int force = -1;
    if (const char* e = std::getenv("NOP_CHAIN_WIDE")) force = e[0] == '0' ? 0 : e[0] == '2' ? 2 : 1;
    return plan_choice(z, max_groups, force, tiles, out);
}

// the layout of Z in the given MMA form (0 narrow, 1 wide, 2 block-wide; falling back to narrow where
// the form does not fit)
constexpr Layout planned(const Sizes& z, int wide) {
    Layout L{};
    plan_choice(z, MAX_GROUPS, wide, 0, &L);
    return L;
}

// A layout known at compile time (Z in MMA form W): every field a constant, so the
// kernel's loops over channels unroll and its tensor- and shared-memory offsets fold into the
// instructions.  The chains of the FNO configurations' models are instantiated this way; every other
// chain (or a layout changed by the environment switches) runs on the launch-time Layout.
template <const Sizes& Z, int W>
struct FixedLayout {
    static constexpr Layout kL = planned(Z, W);
    static constexpr int Kx = kL.Kx, RX = kL.RX, gx = kL.gx, N0 = kL.N0, K1 = kL.K1, N1 = kL.N1, N2 = kL.N2,
                         N3 = kL.N3, N4 = kL.N4, NC1 = kL.NC1, NC3 = kL.NC3, tail = kL.tail, Kt = kL.Kt,
                         KA = kL.KA, cX = kL.cX, cC1 = kL.cC1, cH1 = kL.cH1, cC3 = kL.cC3, cH3 = kL.cH3,
                         cA = kL.cA, cD = kL.cD, cols = kL.cols, groups = kL.groups, o_w0 = kL.o_w0,
                         o_w1 = kL.o_w1, o_w2 = kL.o_w2, o_w3 = kL.o_w3, o_w4 = kL.o_w4, o_wt = kL.o_wt,
                         o_vec = kL.o_vec, o_stash = kL.o_stash, stash_bytes = kL.stash_bytes, o_bar = kL.o_bar,
                         smem = kL.smem, Cx = kL.Cx, Cs = kL.Cs, nd = kL.nd, Ch = kL.Ch, Cy = kL.Cy, Cp = kL.Cp,
                         Co = kL.Co, act0 = kL.act0, act2 = kL.act2, gate = kL.gate, wide = kL.wide, gs = kL.gs;
    __device__ static FixedLayout get(const Layout&) { return FixedLayout{}; }
};

// the launch-time layout
struct LaunchLayout {
    __device__ static const Layout& get(const Layout& l) { return l; }
};

// The FNO configurations' chains (hidden width 32: C1 / C5; 64: C2-C4): lifting with grid channels,
// the inner blocks (skip stage, GELUs, gate), the last block with the projection fused.
constexpr Sizes kLift3dH32{3, 0, 3, 64, 32, 0, 0, 0, 0, 0};
constexpr Sizes kLift1dH32{1, 0, 1, 64, 32, 0, 0, 0, 0, 0};
constexpr Sizes kLift2dH64{1, 0, 2, 128, 64, 0, 0, 0, 0, 0};
constexpr Sizes kBlockH32{32, 32, 0, 16, 32, 0, 0, 1, 1, 1};
constexpr Sizes kBlockH64{64, 64, 0, 32, 64, 0, 0, 1, 1, 1};
constexpr Sizes kLastProj3H32{32, 32, 0, 16, 32, 64, 3, 1, 0, 0};
constexpr Sizes kLastProj1H32{32, 32, 0, 16, 32, 64, 1, 1, 0, 0};
constexpr Sizes kLastH64{64, 64, 0, 32, 64, 0, 0, 1, 0, 0};
constexpr Sizes kProj1H64{64, 0, 0, 128, 1, 0, 0, 0, 0, 0};
// training keeps the projection apart (its backward is a chain of its own): the last block without the
// output GELU, and the projection
constexpr Sizes kLastH32{32, 32, 0, 16, 32, 0, 0, 1, 1, 0};
constexpr Sizes kProj3H32{32, 0, 0, 64, 3, 0, 0, 0, 0, 0};

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// rows [B * C] of P floats, box {128 points, C channels}
bool make_map(CUtensorMap* m, const float* base, int64_t rows, int64_t P, int C) {
    const EncodeTiled enc = reinterpret_cast<EncodeTiled>(tensor_map_encoder());
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)P, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)P * 4};
    const cuuint32_t box[2] = {(cuuint32_t)TP, (cuuint32_t)C};
    const cuuint32_t ones[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int32_t check_desc(const nop_chain_desc* d, Sizes* z, int64_t* P) {
    if (!d) return fail(NOP_E_INVALID, "descriptor is NULL");
    if (d->abi_version != NOP_ABI_VERSION) return fail(NOP_E_INVALID, "ABI version mismatch");
    if (d->ndim < 1 || d->ndim > NOP_MAX_DIMS) return fail(NOP_E_INVALID, "ndim must be in 1..4");
    if (d->batch < 0) return fail(NOP_E_INVALID, "batch must be >= 0");
    if (d->grid_dims != 0 && d->grid_dims != d->ndim) return fail(NOP_E_INVALID, "grid_dims must be 0 or ndim");
    if (d->x_channels < 1 || d->hidden_channels < 1 || d->out_channels < 1)
        return fail(NOP_E_INVALID, "x_channels, hidden_channels and out_channels must be positive");
    if (d->skip_channels < 0 || d->proj_hidden < 0 || (d->proj_hidden > 0 && d->proj_out < 1))
        return fail(NOP_E_INVALID, "skip_channels / proj_hidden must be >= 0 and proj_out >= 1 with a projection");
    if (d->skip_channels && d->grid_dims)
        return fail(NOP_E_INVALID, "grid channels are appended only without the skip stage");
    if (d->gate && d->x_channels != d->out_channels)
        return fail(NOP_E_INVALID, "the soft-gating skip needs x_channels == out_channels");
    const int mx = 256;
    if (d->x_channels + d->grid_dims > mx || d->skip_channels > mx || d->hidden_channels > mx ||
        d->out_channels > mx || d->proj_hidden > mx || d->proj_out > mx)
        return fail(NOP_E_UNSUPPORTED, "channel counts above 256 are not supported");
    int64_t n = 1;
    for (int j = 0; j < d->ndim; ++j) {
        if (d->spatial[j] < 1) return fail(NOP_E_INVALID, "spatial sizes must be >= 1");
        n *= d->spatial[j];
    }
    if (n % 4) return fail(NOP_E_UNSUPPORTED, "points per sample must be a multiple of 4 (16-byte rows)");
    if (n > 0x7fffff80LL) return fail(NOP_E_UNSUPPORTED, "more than 2^31 points per sample");
    if (d->batch * (d->x_channels > d->skip_channels ? d->x_channels : d->skip_channels) > 0x7fffffffLL)
        return fail(NOP_E_UNSUPPORTED, "batch x channels exceeds 2^31 rows");
    if (d->batch * ((n + 127) / 128) > 0x7fffffffLL)
        return fail(NOP_E_UNSUPPORTED, "more than 2^31 tiles of 128 points");
    *P = n;
    z->Cx = d->x_channels;
    z->Cs = d->skip_channels;
    z->nd = d->grid_dims;
    z->Ch = d->hidden_channels;
    z->Cy = d->out_channels;
    z->Cp = d->proj_hidden;
    z->Co = d->proj_hidden ? d->proj_out : 0;
    z->gate = d->gate ? 1 : 0;
    z->act0 = d->act_skip ? 1 : 0;
    z->act2 = d->act_out ? 1 : 0;
    return NOP_OK;
}

}  // namespace chain
}  // namespace nop

using namespace nop;

extern "C" {

int32_t nop_chain_query(const nop_chain_desc* d, int32_t* groups) {
    chain::Sizes z;
    int64_t P = 0;
    int32_t rc = chain::check_desc(d, &z, &P);
    if (rc != NOP_OK) return rc;
    chain::Layout L;
    if (!chain::plan_layout(z, d->batch * ceil_div(P, chain::TP), &L))
        return fail(NOP_E_UNSUPPORTED, "weights and tiles exceed the tensor or shared memory of a CTA");
    if (groups) *groups = L.groups;
    return NOP_OK;
}

int32_t nop_chain_forward(const nop_chain_desc* d, const nop_chain_operands* o, void* stream) {
    chain::Sizes z;
    int64_t P = 0;
    int32_t rc = chain::check_desc(d, &z, &P);
    if (rc != NOP_OK) return rc;
    if (!o) return fail(NOP_E_INVALID, "operands are NULL");
    chain::Layout L;
    if (!chain::plan_layout(z, d->batch * ceil_div(P, chain::TP), &L))
        return fail(NOP_E_UNSUPPORTED, "weights and tiles exceed the tensor or shared memory of a CTA");
    if (d->batch == 0) return NOP_OK;
    if (!o->x || !o->w1 || !o->w2 || !o->y) return fail(NOP_E_INVALID, "x, w1, w2 and y must be non-NULL");
    if (z.Cs && (!o->s || !o->w0)) return fail(NOP_E_INVALID, "s and w0 are needed with skip_channels > 0");
    if (z.gate && !o->g) return fail(NOP_E_INVALID, "g is needed when gate is set");
    if (z.Cp && (!o->w3 || !o->w4)) return fail(NOP_E_INVALID, "w3 and w4 are needed with proj_hidden > 0");
    if ((uintptr_t)o->x % 16 || (o->s && (uintptr_t)o->s % 16))
        return fail(NOP_E_ALIGNMENT, "x and s must be 16-byte aligned (tensor copies)");
    if ((uintptr_t)o->y % 4) return fail(NOP_E_ALIGNMENT, "y must be 4-byte aligned");
    chain::Params p{};
    p.P = P;
    p.tps = ceil_div(P, chain::TP);
    p.tiles = d->batch * p.tps;
    for (int j = 0; j < NOP_MAX_DIMS; ++j) {
        p.sp[j] = j < d->ndim ? d->spatial[j] : 1;
        p.goff[j] = j < d->ndim ? d->grid_offset[j] : 0;
        p.glo[j] = d->grid_lo[j];
        p.gstep[j] = d->grid_step[j];
    }
    p.w0 = o->w0;
    p.w1 = o->w1;
    p.b1 = o->b1;
    p.w2 = o->w2;
    p.b2 = o->b2;
    p.g = o->g;
    p.gb = o->gb;
    p.w3 = o->w3;
    p.b3 = o->b3;
    p.w4 = o->w4;
    p.b4 = o->b4;
    p.y = o->y;
    p.x = o->x;
    CUtensorMap tmx, tms;
    if (!chain::make_map(&tmx, o->x, d->batch * z.Cx, P, z.Cx))
        return fail(NOP_E_CUDA, "cuTensorMapEncodeTiled(x) failed");
    if (z.Cs) {
        if (!chain::make_map(&tms, o->s, d->batch * z.Cs, P, z.Cs))
            return fail(NOP_E_CUDA, "cuTensorMapEncodeTiled(s) failed");
    } else {
        tms = tmx;  // unused
    }
    int dev = 0, sms = 148;
    NOP_CUDA_TRY(cudaGetDevice(&dev));
    NOP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    int* status = status_word(dev);
    if (!status) return fail(NOP_E_CUDA, "status word of the tensor-core kernels is not available");
    const int64_t ctas = ceil_div(p.tiles, L.groups);
    const unsigned grid = (unsigned)(ctas < sms ? ctas : sms);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto launch = [&](auto kernel) -> int32_t {
        NOP_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem));
        kernel<<<grid, L.groups * chain::GT, L.smem, s>>>(tmx, tms, p, L, status);
        NOP_CUDA_TRY(cudaGetLastError());
        return NOP_OK;
    };
    // a configuration layout compiled as constants when the planned layout is exactly it
    bool fixed = false;
    auto try_fixed = [&](auto tag) {
        using F = decltype(tag);
        if (fixed || std::memcmp(&L, &F::kL, sizeof(chain::Layout)) != 0) return;
        fixed = true;
        rc = launch(chain::k_chain<F::groups, F>);
    };
    try_fixed(chain::FixedLayout<chain::kBlockH32, 0>{});
    try_fixed(chain::FixedLayout<chain::kLift3dH32, 0>{});
    try_fixed(chain::FixedLayout<chain::kLastProj3H32, 2>{});
    try_fixed(chain::FixedLayout<chain::kLift1dH32, 0>{});
    try_fixed(chain::FixedLayout<chain::kLastProj1H32, 2>{});
    try_fixed(chain::FixedLayout<chain::kBlockH64, 0>{});
    try_fixed(chain::FixedLayout<chain::kLift2dH64, 0>{});
    try_fixed(chain::FixedLayout<chain::kLastH64, 0>{});
    try_fixed(chain::FixedLayout<chain::kProj1H64, 0>{});
    try_fixed(chain::FixedLayout<chain::kBlockH32, 1>{});  // the chain the planner runs wide
    try_fixed(chain::FixedLayout<chain::kLastProj3H32, 0>{});  // the narrow form (NOP_CHAIN_WIDE=0)
    try_fixed(chain::FixedLayout<chain::kLastH32, 1>{});
    try_fixed(chain::FixedLayout<chain::kLastH32, 0>{});
    try_fixed(chain::FixedLayout<chain::kProj3H32, 0>{});
    if (!fixed) {
        using D = chain::LaunchLayout;
        switch (L.groups) {
            case 5: rc = launch(chain::k_chain<5, D>); break;
            case 4: rc = launch(chain::k_chain<4, D>); break;
            case 3: rc = launch(chain::k_chain<3, D>); break;
            case 2: rc = launch(chain::k_chain<2, D>); break;
            default: rc = launch(chain::k_chain<1, D>); break;
        }
    }
    if (rc != NOP_OK) return rc;
    return NOP_OK;
}

}  // extern "C"

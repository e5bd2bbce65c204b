// Fused per-pixel channel MLP: the FNO layers around the spectral block in one pass over HBM.
//
// At every spatial point of x [B, Cx, P] (P = prod(spatial)):
//     u = [x ; grid]                      grid: coordinate channels generated in the kernel
//     h = act1(W1 u + b1)                 (skipped when Ch == 0: h = u)
//     y = act2(W2 h + b2 + g * r + gb)    soft-gating of a residual r [B, Cy, P]
//     z = W3 y                            (optional, the next FNO block's linear skip)
// A CTA (256 threads, persistent) keeps the transposed weights in shared memory and walks tiles of
// 128 points: the next tile's u arrives by cp.async while the current tile's later layers run; each layer is a small GEMM
// (out channels x 128 points, K = in channels) with a 4 x 4 register tile per thread (a warp covers
// 4 channels x 128 points: broadcast weight loads, conflict-free activation loads), fp32 FMA (the
// same sums as the reference's fp32 Conv1d / SoftGating / GELU ops).  The residual r is read from
// global memory into registers right before the K loop of the layer that adds it.
#include <cstdint>
#include <cstdlib>
#include <string>

#include "nop_internal.cuh"

namespace nop {
namespace pw {

constexpr int THREADS = 256;
constexpr int TP = 128;         // points per tile
constexpr int PG = TP / 4;      // 4-point groups per tile
constexpr int MAX_CH = 256;     // largest channel count of any layer

struct Params {
    const float* x;
    const float* r;
    const float* b1;
    const float* b2;
    const float* g;
    const float* gb;
    const float* w1;
    const float* w2;
    const float* w3;
    float* y;
    float* z;
    int64_t P, tiles;
    int Cx, Ku, Ch, Cy, Cz;    // Ku = Cx + grid channels
    int nd;                    // grid channels (0 or the spatial ndim)
    int64_t sp[NOP_MAX_DIMS];  // spatial sizes
    float glo[NOP_MAX_DIMS], gstep[NOP_MAX_DIMS];
    int act1, act2;
    // shared-memory layout (float offsets)
    int o_w1, o_w2, o_w3, o_b1, o_b2, o_g, o_gb, o_u, o_h, o_yt;
    int slot;  // rows per ring slot: Ku, plus Cy when the residual is staged with u
    int m1, m2, m3;  // row pitches (out channels rounded up to 4) of W1T, W2T, W3T
};

__host__ __device__ inline int up4(int v) { return (v + 3) & ~3; }

__device__ __forceinline__ void cp_async16(float* smem, const float* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}

// issue the loads of tile t (u's data channels, and the residual r when `with_r`) into slot `buf`
// (u rows, then r rows); grid channels are computed
__device__ __forceinline__ void stage_tile(const Params& p, float* sm, int64_t t, int buf, bool with_r) {
    const int64_t tiles_per_sample = p.P / TP;
    const int64_t b = t / tiles_per_sample;
    const int64_t pix0 = (t % tiles_per_sample) * TP;
    float* u = sm + p.o_u + (int64_t)buf * p.slot * TP;
    for (int e = threadIdx.x; e < p.Cx * (TP / 4); e += THREADS) {
        const int c = e / (TP / 4), q = e % (TP / 4);
        cp_async16(u + c * TP + 4 * q, p.x + (b * p.Cx + c) * p.P + pix0 + 4 * q);
    }
    if (with_r) {
        float* r = u + p.Ku * TP;
        for (int e = threadIdx.x; e < p.Cy * (TP / 4); e += THREADS) {
            const int c = e / (TP / 4), q = e % (TP / 4);
            cp_async16(r + c * TP + 4 * q, p.r + (b * p.Cy + c) * p.P + pix0 + 4 * q);
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    // grid coordinates: axis j value lo_j + i_j * (hi_j - lo_j) / N_j, row-major spatial index
    for (int e = threadIdx.x; e < p.nd * TP; e += THREADS) {
        const int j = e / TP, q = e % TP;
        int64_t idx = pix0 + q;
        int64_t ij = 0;
        for (int a = p.nd - 1; a >= 0; --a) {
            const int64_t ia = idx % p.sp[a];
            idx /= p.sp[a];
            if (a == j) ij = ia;
        }
        u[(p.Cx + j) * TP + q] = p.glo[j] + (float)ij * p.gstep[j];
    }
}

// out (M x TP) = W^T-stored weights (K x pitch) times in (K x TP).  Thread tile: channels m0..m0+3,
// points p0..p0+3 (p fastest across a warp).  pre(m0, p0) runs before the K loop (to issue loads the
// epilogue needs), epi(m0, p0, acc) after it.
// The 16 products per K step run as 8 packed two-lane FMAs (__ffma2_rn, each lane rounded like fmaf):
// channel pairs (w0, w1), (w2, w3) times point pairs (x0, x1), (x2, x3) accumulate the diagonal
// entries (acc[2a][2b], acc[2a+1][2b+1]); times the swapped pairs (x1, x0), (x3, x2) the anti-diagonal
// ones (acc[2a][2b+1], acc[2a+1][2b]), so no operand needs a broadcast.
template <class Pre, class Epi>
__device__ __forceinline__ void gemm(const float* __restrict__ WT, int pitch, int M, int K, const float* __restrict__ in,
                                     Pre pre, Epi epi) {
    const int ntiles = (up4(M) / 4) * PG;
    for (int tix = threadIdx.x; tix < ntiles; tix += THREADS) {
        const int m0 = (tix / PG) * 4, p0 = (tix % PG) * 4;
        pre(m0, p0);
        float2 dg[2][2], ad[2][2];
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b) dg[a][b] = ad[a][b] = make_float2(0.f, 0.f);
#pragma unroll 4
        for (int k = 0; k < K; ++k) {
            const float4 w = *reinterpret_cast<const float4*>(WT + k * pitch + m0);
            const float4 v = *reinterpret_cast<const float4*>(in + k * TP + p0);
            const float2 wp[2] = {make_float2(w.x, w.y), make_float2(w.z, w.w)};
            const float2 xp[2] = {make_float2(v.x, v.y), make_float2(v.z, v.w)};
            const float2 xs[2] = {make_float2(v.y, v.x), make_float2(v.w, v.z)};
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    dg[a][b] = __ffma2_rn(wp[a], xp[b], dg[a][b]);
                    ad[a][b] = __ffma2_rn(wp[a], xs[b], ad[a][b]);
                }
        }
        float acc[4][4];
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                acc[2 * a][2 * b] = dg[a][b].x;
                acc[2 * a + 1][2 * b + 1] = dg[a][b].y;
                acc[2 * a][2 * b + 1] = ad[a][b].x;
                acc[2 * a + 1][2 * b] = ad[a][b].y;
            }
        epi(m0, p0, acc);
    }
}

// NS = 1: one u buffer; the next tile's loads start once the last layer reading u is done, and the
// residual is read into registers before the K loop that adds it.
// NS >= 2: a ring of NS slots (u and the residual) with NS - 1 tiles in flight (memory-bound shapes).
template <int NS>
__global__ void __launch_bounds__(THREADS, 2) k_pointwise(Params p) {
    extern __shared__ __align__(16) float sm[];
    // weights, transposed to [in][out] with the out dimension padded to 4 (zeros), and vectors
    auto load_t = [&](const float* w, int rows, int cols, int pitch, int off) {
        for (int e = threadIdx.x; e < cols * pitch; e += THREADS) {
            const int k = e / pitch, m = e % pitch;
            sm[off + e] = m < rows ? __ldg(w + (int64_t)m * cols + k) : 0.f;
        }
    };
    auto load_v = [&](const float* v, int n, int off) {
        for (int e = threadIdx.x; e < up4(n); e += THREADS) sm[off + e] = (v && e < n) ? __ldg(v + e) : 0.f;
    };
    const int Kh = p.Ch > 0 ? p.Ch : p.Ku;
    if (p.Ch > 0) load_t(p.w1, p.Ch, p.Ku, p.m1, p.o_w1);
    load_t(p.w2, p.Cy, Kh, p.m2, p.o_w2);
    if (p.Cz > 0) load_t(p.w3, p.Cz, p.Cy, p.m3, p.o_w3);
    if (p.Ch > 0) load_v(p.b1, p.Ch, p.o_b1);
    load_v(p.b2, p.Cy, p.o_b2);
    load_v(p.g, p.Cy, p.o_g);
    load_v(p.gb, p.Cy, p.o_gb);

    int64_t t = blockIdx.x;
    if constexpr (NS == 1) {
        if (t < p.tiles) stage_tile(p, sm, t, 0, false);
    } else {
#pragma unroll
        for (int k = 0; k < NS - 1; ++k) {
            const int64_t tk = t + (int64_t)k * gridDim.x;
            if (tk < p.tiles) stage_tile(p, sm, tk, k, p.r != nullptr);
            else asm volatile("cp.async.commit_group;\n" ::: "memory");
        }
    }
    for (int it = 0; t < p.tiles; t += gridDim.x, ++it) {
        const int64_t nt = t + gridDim.x;
        const int slot = NS == 1 ? 0 : it % NS;
        if constexpr (NS == 1) {
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group %0;\n" ::"n"(NS - 2) : "memory");
        }
        __syncthreads();
        if constexpr (NS > 1) {  // refill the slot the previous tile used
            const int64_t ft = t + (int64_t)(NS - 1) * gridDim.x;
            if (ft < p.tiles) stage_tile(p, sm, ft, (it + NS - 1) % NS, p.r != nullptr);
            else asm volatile("cp.async.commit_group;\n" ::: "memory");
        }
        const int64_t tiles_per_sample = p.P / TP;
        const int64_t b = t / tiles_per_sample;
        const int64_t pix0 = (t % tiles_per_sample) * TP;
        const float* u = sm + p.o_u + slot * p.slot * TP;
        const float* rs = u + p.Ku * TP;  // staged residual (NS >= 2)
        float* h = sm + p.o_h;
        if (p.Ch > 0) {
            gemm(sm + p.o_w1, p.m1, p.Ch, p.Ku, u, [](int, int) {}, [&](int m0, int p0, float (&acc)[4][4]) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = m0 + i;
                    if (m >= p.Ch) break;
                    const float bias = sm[p.o_b1 + m];
                    float4 o;
                    float* ov = &o.x;
#pragma unroll
                    for (int j = 0; j < 4; ++j) ov[j] = p.act1 ? gelu_erf(acc[i][j] + bias) : acc[i][j] + bias;
                    *reinterpret_cast<float4*>(h + m * TP + p0) = o;
                }
            });
            __syncthreads();
            if (NS == 1 && nt < p.tiles) stage_tile(p, sm, nt, 0, false);
        }
        const float* hin = p.Ch > 0 ? h : u;
        float* yt = sm + p.o_yt;
        float4 rv[4];  // residual of this thread tile, loaded before the K loop
        gemm(
            sm + p.o_w2, p.m2, p.Cy, Kh, hin,
            [&](int m0, int p0) {
                if (NS > 1 || !p.r) return;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    rv[i] = m0 + i < p.Cy ? __ldg(reinterpret_cast<const float4*>(p.r + (b * p.Cy + m0 + i) * p.P +
                                                                                  pix0 + p0))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
            },
            [&](int m0, int p0, float (&acc)[4][4]) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int m = m0 + i;
                if (m >= p.Cy) break;
                const float bias = sm[p.o_b2 + m] + sm[p.o_gb + m];
                const float gw = sm[p.o_g + m];
                const float* rr = NS > 1 ? rs + m * TP + p0 : &rv[i].x;
                float4 o;
                float* ov = &o.x;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float v = acc[i][j] + bias;
                    if (p.r) v = fmaf(gw, rr[j], v);
                    ov[j] = p.act2 ? gelu_erf(v) : v;
                }
                *reinterpret_cast<float4*>(p.y + (b * p.Cy + m) * p.P + pix0 + p0) = o;
                if (p.Cz > 0) *reinterpret_cast<float4*>(yt + m * TP + p0) = o;
            }
        });
        if (NS == 1 && p.Ch == 0 && nt < p.tiles) {  // the single layer read u
            __syncthreads();
            stage_tile(p, sm, nt, 0, false);
        }
        if (p.Cz > 0) {
            __syncthreads();
            gemm(sm + p.o_w3, p.m3, p.Cz, p.Cy, yt, [](int, int) {}, [&](int m0, int p0, float (&acc)[4][4]) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = m0 + i;
                    if (m >= p.Cz) break;
                    *reinterpret_cast<float4*>(p.z + (b * p.Cz + m) * p.P + pix0 + p0) =
                        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
                }
            });
        }
        __syncthreads();  // the next tile reuses h and yt
    }
}

}  // namespace pw
}  // namespace nop

#include "pointwise_tc.cuh"

using namespace nop;

extern "C" int32_t nop_pointwise_smem_bytes(const nop_pointwise_desc* d, size_t* bytes);

namespace {

// NOP_POINTWISE=tc selects the tcgen05 kernel (pointwise_tc.cuh).  It is parity-tested but measured
// slower than the CUDA-core kernel on B200 (C4 model 42.6 vs 40.1 ms, C5 358 vs 209 ms: one tile's
// operands fill the CTA, so each SM runs one serialized GEMM -> epilogue chain at a time), so the
// CUDA-core kernel is the default.
bool pointwise_on_tensor_cores() {
    const char* v = std::getenv("NOP_POINTWISE");
    return v && std::string(v) == "tc";
}

int32_t build_params(const nop_pointwise_desc* d, pw::Params* p, size_t* smem, int* ns) {
    if (!d) return fail(NOP_E_INVALID, "descriptor is NULL");
    if (d->abi_version != NOP_ABI_VERSION) return fail(NOP_E_INVALID, "ABI version mismatch");
    if (d->ndim < 1 || d->ndim > NOP_MAX_DIMS) return fail(NOP_E_INVALID, "ndim must be in 1..4");
    if (d->grid_dims != 0 && d->grid_dims != d->ndim)
        return fail(NOP_E_INVALID, "grid_dims must be 0 or ndim");
    if (d->in_channels < 1 || d->out_channels < 1 || d->hidden_channels < 0 || d->next_channels < 0)
        return fail(NOP_E_INVALID, "channel counts must be positive (hidden / next may be 0)");
    const int Ku = d->in_channels + d->grid_dims;
    if (Ku > pw::MAX_CH || d->hidden_channels > pw::MAX_CH || d->out_channels > pw::MAX_CH ||
        d->next_channels > pw::MAX_CH)
        return fail(NOP_E_UNSUPPORTED, "channel counts above 256 are not supported by the fused kernel");
    if (d->batch < 0) return fail(NOP_E_INVALID, "batch must be >= 0");
    int64_t P = 1;
    for (int j = 0; j < d->ndim; ++j) {
        if (d->spatial[j] < 1) return fail(NOP_E_INVALID, "spatial sizes must be >= 1");
        P *= d->spatial[j];
    }
    if (P % pw::TP) return fail(NOP_E_UNSUPPORTED, "points per sample must be a multiple of 128");
    *p = pw::Params{};
    p->P = P;
    p->tiles = d->batch * (P / pw::TP);
    p->Cx = d->in_channels;
    p->Ku = Ku;
    p->Ch = d->hidden_channels;
    p->Cy = d->out_channels;
    p->Cz = d->next_channels;
    p->nd = d->grid_dims;
    for (int j = 0; j < d->ndim; ++j) {
        p->sp[j] = d->spatial[j];
        p->glo[j] = d->grid_lo[j];
        p->gstep[j] = (d->grid_hi[j] - d->grid_lo[j]) / (float)d->spatial[j];
    }
    p->act1 = d->act_hidden;
    p->act2 = d->act_out;
    const int Kh = p->Ch > 0 ? p->Ch : Ku;
    p->m1 = pw::up4(p->Ch);
    p->m2 = pw::up4(p->Cy);
    p->m3 = pw::up4(p->Cz);
    int off = 0;
    auto take = [&](int n) {
        const int at = off;
        off += pw::up4(n);
        return at;
    };
    p->o_w1 = take(p->Ch > 0 ? Ku * p->m1 : 0);
    p->o_w2 = take(Kh * p->m2);
    p->o_w3 = take(p->Cz > 0 ? p->Cy * p->m3 : 0);
    p->o_b1 = take(p->Ch);
    p->o_b2 = take(p->Cy);
    p->o_g = take(p->Cy);
    p->o_gb = take(p->Cy);
    p->o_h = take(p->Ch * pw::TP);
    p->o_yt = take(p->Cz > 0 ? p->Cy * pw::TP : 0);
    p->o_u = off;  // the ring goes last: NS slots
    // ring depth: two CTAs per SM with the deepest ring that fits, else one CTA; a ring of two or more
    // slots also stages the residual, a single slot holds u only
    const size_t fixed = (size_t)off * sizeof(float);
    const int rows_ring = Ku + (d->gate ? p->Cy : 0);
    *ns = 0;
    for (int ctas : {2, 1}) {
        const size_t budget = ctas == 2 ? 113 * 1024 : 226 * 1024;
        for (int n : {4, 3, 2, 1}) {
            const int rows = n > 1 ? rows_ring : Ku;
            if (fixed + (size_t)n * rows * pw::TP * sizeof(float) <= budget) {
                *ns = n;
                p->slot = rows;
                break;
            }
        }
        if (*ns) break;
    }
    if (!*ns) return fail(NOP_E_UNSUPPORTED, "weights and tiles exceed the shared memory of a CTA");
    *smem = fixed + (size_t)*ns * p->slot * pw::TP * sizeof(float);
    return NOP_OK;
}

}  // namespace

extern "C" {

int32_t nop_pointwise_smem_bytes(const nop_pointwise_desc* d, size_t* bytes) {
    if (!bytes) return fail(NOP_E_INVALID, "bytes is NULL");
    pw::Params p;
    int ns = 0;
    return build_params(d, &p, bytes, &ns);
}

int32_t nop_pointwise_forward(const nop_pointwise_desc* d, const float* x, const float* w1, const float* b1,
                              const float* w2, const float* b2, const float* r, const float* g, const float* gb,
                              const float* w3, float* y, float* z, void* stream) {
    pw::Params p;
    size_t smem = 0;
    int ns = 1;
    int32_t rc = build_params(d, &p, &smem, &ns);
    if (rc != NOP_OK) return rc;
    if (p.tiles == 0) return NOP_OK;
    if (!x || !y || !w2) return fail(NOP_E_INVALID, "x, w2 and y must be non-NULL");
    if (p.Ch > 0 && !w1) return fail(NOP_E_INVALID, "w1 is NULL but hidden_channels > 0");
    if (p.Cz > 0 && (!w3 || !z)) return fail(NOP_E_INVALID, "w3 and z are needed when next_channels > 0");
    if (d->gate && (!r || !g)) return fail(NOP_E_INVALID, "r and g are needed when gate is set");
    if ((uintptr_t)x % 16 || (uintptr_t)y % 16 || (r && (uintptr_t)r % 16) || (z && (uintptr_t)z % 16))
        return fail(NOP_E_ALIGNMENT, "x, r, y and z must be 16-byte aligned");
    p.x = x;
    p.r = d->gate ? r : nullptr;
    p.w1 = w1;
    p.w2 = w2;
    p.w3 = w3;
    p.b1 = d->has_b1 ? b1 : nullptr;
    p.b2 = d->has_b2 ? b2 : nullptr;
    p.g = d->gate ? g : nullptr;
    p.gb = d->gate && d->has_gate_bias ? gb : nullptr;
    p.y = y;
    p.z = z;
    int dev = 0, sms = 148;
    NOP_CUDA_TRY(cudaGetDevice(&dev));
    NOP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    pwtc::Layout L;
    if (pointwise_on_tensor_cores() && pwtc::plan_layout(p, &L)) {
        int* status = status_word(dev);
        if (!status) return fail(NOP_E_CUDA, "status word of the tensor-core kernels is not available");
        NOP_CUDA_TRY(cudaFuncSetAttribute(pwtc::k_pointwise_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem));
        const unsigned grid = (unsigned)(p.tiles < sms ? p.tiles : sms);
        pwtc::k_pointwise_tc<<<grid, pwtc::THREADS, L.smem, static_cast<cudaStream_t>(stream)>>>(p, L, status);
        NOP_CUDA_TRY(cudaGetLastError());
        return NOP_OK;
    }
    auto launch = [&](auto kernel) -> int32_t {
        NOP_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        int per_sm = 0;
        NOP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, pw::THREADS, smem));
        if (per_sm < 1) per_sm = 1;
        const int64_t slots = (int64_t)per_sm * sms;
        const unsigned grid = (unsigned)(p.tiles < slots ? p.tiles : slots);
        kernel<<<grid, pw::THREADS, smem, static_cast<cudaStream_t>(stream)>>>(p);
        return NOP_OK;
    };
    switch (ns) {
        case 4: rc = launch(pw::k_pointwise<4>); break;
        case 3: rc = launch(pw::k_pointwise<3>); break;
        case 2: rc = launch(pw::k_pointwise<2>); break;
        default: rc = launch(pw::k_pointwise<1>); break;
    }
    if (rc != NOP_OK) return rc;
    NOP_CUDA_TRY(cudaGetLastError());
    return NOP_OK;
}

}  // extern "C"

// Allocation-free forward: the generic spectral-block kernels running on a fixed scratch area
// compiled into this library, for callers that must not allocate device memory.
//
// Who needs it: code that runs inside a host that owns all device memory and offers no
// allocation hook (plugin interfaces that hand over only the input and output buffers),
// and latency-critical loops where a cudaMalloc -- which can synchronise the device and
// stall every stream -- is not acceptable.  Such callers pass inputs and outputs only; the
// intermediate spectra and twiddle tables live in g_static_scratch below.
//
// Limits and sharing rules:
//   * the scratch is kStaticScratchBytes (16 MiB) per device; every GPU that loads this
//     library holds it until the process exits.  Larger problems are rejected with
//     NOP_E_WORKSPACE before anything is launched.
//   * every call on a device uses the same scratch and leaves its contents behind.  Each
//     region (twiddle tables, spectra, factor intermediates) is completely rewritten by the
//     kernels of a call before any kernel of that call reads it, so nothing needs clearing.
//     Calls whose kernels overlap on the GPU (different streams without ordering between
//     them, or different host threads) race on the scratch and produce garbage.
//   * the first call in a CUDA context (per device, with that device current) looks up the device
//     address of the scratch with cudaGetSymbolAddress (host code cannot use the symbol itself: in
//     host code its name stands for a host-side shadow, not device memory) and caches it under the
//     context's unique id.  A new context on the device -- after cudaDeviceReset, or a driver-API
//     context made current by the caller -- has another id, so its first call looks the address up
//     again instead of reusing one that belonged to a destroyed context.  Make the first call in each
//     context before any stream capture begins.
#include <mutex>

#include <cuda.h>

#include "nop_internal.cuh"

namespace nop {
namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;
constexpr size_t kScratchAlign = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct ScratchAddr {
    unsigned long long ctx_id = 0;  // id of the context the address belongs to (0: none yet)
    char* addr = nullptr;
};

std::mutex g_addr_mutex;
ScratchAddr g_scratch_addr[kMaxDevices];

size_t round_up(size_t v) { return (v + kScratchAlign - 1) / kScratchAlign * kScratchAlign; }

// cuCtxGetCurrent / cuCtxGetId through the runtime's driver entry point (no link against libcuda)
using CtxGetCurrent = CUresult (*)(CUcontext*);
using CtxGetId = CUresult (*)(CUcontext, unsigned long long*);

template <class F>
F driver_fn(const char* name) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &f, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return nullptr;
    return reinterpret_cast<F>(f);
}

// Unique id of the current context of the calling thread (ids are never reused in a process).
int32_t current_context_id(unsigned long long* id) {
    static const CtxGetCurrent get_current = driver_fn<CtxGetCurrent>("cuCtxGetCurrent");
    static const CtxGetId get_id = driver_fn<CtxGetId>("cuCtxGetId");
    if (!get_current || !get_id) return fail(NOP_E_CUDA, "cuCtxGetCurrent / cuCtxGetId are not available");
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return fail(NOP_E_CUDA, "no current CUDA context");
    if (get_id(ctx, id) != CUDA_SUCCESS) return fail(NOP_E_CUDA, "cuCtxGetId failed");
    return NOP_OK;
}

// Device address of g_static_scratch on device `dev` (the current device) in the current context,
// looked up once per context.
int32_t scratch_address(int dev, char** out) {
    unsigned long long ctx_id = 0;
    int32_t rc = current_context_id(&ctx_id);
    if (rc != NOP_OK) return rc;
    std::lock_guard<std::mutex> lock(g_addr_mutex);
    ScratchAddr& e = g_scratch_addr[dev];
    if (e.ctx_id != ctx_id || !e.addr) {
        void* p = nullptr;
        cudaError_t err = cudaGetSymbolAddress(&p, g_static_scratch);
        if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(static scratch)");
        e.addr = static_cast<char*>(p);
        e.ctx_id = ctx_id;
    }
    *out = e.addr;
    return NOP_OK;
}

// Twiddle table of length n in double and float: (cos 2 pi k / n, sin 2 pi k / n).
__global__ void static_twiddles(double2* d, float2* f, int64_t n) {
    int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (k >= n) return;
    double s, c;
    sincospi(2.0 * (double)k / (double)n, &s, &c);
    if (4 * k == n) { c = 0.0; s = 1.0; }
    if (2 * k == n) { c = -1.0; s = 0.0; }
    if (4 * k == 3 * n) { c = 0.0; s = -1.0; }
    d[k] = make_double2(c, s);
    f[k] = make_float2((float)c, (float)s);
}

}  // namespace
}  // namespace nop

using namespace nop;

extern "C" int32_t nop_spectral_forward_static(const nop_spectral_desc* desc, const void* x,
                                               const void* const* weights, int32_t n_weights, const float* bias,
                                               const float* addend, int32_t apply_gelu, void* y, void* stream) {
    int32_t rc = validate(desc);
    if (rc != NOP_OK) return rc;
    // One plan object per host thread, reused: its table list keeps its capacity, so no call
    // after the first touches the heap.
    thread_local Plan p;
    p.tables.clear();
    p.tables.reserve(2 * NOP_MAX_DIMS);
    p.d = *desc;
    p.fast = false;
    p.fast_kind = FastKind::None;
    p.table_mem = nullptr;
    p.modes_total = 1;
    for (int j = 0; j < p.d.ndim; ++j) p.modes_total *= p.d.kept[j];
    for (int j = p.d.ndim; j < NOP_MAX_DIMS; ++j) {
        p.d.n_in[j] = p.d.n_out[j] = p.d.kept[j] = 1;
        p.d.fwd_off[j] = p.d.inv_off[j] = 0;
    }
    const nop_spectral_desc& d = p.d;
    if (d.engine == NOP_ENGINE_FAST)
        return fail(NOP_E_UNSUPPORTED, "the allocation-free forward runs the generic engine only; "
                                       "pass NOP_ENGINE_AUTO or NOP_ENGINE_GENERIC");
    if (n_weights != expected_weights(d))
        return fail(NOP_E_INVALID, "expected " + std::to_string(expected_weights(d)) + " weight pointers, got " +
                                       std::to_string(n_weights));
    if (d.batch == 0) return NOP_OK;
    if (!x || !y || !weights) return fail(NOP_E_INVALID, "x, y and weights must be non-NULL");
    for (int i = 0; i < n_weights; ++i)
        if (!weights[i]) return fail(NOP_E_INVALID, "weight pointer " + std::to_string(i) + " is NULL");
    if ((addend || apply_gelu) && d.complex_data)
        return fail(NOP_E_UNSUPPORTED, "addend / fused GELU need real data");
    const size_t elem_align = d.complex_data ? 8 : 4;
    if ((uintptr_t)x % elem_align || (uintptr_t)y % elem_align || (bias && (uintptr_t)bias % 4) ||
        (addend && (uintptr_t)addend % 4))
        return fail(NOP_E_ALIGNMENT, "x / y / bias / addend are not aligned to their element size");
    for (int i = 0; i < n_weights; ++i)
        if ((uintptr_t)weights[i] % 8) return fail(NOP_E_ALIGNMENT, "weights must be 8-byte aligned (complex64)");

    // Scratch layout: twiddle tables, then the generic engine's workspace regions.
    int64_t lens[2 * NOP_MAX_DIMS];
    int n_lens = 0;
    for (int j = 0; j < d.ndim; ++j) {
        for (int64_t n : {d.n_in[j], d.n_out[j]}) {
            bool seen = false;
            for (int i = 0; i < n_lens; ++i) seen |= (lens[i] == n);
            if (!seen) lens[n_lens++] = n;
        }
    }
    size_t table_bytes = 0;
    for (int i = 0; i < n_lens; ++i) table_bytes += round_up(lens[i] * sizeof(double2)) + round_up(lens[i] * sizeof(float2));
    size_t off = 0;
    p.ws = WorkspaceLayout{};
    p.ws.buf_elems = generic_buffer_elems(d);
    p.ws.buf_a = off;
    off += round_up((size_t)p.ws.buf_elems * sizeof(float2));
    p.ws.buf_b = off;
    off += round_up((size_t)p.ws.buf_elems * sizeof(float2));
    contraction_layout(p, &off, &p.ws);
    p.ws.bytes = off;
    const size_t need = table_bytes + p.ws.bytes;
    if (need > kStaticScratchBytes)
        return fail(NOP_E_WORKSPACE, "problem needs " + std::to_string(need) + " bytes of scratch; the built-in "
                                     "static scratch holds " + std::to_string(kStaticScratchBytes) +
                                     " bytes (use nop_spectral_forward with a caller-provided workspace)");

    int dev = -1;
    NOP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(NOP_E_UNSUPPORTED, "device index beyond the supported range");
    char* base = nullptr;
    rc = scratch_address(dev, &base);
    if (rc != NOP_OK) return rc;
    p.device = dev;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    size_t at = 0;
    for (int i = 0; i < n_lens; ++i) {
        TwiddleTable t;
        t.n = lens[i];
        double2* dt = reinterpret_cast<double2*>(base + at);
        at += round_up(lens[i] * sizeof(double2));
        float2* ft = reinterpret_cast<float2*>(base + at);
        at += round_up(lens[i] * sizeof(float2));
        static_twiddles<<<(unsigned)ceil_div(lens[i], 256), 256, 0, s>>>(dt, ft, lens[i]);
        cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) return cuda_fail(err, "static twiddle launch");
        t.d_table = dt;
        t.f_table = ft;
        p.tables.push_back(t);
    }
    return generic_forward(p, x, weights, bias, addend, apply_gelu, y, base + table_bytes, s);
}

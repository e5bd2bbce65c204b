// C ABI of libnop_b200: descriptor validation, plans (twiddle tables, workspace layout) and
// dispatch to the fused FFT engine or the generic direct-DFT engine.
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>

#include "nop_internal.cuh"

namespace nop {

namespace {
thread_local std::string g_last_error;
constexpr int64_t kMaxLen = int64_t(1) << 20;     // per-axis transform length limit
constexpr int64_t kMaxElems = int64_t(1) << 40;   // per-tensor element limit
constexpr size_t kAlign = 256;

// NOP_CONTRACTION=simt selects the CUDA-core contraction kernel instead of the tcgen05 one (A/B
// measurements of the two); read once per plan.
bool mix_on_tensor_cores() {
    const char* v = getenv("NOP_CONTRACTION");
    return !(v && strcmp(v, "simt") == 0);
}

// NOP_MIX_TMA=0: the tensor-core contraction with per-thread gathers on the float4 weight packing
bool mix_with_tma() {
    const char* v = getenv("NOP_MIX_TMA");
    return !(v && strcmp(v, "0") == 0);
}

size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

bool mul_ok(int64_t a, int64_t b, int64_t* out) {
    if (a < 0 || b < 0) return false;
    if (a != 0 && b > kMaxElems / a) return false;
    *out = a * b;
    return true;
}
}  // namespace

namespace {
struct LaunchEvents {
    cudaEvent_t ev[32];
    int n = 0;
    int next = 0;
};
thread_local LaunchEvents g_events;
}  // namespace

void launch_mark_begin(cudaStream_t s) {
    if (g_events.n > 0) {
        cudaEventRecord(g_events.ev[0], s);
        g_events.next = 1;
    }
}

void launch_mark(cudaStream_t s) {
    if (g_events.next > 0 && g_events.next < g_events.n) cudaEventRecord(g_events.ev[g_events.next++], s);
}

static int32_t launch_mark_end(int32_t rc) {
    g_events.next = 0;  // marks only follow the launches of one forward call
    return rc;
}

void set_error(const std::string& msg) { g_last_error = msg; }

int32_t fail(int32_t code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int32_t cuda_fail(cudaError_t err, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")";
    return fail(NOP_E_CUDA, m);
}


int expected_weights(const nop_spectral_desc& d) {
    if (d.weight_kind == NOP_WEIGHT_DENSE) return 1;
    return 1 + (d.separable ? 1 : 2) + d.ndim;
}

int32_t validate(const nop_spectral_desc* d) {
    if (!d) return fail(NOP_E_INVALID, "descriptor is NULL");
    if (d->abi_version != NOP_ABI_VERSION)
        return fail(NOP_E_INVALID, "descriptor abi_version " + std::to_string(d->abi_version) +
                                       " != library " + std::to_string(NOP_ABI_VERSION));
    if (d->ndim < 1 || d->ndim > NOP_MAX_DIMS)
        return fail(NOP_E_INVALID, "ndim must be in 1.." + std::to_string(NOP_MAX_DIMS));
    if (d->batch < 0) return fail(NOP_E_INVALID, "batch must be >= 0");
    if (d->in_channels < 1 || d->out_channels < 1) return fail(NOP_E_INVALID, "channel counts must be >= 1");
    if (d->separable && d->in_channels != d->out_channels)
        return fail(NOP_E_INVALID, "separable contraction needs in_channels == out_channels");
    if (d->complex_data != 0 && d->complex_data != 1) return fail(NOP_E_INVALID, "complex_data must be 0 or 1");
    if (d->weight_kind < NOP_WEIGHT_DENSE || d->weight_kind > NOP_WEIGHT_CP)
        return fail(NOP_E_INVALID, "unknown weight_kind");
    if (d->precision != NOP_PRECISION_FP32 && d->precision != NOP_PRECISION_BF16)
        return fail(NOP_E_INVALID, "unknown precision");
    if (d->engine < NOP_ENGINE_AUTO || d->engine > NOP_ENGINE_FAST) return fail(NOP_E_INVALID, "unknown engine");
    if (d->n_zero_imag < 0 || d->n_zero_imag > 3) return fail(NOP_E_INVALID, "n_zero_imag must be in 0..3");
    if (!(std::isfinite(d->fwd_scale) && std::isfinite(d->inv_scale)))
        return fail(NOP_E_INVALID, "scales must be finite");
    const int nd = d->ndim;
    for (int j = 0; j < nd; ++j) {
        const std::string ax = "axis " + std::to_string(j);
        if (d->n_in[j] < 1 || d->n_in[j] > kMaxLen || d->n_out[j] < 1 || d->n_out[j] > kMaxLen)
            return fail(NOP_E_INVALID, ax + ": spatial sizes must be in 1.." + std::to_string(kMaxLen));
        const bool real_last = !d->complex_data && j == nd - 1;
        const int64_t spec = real_last ? d->n_in[j] / 2 + 1 : d->n_in[j];
        if (d->kept[j] < 1 || d->kept[j] > spec)
            return fail(NOP_E_INVALID, ax + ": kept modes " + std::to_string(d->kept[j]) + " outside 1.." +
                                           std::to_string(spec));
        if (d->fwd_off[j] < 0 || d->fwd_off[j] >= d->n_in[j] || d->inv_off[j] < 0 || d->inv_off[j] >= d->n_in[j])
            return fail(NOP_E_INVALID, ax + ": bin offsets must be in 0..n_in-1");
        if (real_last && (d->fwd_off[j] != 0 || d->inv_off[j] != 0))
            return fail(NOP_E_INVALID, "the real last axis keeps rFFT bins from 0 (offsets must be 0)");
    }
    if (d->weight_kind != NOP_WEIGHT_DENSE) {
        const int nr = d->weight_kind == NOP_WEIGHT_CP ? 1 : (d->separable ? 1 : 2) + nd;
        for (int i = 0; i < nr; ++i)
            if (d->ranks[i] < 1 || d->ranks[i] > kMaxLen) return fail(NOP_E_INVALID, "factor ranks must be >= 1");
    }
    // element-count overflow checks on the largest tensors
    int64_t px = 1, py = 1, e;
    for (int j = 0; j < nd; ++j) {
        if (!mul_ok(px, d->n_in[j], &px) || !mul_ok(py, d->n_out[j], &py))
            return fail(NOP_E_INVALID, "spatial size product overflows");
    }
    if (!mul_ok(d->batch, d->in_channels, &e) || !mul_ok(e, px, &e) || !mul_ok(d->batch, d->out_channels, &e) ||
        !mul_ok(e, py, &e))
        return fail(NOP_E_INVALID, "tensor size overflows");
    return NOP_OK;
}

static int64_t tucker_expansion_elems(const nop_spectral_desc& d, int64_t lead, int r0) {
    int64_t best = 0;
    for (int j = 0; j < d.ndim; ++j) {
        int64_t e = lead;
        for (int i = 0; i <= j; ++i) e *= d.kept[i];
        for (int i = j + 1; i < d.ndim; ++i) e *= d.ranks[r0 + i];
        if (e > best) best = e;
    }
    return best;
}

// Workspace regions of the contraction stage (shared by both engines).
void contraction_layout(const Plan& p, size_t* off, WorkspaceLayout* ws) {
    const nop_spectral_desc& d = p.d;
    const int64_t Mt = p.modes_total, B = d.batch, Ci = d.in_channels;
    int64_t g = 0, xf = 0, z = 0;
    if (d.weight_kind == NOP_WEIGHT_TUCKER) {
        if (d.separable) {
            int64_t q = 1;
            for (int j = 0; j < d.ndim; ++j) q *= d.ranks[1 + j];
            xf = Ci * q;
            g = tucker_expansion_elems(d, Ci, 1);
        } else {
            g = tucker_expansion_elems(d, d.ranks[0] * d.ranks[1], 2);
            xf = B * d.ranks[0] * Mt;
            z = B * d.ranks[1] * Mt;
        }
    } else if (d.weight_kind == NOP_WEIGHT_CP) {
        g = (d.separable ? Ci : d.ranks[0]) * Mt;
        if (!d.separable) xf = z = B * d.ranks[0] * Mt;
    }
    auto take = [&](int64_t elems) {
        size_t at = *off;
        *off += align_up((size_t)elems * sizeof(float2));
        return at;
    };
    ws->g = take(g);
    ws->g_tmp = take(d.weight_kind == NOP_WEIGHT_TUCKER ? g : 0);
    ws->xf = take(xf);
    ws->z = take(z);
}

namespace {

int32_t build_tables(Plan* p) {
    const nop_spectral_desc& d = p->d;
    std::vector<int64_t> lens;
    for (int j = 0; j < d.ndim; ++j) {
        for (int64_t n : {d.n_in[j], d.n_out[j]}) {
            bool seen = false;
            for (int64_t v : lens) seen |= (v == n);
            if (!seen) lens.push_back(n);
        }
    }
    size_t bytes = 0;
    for (int64_t n : lens) bytes += align_up(n * sizeof(double2)) + align_up(n * sizeof(float2));
    std::vector<char> host(bytes);
    size_t at = 0;
    std::vector<std::pair<size_t, size_t>> offs;
    for (int64_t n : lens) {
        double2* dt = reinterpret_cast<double2*>(host.data() + at);
        size_t dat = at;
        at += align_up(n * sizeof(double2));
        float2* ft = reinterpret_cast<float2*>(host.data() + at);
        size_t fat = at;
        at += align_up(n * sizeof(float2));
        const long double two_pi = 6.283185307179586476925286766559005768L;
        for (int64_t k = 0; k < n; ++k) {
            // exact values at the quarter points keep the table free of tiny residuals
            long double a = two_pi * (long double)k / (long double)n;
            double c = (double)cosl(a), s = (double)sinl(a);
            if (4 * k == n) { c = 0.0; s = 1.0; }
            if (2 * k == n) { c = -1.0; s = 0.0; }
            if (4 * k == 3 * n) { c = 0.0; s = -1.0; }
            dt[k] = make_double2(c, s);
            ft[k] = make_float2((float)c, (float)s);
        }
        offs.push_back({dat, fat});
    }
    void* mem = nullptr;
    cudaError_t err = cudaMalloc(&mem, bytes ? bytes : 1);
    if (err != cudaSuccess)
        return fail(NOP_E_NOMEM, std::string("twiddle table allocation: ") + cudaGetErrorString(err));
    err = cudaMemcpy(mem, host.data(), bytes, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        cudaFree(mem);
        return cuda_fail(err, "twiddle table upload");
    }
    p->table_mem = mem;
    for (size_t i = 0; i < lens.size(); ++i) {
        TwiddleTable t;
        t.n = lens[i];
        t.d_table = reinterpret_cast<const double2*>(static_cast<char*>(mem) + offs[i].first);
        t.f_table = reinterpret_cast<const float2*>(static_cast<char*>(mem) + offs[i].second);
        p->tables.push_back(t);
    }
    return NOP_OK;
}

}  // namespace
}  // namespace nop

using namespace nop;

extern "C" {

int32_t nop_abi_version(void) { return NOP_ABI_VERSION; }

const char* nop_last_error(void) { return g_last_error.c_str(); }

int32_t nop_spectral_plan_create(const nop_spectral_desc* desc, nop_plan** plan_out) {
    if (!plan_out) return fail(NOP_E_INVALID, "plan_out is NULL");
    *plan_out = nullptr;
    int32_t rc = validate(desc);
    if (rc != NOP_OK) return rc;
    Plan* p = new (std::nothrow) Plan();
    if (!p) return fail(NOP_E_NOMEM, "plan allocation failed");
    p->d = *desc;
    for (int j = 0; j < p->d.ndim; ++j) p->modes_total *= p->d.kept[j];
    for (int j = p->d.ndim; j < NOP_MAX_DIMS; ++j) {
        p->d.n_in[j] = p->d.n_out[j] = p->d.kept[j] = 1;
        p->d.fwd_off[j] = p->d.inv_off[j] = 0;
    }
    std::string why;
    FastKind kind = FastKind::None;
    const bool fast_ok = fast_supported(p->d, &kind, &why);
    if (p->d.engine == NOP_ENGINE_FAST && !fast_ok) {
        delete p;
        return fail(NOP_E_UNSUPPORTED, "fused FFT engine does not cover this shape: " + why);
    }
    cudaError_t err = cudaGetDevice(&p->device);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&p->sm_count, cudaDevAttrMultiProcessorCount, p->device);
    if (err != cudaSuccess) {
        delete p;
        return cuda_fail(err, "cudaGetDevice / multiprocessor count");
    }
    p->fast = fast_ok && p->d.engine != NOP_ENGINE_GENERIC;
    p->fast_kind = p->fast ? kind : FastKind::None;
    p->mix_tc = mix_on_tensor_cores();
    p->mix_tma = p->mix_tc && mix_with_tma();

    size_t off = 0;
    if (p->fast) {
        off = fast_workspace_bytes(*p, &p->ws);
    } else {
        p->ws.buf_elems = generic_buffer_elems(p->d);
        p->ws.buf_a = off;
        off += align_up((size_t)p->ws.buf_elems * sizeof(float2));
        p->ws.buf_b = off;
        off += align_up((size_t)p->ws.buf_elems * sizeof(float2));
        contraction_layout(*p, &off, &p->ws);
    }
    p->ws.bytes = off;

    rc = build_tables(p);
    if (rc != NOP_OK) {
        delete p;
        return rc;
    }
    *plan_out = reinterpret_cast<nop_plan*>(p);
    return NOP_OK;
}

void nop_spectral_plan_destroy(nop_plan* plan) {
    if (!plan) return;
    Plan* p = reinterpret_cast<Plan*>(plan);
    if (p->table_mem) {
        int prev = -1;
        cudaGetDevice(&prev);
        if (prev != p->device) cudaSetDevice(p->device);
        cudaFree(p->table_mem);
        if (prev >= 0 && prev != p->device) cudaSetDevice(prev);
    }
    delete p;
}

int32_t nop_spectral_workspace_size(const nop_plan* plan, size_t* bytes) {
    if (!plan || !bytes) return fail(NOP_E_INVALID, "plan and bytes must be non-NULL");
    *bytes = reinterpret_cast<const Plan*>(plan)->ws.bytes;
    return NOP_OK;
}

int32_t nop_spectral_plan_is_fast(const nop_plan* plan) {
    return plan && reinterpret_cast<const Plan*>(plan)->fast ? 1 : 0;
}

int32_t nop_spectral_launches_per_forward(const nop_plan* plan) {
    if (!plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    return p.fast ? fast_launches(p) : generic_launches(p);
}

static int32_t forward_impl(const nop_plan* plan, const void* x, const void* const* weights, int32_t n_weights,
                            const float* bias, const float* addend, int32_t apply_gelu, void* y, void* workspace,
                            size_t workspace_bytes, void* stream, float2* xs) {
    if (!plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    const nop_spectral_desc& d = p.d;
    if (n_weights != expected_weights(d))
        return fail(NOP_E_INVALID, "expected " + std::to_string(expected_weights(d)) + " weight pointers, got " +
                                       std::to_string(n_weights));
    if (d.batch == 0) return NOP_OK;
    if (!x || !y) return fail(NOP_E_INVALID, "x and y must be non-NULL");
    if (!weights) return fail(NOP_E_INVALID, "weights array is NULL");
    for (int i = 0; i < n_weights; ++i)
        if (!weights[i]) return fail(NOP_E_INVALID, "weight pointer " + std::to_string(i) + " is NULL");
    if (addend && d.complex_data) return fail(NOP_E_UNSUPPORTED, "addend / fused skip needs real data");
    if (apply_gelu && d.complex_data) return fail(NOP_E_UNSUPPORTED, "fused GELU needs real data");
    const size_t elem_align = d.complex_data ? 8 : 4;
    if ((uintptr_t)x % elem_align || (uintptr_t)y % elem_align || (bias && (uintptr_t)bias % 4) ||
        (addend && (uintptr_t)addend % 4))
        return fail(NOP_E_ALIGNMENT, "x / y / bias / addend are not aligned to their element size");
    for (int i = 0; i < n_weights; ++i)
        if ((uintptr_t)weights[i] % 8) return fail(NOP_E_ALIGNMENT, "weights must be 8-byte aligned (complex64)");
    if (p.ws.bytes > 0) {
        if (!workspace) return fail(NOP_E_WORKSPACE, "workspace is NULL");
        if (workspace_bytes < p.ws.bytes)
            return fail(NOP_E_WORKSPACE, "workspace has " + std::to_string(workspace_bytes) + " bytes, plan needs " +
                                             std::to_string(p.ws.bytes));
        if ((uintptr_t)workspace % kAlign) return fail(NOP_E_ALIGNMENT, "workspace must be 256-byte aligned");
    }
    int dev = -1;
    NOP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != p.device)
        return fail(NOP_E_INVALID, "plan was created on device " + std::to_string(p.device) +
                                       " but the current device is " + std::to_string(dev));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* ws = static_cast<char*>(workspace);
    launch_mark_begin(s);
    if (p.fast) return launch_mark_end(fast_forward(p, x, weights, bias, addend, apply_gelu, y, ws, s, xs));
    return launch_mark_end(generic_forward(p, x, weights, bias, addend, apply_gelu, y, ws, s, xs));
}

int32_t nop_spectral_forward(const nop_plan* plan, const void* x, const void* const* weights, int32_t n_weights,
                             const float* bias, const float* addend, int32_t apply_gelu, void* y, void* workspace,
                             size_t workspace_bytes, void* stream) {
    return forward_impl(plan, x, weights, n_weights, bias, addend, apply_gelu, y, workspace, workspace_bytes, stream,
                        nullptr);
}

static int32_t check_workspace(const Plan& p, const void* workspace, size_t workspace_bytes) {
    if (p.ws.bytes == 0) return NOP_OK;
    if (!workspace) return fail(NOP_E_WORKSPACE, "workspace is NULL");
    if (workspace_bytes < p.ws.bytes)
        return fail(NOP_E_WORKSPACE, "workspace has " + std::to_string(workspace_bytes) + " bytes, plan needs " +
                                         std::to_string(p.ws.bytes));
    if ((uintptr_t)workspace % kAlign) return fail(NOP_E_ALIGNMENT, "workspace must be 256-byte aligned");
    return NOP_OK;
}

static int32_t check_device(const Plan& p) {
    int dev = -1;
    NOP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != p.device)
        return fail(NOP_E_INVALID, "plan was created on device " + std::to_string(p.device) +
                                       " but the current device is " + std::to_string(dev));
    return NOP_OK;
}

int32_t nop_spectral_slab_plan_create(const nop_spectral_desc* desc, int32_t rank, int32_t world,
                                      nop_plan** plan_out) {
    if (!plan_out) return fail(NOP_E_INVALID, "plan_out is NULL");
    *plan_out = nullptr;
    if (world < 1 || world > NOP_MAX_SLAB_RANKS || rank < 0 || rank >= world)
        return fail(NOP_E_INVALID, "rank / world outside 0 <= rank < world <= " + std::to_string(NOP_MAX_SLAB_RANKS));
    int32_t rc = validate(desc);
    if (rc != NOP_OK) return rc;
    FastKind kind;
    std::string why;
    if (!fast_supported(*desc, &kind, &why) || kind != FastKind::Vol3D)
        return fail(NOP_E_UNSUPPORTED, "slab decomposition needs a fused 3D shape: " + why);
    if (desc->n_in[0] % world)
        return fail(NOP_E_INVALID, "first-axis size must be a multiple of the number of ranks");
    Plan* p = new (std::nothrow) Plan();
    if (!p) return fail(NOP_E_NOMEM, "plan allocation failed");
    p->d = *desc;
    for (int j = 0; j < p->d.ndim; ++j) p->modes_total *= p->d.kept[j];
    for (int j = p->d.ndim; j < NOP_MAX_DIMS; ++j) {
        p->d.n_in[j] = p->d.n_out[j] = p->d.kept[j] = 1;
        p->d.fwd_off[j] = p->d.inv_off[j] = 0;
    }
    p->fast = true;
    p->fast_kind = FastKind::Vol3DSlab;
    p->mix_tc = mix_on_tensor_cores();
    p->mix_tma = p->mix_tc && mix_with_tma();
    p->slab_rank = rank;
    p->slab_world = world;
    p->slab_nx = p->d.n_in[0] / world;
    const int64_t qp = p->d.kept[1] * p->d.kept[2] / 8;  // fused 3D shapes keep a multiple of 8 plane modes
    for (int r = 0; r < world; ++r) {  // balanced split of the plane-mode blocks
        p->slab_qcount[r] = qp / world + (r < qp % world ? 1 : 0);
        p->slab_qbegin[r] = r * (qp / world) + (r < qp % world ? r : qp % world);
    }
    cudaError_t err = cudaGetDevice(&p->device);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&p->sm_count, cudaDevAttrMultiProcessorCount, p->device);
    if (err != cudaSuccess) {
        delete p;
        return cuda_fail(err, "cudaGetDevice / multiprocessor count");
    }
    p->ws.bytes = fast_workspace_bytes(*p, &p->ws);
    rc = build_tables(p);
    if (rc != NOP_OK) {
        delete p;
        return rc;
    }
    *plan_out = reinterpret_cast<nop_plan*>(p);
    return NOP_OK;
}

int32_t nop_spectral_slab_info(const nop_plan* plan, nop_slab_info* info) {
    if (!plan || !info) return fail(NOP_E_INVALID, "plan and info must be non-NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    if (p.fast_kind != FastKind::Vol3DSlab) return fail(NOP_E_INVALID, "not a slab plan");
    *info = nop_slab_info{};
    const nop_spectral_desc& d = p.d;
    const int64_t nx = p.slab_nx, r = p.slab_rank;
    const size_t blk_in = (size_t)d.batch * d.in_channels * nx * 8 * sizeof(float2);   // one block, one slab
    const size_t blk_out = (size_t)d.batch * d.out_channels * nx * 8 * sizeof(float2);
    info->rank = p.slab_rank;
    info->world = p.slab_world;
    info->x_begin = r * nx;
    info->x_count = nx;
    info->plane_blocks = d.kept[1] * d.kept[2] / 8;
    for (int s = 0; s < p.slab_world; ++s) {
        info->block_begin[s] = p.slab_qbegin[s];
        info->block_count[s] = p.slab_qcount[s];
        info->send1_split[s] = p.slab_qcount[s] * blk_in;   // my planes of s's blocks
        info->recv1_split[s] = p.slab_qcount[r] * blk_in;   // s's planes of my blocks
        info->send2_split[s] = p.slab_qcount[r] * blk_out;  // my blocks on s's planes
        info->recv2_split[s] = p.slab_qcount[s] * blk_out;  // s's blocks on my planes
        info->send1_bytes += info->send1_split[s];
        info->recv1_bytes += info->recv1_split[s];
        info->send2_bytes += info->send2_split[s];
        info->recv2_bytes += info->recv2_split[s];
    }
    return NOP_OK;
}

static int32_t slab_plan(const nop_plan* plan, const Plan** out) {
    if (!plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan* p = reinterpret_cast<const Plan*>(plan);
    if (p->fast_kind != FastKind::Vol3DSlab) return fail(NOP_E_INVALID, "not a slab plan");
    *out = p;
    return check_device(*p);
}

int32_t nop_spectral_slab_forward_planes(const nop_plan* plan, const float* x, void* send1, void* stream) {
    const Plan* p;
    int32_t rc = slab_plan(plan, &p);
    if (rc != NOP_OK) return rc;
    if (!x || !send1) return fail(NOP_E_INVALID, "x and send1 must be non-NULL");
    if ((uintptr_t)send1 % 16 || (uintptr_t)x % 4) return fail(NOP_E_ALIGNMENT, "send1 must be 16-byte aligned");
    return fast_slab_planes_fwd(*p, x, send1, static_cast<cudaStream_t>(stream));
}

int32_t nop_spectral_slab_modes(const nop_plan* plan, const void* recv1, const void* packed, size_t packed_bytes,
                                void* send2, void* workspace, size_t workspace_bytes, void* stream) {
    const Plan* p;
    int32_t rc = slab_plan(plan, &p);
    if (rc != NOP_OK) return rc;
    if (!recv1 || !send2) return fail(NOP_E_INVALID, "recv1 and send2 must be non-NULL");
    if (!packed || packed_bytes < p->packed_bytes)
        return fail(NOP_E_WORKSPACE, "packed-weight buffer missing or smaller than nop_spectral_packed_size");
    if ((uintptr_t)recv1 % 16 || (uintptr_t)send2 % 16 || (uintptr_t)packed % 16)
        return fail(NOP_E_ALIGNMENT, "exchange and packed buffers must be 16-byte aligned");
    if ((rc = check_workspace(*p, workspace, workspace_bytes)) != NOP_OK) return rc;
    return fast_slab_modes(*p, recv1, static_cast<const char*>(packed), send2, static_cast<char*>(workspace),
                           static_cast<cudaStream_t>(stream));
}

int32_t nop_spectral_slab_inverse_planes(const nop_plan* plan, const void* recv2, const float* bias,
                                         const float* addend, int32_t apply_gelu, float* y, void* stream) {
    const Plan* p;
    int32_t rc = slab_plan(plan, &p);
    if (rc != NOP_OK) return rc;
    if (!recv2 || !y) return fail(NOP_E_INVALID, "recv2 and y must be non-NULL");
    if ((uintptr_t)recv2 % 16) return fail(NOP_E_ALIGNMENT, "recv2 must be 16-byte aligned");
    return fast_slab_planes_inv(*p, recv2, bias, addend, apply_gelu, y, static_cast<cudaStream_t>(stream));
}

int32_t nop_device_status(int32_t* status, int32_t clear) {
    if (!status) return fail(NOP_E_INVALID, "status is NULL");
    int v = 0;
    int32_t rc = fast_device_status(&v, clear != 0);
    if (rc == NOP_OK) *status = v;
    return rc;
}

int32_t nop_set_launch_events(void* const* events, int32_t n) {
    if (n < 0 || n > 32) return fail(NOP_E_INVALID, "event count must be in 0..32");
    if (n > 0 && !events) return fail(NOP_E_INVALID, "events is NULL");
    for (int i = 0; i < n; ++i) g_events.ev[i] = static_cast<cudaEvent_t>(events[i]);
    g_events.n = n;
    g_events.next = 0;
    return NOP_OK;
}

int32_t nop_spectral_packed_size(const nop_plan* plan, size_t* bytes) {
    if (!plan || !bytes) return fail(NOP_E_INVALID, "plan and bytes must be non-NULL");
    *bytes = reinterpret_cast<const Plan*>(plan)->packed_bytes;
    return NOP_OK;
}

int32_t nop_spectral_pack_weights(const nop_plan* plan, const void* const* weights, int32_t n_weights, void* packed,
                                  size_t packed_bytes, void* workspace, size_t workspace_bytes, void* stream) {
    if (!plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    if (p.packed_bytes == 0) return fail(NOP_E_UNSUPPORTED, "this plan takes its weights unpacked");
    if (n_weights != expected_weights(p.d))
        return fail(NOP_E_INVALID, "expected " + std::to_string(expected_weights(p.d)) + " weight pointers, got " +
                                       std::to_string(n_weights));
    if (!weights) return fail(NOP_E_INVALID, "weights array is NULL");
    for (int i = 0; i < n_weights; ++i) {
        if (!weights[i]) return fail(NOP_E_INVALID, "weight pointer " + std::to_string(i) + " is NULL");
        if ((uintptr_t)weights[i] % 8) return fail(NOP_E_ALIGNMENT, "weights must be 8-byte aligned (complex64)");
    }
    if (!packed || packed_bytes < p.packed_bytes)
        return fail(NOP_E_WORKSPACE, "packed-weight buffer missing or smaller than nop_spectral_packed_size");
    if ((uintptr_t)packed % kAlign) return fail(NOP_E_ALIGNMENT, "packed-weight buffer must be 256-byte aligned");
    int32_t rc = check_workspace(p, workspace, workspace_bytes);
    if (rc != NOP_OK) return rc;
    if ((rc = check_device(p)) != NOP_OK) return rc;
    return fast_pack(p, weights, static_cast<char*>(packed), static_cast<char*>(workspace),
                     static_cast<cudaStream_t>(stream));
}

int32_t nop_spectral_pack_weights_adjoint(const nop_plan* adjoint_plan, const void* forward_weight, void* packed,
                                          size_t packed_bytes, void* stream) {
    if (!adjoint_plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(adjoint_plan);
    if (p.packed_bytes == 0) return fail(NOP_E_UNSUPPORTED, "this plan takes its weights unpacked");
    if (p.d.weight_kind != NOP_WEIGHT_DENSE || p.d.separable)
        return fail(NOP_E_UNSUPPORTED, "adjoint packing needs a dense, non-separable weight");
    if (!forward_weight) return fail(NOP_E_INVALID, "weight pointer is NULL");
    if ((uintptr_t)forward_weight % 8) return fail(NOP_E_ALIGNMENT, "weights must be 8-byte aligned (complex64)");
    if (!packed || packed_bytes < p.packed_bytes)
        return fail(NOP_E_WORKSPACE, "packed-weight buffer missing or smaller than nop_spectral_packed_size");
    if ((uintptr_t)packed % kAlign) return fail(NOP_E_ALIGNMENT, "packed-weight buffer must be 256-byte aligned");
    int32_t rc = check_device(p);
    if (rc != NOP_OK) return rc;
    return fast_pack_adjoint(p, forward_weight, static_cast<char*>(packed), static_cast<cudaStream_t>(stream));
}

static int32_t forward_packed_impl(const nop_plan* plan, const void* x, const void* packed, size_t packed_bytes,
                                   const float* bias, const float* addend, int32_t apply_gelu, void* y,
                                   void* workspace, size_t workspace_bytes, void* stream, float2* xs) {
    if (!plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    const nop_spectral_desc& d = p.d;
    if (p.packed_bytes == 0) return fail(NOP_E_UNSUPPORTED, "this plan takes its weights unpacked");
    if (d.batch == 0) return NOP_OK;
    if (!x || !y) return fail(NOP_E_INVALID, "x and y must be non-NULL");
    if (!packed || packed_bytes < p.packed_bytes)
        return fail(NOP_E_WORKSPACE, "packed-weight buffer missing or smaller than nop_spectral_packed_size");
    if ((uintptr_t)packed % kAlign) return fail(NOP_E_ALIGNMENT, "packed-weight buffer must be 256-byte aligned");
    if ((uintptr_t)x % 4 || (uintptr_t)y % 4 || (bias && (uintptr_t)bias % 4) || (addend && (uintptr_t)addend % 4))
        return fail(NOP_E_ALIGNMENT, "x / y / bias / addend are not aligned to their element size");
    int32_t rc = check_workspace(p, workspace, workspace_bytes);
    if (rc != NOP_OK) return rc;
    if ((rc = check_device(p)) != NOP_OK) return rc;
    launch_mark_begin(static_cast<cudaStream_t>(stream));
    return launch_mark_end(fast_forward_packed(p, x, static_cast<const char*>(packed), bias, addend, apply_gelu, y,
                                               static_cast<char*>(workspace), static_cast<cudaStream_t>(stream), xs));
}

int32_t nop_spectral_forward_packed(const nop_plan* plan, const void* x, const void* packed, size_t packed_bytes,
                                    const float* bias, const float* addend, int32_t apply_gelu, void* y,
                                    void* workspace, size_t workspace_bytes, void* stream) {
    return forward_packed_impl(plan, x, packed, packed_bytes, bias, addend, apply_gelu, y, workspace, workspace_bytes,
                               stream, nullptr);
}

/* ---- backward support ----------------------------------------------------------------------- */

int32_t nop_spectral_spectrum_layout(const nop_plan* plan, int64_t* strides, size_t* bytes) {
    if (!plan || !strides || !bytes) return fail(NOP_E_INVALID, "NULL argument");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    return spectrum_layout(p, &strides[0], &strides[1], &strides[2], bytes);
}

int32_t nop_spectral_forward_keep(const nop_plan* plan, const void* x, const void* const* weights, int32_t n_weights,
                                  const void* packed, size_t packed_bytes, const float* bias, const float* addend,
                                  int32_t apply_gelu, void* y, void* x_spec, size_t x_spec_bytes, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    if (!plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    int64_t st[3];
    size_t need = 0;
    int32_t rc = spectrum_layout(p, &st[0], &st[1], &st[2], &need);
    if (rc != NOP_OK) return rc;
    if (p.d.batch == 0) return NOP_OK;
    if (!x_spec || x_spec_bytes < need)
        return fail(NOP_E_WORKSPACE, "spectrum buffer missing or smaller than nop_spectral_spectrum_layout's size");
    if ((uintptr_t)x_spec % kAlign) return fail(NOP_E_ALIGNMENT, "spectrum buffer must be 256-byte aligned");
    float2* xs = static_cast<float2*>(x_spec);
    if (packed)
        return forward_packed_impl(plan, x, packed, packed_bytes, bias, addend, apply_gelu, y, workspace,
                                   workspace_bytes, stream, xs);
    return forward_impl(plan, x, weights, n_weights, bias, addend, apply_gelu, y, workspace, workspace_bytes, stream,
                        xs);
}

int32_t nop_spectral_weight_grad_workspace_size(const nop_plan* plan, size_t* bytes) {
    if (!plan || !bytes) return fail(NOP_E_INVALID, "NULL argument");
    *bytes = weight_grad_workspace(*reinterpret_cast<const Plan*>(plan));
    return NOP_OK;
}

int32_t nop_spectral_weight_grad(const nop_plan* plan, const void* x_spec, const nop_plan* adjoint_plan,
                                 const void* g_spec, void* grad_w, float* grad_bias, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    if (!plan || !adjoint_plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    const Plan& a = *reinterpret_cast<const Plan*>(adjoint_plan);
    if (p.device != a.device) return fail(NOP_E_INVALID, "plans live on different devices");
    if ((x_spec && (uintptr_t)x_spec % 8) || (g_spec && (uintptr_t)g_spec % 8) || (grad_w && (uintptr_t)grad_w % 8) ||
        (grad_bias && (uintptr_t)grad_bias % 4))
        return fail(NOP_E_ALIGNMENT, "spectra / gradients are not aligned to their element size");
    int32_t rc = check_device(p);
    if (rc != NOP_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    launch_mark_begin(s);
    if (workspace && (uintptr_t)workspace % kAlign) return fail(NOP_E_ALIGNMENT, "workspace must be 256-byte aligned");
    return launch_mark_end(weight_grad(p, x_spec, a, g_spec, grad_w, grad_bias, workspace, workspace_bytes, s));
}

/* ---- forward from host memory ------------------------------------------------------------- */

struct HostChunkLayout {
    size_t x_bytes, y_bytes;   // one chunk of desc.batch samples
    size_t x_off, y_off, a_off, ws_off, per_stream;
};

static HostChunkLayout host_layout(const Plan& p) {
    const nop_spectral_desc& d = p.d;
    const size_t esz = d.complex_data ? 8 : 4;
    int64_t pin = 1, pout = 1;
    for (int j = 0; j < d.ndim; ++j) {
        pin *= d.n_in[j];
        pout *= d.n_out[j];
    }
    HostChunkLayout h{};
    h.x_bytes = (size_t)d.batch * d.in_channels * pin * esz;
    h.y_bytes = (size_t)d.batch * d.out_channels * pout * esz;
    h.x_off = 0;
    h.y_off = align_up(h.x_bytes);
    h.a_off = h.y_off + align_up(h.y_bytes);
    h.ws_off = h.a_off + align_up(h.y_bytes);
    h.per_stream = h.ws_off + align_up(p.ws.bytes);
    return h;
}

int32_t nop_spectral_host_workspace_size(const nop_plan* plan, int32_t n_streams, size_t* bytes) {
    if (!plan || !bytes) return fail(NOP_E_INVALID, "plan and bytes must be non-NULL");
    if (n_streams < 1 || n_streams > 8) return fail(NOP_E_INVALID, "n_streams must be in 1..8");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    if (p.fast_kind == FastKind::Vol3DSlab) return fail(NOP_E_INVALID, "slab plans have no host forward");
    // [packed weights][stream 0 region][stream 1 region]...
    *bytes = align_up(p.packed_bytes) + (size_t)n_streams * host_layout(p).per_stream;
    return NOP_OK;
}

int32_t nop_spectral_forward_host(const nop_plan* plan, const void* x_host, int64_t total_batch,
                                  const void* const* weights, int32_t n_weights, const void* packed,
                                  size_t packed_bytes, const float* bias, const float* addend_host,
                                  int32_t apply_gelu, void* y_host, void* workspace, size_t workspace_bytes,
                                  int32_t n_streams, void* stream) {
    if (!plan) return fail(NOP_E_INVALID, "plan is NULL");
    const Plan& p = *reinterpret_cast<const Plan*>(plan);
    const nop_spectral_desc& d = p.d;
    size_t need = 0;
    int32_t rc = nop_spectral_host_workspace_size(plan, n_streams, &need);
    if (rc != NOP_OK) return rc;
    if (total_batch < 0) return fail(NOP_E_INVALID, "total_batch is negative");
    if (total_batch == 0) return NOP_OK;
    if (d.batch == 0 || total_batch % d.batch)
        return fail(NOP_E_INVALID, "total_batch (" + std::to_string(total_batch) +
                                       ") must be a multiple of the plan's batch (" + std::to_string(d.batch) + ")");
    if (!x_host || !y_host) return fail(NOP_E_INVALID, "x_host and y_host must be non-NULL");
    if ((addend_host || apply_gelu) && d.complex_data)
        return fail(NOP_E_UNSUPPORTED, "addend / fused GELU need real data");
    if (bias && (uintptr_t)bias % 4) return fail(NOP_E_ALIGNMENT, "bias must be 4-byte aligned");
    const bool use_packed = packed != nullptr;
    if (use_packed) {
        if (p.packed_bytes == 0) return fail(NOP_E_UNSUPPORTED, "this plan takes its weights unpacked");
        if (packed_bytes < p.packed_bytes)
            return fail(NOP_E_WORKSPACE, "packed-weight buffer smaller than nop_spectral_packed_size");
        if ((uintptr_t)packed % kAlign) return fail(NOP_E_ALIGNMENT, "packed-weight buffer must be 256-byte aligned");
    } else {
        if (n_weights != expected_weights(d))
            return fail(NOP_E_INVALID, "expected " + std::to_string(expected_weights(d)) +
                                           " weight pointers, got " + std::to_string(n_weights));
        if (!weights) return fail(NOP_E_INVALID, "give either packed weights or the weights array");
        for (int i = 0; i < n_weights; ++i) {
            if (!weights[i]) return fail(NOP_E_INVALID, "weight pointer " + std::to_string(i) + " is NULL");
            if ((uintptr_t)weights[i] % 8) return fail(NOP_E_ALIGNMENT, "weights must be 8-byte aligned (complex64)");
        }
    }
    if (!workspace || workspace_bytes < need)
        return fail(NOP_E_WORKSPACE, "host-forward workspace has " + std::to_string(workspace_bytes) +
                                         " bytes, nop_spectral_host_workspace_size gives " + std::to_string(need));
    if ((uintptr_t)workspace % kAlign) return fail(NOP_E_ALIGNMENT, "workspace must be 256-byte aligned");
    if ((rc = check_device(p)) != NOP_OK) return rc;

    const HostChunkLayout h = host_layout(p);
    char* base = static_cast<char*>(workspace);
    char* packed_ws = base;
    char* regions = base + align_up(p.packed_bytes);
    cudaStream_t caller = static_cast<cudaStream_t>(stream);

    // Streams and events live for this call only: destroying them with work still queued is legal
    // (their resources are released once that work completes), so nothing outlives the call.
    cudaStream_t st[8] = {};
    cudaEvent_t ev[9] = {};
    auto release = [&]() {
        for (auto& e : ev)
            if (e) cudaEventDestroy(e);
        for (auto& q : st)
            if (q) cudaStreamDestroy(q);
    };
    auto cuda_err = [&](cudaError_t err, const char* what) {
        release();
        return cuda_fail(err, what);
    };
    cudaError_t err;
    for (int i = 0; i <= n_streams; ++i)
        if ((err = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming)) != cudaSuccess)
            return cuda_err(err, "cudaEventCreateWithFlags");
    for (int i = 0; i < n_streams; ++i)
        if ((err = cudaStreamCreateWithFlags(&st[i], cudaStreamNonBlocking)) != cudaSuccess)
            return cuda_err(err, "cudaStreamCreateWithFlags");
    if ((err = cudaEventRecord(ev[n_streams], caller)) != cudaSuccess) return cuda_err(err, "cudaEventRecord");
    for (int i = 0; i < n_streams; ++i)
        if ((err = cudaStreamWaitEvent(st[i], ev[n_streams], 0)) != cudaSuccess)
            return cuda_err(err, "cudaStreamWaitEvent");

    // Fused plans given unpacked weights pack them once; every stream then waits for the packing.
    const char* pk = static_cast<const char*>(packed);
    if (!use_packed && p.fast) {
        if ((rc = fast_pack(p, weights, packed_ws, regions + h.ws_off, st[0])) != NOP_OK) {
            release();
            return rc;
        }
        if ((err = cudaEventRecord(ev[n_streams], st[0])) != cudaSuccess) return cuda_err(err, "cudaEventRecord");
        for (int i = 1; i < n_streams; ++i)
            if ((err = cudaStreamWaitEvent(st[i], ev[n_streams], 0)) != cudaSuccess)
                return cuda_err(err, "cudaStreamWaitEvent");
        pk = packed_ws;
    }

    const int64_t chunks = total_batch / d.batch;
    const char* xh = static_cast<const char*>(x_host);
    const char* ah = reinterpret_cast<const char*>(addend_host);
    char* yh = static_cast<char*>(y_host);
    for (int64_t c = 0; c < chunks; ++c) {
        const int i = (int)(c % n_streams);
        cudaStream_t s = st[i];
        char* r = regions + (size_t)i * h.per_stream;
        if ((err = cudaMemcpyAsync(r + h.x_off, xh + c * h.x_bytes, h.x_bytes, cudaMemcpyHostToDevice, s)) !=
            cudaSuccess)
            return cuda_err(err, "cudaMemcpyAsync (x chunk)");
        const float* a_dev = nullptr;
        if (ah) {
            if ((err = cudaMemcpyAsync(r + h.a_off, ah + c * h.y_bytes, h.y_bytes, cudaMemcpyHostToDevice, s)) !=
                cudaSuccess)
                return cuda_err(err, "cudaMemcpyAsync (addend chunk)");
            a_dev = reinterpret_cast<const float*>(r + h.a_off);
        }
        if (p.fast)
            rc = fast_forward_packed(p, r + h.x_off, pk, bias, a_dev, apply_gelu, r + h.y_off, r + h.ws_off, s);
        else
            rc = generic_forward(p, r + h.x_off, weights, bias, a_dev, apply_gelu, r + h.y_off, r + h.ws_off, s);
        if (rc != NOP_OK) {
            release();
            return rc;
        }
        if ((err = cudaMemcpyAsync(yh + c * h.y_bytes, r + h.y_off, h.y_bytes, cudaMemcpyDeviceToHost, s)) !=
            cudaSuccess)
            return cuda_err(err, "cudaMemcpyAsync (y chunk)");
    }
    for (int i = 0; i < n_streams; ++i) {
        if ((err = cudaEventRecord(ev[i], st[i])) != cudaSuccess) return cuda_err(err, "cudaEventRecord");
        if ((err = cudaStreamWaitEvent(caller, ev[i], 0)) != cudaSuccess) return cuda_err(err, "cudaStreamWaitEvent");
    }
    release();
    return NOP_OK;
}

}  // extern "C"

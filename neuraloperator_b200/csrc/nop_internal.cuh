// Internal declarations shared by the libnop_b200 translation units.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "nop_spectral.h"

namespace nop {

// ------------------------------------------------------------------------------------------
// error reporting (thread-local message behind nop_last_error)
// ------------------------------------------------------------------------------------------
void set_error(const std::string& msg);
int32_t fail(int32_t code, const std::string& msg);
int32_t cuda_fail(cudaError_t err, const char* what);

#define NOP_CUDA_TRY(call)                                         \
    do {                                                           \
        cudaError_t e_ = (call);                                   \
        if (e_ != cudaSuccess) return ::nop::cuda_fail(e_, #call); \
    } while (0)

// ------------------------------------------------------------------------------------------
// plan
// ------------------------------------------------------------------------------------------
struct TwiddleTable {
    int64_t n = 0;
    const double2* d_table = nullptr;  // (cos 2 pi k / n, sin 2 pi k / n), k < n   (generic path)
    const float2* f_table = nullptr;   // same values rounded to float               (fused path)
};

struct WorkspaceLayout {
    size_t bytes = 0;
    size_t buf_a = 0, buf_b = 0;       // ping-pong spectra (complex64)
    size_t g = 0, g_tmp = 0;           // factorized weight expansions
    size_t xf = 0, z = 0;              // factorized contraction intermediates
    size_t packed = 0;                 // packed weights (fused engine, unpacked forward only)
    size_t pl_a = 0, pl_b = 0;         // 3D: plane spectra before / after the outer-axis transform
    int64_t buf_elems = 0;
};

enum class FastKind : int32_t { None = 0, Plane2D = 1, Row1D = 2, Vol3D = 3, Vol3DSlab = 4 };

constexpr int kMaxSlabRanks = 64;

struct Plan {
    nop_spectral_desc d{};
    int device = 0;
    int sm_count = 148;                // multiprocessors of `device` (persistent grids)
    bool fast = false;
    FastKind fast_kind = FastKind::None;
    int64_t modes_total = 1;           // prod(kept)
    std::vector<TwiddleTable> tables;  // one per distinct transform length
    void* table_mem = nullptr;         // single device allocation holding every table
    WorkspaceLayout ws;
    size_t packed_bytes = 0;           // fused engine: packed-weight buffer size (0: no packing)
    bool mix_tc = true;                // fused engine: contraction on the tensor cores (tcgen05)
    bool mix_tma = true;               // ... by the TMA kernel on pre-split weight tiles (packed layout)
    // 3D slab decomposition (FastKind::Vol3DSlab): this rank's x planes and everyone's mode blocks
    int slab_rank = 0, slab_world = 1;
    int64_t slab_nx = 0;                                   // x planes per rank
    int64_t slab_qbegin[kMaxSlabRanks] = {}, slab_qcount[kMaxSlabRanks] = {};
    size_t pk_w = 0, pk_uin = 0, pk_uout = 0;  // offsets inside the packed-weight buffer

    const TwiddleTable* table(int64_t n) const {
        for (const auto& t : tables)
            if (t.n == n) return &t;
        return nullptr;
    }
};

// measurement hook: record the caller's events around kernel launches (api.cu)
void launch_mark_begin(cudaStream_t s);
void launch_mark(cudaStream_t s);

// descriptor checks and contraction workspace regions (api.cu)
int expected_weights(const nop_spectral_desc& d);
int32_t validate(const nop_spectral_desc* d);
void contraction_layout(const Plan& p, size_t* off, WorkspaceLayout* ws);

// ------------------------------------------------------------------------------------------
// generic direct-DFT engine (any sizes, any ndim): generic.cu
// ------------------------------------------------------------------------------------------
int64_t generic_buffer_elems(const nop_spectral_desc& d);
// xs (nullable): also leave the kept input spectrum there (layout: spectrum_layout)
int32_t generic_forward(const Plan& p, const void* x, const void* const* weights, const float* bias,
                        const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s,
                        float2* xs = nullptr);

int32_t generic_launches(const Plan& p);
// Tucker core expanded along the spatial modes into the g / g_tmp workspace regions
float2* expand_tucker_core(const Plan& p, const float2* core, const void* const* weights, int first_spatial_w,
                           int64_t lead, char* ws, cudaError_t* err, cudaStream_t s);
int32_t contract_launches(const Plan& p);

// contraction stage shared by both engines: X [B, Ci, Mt] -> Y [B, Co, Mt]
int32_t contract_stage(const Plan& p, const float2* X, const void* const* weights, float2* Y, char* ws,
                       cudaStream_t s);

// fused FFT engine: fast.cu
bool fast_supported(const nop_spectral_desc& d, FastKind* kind, std::string* why);
size_t fast_workspace_bytes(Plan& p, WorkspaceLayout* ws);
int32_t fast_launches(const Plan& p);
// status word of the tensor-core kernels on the current device (synchronous read, optional reset)
int32_t fast_device_status(int* status, bool clear);
// device address of that status word on `device` (kernels write it when a bounded wait expires)
int* status_word(int device);
// cuTensorMapEncodeTiled looked up through the runtime (nullptr when the driver lacks it)
void* tensor_map_encoder();
int32_t fast_pack(const Plan& p, const void* const* weights, char* packed, char* ws, cudaStream_t s);
// adjoint plan's packed weights straight from the forward's dense weight (conjugate transpose in the pack)
int32_t fast_pack_adjoint(const Plan& p, const void* W, char* packed, cudaStream_t s);
// xs (nullable): the contraction reads the kept input spectrum from xs instead of the workspace,
// so it is still there after the call
int32_t fast_forward_packed(const Plan& p, const void* x, const char* packed, const float* bias,
                            const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s,
                            float2* xs = nullptr);
int32_t fast_forward(const Plan& p, const void* x, const void* const* weights, const float* bias,
                     const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s, float2* xs = nullptr);
int32_t fast_slab_planes_fwd(const Plan& p, const float* x, void* send1, cudaStream_t s);
int32_t fast_slab_modes(const Plan& p, const void* recv1, const char* packed, void* send2, char* ws,
                        cudaStream_t s);
int32_t fast_slab_planes_inv(const Plan& p, const void* recv2, const float* bias, const float* addend,
                             int apply_gelu, float* y, cudaStream_t s);

// backward: kept-spectrum layout of a plan's input side and the weight / bias gradients (grad.cu)
int32_t spectrum_layout(const Plan& p, int64_t* q_stride, int64_t* b_stride, int64_t* c_stride, size_t* bytes);
size_t weight_grad_workspace(const Plan& p);
int32_t weight_grad(const Plan& p, const void* x_spec, const Plan& adjoint, const void* g_spec, void* grad_w,
                    float* grad_bias, void* workspace, size_t workspace_bytes, cudaStream_t s);

// ------------------------------------------------------------------------------------------
// small device helpers
// ------------------------------------------------------------------------------------------
__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

__device__ __forceinline__ float gelu_erf(float v) {
    // exact GELU, as torch.nn.functional.gelu(approximate="none")
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
}

__device__ __forceinline__ float round_bf16(float v) {
    // value after rounding to bfloat16 (round to nearest even), as float
    return __bfloat162float(__float2bfloat16_rn(v));
}

}  // namespace nop

// Fused FFT engine (placeholder until the fused kernels land): covers no shape yet.
#include "nop_internal.cuh"

namespace nop {

bool fast_supported(const nop_spectral_desc& d, FastKind* kind, std::string* why) {
    (void)d;
    *kind = FastKind::None;
    *why = "no fused kernels built";
    return false;
}

size_t fast_workspace_bytes(const Plan& p, WorkspaceLayout* ws) {
    (void)p;
    (void)ws;
    return 0;
}

int32_t fast_launches(const Plan& p) {
    (void)p;
    return 0;
}

int32_t fast_forward(const Plan& p, const void* x, const void* const* weights, const float* bias,
                     const float* addend, int apply_gelu, void* y, char* ws, cudaStream_t s) {
    (void)p; (void)x; (void)weights; (void)bias; (void)addend; (void)apply_gelu; (void)y; (void)ws; (void)s;
    return fail(NOP_E_UNSUPPORTED, "fused FFT engine not available");
}

}  // namespace nop

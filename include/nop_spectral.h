/*
 * nop_spectral.h — C ABI of the B200 FNO spectral block (libnop_b200.so).
 *
 * One SpectralConv forward (neuralop/layers/spectral_convolution.py:417-570) is
 *   truncated forward real FFT over every spatial axis  ->  per-mode channel contraction
 *   (dense, separable, Tucker or CP weights)  ->  truncated inverse FFT  ->  + bias
 * optionally followed by the FNOBlocks epilogue  y = gelu(y + skip)
 * (neuralop/layers/fno_block.py:356-361).
 *
 * Conventions
 *   - All device pointers are CUDA device memory of the current device.  Complex data are
 *     interleaved float pairs (complex64).  Every tensor is contiguous, row-major.
 *   - x   : [B, Ci, n_in[0..ndim-1]]   float32 (complex64 when complex_data)
 *   - y   : [B, Co, n_out[0..ndim-1]]  float32 (complex64 when complex_data)
 *   - The caller owns every buffer, including the workspace, whose size the plan reports.
 *     Forward calls never allocate; plan creation allocates the plan's twiddle tables.
 *   - Kernels are enqueued on `stream` (a cudaStream_t; NULL = legacy default stream).
 *   - Functions return NOP_OK (0) or a negative nop_status; nop_last_error() then returns
 *     a message for the calling thread.  All argument checks run on the host before any
 *     launch; no kernel traps.
 *
 * Geometry: kept mode m of axis j is DFT bin u = (m - fwd_off[j]) mod n_in[j] in the forward
 * transform and bin index u = (m - inv_off[j]) mod n_in[j] in the inverse, where bins with
 * u >= n_out[j] are dropped (ifftn with s=n_out truncates / zero-pads at the end).  For real
 * data the last axis keeps rFFT bins 0..kept-1 (offsets 0) and is inverted with the Hermitian
 * c2r rule; the bins listed in zero_imag_bins contribute only their real part.  The Python
 * layer fills these from the reference's fftshift / slice / ifftshift bookkeeping
 * (spectral_convolution.py:443-559).
 */
#ifndef NOP_SPECTRAL_H
#define NOP_SPECTRAL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NOP_ABI_VERSION 1
#define NOP_MAX_DIMS 4

typedef enum nop_status {
    NOP_OK = 0,
    NOP_E_INVALID = -1,      /* malformed descriptor or argument */
    NOP_E_UNSUPPORTED = -2,  /* well-formed request this library does not implement */
    NOP_E_ALIGNMENT = -3,    /* a pointer is not aligned as required */
    NOP_E_WORKSPACE = -4,    /* workspace missing or smaller than nop_spectral_workspace_size */
    NOP_E_CUDA = -5,         /* CUDA runtime error (message names the call) */
    NOP_E_NOMEM = -6         /* host or device allocation failed during plan creation */
} nop_status;

typedef enum nop_weight_kind {
    NOP_WEIGHT_DENSE = 0,    /* weights[0] = W [Ci, Co, kept...] (separable: [C, kept...])            */
    NOP_WEIGHT_TUCKER = 1,   /* weights = core, U_in, U_out, U_1..U_ndim (separable: core, U_c, U_j)  */
    NOP_WEIGHT_CP = 2        /* weights = lambda, U_in, U_out, U_1..U_ndim (separable: lambda, U_c, U_j) */
} nop_weight_kind;

typedef enum nop_precision {
    NOP_PRECISION_FP32 = 0,  /* float32 transforms and contraction                                  */
    NOP_PRECISION_BF16 = 1   /* contraction operands rounded to bfloat16, float32 accumulation        */
} nop_precision;

typedef enum nop_engine {
    NOP_ENGINE_AUTO = 0,     /* fused FFT kernels where the shape is supported, else generic         */
    NOP_ENGINE_GENERIC = 1,  /* direct-DFT kernels: any sizes, any ndim; slower                         */
    NOP_ENGINE_FAST = 2      /* fused FFT kernels only; NOP_E_UNSUPPORTED when the shape is not covered */
} nop_engine;

typedef struct nop_spectral_desc {
    int32_t abi_version;                 /* must be NOP_ABI_VERSION                                 */
    int32_t ndim;                        /* spatial dims, 1..NOP_MAX_DIMS                            */
    int32_t complex_data;                /* 1: x and y are complex64                                 */
    int32_t separable;                   /* 1: diagonal in channels (Ci == Co)                       */
    int32_t weight_kind;                 /* nop_weight_kind                                          */
    int32_t precision;                   /* nop_precision                                            */
    int32_t engine;                      /* nop_engine                                               */
    int32_t n_zero_imag;                 /* entries used in zero_imag_bins (0..3)                    */
    int64_t batch;                       /* B (0 is allowed: calls return immediately)               */
    int64_t in_channels;                 /* Ci                                                       */
    int64_t out_channels;                /* Co                                                       */
    int64_t n_in[NOP_MAX_DIMS];          /* input spatial sizes                                      */
    int64_t n_out[NOP_MAX_DIMS];         /* output spatial sizes                                     */
    int64_t kept[NOP_MAX_DIMS];          /* kept modes per axis (the weight's mode dims)             */
    int64_t fwd_off[NOP_MAX_DIMS];       /* forward bin offset per axis                              */
    int64_t inv_off[NOP_MAX_DIMS];       /* inverse bin offset per axis                              */
    int64_t ranks[NOP_MAX_DIMS + 2];     /* Tucker: r_in, r_out, r_1..r_ndim (separable: r_c, r_j);
                                            CP: ranks[0] = R                                         */
    int64_t zero_imag_bins[3];           /* real data: last-axis bins read as real                   */
    double fwd_scale;                    /* forward normalisation (1/prod(n_in) for norm="forward")  */
    double inv_scale;                    /* inverse normalisation (1 for norm="forward")             */
} nop_spectral_desc;

typedef struct nop_plan nop_plan;        /* opaque, immutable after creation, thread-safe to share  */

/* ABI version of the loaded library (NOP_ABI_VERSION it was built with). */
int32_t nop_abi_version(void);

/* Message for the last failing call on this thread ("" if none). */
const char* nop_last_error(void);

/* Validate `desc`, pick the kernels and upload twiddle tables for the current device.
 * Replaces the per-call shape bookkeeping of SpectralConv.forward
 * (neuralop/layers/spectral_convolution.py:429-519). */
int32_t nop_spectral_plan_create(const nop_spectral_desc* desc, nop_plan** plan_out);

/* Release a plan (frees its device tables).  NULL is ignored. */
void nop_spectral_plan_destroy(nop_plan* plan);

/* Bytes of device workspace nop_spectral_forward needs (256-byte aligned buffer). */
int32_t nop_spectral_workspace_size(const nop_plan* plan, size_t* bytes);

/* 1 when the plan runs the fused FFT kernels, 0 when it runs the generic direct-DFT kernels. */
int32_t nop_spectral_plan_is_fast(const nop_plan* plan);

/* Number of kernel launches one nop_spectral_forward call with this plan enqueues. */
int32_t nop_spectral_launches_per_forward(const nop_plan* plan);

/* One forward of the spectral block.
 * Replaces SpectralConv.forward (neuralop/layers/spectral_convolution.py:417-570); with
 * `addend` / `apply_gelu` it also replaces the skip add and activation of
 * FNOBlocks.forward_with_postactivation (neuralop/layers/fno_block.py:356-361):
 *     y = spec(x) + bias;  if addend: y += addend;  if apply_gelu: y = gelu_erf(y)
 *   weights   : n_weights device pointers, layout per nop_weight_kind (complex64, contiguous)
 *   bias      : [Co] float32, or NULL
 *   addend    : [B, Co, n_out...] float32, or NULL (real data only)
 *   workspace : >= nop_spectral_workspace_size bytes, 256-byte aligned */
int32_t nop_spectral_forward(const nop_plan* plan, const void* x, const void* const* weights,
                             int32_t n_weights, const float* bias, const float* addend,
                             int32_t apply_gelu, void* y, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Bytes of the packed-weight buffer of a fused-engine plan; 0 when the plan takes weights unpacked
 * (generic engine).  Packing moves the per-forward weight reformatting (mode-blocked layout, Tucker
 * core expansion) out of the forward, as the reference's weights are fixed between updates. */
int32_t nop_spectral_packed_size(const nop_plan* plan, size_t* bytes);

/* Pack `weights` (layout as for nop_spectral_forward) into `packed` (>= nop_spectral_packed_size
 * bytes, 256-byte aligned).  Weight-only work on `stream`; redo it whenever the weights change.
 * Replaces the weight slicing / factor handling of SpectralConv.forward
 * (neuralop/layers/spectral_convolution.py:465-489) and the weight side of _contract_tucker (:76-103). */
int32_t nop_spectral_pack_weights(const nop_plan* plan, const void* const* weights, int32_t n_weights,
                                  void* packed, size_t packed_bytes, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* nop_spectral_forward with weights packed by nop_spectral_pack_weights.
 * Replaces SpectralConv.forward (neuralop/layers/spectral_convolution.py:417-570) and, with
 * addend / apply_gelu, the skip add + activation of neuralop/layers/fno_block.py:356-361. */
int32_t nop_spectral_forward_packed(const nop_plan* plan, const void* x, const void* packed,
                                    size_t packed_bytes, const float* bias, const float* addend,
                                    int32_t apply_gelu, void* y, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* ---- 3D slab decomposition over the first spatial axis (one process per GPU) ------------------
 * Replaces the unused all-to-all transpose helper of the reference's model-parallel layer
 * (neuralop/mpu/helpers.py:81-99) with a data path that exchanges only kept modes.  Every rank holds
 * x planes [x_begin, x_begin + x_count) of a 3D input (all batch entries and channels) and the full
 * weights.  One forward is:
 *   nop_spectral_slab_forward_planes  local (y, z) transforms -> send1
 *   all-to-all #1 (send1 -> recv1, per-peer byte counts in nop_slab_info)
 *   nop_spectral_slab_modes           x transforms, contraction, inverse x transforms -> send2
 *   all-to-all #2 (send2 -> recv2)
 *   nop_spectral_slab_inverse_planes  local inverse (y, z) transforms + epilogue -> y planes
 * Rank r contracts plane-mode blocks [block_begin[r], block_begin[r] + block_count[r]) for every
 * kept x mode.  Buffers are caller-owned device memory (256-byte aligned). */
#define NOP_MAX_SLAB_RANKS 64

typedef struct nop_slab_info {
    int32_t rank, world;
    int64_t x_begin, x_count;                      /* this rank's first-axis planes              */
    int64_t plane_blocks;                          /* blocks of 8 kept (y, z) modes               */
    int64_t block_begin[NOP_MAX_SLAB_RANKS];       /* plane-mode blocks contracted by each rank   */
    int64_t block_count[NOP_MAX_SLAB_RANKS];
    size_t send1_bytes, recv1_bytes, send2_bytes, recv2_bytes;
    size_t send1_split[NOP_MAX_SLAB_RANKS];        /* bytes to / from each peer, in rank order     */
    size_t recv1_split[NOP_MAX_SLAB_RANKS];
    size_t send2_split[NOP_MAX_SLAB_RANKS];
    size_t recv2_split[NOP_MAX_SLAB_RANKS];
} nop_slab_info;

/* Plan for rank `rank` of `world`; `desc` describes the whole (global) problem. */
int32_t nop_spectral_slab_plan_create(const nop_spectral_desc* desc, int32_t rank, int32_t world,
                                      nop_plan** plan_out);
int32_t nop_spectral_slab_info(const nop_plan* plan, nop_slab_info* info);
/* x: [B, Ci, x_count, n_in[1], n_in[2]] float32; send1: send1_bytes. */
int32_t nop_spectral_slab_forward_planes(const nop_plan* plan, const float* x, void* send1, void* stream);
/* recv1: recv1_bytes; packed: nop_spectral_pack_weights of the same plan; send2: send2_bytes. */
int32_t nop_spectral_slab_modes(const nop_plan* plan, const void* recv1, const void* packed,
                                size_t packed_bytes, void* send2, void* workspace, size_t workspace_bytes,
                                void* stream);
/* recv2: recv2_bytes; y: [B, Co, x_count, n_out[1], n_out[2]]; epilogue as nop_spectral_forward. */
int32_t nop_spectral_slab_inverse_planes(const nop_plan* plan, const void* recv2, const float* bias,
                                         const float* addend, int32_t apply_gelu, float* y, void* stream);

/* Measurement hook (no counterpart in the reference, which has no kernels of its own): while n > 0
 * on the calling thread, every forward call records events[0] on its stream before its first
 * kernel and events[i] after its i-th kernel launch (i = 1 .. n-1).  `events` are cudaEvent_t
 * created by the caller; n = 0 disables.  Lets a caller time each kernel of the block with CUDA
 * events on the launching stream. */
int32_t nop_set_launch_events(void* const* events, int32_t n);

/* Device status word (no counterpart in the reference).  The tensor-core contraction bounds every
 * wait for its MMAs (about one second); a wait that expires makes the kernel stop, free its tensor
 * memory and record NOP_DEVICE_MMA_TIMEOUT here instead of hanging the GPU.  Reads the word of the
 * current device into *status (0: nothing recorded) and resets it when `clear` is non-zero.
 * Synchronises with the device. */
#define NOP_DEVICE_MMA_TIMEOUT 1
int32_t nop_device_status(int32_t* status, int32_t clear);

/* Allocation-free forward.  No counterpart in the reference: it exists for callers that may not
 * allocate device memory at all -- code hosted by a runtime that owns every byte of device memory
 * and hands a plugin only its input and output buffers, or a latency-bound loop that cannot afford
 * a cudaMalloc, which may synchronise the device.  It takes the descriptor directly (no plan, no
 * workspace), runs the generic direct-DFT kernels and keeps their twiddle tables and intermediate
 * spectra in a 16 MiB scratch area compiled into the library (held by every GPU that loads the
 * library until the process exits).  Problems that need more scratch fail with NOP_E_WORKSPACE.
 * The descriptor's engine field must be NOP_ENGINE_AUTO or NOP_ENGINE_GENERIC (NOP_ENGINE_FAST:
 * NOP_E_UNSUPPORTED).  The first call in each CUDA context (per device; again after a
 * cudaDeviceReset or in another driver-API context) looks up that area's device address; make it
 * before any stream capture starts.  All calls on a device share the area and leave their contents in it (every
 * region is fully rewritten before it is read); calls that run concurrently on the GPU race on it,
 * so order them on one stream.  Arguments are those of nop_spectral_forward minus plan and
 * workspace; it never calls cudaMalloc or cudaFree. */
int32_t nop_spectral_forward_static(const nop_spectral_desc* desc, const void* x, const void* const* weights,
                                    int32_t n_weights, const float* bias, const float* addend,
                                    int32_t apply_gelu, void* y, void* stream);

/* ---- per-pixel layer chain on the tensor cores (the FNO layers around each spectral block) ----
 * One pass over HBM evaluates, at every spatial point of x [B, Cx, *spatial] (float32, contiguous):
 *     u = skip_channels ? act_skip(W0 x + s) : [x ; grid]   s [B, skip_channels, *spatial]: the block's
 *                                                          spectral output (bias included)
 *     h = GELU(W1 u + b1)
 *     y = act_out(W2 h + b2 + g * x + gb)                   g, gb [out_channels]: soft-gating of x (gate)
 *     p = GELU(W3 y + b3),  out = W4 p + b4                 when proj_hidden > 0
 * and writes y [B, out_channels, *spatial] (proj_hidden == 0) or out [B, proj_out, *spatial] to `y`.
 * GELU is the exact (erf) one.  Grid channels (lifting, skip_channels == 0 only): axis j's coordinate
 * grid_lo[j] + (i_j + grid_offset[j]) * grid_step[j] for index i_j of this call's points (grid_offset:
 * the first index of a slab of a larger grid).  Weights are torch Conv1d weights [out, in(, 1)]
 * row-major; b1, b2, gb, b3, b4 may be NULL (zero).  Every GEMM runs on tcgen05 (tf32, three-pass
 * split: float32 accuracy).
 * Replaces, in one kernel: FNOBlocks.forward_with_postactivation after the spectral convolution
 * (neuralop/layers/fno_block.py:339-381: the linear skip (skip_connections.py:96-127) added to the
 * SpectralConv output, GELU, ChannelMLP (neuralop/layers/channel_mlp.py:82-119), the soft-gating skip
 * (skip_connections.py:53-94), GELU), the lifting ChannelMLP with GridEmbeddingND
 * (neuralop/models/fno.py:387-396, neuralop/layers/embeddings.py:147-164) and the projection
 * ChannelMLP (fno.py:404-406), fused into the last block when proj_hidden > 0.
 * Limits: channel counts <= 256, points per sample a multiple of 4, x and s 16-byte aligned. */
typedef struct nop_chain_desc {
    int32_t abi_version;                 /* NOP_ABI_VERSION                                          */
    int32_t ndim;                        /* spatial dims, 1..NOP_MAX_DIMS                             */
    int64_t batch;
    int64_t spatial[NOP_MAX_DIMS];       /* sizes of this call's x                                   */
    int32_t x_channels;                  /* Cx                                                       */
    int32_t grid_dims;                   /* 0 or ndim (only with skip_channels == 0)                 */
    float grid_lo[NOP_MAX_DIMS], grid_step[NOP_MAX_DIMS];
    int64_t grid_offset[NOP_MAX_DIMS];
    int32_t skip_channels;               /* rows of W0 = channels of s (0: no skip stage)            */
    int32_t act_skip;                    /* 1: GELU after the skip add                               */
    int32_t hidden_channels;             /* rows of W1 (> 0)                                         */
    int32_t out_channels;                /* rows of W2                                               */
    int32_t act_out;                     /* 1: GELU on y                                             */
    int32_t gate;                        /* 1: add g * x (+ gb); needs x_channels == out_channels    */
    int32_t proj_hidden;                 /* rows of W3 (0: no projection)                            */
    int32_t proj_out;                    /* rows of W4                                               */
} nop_chain_desc;

typedef struct nop_chain_operands {
    const float* x;
    const float* s;
    const float* w0;
    const float* w1;
    const float* b1;
    const float* w2;
    const float* b2;
    const float* g;
    const float* gb;
    const float* w3;
    const float* b3;
    const float* w4;
    const float* b4;
    float* y;
} nop_chain_operands;

/* NOP_OK when the kernel takes this descriptor; *groups (nullable) = tiles in flight per CTA. */
int32_t nop_chain_query(const nop_chain_desc* desc, int32_t* groups);
int32_t nop_chain_forward(const nop_chain_desc* desc, const nop_chain_operands* operands, void* stream);

/* ---- backward of the chain (training) ---------------------------------------------------------
 * Gradients of one chain call without the projection (proj_hidden = 0) given dL/dy: what torch autograd
 * computes through the reference modules (linear skip, ChannelMLP with GELU, SoftGating, the GELUs,
 * GridEmbeddingND's channels as inputs without a gradient).  The forward's intermediates are recomputed
 * from x and s, in fp32 on CUDA cores; the weight and bias gradients are per-CTA sums over points added
 * in a fixed order (deterministic).  Every output pointer may be NULL when that gradient is not wanted,
 * except that the kernel always needs the operands' x, s (with skip), weights and dy.  dw* have the
 * weights' shapes ([out, in]), db* / dg / dgb [channels]; dx [B, Cx, P], ds [B, Cs, P].  Outputs are
 * overwritten, not accumulated.  Supported for channel counts <= 128 (nop_chain_backward_query). */
typedef struct nop_chain_grads {
    const float* dy;             /* dL/dy [B, out_channels, P] */
    float* dx;
    float* ds;
    float* dw0;
    float* dw1;
    float* db1;
    float* dw2;
    float* db2;
    float* dg;
    float* dgb;
} nop_chain_grads;

/* NOP_OK when the backward takes this descriptor; *workspace_bytes (nullable) = the device workspace
 * nop_chain_backward needs (256-byte aligned). */
int32_t nop_chain_backward_query(const nop_chain_desc* desc, size_t* workspace_bytes);
int32_t nop_chain_backward(const nop_chain_desc* desc, const nop_chain_operands* operands,
                           const nop_chain_grads* grads, void* workspace, size_t workspace_bytes, void* stream);

/* ---- forward from host memory, copies overlapped with the kernels ---------------------------
 * The reference's SpectralConv.forward runs wherever its input lives; a serving caller that holds
 * inputs in host memory would copy the whole batch in, run, and copy the whole batch out, so the
 * two PCIe transfers and the kernels follow one another.  nop_spectral_forward_host cuts a batch of
 * `total_batch` samples (a multiple of desc.batch) into chunks of desc.batch samples and runs each
 * chunk's host-to-device copy, forward and device-to-host copy on one of `n_streams` (1..8)
 * internal streams, so the copies of neighbouring chunks in both directions overlap each other and
 * the kernels.  x_host / addend_host / y_host: host buffers laid out like x / addend / y of
 * nop_spectral_forward with batch total_batch; page-locked memory is needed for the copies to
 * overlap (pageable memory gives the same result, serialised).  Weights: `packed` (from
 * nop_spectral_pack_weights, device) for plans with a packed form, else `weights` / `n_weights`
 * (device pointers as for nop_spectral_forward), which fused plans pack once into the workspace.
 * bias: device pointer or NULL.  workspace: device memory of nop_spectral_host_workspace_size
 * bytes, 256-byte aligned.  Ordering: the chunks start after work already queued on `stream`, and
 * work queued on `stream` after the call waits for every chunk; the call itself does not block the
 * host.  Returns without touching the buffers when total_batch is 0. */
int32_t nop_spectral_host_workspace_size(const nop_plan* plan, int32_t n_streams, size_t* bytes);
int32_t nop_spectral_forward_host(const nop_plan* plan, const void* x_host, int64_t total_batch,
                                  const void* const* weights, int32_t n_weights, const void* packed,
                                  size_t packed_bytes, const float* bias, const float* addend_host,
                                  int32_t apply_gelu, void* y_host, void* workspace, size_t workspace_bytes,
                                  int32_t n_streams, void* stream);

/* ---- backward (training) ------------------------------------------------------------------
 * Gradients of y = SpectralConv(x) for a real loss with g = dL/dy, equal to what torch autograd
 * computes through the reference forward (neuralop/layers/spectral_convolution.py:417-570:
 * rfftn, fftshift, slicing, the contraction einsum :21-103, ifftn, irfft, bias).
 *   dL/dx    = the forward of the ADJOINT plan on g, with the conjugate-transposed weights
 *              (dense: W'[o][i] = conj W[i][o]; Tucker / CP: in- and out-factors swapped, every
 *              factor conjugated, the core's first two modes swapped) and no bias.  The adjoint
 *              descriptor is the forward's with in/out channels, n_in/n_out, fwd_off/inv_off and
 *              fwd_scale/inv_scale swapped; the doubling of interior last-axis bins in the c2r
 *              adjoint cancels the halving in the r2c adjoint, so nothing else changes.
 *   dL/dW, dL/dbias from nop_spectral_weight_grad, given the kept spectra of x (forward plan) and of
 *              g (adjoint plan), both left by nop_spectral_forward_keep.
 * Supported when n_out == n_in (no output resampling) and for every plan but slab plans. */

/* Layout of the kept input-side spectrum a plan's forward computes: element (b, c, mode t) at complex
 * index (t / 8) * strides[0] + b * strides[1] + c * strides[2] + t % 8; `bytes` = buffer size. Mode
 * t runs over the kept modes of the weight's mode dims in row-major order. */
int32_t nop_spectral_spectrum_layout(const nop_plan* plan, int64_t* strides, size_t* bytes);

/* nop_spectral_forward (weights / n_weights; packed = NULL) or nop_spectral_forward_packed (packed /
 * packed_bytes) that also leaves the kept input spectrum in x_spec (>= the layout's bytes, 256-byte
 * aligned) for nop_spectral_weight_grad.  Same results in y. */
int32_t nop_spectral_forward_keep(const nop_plan* plan, const void* x, const void* const* weights,
                                  int32_t n_weights, const void* packed, size_t packed_bytes,
                                  const float* bias, const float* addend, int32_t apply_gelu, void* y,
                                  void* x_spec, size_t x_spec_bytes, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* Weight and bias gradients.  x_spec: kept spectrum of x from the forward plan; g_spec: kept
 * spectrum of g from the adjoint plan (nop_spectral_forward_keep on each).  workspace:
 * nop_spectral_weight_grad_workspace_size bytes (256-byte aligned), or NULL when that is 0.  grad_w (or NULL):
 * [Ci, Co, kept...] complex64 (separable: [C, kept...]), the gradient of the dense weight slice the
 * forward used (for Tucker / CP weights, of the reconstructed weight; the factor gradients follow
 * from it by the chain rule).  grad_bias (or NULL): [Co] float32.  Replaces the autograd of the
 * contraction einsum (spectral_convolution.py:21-52) and of the bias add (:567-568). */
int32_t nop_spectral_weight_grad(const nop_plan* plan, const void* x_spec, const nop_plan* adjoint_plan,
                                 const void* g_spec, void* grad_w, float* grad_bias, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Packed weights of an ADJOINT plan (dense, fused engine) straight from the forward's dense weight
 * [Ci, Co, kept...] (the adjoint's Co, Ci): the conjugate transpose is taken while packing, so no
 * transposed copy of the weight is made.  Same result as nop_spectral_pack_weights on conj(W)^T. */
int32_t nop_spectral_pack_weights_adjoint(const nop_plan* adjoint_plan, const void* forward_weight, void* packed,
                                          size_t packed_bytes, void* stream);

/* Device workspace of nop_spectral_weight_grad for the forward plan (0: none needed).  Small mode
 * counts with a large batch split the batch sum over more CTAs; the partial sums live here and are
 * reduced in a fixed order, so results do not depend on scheduling. */
int32_t nop_spectral_weight_grad_workspace_size(const nop_plan* plan, size_t* bytes);

/* Gradients of a Tucker-factorized weight W = core x_0 U_0 x_1 U_1 ... x_{n-1} U_{n-1} (n = ndim + 2
 * modes; U_0 = U_in [Ci, r_in], U_1 = U_out [Co, r_out], U_{k+2} = [kept_k, r_k]; core [r_0, ..., r_{n-1}];
 * all complex64, row-major) from grad_w = dL/dW ([Ci, Co, kept...], from nop_spectral_weight_grad):
 *   grad_core = grad_w x_0 conj(U_0) ... x_{n-1} conj(U_{n-1}),
 *   grad_factors[k] = sum over every mode but k of (grad_w x_j conj(U_j) for j != k) * conj(core),
 * torch's convention for complex leaves.  Replaces autograd through the reconstruction einsum of
 * _contract_tucker (spectral_convolution.py:76-103).  dims / ranks: the n mode sizes and ranks.  workspace:
 * nop_tucker_grads_workspace_size bytes, 256-byte aligned.  fp32 arithmetic, deterministic order. */
int32_t nop_tucker_grads_workspace_size(int32_t n, const int64_t* dims, const int64_t* ranks, size_t* bytes);
int32_t nop_tucker_grads(int32_t n, const int64_t* dims, const int64_t* ranks, const void* core,
                         const void* const* factors, const void* grad_w, void* grad_core, void* const* grad_factors,
                         void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NOP_SPECTRAL_H */

"""ctypes binding of libnop_b200.so (C ABI declared in include/nop_spectral.h).

The library is loaded from this package directory.  If it is missing or older than its
sources it is rebuilt with nvcc; if that is impossible the import of the compute path
fails with a RuntimeError -- there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnop_b200.so")

ABI_VERSION = 1
MAX_DIMS = 4

NOP_OK = 0
STATUS_NAMES = {0: "NOP_OK", -1: "NOP_E_INVALID", -2: "NOP_E_UNSUPPORTED", -3: "NOP_E_ALIGNMENT",
                -4: "NOP_E_WORKSPACE", -5: "NOP_E_CUDA", -6: "NOP_E_NOMEM"}

WEIGHT_DENSE, WEIGHT_TUCKER, WEIGHT_CP = 0, 1, 2
PRECISION_FP32, PRECISION_BF16 = 0, 1
ENGINE_AUTO, ENGINE_GENERIC, ENGINE_FAST = 0, 1, 2

EXPORTED_SYMBOLS = (
    "nop_abi_version", "nop_last_error", "nop_spectral_plan_create", "nop_spectral_plan_destroy",
    "nop_spectral_workspace_size", "nop_spectral_plan_is_fast", "nop_spectral_launches_per_forward",
    "nop_spectral_forward", "nop_spectral_packed_size", "nop_spectral_pack_weights",
    "nop_spectral_forward_packed", "nop_set_launch_events", "nop_spectral_slab_plan_create",
    "nop_spectral_slab_info", "nop_spectral_slab_forward_planes", "nop_spectral_slab_modes",
    "nop_spectral_slab_inverse_planes", "nop_spectral_host_workspace_size", "nop_spectral_forward_host",
    "nop_device_status", "nop_chain_query", "nop_chain_forward", "nop_chain_backward_query", "nop_chain_backward",
    "nop_spectral_spectrum_layout", "nop_spectral_forward_keep", "nop_spectral_weight_grad",
    "nop_spectral_weight_grad_workspace_size", "nop_spectral_pack_weights_adjoint",
    "nop_tucker_grads_workspace_size", "nop_tucker_grads",
)

MAX_SLAB_RANKS = 64


class NopSpectralDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("complex_data", ctypes.c_int32),
        ("separable", ctypes.c_int32),
        ("weight_kind", ctypes.c_int32),
        ("precision", ctypes.c_int32),
        ("engine", ctypes.c_int32),
        ("n_zero_imag", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("in_channels", ctypes.c_int64),
        ("out_channels", ctypes.c_int64),
        ("n_in", ctypes.c_int64 * MAX_DIMS),
        ("n_out", ctypes.c_int64 * MAX_DIMS),
        ("kept", ctypes.c_int64 * MAX_DIMS),
        ("fwd_off", ctypes.c_int64 * MAX_DIMS),
        ("inv_off", ctypes.c_int64 * MAX_DIMS),
        ("ranks", ctypes.c_int64 * (MAX_DIMS + 2)),
        ("zero_imag_bins", ctypes.c_int64 * 3),
        ("fwd_scale", ctypes.c_double),
        ("inv_scale", ctypes.c_double),
    ]


class NopSlabInfo(ctypes.Structure):
    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("x_begin", ctypes.c_int64),
        ("x_count", ctypes.c_int64),
        ("plane_blocks", ctypes.c_int64),
        ("block_begin", ctypes.c_int64 * 64),
        ("block_count", ctypes.c_int64 * 64),
        ("send1_bytes", ctypes.c_size_t),
        ("recv1_bytes", ctypes.c_size_t),
        ("send2_bytes", ctypes.c_size_t),
        ("recv2_bytes", ctypes.c_size_t),
        ("send1_split", ctypes.c_size_t * 64),
        ("recv1_split", ctypes.c_size_t * 64),
        ("send2_split", ctypes.c_size_t * 64),
        ("recv2_split", ctypes.c_size_t * 64),
    ]


class NopError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {message}")
        self.code = code


_lib = None
_lock = threading.Lock()


def _declare(lib):
    c_plan_p = ctypes.c_void_p
    lib.nop_abi_version.restype = ctypes.c_int32
    lib.nop_abi_version.argtypes = []
    lib.nop_last_error.restype = ctypes.c_char_p
    lib.nop_last_error.argtypes = []
    lib.nop_spectral_plan_create.restype = ctypes.c_int32
    lib.nop_spectral_plan_create.argtypes = [ctypes.POINTER(NopSpectralDesc), ctypes.POINTER(c_plan_p)]
    lib.nop_spectral_plan_destroy.restype = None
    lib.nop_spectral_plan_destroy.argtypes = [c_plan_p]
    lib.nop_spectral_workspace_size.restype = ctypes.c_int32
    lib.nop_spectral_workspace_size.argtypes = [c_plan_p, ctypes.POINTER(ctypes.c_size_t)]
    lib.nop_spectral_plan_is_fast.restype = ctypes.c_int32
    lib.nop_spectral_plan_is_fast.argtypes = [c_plan_p]
    lib.nop_spectral_launches_per_forward.restype = ctypes.c_int32
    lib.nop_spectral_launches_per_forward.argtypes = [c_plan_p]
    lib.nop_spectral_packed_size.restype = ctypes.c_int32
    lib.nop_spectral_packed_size.argtypes = [c_plan_p, ctypes.POINTER(ctypes.c_size_t)]
    lib.nop_spectral_pack_weights.restype = ctypes.c_int32
    lib.nop_spectral_pack_weights.argtypes = [
        c_plan_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.nop_spectral_forward_packed.restype = ctypes.c_int32
    lib.nop_spectral_forward_packed.argtypes = [
        c_plan_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.nop_set_launch_events.restype = ctypes.c_int32
    lib.nop_set_launch_events.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32]
    lib.nop_spectral_slab_plan_create.restype = ctypes.c_int32
    lib.nop_spectral_slab_plan_create.argtypes = [ctypes.POINTER(NopSpectralDesc), ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.POINTER(c_plan_p)]
    lib.nop_spectral_slab_info.restype = ctypes.c_int32
    lib.nop_spectral_slab_info.argtypes = [c_plan_p, ctypes.POINTER(NopSlabInfo)]
    lib.nop_spectral_slab_forward_planes.restype = ctypes.c_int32
    lib.nop_spectral_slab_forward_planes.argtypes = [c_plan_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.nop_spectral_slab_modes.restype = ctypes.c_int32
    lib.nop_spectral_slab_modes.argtypes = [c_plan_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.nop_spectral_slab_inverse_planes.restype = ctypes.c_int32
    lib.nop_spectral_slab_inverse_planes.argtypes = [c_plan_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                     ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
    lib.nop_spectral_spectrum_layout.restype = ctypes.c_int32
    lib.nop_spectral_spectrum_layout.argtypes = [c_plan_p, ctypes.POINTER(ctypes.c_int64),
                                                 ctypes.POINTER(ctypes.c_size_t)]
    lib.nop_spectral_forward_keep.restype = ctypes.c_int32
    lib.nop_spectral_forward_keep.argtypes = [
        c_plan_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.nop_spectral_weight_grad.restype = ctypes.c_int32
    lib.nop_spectral_weight_grad.argtypes = [c_plan_p, ctypes.c_void_p, c_plan_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.nop_spectral_pack_weights_adjoint.restype = ctypes.c_int32
    lib.nop_spectral_pack_weights_adjoint.argtypes = [c_plan_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                                      ctypes.c_void_p]
    lib.nop_spectral_weight_grad_workspace_size.restype = ctypes.c_int32
    lib.nop_spectral_weight_grad_workspace_size.argtypes = [c_plan_p, ctypes.POINTER(ctypes.c_size_t)]
    lib.nop_tucker_grads_workspace_size.restype = ctypes.c_int32
    lib.nop_tucker_grads_workspace_size.argtypes = [ctypes.c_int32, ctypes.POINTER(ctypes.c_int64),
                                                    ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_size_t)]
    lib.nop_tucker_grads.restype = ctypes.c_int32
    lib.nop_tucker_grads.argtypes = [
        ctypes.c_int32, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p,
        ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.nop_device_status.restype = ctypes.c_int32
    lib.nop_device_status.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_int32]
    lib.nop_spectral_host_workspace_size.restype = ctypes.c_int32
    lib.nop_spectral_host_workspace_size.argtypes = [c_plan_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_size_t)]
    lib.nop_spectral_forward_host.restype = ctypes.c_int32
    lib.nop_spectral_forward_host.argtypes = [
        c_plan_p, ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.c_int32, ctypes.c_void_p]
    lib.nop_spectral_forward.restype = ctypes.c_int32
    lib.nop_spectral_forward.argtypes = [
        c_plan_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]


def library():
    """The loaded CDLL (built on first use when the in-tree .so is missing or stale)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if os.environ.get("NOP_SKIP_BUILD") != "1":
            try:
                from . import build as _build
                _build.build()
            except Exception as exc:  # noqa: BLE001
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"libnop_b200.so is not built and building it failed: {exc}") from exc
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libnop_b200.so not found; run `python -m neuraloperator_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        _declare(lib)
        v = lib.nop_abi_version()
        if v != ABI_VERSION:
            raise RuntimeError(f"libnop_b200.so ABI {v} != binding ABI {ABI_VERSION}; rebuild the library")
        _lib = lib
        return lib


class LaunchEvents:
    """Context manager: time every kernel of the forward calls made inside it with CUDA events.

    ``LaunchEvents(n_kernels)`` records events[0] before the first kernel and events[i] after the
    i-th; ``durations_ms()`` returns the per-kernel times of the last forward.
    """

    def __init__(self, n_kernels: int):
        import torch
        self.events = [torch.cuda.Event(enable_timing=True) for _ in range(n_kernels + 1)]
        for e in self.events:  # torch creates the underlying cudaEvent_t on first record
            e.record()

    def __enter__(self):
        arr = (ctypes.c_void_p * len(self.events))(*[e.cuda_event for e in self.events])
        check(library().nop_set_launch_events(arr, len(self.events)))
        return self

    def __exit__(self, *exc):
        library().nop_set_launch_events(None, 0)
        return False

    def durations_ms(self):
        return [self.events[i].elapsed_time(self.events[i + 1]) for i in range(len(self.events) - 1)]


def last_error() -> str:
    return library().nop_last_error().decode(errors="replace")


def check(code: int):
    if code != NOP_OK:
        raise NopError(code, last_error())


class Plan:
    """Owns one nop_plan (created on the current CUDA device).  With ``slab=(rank, world)`` the plan
    is a 3D slab-decomposition plan (nop_spectral_slab_plan_create) and ``slab_info`` is filled."""

    def __init__(self, desc: NopSpectralDesc, slab=None):
        lib = library()
        handle = ctypes.c_void_p()
        if slab is None:
            check(lib.nop_spectral_plan_create(ctypes.byref(desc), ctypes.byref(handle)))
        else:
            check(lib.nop_spectral_slab_plan_create(ctypes.byref(desc), int(slab[0]), int(slab[1]),
                                                    ctypes.byref(handle)))
        self.slab_info = None
        if slab is not None:
            info = NopSlabInfo()
            check(lib.nop_spectral_slab_info(handle, ctypes.byref(info)))
            self.slab_info = info
        self._lib = lib
        self.handle = handle
        self.desc = desc
        size = ctypes.c_size_t()
        check(lib.nop_spectral_workspace_size(handle, ctypes.byref(size)))
        self.workspace_bytes = int(size.value)
        self.spectrum_strides, self.spectrum_bytes = None, 0
        if slab is None:
            strides = (ctypes.c_int64 * 3)()
            sb = ctypes.c_size_t()
            check(lib.nop_spectral_spectrum_layout(handle, strides, ctypes.byref(sb)))
            self.spectrum_strides, self.spectrum_bytes = tuple(strides), int(sb.value)
        self.is_fast = bool(lib.nop_spectral_plan_is_fast(handle))
        self.launches_per_forward = int(lib.nop_spectral_launches_per_forward(handle))
        check(lib.nop_spectral_packed_size(handle, ctypes.byref(size)))
        self.packed_bytes = int(size.value)

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                self._lib.nop_spectral_plan_destroy(h)
            except Exception:  # noqa: BLE001  (interpreter shutdown)
                pass
            self.handle = None


def device_status(clear: bool = True) -> int:
    """Status word the tensor-core kernels set when a bounded wait expires (0: none); see
    nop_device_status.  Synchronises with the current device."""
    v = ctypes.c_int32()
    check(library().nop_device_status(ctypes.byref(v), int(bool(clear))))
    return int(v.value)

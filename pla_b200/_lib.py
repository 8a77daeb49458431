"""ctypes binding of libpla_b200.so (the C ABI declared in include/pla_b200.h).

The shared library is built in-tree (``python -m pla_b200.build``); importing
the ops without it, or calling them on a non-CUDA tensor, raises: there is no
CPU or eager-PyTorch fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpla_b200.so")
TORCH_LIB_PATH = os.path.join(_HERE, "libpla_b200_torch.so")

PLA_F16, PLA_F32, PLA_F64, PLA_BF16 = 0, 1, 2, 3
PLA_OK, PLA_ERR_UNSUPPORTED = 0, 2
PLA_NCHW, PLA_NHWC = 0, 1

DTYPE_CODE = {
    torch.float16: PLA_F16,
    torch.float32: PLA_F32,
    torch.float64: PLA_F64,
    torch.bfloat16: PLA_BF16,
}

# Every symbol include/pla_b200.h declares, with its ctypes signature.
_vp, _i32, _i64, _u32p = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.POINTER(ctypes.c_uint)
_f32p = ctypes.POINTER(ctypes.c_float)
SIGNATURES = {
    "pla_status_string": ([_i32], ctypes.c_char_p),
    "pla_last_cuda_error": ([], ctypes.c_char_p),
    "pla_version": ([], _i32),
    "pla_stencil7x7_forward": ([_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i64, _i64, _i64, _i32, _vp], _i32),
    "pla_stencil7x7_forward_taps": ([_vp, _f32p, _f32p, _vp, _i32, _i32, _i32, _i64, _i64, _i64, _i32, _vp], _i32),
    "pla_depthwise7x7_forward": ([_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp], _i32),
    "pla_depthwise_forward": ([_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp], _i32),
    "pla_depthwise7x7_forward_many": ([_vp, _i32, _i32, _i32, _vp], _i32),
    "pla_depthwise7x7_layernorm_nhwc": ([_vp, _vp, _vp, _vp, _vp, ctypes.c_float, _vp, _i32, _i32, _i32, _i32, _i32,
                                         _vp], _i32),
    "pla_stencil7x7_iterate": ([_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp], _i32),
    "pla_stencil7x7_iterate_noalloc": ([_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp], _i32),
    "pla_stencil7x7_iterate_taps": ([_vp, _f32p, _f32p, _vp, _vp, _i32, _i32, _i32, _i32, _vp], _i32),
    "pla_stencil7x7_band_step": ([_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp], _i32),
    "pla_stencil7x7_band_step_taps": ([_vp, _f32p, _f32p, _vp, _i32, _i32, _i32, _i32, _i32, _vp], _i32),
    "pla_stencil7x7_band_step_halo": ([_vp, _f32p, _f32p, _vp, _i32, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp,
                                       _vp, ctypes.c_uint, _vp], _i32),
    "pla_ipc_export": ([_vp, _vp, ctypes.POINTER(ctypes.c_uint64)], _i32),
    "pla_ipc_import": ([_vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)], _i32),
    "pla_ipc_close": ([_vp, ctypes.c_uint64], _i32),
    "pla_read_device_faults": ([_u32p], _i32),
    "pla_clear_device_faults": ([], _i32),
}

class DwProblem(ctypes.Structure):
    """pla_dw_problem (include/pla_b200.h): one problem of pla_depthwise7x7_forward_many."""

    _fields_ = [("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("b", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("n", ctypes.c_int), ("c", ctypes.c_int), ("h", ctypes.c_int), ("width", ctypes.c_int)]


_lib = None


class PlaError(RuntimeError):
    """A non-zero status from the C ABI (mirrors the reference's TORCH_CHECK -> RuntimeError)."""


def lib() -> ctypes.CDLL:
    """Load libpla_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build the CUDA library first (python -m pla_b200.build); "
                "this package has no CPU fallback")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (argtypes, restype) in SIGNATURES.items():
            try:
                fn = getattr(handle, name)
            except AttributeError:
                raise ImportError(f"{LIB_PATH} does not export {name}: it is older than the package; "
                                  "rebuild it (python -m pla_b200.build)") from None
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = handle
    return _lib


_ops = None


def ops():
    """``torch.ops.pla_b200``: the torch custom ops of libpla_b200_torch.so
    (csrc/torch_ops.cpp) over the C ABI, loaded once; raise if not built."""
    global _ops
    if _ops is None:
        lib()
        if not os.path.exists(TORCH_LIB_PATH):
            raise ImportError(f"{TORCH_LIB_PATH} is missing: build it first (python -m pla_b200.build)")
        torch.ops.load_library(TORCH_LIB_PATH)
        _ops = torch.ops.pla_b200
    return _ops


def check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        msg = L.pla_status_string(status).decode()
        detail = L.pla_last_cuda_error().decode()
        raise PlaError(f"{what}: {msg}" + (f" ({detail})" if detail and status == 4 else ""))


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def overlaps(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Whether the memory spans of two CUDA tensors intersect.

    The single-step kernels read each input halo after other CTAs may have
    stored their outputs, so an output that overlaps its input would give
    wrong results; the ops reject it instead.
    """
    if a.numel() == 0 or b.numel() == 0 or a.device != b.device:
        return False

    def span(t):
        lo = hi = t.data_ptr()
        for size, stride in zip(t.shape, t.stride()):
            ext = (size - 1) * stride * t.element_size()
            if ext < 0:
                lo += ext
            else:
                hi += ext
        return lo, hi + t.element_size()

    (a0, a1), (b0, b1) = span(a), span(b)
    return a0 < b1 and b0 < a1


class HostTaps:
    """A 7x7 filter (+ optional bias) copied to host fp32 memory for the *_taps entry points.

    Mirrors the reference's weight cache (data/depthwise_conv_7x7_cuda/
    model_cutlass_autotune_v6.py:507-513, keyed on the parameter's _version
    and storage): the device->host copy (a stream sync) happens only when the
    weight or bias tensor changed since the last call.
    """

    def __init__(self):
        self._key = None
        self.taps = (ctypes.c_float * 49)()
        self.bias = ctypes.c_float(0.0)
        self.has_bias = False

    @staticmethod
    def _tkey(t):
        return None if t is None else (t.data_ptr(), t._version, t.dtype, str(t.device))

    def update(self, weight: torch.Tensor, bias: torch.Tensor | None) -> "HostTaps":
        key = (self._tkey(weight), self._tkey(bias))
        if key != self._key:
            w = weight.detach().reshape(49).float().cpu()
            for k in range(49):
                self.taps[k] = float(w[k])
            self.has_bias = bias is not None
            if bias is not None:
                self.bias.value = float(bias.detach().reshape(-1)[0].float().cpu())
            self._key = key
        return self

    def args(self):
        return self.taps, (ctypes.byref(self.bias) if self.has_bias else None)

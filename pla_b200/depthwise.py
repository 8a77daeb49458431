"""Depthwise 7x7 convolution with the reference's KernelBench module contract.

Drop-in for the generated depthwise modules of the reference
(``data/depthwise_conv_7x7_cuda/model_cutlass_autotune_v6.py:495-524``,
``model_cutlass.py:316-345``); the op they replace is
``data/depthwise_conv_7x7.py:15-29``
(``nn.Conv2d(C, C, k, stride, padding, groups=C, bias)``).  Same names:
``ModelNew(in_channels, kernel_size, stride=1, padding=1, bias=False)`` with a
``conv2d`` submodule (``conv2d.weight`` [C,1,7,7], ``conv2d.bias`` [C] when
bias=True), ``get_inputs()``, ``get_init_inputs()``.

Beyond the reference kernels (fp16/fp32, NCHW, no bias, weights repacked to
[C,8,80]): fp32 / bf16 / fp16 / fp64, NCHW and channels_last (NHWC), optional
bias, and no weight repack (the kernels read the module's own weight).

``depthwise_kxk()`` also takes 3x3 and 5x5 filters (padding k // 2): the operator
of the reference's MetaSchedule benchmark
(``benchmark/MetaSchedule/depthwise_conv.py:7-13, 32-33``, kernel 3 or 7).
"""
from __future__ import annotations

import torch

if __package__:
    from . import _lib
else:  # loaded from its path by a KernelBench-style harness (run_and_check)
    import os
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from pla_b200 import _lib


def depthwise7x7(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """y = conv2d(x, weight, bias, stride=1, padding=3, groups=C) for CUDA x [N,C,H,W].

    A channels_last input runs the NHWC kernels and returns channels_last (as
    torch does); a contiguous input runs NCHW; anything else is made
    contiguous first.
    """
    return depthwise_kxk(x, weight, bias, out, k=7)


def depthwise_kxk(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
              out: torch.Tensor | None = None, k: int | None = None) -> torch.Tensor:
    """y = conv2d(x, weight, bias, stride=1, padding=k // 2, groups=C), k in {3, 5, 7}.

    ``k`` defaults to ``weight.shape[-1]``; ``weight`` is [C,1,k,k] (or any
    shape with C*k*k elements).  Same layouts and dtypes as depthwise7x7.
    Without ``out`` this is the torch op ``torch.ops.pla_b200.depthwise7x7``
    (k = 7) or ``torch.ops.pla_b200.depthwise``; ``out`` writes into a caller
    tensor through the same C ABI.
    """
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError("depthwise7x7 requires a CUDA input")
    if x.dim() != 4:
        raise RuntimeError("input must have shape [N,C,H,W]")
    N, C, H, W = x.shape
    if not weight.is_cuda or weight.device != x.device:
        raise RuntimeError("weight must be a CUDA tensor on the input's device")
    if k is None:
        k = int(weight.shape[-1]) if weight.dim() == 4 else 7
    if k not in (3, 5, 7):
        raise RuntimeError("only 3x3, 5x5 and 7x7 filters are supported")
    if weight.numel() != C * k * k or (weight.dim() == 4 and tuple(weight.shape) != (C, 1, k, k)):
        raise RuntimeError(f"weight must have shape [C,1,{k},{k}]")
    if weight.dtype != x.dtype:
        raise RuntimeError("dtype mismatch")
    if x.dtype not in _lib.DTYPE_CODE:
        raise RuntimeError("unsupported dtype")
    if bias is not None and (not bias.is_cuda or bias.device != x.device or bias.dtype != x.dtype
                             or bias.numel() != C):
        raise RuntimeError("bias device/dtype/shape mismatch")
    if x.is_contiguous():
        layout, fmt = _lib.PLA_NCHW, torch.contiguous_format
    elif x.is_contiguous(memory_format=torch.channels_last):
        layout, fmt = _lib.PLA_NHWC, torch.channels_last
    else:
        x = x.contiguous()
        layout, fmt = _lib.PLA_NCHW, torch.contiguous_format
    if out is None:
        # torch op (device-resident filter, output in x's memory format)
        op = _lib.ops().depthwise7x7 if k == 7 else _lib.ops().depthwise
        return op(x, weight.detach().reshape(C, 1, k, k), None if bias is None else bias.detach())
    elif out.shape != x.shape or not out.is_contiguous(memory_format=fmt) or out.dtype != x.dtype:
        raise RuntimeError("out must match x's shape, dtype and memory format")
    elif _lib.overlaps(out, x):
        raise RuntimeError("out must not overlap x")
    if out.numel() == 0:
        return out
    weight = weight.detach().contiguous()
    bias = None if bias is None else bias.detach().contiguous()
    with torch.cuda.device(x.device):
        st = _lib.lib().pla_depthwise_forward(
            x.data_ptr(), weight.data_ptr(), _lib.ptr(bias), out.data_ptr(), N, C, H, W, k,
            _lib.DTYPE_CODE[x.dtype], layout, _lib.stream_ptr(x.device))
    _lib.check(st, "pla_depthwise_forward")
    return out


def depthwise7x7_many(problems, outs=None) -> list[torch.Tensor]:
    """Several independent 7x7 depthwise convolutions in one call, run
    concurrently (``pla_depthwise7x7_forward_many``): ``problems`` is a list of
    ``(x, weight, bias_or_None)`` CUDA tensors of one dtype and one layout
    (all contiguous NCHW or all channels_last), e.g. the four stages of a
    ConvNeXt-T-shaped sweep.  Returns the outputs in order, in x's memory
    format (or writes into ``outs``).  Each result equals
    ``depthwise7x7(x, weight, bias)`` bit for bit.
    """
    problems = list(problems)
    if not problems:
        return []
    x0 = problems[0][0]
    if not isinstance(x0, torch.Tensor) or not x0.is_cuda:
        raise ValueError("depthwise7x7_many requires CUDA inputs")
    if x0.dtype not in _lib.DTYPE_CODE:
        raise RuntimeError("unsupported dtype")
    if x0.dim() == 4 and x0.is_contiguous():
        layout, fmt = _lib.PLA_NCHW, torch.contiguous_format
    elif x0.dim() == 4 and x0.is_contiguous(memory_format=torch.channels_last):
        layout, fmt = _lib.PLA_NHWC, torch.channels_last
    else:
        raise RuntimeError("depthwise7x7_many takes dense NCHW or channels_last [N,C,H,W] inputs")
    arr = (_lib.DwProblem * len(problems))()
    keep = []
    results = []
    for i, (x, w, b) in enumerate(problems):
        if not isinstance(x, torch.Tensor) or not x.is_cuda or x.device != x0.device or x.dtype != x0.dtype:
            raise RuntimeError("every problem's input must be a CUDA tensor of the first one's device and dtype")
        if x.dim() != 4 or not x.is_contiguous(memory_format=fmt):
            raise RuntimeError("every problem's input must have the first one's layout")
        N, C, H, W = x.shape
        if not w.is_cuda or w.device != x.device or w.dtype != x.dtype or w.numel() != C * 49:
            raise RuntimeError("weight must be a [C,1,7,7] CUDA tensor of x's dtype on x's device")
        if b is not None and (not b.is_cuda or b.device != x.device or b.dtype != x.dtype or b.numel() != C):
            raise RuntimeError("bias device/dtype/shape mismatch")
        if outs is None:
            y = torch.empty(x.shape, dtype=x.dtype, device=x.device, memory_format=fmt)
        else:
            y = outs[i]
            if y.shape != x.shape or y.dtype != x.dtype or not y.is_contiguous(memory_format=fmt):
                raise RuntimeError("out must match x's shape, dtype and memory format")
        w = w.detach().contiguous()
        b = None if b is None else b.detach().contiguous()
        keep += [w, b]
        arr[i] = _lib.DwProblem(x.data_ptr(), w.data_ptr(), _lib.ptr(b), y.data_ptr(), N, C, H, W)
        results.append(y)
    with torch.cuda.device(x0.device):
        st = _lib.lib().pla_depthwise7x7_forward_many(arr, len(problems), _lib.DTYPE_CODE[x0.dtype], layout,
                                                      _lib.stream_ptr(x0.device))
    _lib.check(st, "pla_depthwise7x7_forward_many")
    return results


def depthwise7x7_layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                           norm_weight: torch.Tensor | None = None, norm_bias: torch.Tensor | None = None,
                           eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm over channels of depthwise7x7(x), fused into one pass (ConvNeXt's dwconv -> norm).

    ``x`` is a channels_last CUDA tensor [N, C, H, W] (fp32 / bf16 / fp16);
    the result is channels_last too, so ``result.permute(0, 2, 3, 1)`` is the
    contiguous [N, H, W, C] tensor that ``nn.LayerNorm(C)`` returns in a
    ConvNeXt block.  ``weight`` [C,1,7,7], ``bias`` / ``norm_weight`` /
    ``norm_bias`` [C] or None, all of x's dtype.  The normalisation works on
    the depthwise outputs rounded to x's dtype (what the unfused pair sees)
    in fp32.  No reference counterpart: the reference's operator is the
    depthwise half (data/depthwise_conv_7x7.py:15-29).
    """
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError("depthwise7x7_layernorm requires a CUDA input")
    if x.dim() != 4:
        raise RuntimeError("input must have shape [N,C,H,W]")
    if not x.is_contiguous(memory_format=torch.channels_last):
        raise RuntimeError("depthwise7x7_layernorm normalises NHWC pixels: pass a channels_last input")
    N, C, H, W = x.shape
    if x.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise RuntimeError("unsupported dtype")
    if not weight.is_cuda or weight.device != x.device or weight.dtype != x.dtype or weight.numel() != C * 49:
        raise RuntimeError("weight must be a [C,1,7,7] CUDA tensor of x's dtype on x's device")
    for name, t in (("bias", bias), ("norm_weight", norm_weight), ("norm_bias", norm_bias)):
        if t is not None and (not t.is_cuda or t.device != x.device or t.dtype != x.dtype or t.numel() != C):
            raise RuntimeError(f"{name} device/dtype/shape mismatch")
    if out is None:
        vecs = [None if t is None else t.detach() for t in (bias, norm_weight, norm_bias)]
        return _lib.ops().depthwise7x7_layernorm(x, weight.detach(), *vecs, eps=float(eps))
    elif out.shape != x.shape or not out.is_contiguous(memory_format=torch.channels_last) or out.dtype != x.dtype:
        raise RuntimeError("out must match x's shape, dtype and channels_last format")
    elif _lib.overlaps(out, x):
        raise RuntimeError("out must not overlap x")
    if out.numel() == 0:
        return out
    vecs = [None if t is None else t.detach().contiguous() for t in (bias, norm_weight, norm_bias)]
    weight = weight.detach().contiguous()
    with torch.cuda.device(x.device):
        st = _lib.lib().pla_depthwise7x7_layernorm_nhwc(
            x.data_ptr(), weight.data_ptr(), _lib.ptr(vecs[0]), _lib.ptr(vecs[1]), _lib.ptr(vecs[2]), float(eps),
            out.data_ptr(), N, C, H, W, _lib.DTYPE_CODE[x.dtype], _lib.stream_ptr(x.device))
    _lib.check(st, "pla_depthwise7x7_layernorm_nhwc")
    return out


class DepthwiseLayerNorm(torch.nn.Module):
    """ConvNeXt block head: ``dwconv`` (7x7 depthwise, bias) then ``norm`` (LayerNorm over C), fused.

    Parameter names follow the ConvNeXt block (``dwconv.weight`` [C,1,7,7],
    ``dwconv.bias`` [C], ``norm.weight`` / ``norm.bias`` [C]), so its state
    dict slots into one.  ``forward`` takes a channels_last [N, C, H, W]
    tensor and returns the normalised channels_last tensor.
    """

    def __init__(self, dim: int, eps: float = 1e-6, bias: bool = True):
        super().__init__()
        self.dwconv = torch.nn.Conv2d(dim, dim, 7, padding=3, groups=dim, bias=bias)
        self.norm = torch.nn.LayerNorm(dim, eps=eps)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return depthwise7x7_layernorm(x, self.dwconv.weight, self.dwconv.bias, self.norm.weight, self.norm.bias,
                                      self.norm.eps)


class ModelNew(torch.nn.Module):
    """KernelBench drop-in for data/depthwise_conv_7x7.py's Model (parameter ``conv2d``).

    kernel_size 7 with padding 3 is the reference module's case; 3 (padding 1)
    and 5 (padding 2) cover the MetaSchedule benchmark's other filter size.
    """

    def __init__(self, in_channels: int, kernel_size: int, stride: int = 1, padding: int = 1,
                 bias: bool = False):
        super().__init__()
        if kernel_size not in (3, 5, 7) or stride != 1 or padding != kernel_size // 2:
            raise ValueError("only kernel_size 3, 5 or 7 with stride=1 and padding=kernel_size // 2 is supported")
        self.conv2d = torch.nn.Conv2d(in_channels, in_channels, kernel_size, stride=1, padding=kernel_size // 2,
                                      groups=in_channels, bias=bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return depthwise_kxk(x, self.conv2d.weight, self.conv2d.bias)


# Harness shape of the reference problem (data/depthwise_conv_7x7.py:64-85).
batch_size, in_channels, kernel_size, height, width, stride, padding = 1, 8, 7, 2048, 2048, 1, 3


def get_inputs():
    return [torch.rand(batch_size, in_channels, height, width)]


def get_init_inputs():
    return [in_channels, kernel_size, stride, padding]

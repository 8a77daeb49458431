"""B200-native (sm_100a) 7x7 depthwise convolution and 7x7 stencil.

Drop-in for the hot path of Raymond0715/PLA: the KernelBench modules that
replace ``data/depthwise_conv_7x7.py`` and ``data/stencil_7x7.py``.

* ``pla_b200.stencil``   — ``ModelNew`` (``conv1``), ``stencil7x7()``
* ``pla_b200.depthwise`` — ``ModelNew`` (``conv2d``), ``depthwise7x7()``, ``depthwise7x7_many()`` (independent
  problems, run concurrently), ``depthwise_kxk()`` (k = 3, 5, 7),
  ``depthwise7x7_layernorm()`` / ``DepthwiseLayerNorm`` (depthwise + channel LayerNorm, NHWC, fused)
* ``pla_b200.iterate``   — ``stencil7x7_iterate()``, ``BandedStencil`` (multi-GPU)

All compute goes through the C ABI in ``include/pla_b200.h``
(``libpla_b200.so``, built by ``python -m pla_b200.build``).  The functional
forms without ``out=`` run as torch custom ops, ``torch.ops.pla_b200.*``
(``libpla_b200_torch.so``: TORCH_CHECK errors, device guard, current stream,
Meta kernels for fake tensors), so they trace under ``torch.compile`` and
replay in CUDA graphs with the weights current at replay time.
"""
from . import _lib

try:  # registered at import so that compiled code never traces the loading
    _lib.ops()
except ImportError:  # not built yet (e.g. while pla_b200.build runs): the ops raise when called
    pass

from .depthwise import DepthwiseLayerNorm, depthwise7x7, depthwise7x7_layernorm, depthwise7x7_many, depthwise_kxk
from .iterate import BandedStencil, band_rows, stencil7x7_iterate
from .stencil import stencil7x7

__all__ = ["stencil7x7", "depthwise7x7", "depthwise7x7_many", "depthwise_kxk", "depthwise7x7_layernorm", "DepthwiseLayerNorm",
           "stencil7x7_iterate", "BandedStencil", "band_rows"]

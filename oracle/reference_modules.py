"""The reference's two problem modules, re-declared — TEST AND CPU-BASELINE INFRASTRUCTURE ONLY.

The reference computes its hot path on the CPU with PyTorch's own
torch.nn.Conv2d; its problem files are thin wrappers:

* ``data/stencil_7x7.py:5-12`` —
  ``Model`` holding ``conv1 = nn.Conv2d(1, 1, kernel_size=7, stride=1, padding=3)``;
* ``data/depthwise_conv_7x7.py:15-29`` —
  ``Model(in_channels, kernel_size, stride=1, padding=1, bias=False)`` holding
  ``conv2d = nn.Conv2d(C, C, k, stride, padding, groups=C, bias)``.

The reference tree does not travel to the GPU host, so ``bench.py``'s CPU
baseline (and its ``--impl reference`` arm) builds these equivalent modules
here: the attribute names and constructor arguments are kept identical so the
timed code path is the reference's (ATen's CPU convolution).  Nothing in the
product package imports this file.
"""
from __future__ import annotations

import torch
import torch.nn as nn


class StencilModel(nn.Module):
    """data/stencil_7x7.py:5-12."""

    def __init__(self):
        super().__init__()
        self.conv1 = nn.Conv2d(in_channels=1, out_channels=1, kernel_size=7, stride=1, padding=3)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.conv1(x)


class DepthwiseModel(nn.Module):
    """data/depthwise_conv_7x7.py:15-29."""

    def __init__(self, in_channels: int, kernel_size: int, stride: int = 1, padding: int = 1, bias: bool = False):
        super().__init__()
        self.conv2d = nn.Conv2d(in_channels, in_channels, kernel_size, stride=stride, padding=padding,
                                groups=in_channels, bias=bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.conv2d(x)

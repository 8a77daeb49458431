"""A small KernelBench-style problem file (test input for pla_b200.runner):
a Model built like data/stencil_7x7.py's (one nn.Conv2d(1, 1, 7, padding=3),
attribute `conv1`), with its own small input shape."""
import torch
import torch.nn as nn


class Model(nn.Module):
    def __init__(self):
        super().__init__()
        self.conv1 = nn.Conv2d(in_channels=1, out_channels=1, kernel_size=7, stride=1, padding=3)

    def forward(self, x):
        return self.conv1(x)


def get_inputs():
    return [torch.rand(2, 1, 96, 200)]


def get_init_inputs():
    return []

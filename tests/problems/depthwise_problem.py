"""A small KernelBench-style problem file (test input for pla_b200.runner):
a depthwise Model built like data/depthwise_conv_7x7.py's (attribute
`conv2d`, groups = in_channels), with its own small shapes."""
import torch
import torch.nn as nn


class Model(nn.Module):
    def __init__(self, in_channels, kernel_size, stride=1, padding=1, bias=False):
        super().__init__()
        self.conv2d = nn.Conv2d(in_channels, in_channels, kernel_size, stride=stride, padding=padding,
                                groups=in_channels, bias=bias)

    def forward(self, x):
        return self.conv2d(x)


def get_inputs():
    return [torch.rand(4, 64, 14, 14)]


def get_init_inputs():
    return [64, 7, 1, 3]

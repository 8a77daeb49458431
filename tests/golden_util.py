"""Reader of tests/golden/golden.npz (written by tests/golden/make_golden.py)."""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "f64": torch.float64}
TOL = {"f32": 1e-5, "bf16": 2e-2, "f16": 2e-3, "f64": 1e-10}
# k x k cases of the MetaSchedule benchmark: its own check's tolerance
# (benchmark/MetaSchedule/common.py:175: 1e-4 for fp32, 1e-2 otherwise).
MS_TOL = {"f32": 1e-4, "bf16": 1e-2, "f16": 1e-2}


@dataclass
class Case:
    name: str
    op: str
    dtype: str
    layout: str
    steps: int
    shape: tuple
    x: torch.Tensor
    w: torch.Tensor
    b: torch.Tensor | None
    y: torch.Tensor
    y_native: torch.Tensor | None

    @property
    def tol(self) -> float:
        return MS_TOL[self.dtype] if self.op == "depthwise_ms" else TOL[self.dtype]

    @property
    def k(self) -> int:
        """Filter side (7 except for the k x k depthwise cases)."""
        return int(round((self.w.numel() // self.shape[1]) ** 0.5)) if self.op == "depthwise_ms" else 7


def _tensor(arr: np.ndarray, dtype: str, shape, layout: str) -> torch.Tensor:
    td = DT[dtype]
    if td in (torch.bfloat16, torch.float16):
        t = torch.from_numpy(arr.view(np.int16).copy()).view(td)
    else:
        t = torch.from_numpy(arr.copy())
    if layout == "nhwc":  # stored physically as [N, H, W, C]
        N, C, H, W = shape
        return t.reshape(N, H, W, C).permute(0, 3, 1, 2)
    return t.reshape(shape)


def load_cases() -> list[Case]:
    data = np.load(GOLDEN)
    cases = []
    for entry in data["__index__"]:
        name, op, dtype, layout, steps, has_b, has_native, shape = str(entry).split("|")
        shape = tuple(int(s) for s in shape.split(","))
        yshape = shape
        x = _tensor(data[name + ".x"], dtype, shape, layout)
        w = _tensor(data[name + ".w"], dtype, (-1,), "nchw")
        b = _tensor(data[name + ".b"], dtype, (-1,), "nchw") if has_b == "1" else None
        y = _tensor(data[name + ".y"], dtype, yshape, layout)
        yn = _tensor(data[name + ".y_native"], dtype, yshape, layout) if has_native == "1" else None
        cases.append(Case(name, op, dtype, layout, int(steps), shape, x, w, b, y, yn))
    return cases

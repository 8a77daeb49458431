"""Generate the golden vectors in tests/golden/golden.npz from the REFERENCE modules.

Run in a checkout that has the reference tree (PLA) next to it:

    python tests/golden/make_golden.py --reference-root <PLA checkout> [--out tests/golden/golden.npz]

It imports the reference's own ``data/stencil_7x7.py`` and
``data/depthwise_conv_7x7.py`` (their ``Model`` classes are plain
torch.nn.Conv2d wrappers), loads seeded parameters into them and records their
CPU outputs for seeded inputs.  Inputs follow the benchmark configurations' recipes (x, w, b drawn
in that order from ``torch.Generator().manual_seed(seed)`` on the CPU) at
reduced sizes, plus the odd/tail shapes of the reference's own tests
(data/stencil_direct_cuda_v7/test_stencil.py:31-37).

Low-precision expected values follow the reference tests' convention
(data/stencil_direct_cuda_v7/test_stencil.py:49-54): the module evaluated in
fp32 (fp64 for fp64) on the widened inputs, then cast to the data type.  For
bf16 the module is also run natively in bf16 and stored as ``y_native``.

The k x k depthwise cases (op "depthwise_ms") come from the reference's
MetaSchedule benchmark instead: its own numpy check ``ref`` (nested in
``main`` of benchmark/MetaSchedule/depthwise_conv.py:41-46; fp32 products
summed in (ry, rx) order, cast to the data type) is lifted out of the source
with ``ast`` and run on inputs drawn as its harness draws them
(benchmark/MetaSchedule/common.py:176-177: ``np.random.default_rng(seed)``,
x then w ~ U(-1, 1), cast to the dtype).  The TVM parts of that file are not
imported or run.

The fixtures are read at test time; the reference tree is not needed then.
"""
from __future__ import annotations

import argparse
import ast
import importlib.util
import os
import sys

import numpy as np
import torch


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bits(t: torch.Tensor) -> np.ndarray:
    """Raw storage of a CPU tensor in its own memory order (16-bit types as uint16)."""
    t = t.detach()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.contiguous().numpy().copy()


def _nhwc_bits(t: torch.Tensor) -> np.ndarray:
    """Storage of a channels_last tensor as its physical [N, H, W, C] array."""
    return _bits(t.permute(0, 2, 3, 1))


DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "f64": torch.float64}


def _metaschedule_ref(reference_root):
    """Factory for the reference's numpy depthwise check, bound to (k, h, w)."""
    path = os.path.join(reference_root, "benchmark", "MetaSchedule", "depthwise_conv.py")
    with open(path) as f:
        tree = ast.parse(f.read())
    main = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "main")
    fn = next(n for n in ast.walk(main) if isinstance(n, ast.FunctionDef) and n.name == "ref")
    code = compile(ast.Module(body=[fn], type_ignores=[]), path, "exec")

    def make(k, h, w):
        ns = {"np": np, "k": k, "pad": k // 2, "h": h, "w": w}  # the names `ref` reads from main's scope
        exec(code, ns)
        return ns["ref"]

    return make


def _np_to_torch(a: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype in ("bf16", "f16"):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).view(DT[dtype])
    return torch.from_numpy(np.ascontiguousarray(a))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference-root", required=True)
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz"))
    args = ap.parse_args(argv)

    stencil_mod = _load(os.path.join(args.reference_root, "data", "stencil_7x7.py"), "ref_stencil_7x7")
    dw_mod = _load(os.path.join(args.reference_root, "data", "depthwise_conv_7x7.py"), "ref_depthwise_conv_7x7")
    torch.backends.mkldnn.deterministic = True

    out = {}
    index = []

    def record(name, op, dtype, layout, x, w, b, y, steps=0, y_native=None):
        index.append(f"{name}|{op}|{dtype}|{layout}|{steps}|{int(b is not None)}|{int(y_native is not None)}|"
                     + ",".join(str(s) for s in x.shape))
        if layout == "nhwc":
            out[name + ".x"] = _nhwc_bits(x)
            out[name + ".y"] = _nhwc_bits(y)
            if y_native is not None:
                out[name + ".y_native"] = _nhwc_bits(y_native)
        else:
            out[name + ".x"] = _bits(x)
            out[name + ".y"] = _bits(y)
            if y_native is not None:
                out[name + ".y_native"] = _bits(y_native)
        out[name + ".w"] = _bits(w)
        if b is not None:
            out[name + ".b"] = _bits(b)

    # ---------------- single-step stencil (data/stencil_7x7.py) ----------------
    def stencil_case(name, shape, seed, dtype, dist="uniform", bias=True):
        g = torch.Generator().manual_seed(seed)
        if dist == "uniform":  # cfg2 recipe: x~U(-1,1), w~U(-1,1)/49
            x = torch.rand(shape, generator=g) * 2 - 1
            w = (torch.rand(1, 1, 7, 7, generator=g) * 2 - 1) / 49
            b = (torch.rand(1, generator=g) * 2 - 1) / 49
        else:
            x = torch.randn(shape, generator=g)
            w = torch.randn(1, 1, 7, 7, generator=g) / 7
            b = torch.randn(1, generator=g) * 0.1
        td = DT[dtype]
        x, w, b = x.to(td), w.to(td), b.to(td)
        acc = torch.float64 if td == torch.float64 else torch.float32
        m = stencil_mod.Model().to(acc)
        with torch.no_grad():
            m.conv1.weight.copy_(w.to(acc))
            if bias:
                m.conv1.bias.copy_(b.to(acc))
            else:
                m.conv1.bias = None
            y = m(x.to(acc)).to(td)
            y_native = None
            if td == torch.bfloat16:
                y_native = m.to(td)(x)
        record(name, "stencil", dtype, "nchw", x, w, b if bias else None, y, y_native=y_native)

    stencil_case("st_cfg2_64", (1, 1, 64, 64), 1, "f32")
    stencil_case("st_cfg2_64_nobias", (1, 1, 64, 64), 1, "f32", bias=False)
    stencil_case("st_odd_1x1", (2, 1, 1, 1), 42, "f32", "normal")
    stencil_case("st_odd_3d", (1, 7, 9), 43, "f32", "normal")
    stencil_case("st_odd_17x257", (2, 1, 17, 257), 44, "f32", "normal")
    stencil_case("st_odd_2x4", (1, 1, 2, 4), 45, "f32", "normal")
    stencil_case("st_odd_20x769", (1, 1, 20, 769), 46, "f32", "normal")
    stencil_case("st_wide_12x1024", (1, 1, 12, 1024), 47, "f32", "normal")
    stencil_case("st_bf16_40x136", (2, 1, 40, 136), 48, "bf16", "normal")
    stencil_case("st_f16_33x96", (1, 1, 33, 96), 49, "f16", "normal")
    stencil_case("st_f64_17x29", (1, 1, 17, 29), 50, "f64", "normal")

    # ---------------- depthwise (data/depthwise_conv_7x7.py) -------------------
    def dw_case(name, shape, seed, dtype, layout="nchw", bias=True):
        g = torch.Generator().manual_seed(seed)
        N, C, H, W = shape
        x = torch.randn(shape, generator=g)                 # ~N(0,1)
        w = torch.randn(C, 1, 7, 7, generator=g) / 7        # ~N(0,1/49)
        b = torch.randn(C, generator=g) * 0.1               # ~N(0,0.01)
        td = DT[dtype]
        x, w, b = x.to(td), w.to(td), b.to(td)
        acc = torch.float64 if td == torch.float64 else torch.float32
        m = dw_mod.Model(C, 7, 1, 3, bias=bias).to(acc)
        with torch.no_grad():
            m.conv2d.weight.copy_(w.to(acc))
            if bias:
                m.conv2d.bias.copy_(b.to(acc))
            xin = x
            if layout == "nhwc":
                xin = x.contiguous(memory_format=torch.channels_last)
            y = m(xin.to(acc)).to(td)
            y_native = None
            if td == torch.bfloat16:
                y_native = m.to(td)(xin)
            if layout == "nhwc":
                y = y.contiguous(memory_format=torch.channels_last)
                if y_native is not None:
                    y_native = y_native.contiguous(memory_format=torch.channels_last)
        record(name, "depthwise", dtype, layout, xin, w, b if bias else None, y, y_native=y_native)

    dw_case("dw_cfg1_c8", (1, 8, 56, 56), 0, "f32")
    dw_case("dw_cfg3_nchw", (2, 32, 14, 14), 2, "bf16")
    dw_case("dw_cfg3_nhwc", (2, 32, 14, 14), 2, "bf16", "nhwc")
    dw_case("dw_cfg4_s4", (2, 40, 7, 7), 3, "bf16", bias=False)
    dw_case("dw_cfg4_s2", (1, 8, 28, 28), 3, "bf16", bias=False)
    dw_case("dw_cfg4_s1_nhwc", (1, 16, 56, 56), 3, "bf16", "nhwc", bias=False)
    dw_case("dw_odd_5x9", (1, 3, 5, 9), 5, "f32")
    dw_case("dw_odd_1x1", (2, 2, 1, 1), 6, "f32")
    dw_case("dw_odd_13x70", (1, 4, 13, 70), 7, "f32")
    dw_case("dw_wide_20x128", (1, 2, 20, 128), 8, "f32")
    dw_case("dw_wide_bf16_9x136", (2, 3, 9, 136), 9, "bf16")
    dw_case("dw_f64_9x11", (1, 2, 9, 11), 10, "f64")
    dw_case("dw_f16_14", (1, 4, 14, 14), 11, "f16")
    dw_case("dw_f32_nhwc_odd", (2, 35, 9, 10), 12, "f32", "nhwc")

    # ------- k x k depthwise of the MetaSchedule benchmark (its numpy check) -------
    ms_ref = _metaschedule_ref(args.reference_root)

    def ms_case(name, shape, k, seed, dtype):
        import ml_dtypes

        npdt = {"f32": np.float32, "f16": np.float16, "bf16": ml_dtypes.bfloat16}[dtype]
        n, c, h, w = shape
        rng = np.random.default_rng(seed)
        x = rng.uniform(-1, 1, (n, c, h, w)).astype(npdt)
        wt = rng.uniform(-1, 1, (c, 1, k, k)).astype(npdt)
        y = ms_ref(k, h, w)(x, wt)
        assert y.dtype == x.dtype
        record(name, "depthwise_ms", dtype, "nchw", _np_to_torch(x, dtype), _np_to_torch(wt, dtype), None,
               _np_to_torch(y, dtype))

    ms_case("ms_k3_f32", (1, 8, 64, 64), 3, 0, "f32")
    ms_case("ms_k3_f16", (1, 8, 64, 64), 3, 1, "f16")
    ms_case("ms_k3_bf16", (2, 4, 40, 72), 3, 2, "bf16")
    ms_case("ms_k3_f32_odd", (2, 3, 9, 13), 3, 3, "f32")
    ms_case("ms_k7_f32", (1, 4, 48, 64), 7, 4, "f32")

    # ---------------- iterated stencil (iterated-stencil recipe, reduced) --------
    g = torch.Generator().manual_seed(4)
    H = W = 64
    x = torch.rand(H, W, generator=g) * 2 - 1
    w = torch.rand(1, 1, 7, 7, generator=g) * 2 - 1
    w = w / w.sum()
    m = stencil_mod.Model()
    with torch.no_grad():
        m.conv1.weight.copy_(w)
        m.conv1.bias = None
        u = x.view(1, 1, H, W)
        for _ in range(10):
            u = m(u)
    record("it_cfg5_64_s10", "iterate", "f32", "nchw", x, w, None, u.view(H, W), steps=10)

    out["__index__"] = np.array(index)
    np.savez_compressed(args.out, **out)
    print(f"wrote {len(index)} cases to {args.out}")


if __name__ == "__main__":
    sys.exit(main())

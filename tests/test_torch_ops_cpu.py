"""The torch custom ops (torch.ops.pla_b200.*, csrc/torch_ops.cpp) without a GPU:
they are registered with their schemas, their Meta kernels give the shapes,
dtypes and memory formats the CUDA kernels return (what fake tensors and
torch.compile see), and a CPU tensor has no kernel to run on (no CPU
fallback)."""
import pytest
import torch

import pla_b200  # noqa: F401  (loads the ops)
from pla_b200 import _lib

OPS = ("stencil7x7", "depthwise7x7", "depthwise", "depthwise7x7_layernorm", "stencil7x7_iterate")


def test_ops_are_registered_with_schemas():
    ns = _lib.ops()
    for name in OPS:
        schema = str(getattr(ns, name).default._schema)
        assert schema.startswith(f"pla_b200::{name}(Tensor x, Tensor weight"), schema
        assert schema.endswith("-> Tensor")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.float64])
def test_meta_kernels_match_the_kernels_output_contract(dtype):
    ops = _lib.ops()
    m = dict(device="meta", dtype=dtype)
    # stencil: contiguous output shaped like x, whatever x's strides
    x = torch.empty(2, 1, 40, 96, **m)[:, :, :, ::2]
    y = ops.stencil7x7(x, torch.empty(1, 1, 7, 7, **m), torch.empty(1, **m))
    assert y.shape == x.shape and y.is_contiguous() and y.dtype == dtype
    # depthwise: the input's memory format (channels_last stays channels_last)
    for fmt in (torch.contiguous_format, torch.channels_last):
        x = torch.empty(3, 8, 14, 14, **m).contiguous(memory_format=fmt)
        for op, k in ((ops.depthwise7x7, 7), (ops.depthwise, 3), (ops.depthwise, 5)):
            y = op(x, torch.empty(8, 1, k, k, **m), None)
            assert y.shape == x.shape and y.stride() == x.stride()
    # a strided input that is neither format comes back contiguous
    x = torch.empty(3, 8, 14, 28, **m)[..., ::2]
    assert ops.depthwise7x7(x, torch.empty(8, 1, 7, 7, **m)).is_contiguous()
    # iterate: [H, W] grid
    g = torch.empty(64, 48, **m)
    assert ops.stencil7x7_iterate(g, torch.empty(7, 7, **m), 3).shape == (64, 48)


def test_meta_layernorm_is_channels_last():
    ops = _lib.ops()
    x = torch.empty(2, 64, 14, 14, device="meta", dtype=torch.bfloat16).contiguous(memory_format=torch.channels_last)
    w = torch.empty(64, 1, 7, 7, device="meta", dtype=torch.bfloat16)
    y = ops.depthwise7x7_layernorm(x, w, None, None, None, 1e-6)
    assert y.is_contiguous(memory_format=torch.channels_last) and y.shape == x.shape


def test_cpu_tensors_have_no_kernel():
    ops = _lib.ops()
    with pytest.raises(NotImplementedError):
        ops.stencil7x7(torch.zeros(1, 1, 8, 8), torch.zeros(1, 1, 7, 7), None)
    with pytest.raises(NotImplementedError):
        ops.depthwise7x7(torch.zeros(1, 4, 8, 8), torch.zeros(4, 1, 7, 7), None)
    # the Python API refuses a CPU input before reaching the op, as the
    # reference module does (data/stencil_direct_cuda_v7/generate_model.py:50-51)
    with pytest.raises(ValueError):
        pla_b200.stencil7x7(torch.zeros(1, 1, 8, 8), torch.zeros(1, 1, 7, 7))


def test_meta_kernels_reject_bad_shapes():
    ops = _lib.ops()
    with pytest.raises(RuntimeError):
        ops.stencil7x7_iterate(torch.empty(2, 8, 8, device="meta"), torch.empty(7, 7, device="meta"), 1)
    with pytest.raises(RuntimeError):
        ops.depthwise(torch.empty(8, 8, device="meta"), torch.empty(8, 1, 7, 7, device="meta"), None)


def test_dynamic_shapes_stay_symbolic_through_export():
    """torch.export with dynamic batch / height / width: the Meta kernels use
    symbolic sizes, so nothing is specialised."""
    from torch.export import Dim

    ops = _lib.ops()

    class Dw(torch.nn.Module):
        def forward(self, x, w):
            return ops.depthwise7x7(x, w, None) + 1

    class St(torch.nn.Module):
        def forward(self, x, w):
            return ops.stencil7x7(x, w, None) * 2

    dyn = {"x": {0: Dim("n"), 2: Dim("h"), 3: Dim("w")}, "w": None}
    for mod, x, w in ((Dw(), torch.empty(4, 8, 14, 20, device="meta").contiguous(memory_format=torch.channels_last),
                       torch.empty(8, 1, 7, 7, device="meta")),
                      (St(), torch.empty(4, 1, 14, 20, device="meta"), torch.empty(1, 1, 7, 7, device="meta"))):
        ep = torch.export.export(mod, (x, w), dynamic_shapes=dyn)
        out = [n for n in ep.graph.nodes if n.op == "call_function"][0].meta["val"]
        assert not any(isinstance(d, int) for d in (out.shape[0], out.shape[2], out.shape[3]))


def test_opcheck_on_meta_tensors():
    """torch.library.opcheck's schema, autograd-registration, fake-tensor and
    dynamic aot-dispatch tests, run on meta tensors (the CUDA run is in
    tests/test_gpu_torch_ops.py)."""
    ops = _lib.ops()
    m = dict(device="meta")
    cases = [
        (ops.stencil7x7, (torch.empty(2, 1, 40, 48, **m), torch.empty(1, 1, 7, 7, **m), torch.empty(1, **m))),
        (ops.depthwise7x7, (torch.empty(2, 8, 14, 14, **m).contiguous(memory_format=torch.channels_last),
                            torch.empty(8, 1, 7, 7, **m), None)),
        (ops.depthwise, (torch.empty(2, 8, 30, 30, **m), torch.empty(8, 1, 3, 3, **m), torch.empty(8, **m))),
        (ops.stencil7x7_iterate, (torch.empty(32, 40, **m), torch.empty(7, 7, **m), 3, None)),
    ]
    for op, args in cases:
        res = torch.library.opcheck(op.default, args)
        assert all(v == "SUCCESS" for v in res.values()), res

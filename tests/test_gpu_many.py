"""pla_depthwise7x7_forward_many on the GPU: the four ConvNeXt-T-shaped stages
(cfg4's shapes at a small batch) run concurrently in one call and give the
same bits as one pla_depthwise7x7_forward call each, and as the CPU oracle;
also when the call is captured in a CUDA graph and replayed."""
import pytest
import torch

from oracle import oracle
from pla_b200 import depthwise7x7, depthwise7x7_many

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
STAGES = [(96, 56), (192, 28), (384, 14), (768, 7)]


def _problems(n, dtype, fmt, seed, bias):
    g = torch.Generator().manual_seed(seed)
    out = []
    for C, S in STAGES:
        x = torch.randn(n, C, S, S, generator=g).to(dtype)
        w = (torch.randn(C, 1, 7, 7, generator=g) / 7).to(dtype)
        b = (torch.randn(C, generator=g) * 0.1).to(dtype) if bias else None
        out.append((x, w, b, x.to(DEV).contiguous(memory_format=fmt), w.to(DEV),
                    None if b is None else b.to(DEV)))
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("fmt", [torch.contiguous_format, torch.channels_last])
def test_many_equals_single_calls_and_oracle(dtype, fmt):
    probs = _problems(3, dtype, fmt, 31, bias=dtype == torch.float32)
    ys = depthwise7x7_many([(xd, wd, bd) for (_, _, _, xd, wd, bd) in probs])
    for y, (x, w, b, xd, wd, bd) in zip(ys, probs):
        assert y.is_contiguous(memory_format=fmt)
        assert torch.equal(y, depthwise7x7(xd, wd, bd))
        assert torch.equal(y.cpu(), oracle.depthwise7x7(x, w, b))


def test_many_in_a_cuda_graph_and_on_a_side_stream():
    probs = _problems(2, torch.bfloat16, torch.contiguous_format, 32, bias=False)
    args = [(xd, wd, bd) for (_, _, _, xd, wd, bd) in probs]
    refs = [depthwise7x7(*a) for a in args]
    outs = [torch.empty_like(r) for r in refs]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        depthwise7x7_many(args, outs=outs)
    torch.cuda.current_stream().wait_stream(s)
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
    for o in outs:
        o.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        depthwise7x7_many(args, outs=outs)
    graph.replay()
    torch.cuda.synchronize()
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
    # new inputs in place, replay again
    for (xd, _, _) in args:
        xd.mul_(-1)
    graph.replay()
    torch.cuda.synchronize()
    for o, (xd, wd, bd) in zip(outs, args):
        assert torch.equal(o, depthwise7x7(xd, wd, bd))


def test_many_rejects_an_output_that_is_another_problems_input():
    probs = _problems(1, torch.float32, torch.contiguous_format, 33, bias=False)
    args = [(xd, wd, bd) for (_, _, _, xd, wd, bd) in probs[:2]]
    x0, x1 = args[0][0], args[1][0]
    inside_x0 = x0.view(-1)[:x1.numel()].view(x1.shape)  # problem 1's output inside problem 0's input
    with pytest.raises(RuntimeError, match="invalid argument"):
        depthwise7x7_many(args, outs=[torch.empty_like(x0), inside_x0])

"""Dependent launches back to back on one stream.

The persistent depthwise kernels (plane stack, plane pair, NHWC spatial tile,
static-striding plane tile) launch with programmatic dependent launch: the
next launch's CTAs start while the previous grid drains and wait
(griddepcontrol.wait) before their first global access.  Each case chains
depthwise calls through two buffers, so every launch reads what the previous
one wrote (read after write) and writes what it read (write after read), with
no host synchronisation in between; the result must equal, bit for bit, the
same chain with a device synchronisation after every call, and a replay of the
chain captured in a CUDA graph."""
import pytest
import torch

from pla_b200 import depthwise7x7

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

# (n, c, s, dtype, memory format, kernel the shape dispatches to)
CASES = [
    (8, 64, 14, torch.bfloat16, torch.contiguous_format, "plane stack 14x14"),
    (8, 128, 7, torch.bfloat16, torch.contiguous_format, "plane stack 7x7"),
    (4, 64, 28, torch.bfloat16, torch.contiguous_format, "plane stack 28x28"),
    (6, 32, 14, torch.float32, torch.contiguous_format, "plane stack 14x14 fp32"),
    (8, 64, 14, torch.bfloat16, torch.channels_last, "plane stack 14x14 NHWC"),
    (32, 48, 56, torch.bfloat16, torch.contiguous_format, "plane pair 56x56"),
    (4, 64, 56, torch.bfloat16, torch.channels_last, "NHWC spatial tile 56x56"),
    (2, 8, 64, torch.float32, torch.contiguous_format, "plane tile, static striding"),
]
LINKS = 6


def _setup(n, c, s, dtype, fmt, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, c, s, s, generator=g).to(dtype).to(DEV).contiguous(memory_format=fmt)
    ws = [(torch.randn(c, 1, 7, 7, generator=g) / 7).to(dtype).to(DEV) for _ in range(3)]
    return x, ws


def _chain(x, ws, sync):
    a, b = x.clone(), torch.empty_like(x)
    for i in range(LINKS):
        src, dst = (a, b) if i % 2 == 0 else (b, a)
        depthwise7x7(src, ws[i % len(ws)], None, out=dst)
        if sync:
            torch.cuda.synchronize()
    return a if LINKS % 2 == 0 else b


@pytest.mark.parametrize("n,c,s,dtype,fmt,kernel", CASES, ids=[c[-1] for c in CASES])
def test_dependent_launch_chain(n, c, s, dtype, fmt, kernel):
    x, ws = _setup(n, c, s, dtype, fmt, 7 + s + c)
    want = _chain(x, ws, sync=True).clone()
    got = _chain(x, ws, sync=False)
    torch.cuda.synchronize()
    assert torch.equal(got, want), kernel
    # The chain as one CUDA graph, replayed twice from a fresh input.
    a, b = x.clone(), torch.empty_like(x)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(LINKS):
            src, dst = (a, b) if i % 2 == 0 else (b, a)
            depthwise7x7(src, ws[i % len(ws)], None, out=dst)
    for _ in range(2):
        a.copy_(x)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(a if LINKS % 2 == 0 else b, want), kernel

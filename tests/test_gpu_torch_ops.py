"""torch.ops.pla_b200.* on the GPU: opcheck on real CUDA inputs, the modules
under torch.compile(fullgraph=True) bit-identical to the CPU oracle, and CUDA
graph replays that see in-place weight updates (the kernels read the filter
from device memory when they run, as the reference's kernels do)."""
import pytest
import torch

from oracle import oracle
from pla_b200 import _lib
from pla_b200.depthwise import ModelNew as DwModel
from pla_b200.stencil import ModelNew as StencilModel

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _gen(seed=0):
    return torch.Generator().manual_seed(seed)


def test_opcheck_on_cuda_inputs():
    ops = _lib.ops()
    g = _gen()
    x = torch.randn(2, 1, 40, 36, generator=g).to(DEV)
    w = (torch.randn(1, 1, 7, 7, generator=g) / 7).to(DEV)
    b = torch.randn(1, generator=g).to(DEV)
    xb = torch.randn(3, 16, 14, 14, generator=g).bfloat16().to(DEV)
    wb = (torch.randn(16, 1, 7, 7, generator=g) / 7).bfloat16().to(DEV)
    x3 = torch.randn(2, 8, 64, 64, generator=g).to(DEV)
    w3 = torch.randn(8, 1, 3, 3, generator=g).to(DEV)
    xl = xb.contiguous(memory_format=torch.channels_last)
    gam, bet = torch.ones(16, dtype=torch.bfloat16, device=DEV), torch.zeros(16, dtype=torch.bfloat16, device=DEV)
    grid = torch.rand(48, 64, generator=g).to(DEV)
    cases = [
        (ops.stencil7x7, (x, w, b)),
        (ops.stencil7x7, (x[:, :, :, ::2], w, None)),
        (ops.depthwise7x7, (xb, wb, None)),
        (ops.depthwise7x7, (xl, wb, None)),
        (ops.depthwise, (x3, w3, None)),
        (ops.depthwise7x7_layernorm, (xl, wb, None, gam, bet, 1e-6)),
        (ops.stencil7x7_iterate, (grid, w.reshape(7, 7), 3, None)),
    ]
    for op, args in cases:
        res = torch.library.opcheck(op.default, args)
        assert all(v == "SUCCESS" for v in res.values()), (op, res)


def test_compiled_modules_match_the_oracle():
    g = _gen(1)
    m = StencilModel().to(DEV)
    with torch.no_grad():
        m.conv1.weight.copy_(torch.randn(1, 1, 7, 7, generator=g) / 7)
    x = torch.rand(2, 1, 96, 160, generator=g) * 2 - 1
    cm = torch.compile(m, fullgraph=True)
    with torch.no_grad():
        y = cm(x.to(DEV))
    ref = oracle.stencil7x7(x, m.conv1.weight.detach().cpu(), m.conv1.bias.detach().cpu())
    assert torch.equal(y.cpu(), ref)

    d = DwModel(32, 7, 1, 3, bias=True).to(DEV).bfloat16()
    xd = torch.randn(4, 32, 14, 14, generator=g).bfloat16()
    cd = torch.compile(d, fullgraph=True)
    for fmt in (torch.contiguous_format, torch.channels_last):
        with torch.no_grad():
            yd = cd(xd.to(DEV).contiguous(memory_format=fmt))
        assert yd.is_contiguous(memory_format=fmt)
        refd = oracle.depthwise7x7(xd, d.conv2d.weight.detach().cpu(), d.conv2d.bias.detach().cpu())
        assert torch.equal(yd.cpu(), refd)


@pytest.mark.parametrize("via_data", [False, True])
def test_graph_replay_sees_in_place_weight_updates(via_data):
    """Capture the module, update conv1.weight / conv1.bias in place (under
    no_grad, or through .data, which bypasses the version counter), replay:
    the output uses the new weights (the reference's own test updates the
    weights after construction, data/stencil_cuda_v2/test_stencil.py:85-96)."""
    g = _gen(2)
    m = StencilModel().to(DEV)
    x = (torch.rand(1, 1, 128, 192, generator=g) * 2 - 1).to(DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.no_grad():
        m(x)  # warm-up off the capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph), torch.no_grad():
        y = m(x)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), oracle.stencil7x7(x.cpu(), m.conv1.weight.detach().cpu(), m.conv1.bias.detach().cpu()))
    w2 = torch.randn(1, 1, 7, 7, generator=g) / 7
    b2 = torch.tensor([0.25])
    if via_data:
        m.conv1.weight.data.copy_(w2)
        m.conv1.bias.data.copy_(b2)
    else:
        with torch.no_grad():
            m.conv1.weight.copy_(w2)
            m.conv1.bias.copy_(b2)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), oracle.stencil7x7(x.cpu(), w2, b2))
    # eager calls see it too
    with torch.no_grad():
        assert torch.equal(m(x).cpu(), oracle.stencil7x7(x.cpu(), w2, b2))


def test_depthwise_graph_replay_sees_weight_updates():
    g = _gen(3)
    d = DwModel(24, 7, 1, 3, bias=True).to(DEV)
    x = torch.randn(2, 24, 28, 28, generator=g).to(DEV)
    with torch.no_grad():
        d(x)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph), torch.no_grad():
        y = d(x)
    w2 = torch.randn(24, 1, 7, 7, generator=g) / 7
    d.conv2d.weight.data.copy_(w2)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), oracle.depthwise7x7(x.cpu(), w2, d.conv2d.bias.detach().cpu()))


def test_frozen_taps_opt_in_matches_and_follows_versioned_updates():
    g = _gen(4)
    m = StencilModel(frozen_taps=True).to(DEV)
    x = (torch.rand(1, 1, 64, 128, generator=g) * 2 - 1).to(DEV)
    with torch.no_grad():
        y = m(x)
        assert torch.equal(y.cpu(), oracle.stencil7x7(x.cpu(), m.conv1.weight.cpu(), m.conv1.bias.cpu()))
        w2 = torch.randn(1, 1, 7, 7, generator=g) / 7
        m.conv1.weight.copy_(w2)  # bumps the version counter: the host copy follows
        assert torch.equal(m(x).cpu(), oracle.stencil7x7(x.cpu(), w2, m.conv1.bias.cpu()))


def test_op_errors_are_runtime_errors():
    ops = _lib.ops()
    x = torch.zeros(1, 1, 16, 16, device=DEV)
    with pytest.raises(RuntimeError, match="dtype"):
        ops.stencil7x7(x, torch.zeros(1, 1, 7, 7, device=DEV, dtype=torch.float16), None)
    with pytest.raises(RuntimeError, match="elements"):
        ops.stencil7x7(x, torch.zeros(1, 1, 5, 5, device=DEV), None)
    with pytest.raises(RuntimeError):
        ops.depthwise(torch.zeros(1, 4, 16, 16, device=DEV), torch.zeros(4, 1, 9, 9, device=DEV), None)

"""GPU parity of the fused depthwise 7x7 + channel LayerNorm (NHWC) against
the CPU oracle (bit for bit) and against torch's own conv + layer_norm
(within rtol = atol = 1e-5 fp32 / 2e-2 for 16-bit data).

The shapes cover both kernels and every cluster geometry: the ConvNeXt-T
stages of the benchmark configuration at small batch (56x56 planes on the
NHWC tile kernel with 3-CTA clusters; 28 / 14 / 7 on the plane-stack kernel
with 6 / 12 / 6-CTA clusters), channel counts that leave a partial
32-channel group, plane sizes with clipped edge tiles, and the
bias / scale / shift options.
"""
import pytest
import torch

from oracle import oracle
from tests.test_oracle import _torch_dw_ln

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _inputs(shape, dtype, seed, affine=True):
    g = torch.Generator().manual_seed(seed)
    N, C, H, W = shape
    x = torch.randn(*shape, generator=g).to(dtype).contiguous(memory_format=torch.channels_last)
    w = (torch.randn(C, 1, 7, 7, generator=g) / 7).to(dtype)
    vec = lambda s, o: (o + s * torch.randn(C, generator=g)).to(dtype) if affine else None  # noqa: E731
    return x, w, vec(0.1, 0.0), vec(0.2, 1.0), vec(0.1, 0.0)


def _run(x, w, b, gamma, beta, eps=1e-6):
    from pla_b200 import depthwise7x7_layernorm

    dev = [None if t is None else t.to(DEV) for t in (b, gamma, beta)]
    y = depthwise7x7_layernorm(x.to(DEV), w.to(DEV), *dev, eps=eps)
    torch.cuda.synchronize()
    assert y.is_contiguous(memory_format=torch.channels_last)
    return y.cpu()


def _check(shape, dtype, seed, affine=True, eps=1e-6):
    x, w, b, gamma, beta = _inputs(shape, dtype, seed, affine)
    got = _run(x, w, b, gamma, beta, eps)
    ref = oracle.depthwise7x7_layernorm(x, w, b, gamma, beta, eps)
    if not torch.equal(got, ref):
        diff = (got.double() - ref.double()).abs()
        raise AssertionError(f"not bit-identical: {int((diff > 0).sum())} of {diff.numel()} differ, "
                             f"max |diff| {diff.max().item():.3e}")
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(got.float(), _torch_dw_ln(x, w, b, gamma, beta, eps).float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("shape", [(4, 96, 56, 56), (4, 192, 28, 28), (4, 384, 14, 14), (4, 768, 7, 7)],
                         ids=["stage1", "stage2", "stage3", "stage4"])
def test_convnext_stages_bf16(shape):
    _check(shape, torch.bfloat16, seed=3)


@pytest.mark.parametrize("shape,dtype", [
    ((2, 96, 14, 14), torch.float32),
    ((2, 64, 28, 28), torch.float32),     # fp32 28x28 goes to the tile kernel
    ((1, 128, 7, 7), torch.float32),
    ((2, 64, 14, 14), torch.float16),
    ((2, 96, 56, 56), torch.float16),
])
def test_dtypes(shape, dtype):
    _check(shape, dtype, seed=5)


@pytest.mark.parametrize("shape,dtype", [
    ((2, 40, 14, 14), torch.bfloat16),    # partial second group (8 channels)
    ((3, 200, 7, 7), torch.bfloat16),     # 128-channel stages, 7 groups of 32
    ((2, 72, 20, 20), torch.bfloat16),    # clipped edge tiles
    ((1, 36, 30, 17), torch.float32),     # non-square plane, 4 channels left over
    ((5, 512, 14, 14), torch.bfloat16),   # 16-CTA clusters (the largest)
])
def test_odd_shapes(shape, dtype):
    _check(shape, dtype, seed=7)


def test_without_bias_scale_shift_and_large_eps():
    _check((2, 96, 14, 14), torch.bfloat16, seed=11, affine=False)
    _check((2, 96, 28, 28), torch.float16, seed=12, eps=0.5)


def test_module_matches_oracle_and_unfused_pair():
    from pla_b200 import DepthwiseLayerNorm, depthwise7x7

    torch.manual_seed(0)
    m = DepthwiseLayerNorm(192).to(DEV).to(torch.bfloat16)
    with torch.no_grad():
        m.norm.weight.normal_(1.0, 0.2)
        m.norm.bias.normal_(0.0, 0.1)
    x = torch.randn(3, 192, 28, 28, device=DEV).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    z = m(x)
    p = [t.detach().cpu() for t in (m.dwconv.weight, m.dwconv.bias, m.norm.weight, m.norm.bias)]
    assert torch.equal(z.cpu(), oracle.depthwise7x7_layernorm(x.cpu(), *p, 1e-6))
    # the unfused pair: this library's depthwise, then torch's LayerNorm on the NHWC view
    y = depthwise7x7(x, m.dwconv.weight, m.dwconv.bias)
    ref = m.norm(y.permute(0, 2, 3, 1)).permute(0, 3, 1, 2)
    torch.testing.assert_close(z.float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_repeated_calls_and_side_stream():
    x, w, b, gamma, beta = _inputs((8, 384, 14, 14), torch.bfloat16, seed=13)
    ref = oracle.depthwise7x7_layernorm(x, w, b, gamma, beta, 1e-6)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        outs = [_run(x, w, b, gamma, beta) for _ in range(3)]
    for o in outs:
        assert torch.equal(o, ref)


def test_unsupported_inputs_raise():
    from pla_b200 import _lib, depthwise7x7_layernorm

    w = torch.randn(1024, 1, 7, 7, device=DEV)
    x = torch.randn(1, 1024, 14, 14, device=DEV).contiguous(memory_format=torch.channels_last)
    # The functional form runs the torch op (TORCH_CHECK -> RuntimeError with
    # the C ABI's status text); the out= form calls the C ABI through ctypes
    # (PlaError, a RuntimeError).
    with pytest.raises(RuntimeError, match="unsupported"):  # 32 channel groups: more CTAs than a cluster holds
        depthwise7x7_layernorm(x, w)
    with pytest.raises(_lib.PlaError):
        depthwise7x7_layernorm(x, w, out=torch.empty_like(x))
    with pytest.raises(RuntimeError):  # NCHW input
        depthwise7x7_layernorm(torch.randn(1, 32, 14, 14, device=DEV), torch.randn(32, 1, 7, 7, device=DEV))
    with pytest.raises(RuntimeError, match="unsupported"):  # 12 bf16 channels: 24-byte pixel rows, not TMA-addressable
        depthwise7x7_layernorm(torch.randn(1, 12, 14, 14, device=DEV).bfloat16()
                               .contiguous(memory_format=torch.channels_last),
                               torch.randn(12, 1, 7, 7, device=DEV).bfloat16())


def test_no_device_faults_after_layernorm():
    from pla_b200 import _lib

    L = _lib.lib()
    _check((2, 192, 28, 28), torch.bfloat16, seed=17)
    import ctypes

    f = ctypes.c_uint(0)
    assert L.pla_read_device_faults(ctypes.byref(f)) == 0
    assert f.value == 0

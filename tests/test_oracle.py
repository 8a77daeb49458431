"""Pin the CPU oracle (oracle/oracle.py + oracle/pla_oracle.c) against the
golden vectors produced by the reference modules (tests/golden/make_golden.py).

Tolerances are the ones the north star states (rtol = atol = 1e-5 for fp32,
2e-2 for bf16) and the reference tests use for fp16 / fp64
(data/stencil_direct_cuda_v7/test_stencil.py:39-40).
"""
import pytest
import torch

from oracle import oracle
from tests.golden_util import load_cases

CASES = load_cases()


def _oracle(case):
    if case.op == "stencil":
        return oracle.stencil7x7(case.x, case.w, case.b)
    if case.op == "depthwise":
        C = case.shape[1]
        return oracle.depthwise7x7(case.x, case.w.reshape(C, 1, 7, 7), case.b)
    if case.op == "depthwise_ms":
        C, k = case.shape[1], case.k
        return oracle.depthwise(case.x, case.w.reshape(C, 1, k, k), case.b)
    return oracle.stencil7x7_iterate(case.x, case.w, case.steps, case.b)


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference_golden(case):
    got = _oracle(case)
    assert got.shape == case.y.shape and got.dtype == case.y.dtype
    if case.layout == "nhwc":
        assert got.is_contiguous(memory_format=torch.channels_last)
    if case.op == "iterate":
        # Values grow step by step (coefficients summing to 1 are not a
        # contraction); compare relative to the largest magnitude.
        scale = case.y.abs().max().item()
        torch.testing.assert_close(got / scale, case.y / scale, rtol=1e-5, atol=1e-5)
    else:
        torch.testing.assert_close(got.float(), case.y.float(), rtol=case.tol, atol=case.tol)
    if case.y_native is not None:
        # The reference module run natively in bf16 on the CPU.
        torch.testing.assert_close(got.float(), case.y_native.float(), rtol=2e-2, atol=2e-2)


def test_oracle_bf16_rounding_is_rne():
    # Exactly representable sums, then ties: 1 + 2^-8 rounds to 1 (even), 1 + 3*2^-8 rounds up.
    x = torch.zeros(1, 1, 1, 2)
    x[0, 0, 0, 0] = 1.0
    w = torch.zeros(1, 1, 7, 7)
    w[0, 0, 3, 3] = 1.0
    for extra, expect in [(2.0 ** -8, 1.0), (3 * 2.0 ** -8, 1.0 + 2.0 ** -6)]:
        b = torch.tensor([extra])
        y = oracle.depthwise7x7(x.bfloat16(), w.bfloat16(), None)
        assert y[0, 0, 0, 0].item() == 1.0
        # fp32 accumulate + bias, single rounding to bf16
        yf = oracle.depthwise7x7(x, w, b)
        assert yf[0, 0, 0, 0].item() == 1.0 + extra
        assert yf.bfloat16()[0, 0, 0, 0].item() == expect


def test_oracle_rows_band_equals_full():
    g = torch.Generator().manual_seed(0)
    x = torch.rand(50, 40, generator=g) * 2 - 1
    w = torch.rand(7, 7, generator=g)
    full = oracle.stencil7x7(x.view(1, 1, 50, 40), w).view(50, 40)
    for r0, r1 in [(0, 5), (10, 30), (45, 50), (0, 50)]:
        band = oracle.stencil7x7_rows(x, w, r0, r1)
        assert torch.equal(band, full[r0:r1])


def test_oracle_threads_do_not_change_results():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 5, 21, 33, generator=g)
    w = torch.randn(5, 1, 7, 7, generator=g)
    b = torch.randn(5, generator=g)
    a = oracle.depthwise7x7(x, w, b, threads=1)
    c = oracle.depthwise7x7(x, w, b, threads=7)
    assert torch.equal(a, c)


# --------------------------------------------------------------------------
# depthwise 7x7 + channel LayerNorm (NHWC).  No reference counterpart: the
# LayerNorm half is pinned to torch's own F.layer_norm on the reference
# depthwise module's output (data/depthwise_conv_7x7.py:15-29 run through
# oracle/reference_modules.py), the depthwise half to the golden vectors above.
# --------------------------------------------------------------------------
def _torch_dw_ln(x, w, b, gamma, beta, eps):
    import torch.nn.functional as F

    C = x.shape[1]
    y = F.conv2d(x.float(), w.float(), None if b is None else b.float(), padding=3, groups=C).to(x.dtype)
    z = F.layer_norm(y.float().permute(0, 2, 3, 1), (C,), None if gamma is None else gamma.float(),
                     None if beta is None else beta.float(), eps)
    return z.permute(0, 3, 1, 2).to(x.dtype)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2), (torch.float16, 2e-2)])
@pytest.mark.parametrize("shape", [(2, 96, 14, 14), (1, 40, 7, 7), (2, 72, 20, 20), (1, 200, 7, 7)])
@pytest.mark.parametrize("affine", [True, False])
def test_oracle_depthwise_layernorm_matches_torch(dtype, tol, shape, affine):
    g = torch.Generator().manual_seed(hash((shape, affine)) % 1000)
    N, C, H, W = shape
    x = torch.randn(*shape, generator=g).to(dtype)
    w = (torch.randn(C, 1, 7, 7, generator=g) / 7).to(dtype)
    b = (torch.randn(C, generator=g) * 0.1).to(dtype) if affine else None
    gamma = (1 + 0.2 * torch.randn(C, generator=g)).to(dtype) if affine else None
    beta = (0.1 * torch.randn(C, generator=g)).to(dtype) if affine else None
    got = oracle.depthwise7x7_layernorm(x, w, b, gamma, beta, 1e-6)
    assert got.is_contiguous(memory_format=torch.channels_last)
    ref = _torch_dw_ln(x, w, b, gamma, beta, 1e-6)
    torch.testing.assert_close(got.float(), ref.float(), rtol=tol, atol=tol)
    # the depthwise half is the plain oracle's output
    if not affine:
        y = oracle.depthwise7x7(x.contiguous(memory_format=torch.channels_last), w, None)
        assert torch.equal(got, oracle.depthwise7x7_layernorm(y.contiguous(memory_format=torch.channels_last),
                                                              _identity_filter(C, dtype), None, None, None, 1e-6))


def _identity_filter(C, dtype):
    w = torch.zeros(C, 1, 7, 7)
    w[:, 0, 3, 3] = 1.0
    return w.to(dtype)


def test_oracle_depthwise_layernorm_constant_pixels():
    # A pixel whose channels are all equal has zero variance: z = beta exactly.
    C = 64
    x = torch.zeros(1, C, 7, 7)
    w = torch.zeros(C, 1, 7, 7)
    b = torch.full((C,), 0.75)
    beta = torch.linspace(-1, 1, C)
    z = oracle.depthwise7x7_layernorm(x, w, b, torch.ones(C), beta, 1e-6)
    assert torch.equal(z, beta.view(1, C, 1, 1).expand(1, C, 7, 7).contiguous(memory_format=torch.channels_last))

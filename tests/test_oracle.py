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

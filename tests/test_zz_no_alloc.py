"""pla_stencil7x7_iterate_noalloc: the iterated stencil for callers that
cannot allocate device memory (plugins inside a framework that owns all
device allocations, fixed-budget runtimes, real-time loops that cannot take
cudaMalloc's implicit synchronisation).  Its ping-pong plane is a static
16 MiB array inside the library instead of a caller buffer.

The test goes through the C ABI and checks the allocation-free entry point
against pla_stencil7x7_iterate (same kernels, caller scratch) on two calls in
a row: results must agree bit for bit, the same bar as every other parity test
here.  This file is collected last so that a failure here comes after all
other tests have run; it also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _inputs(seed, H, W, dtype):
    g = torch.Generator().manual_seed(seed)
    x = (torch.rand(H, W, generator=g) * 2 - 1).to(dtype)
    w = torch.rand(7, 7, generator=g) * 2 - 1
    w = (w / w.sum()).to(dtype)
    b = ((torch.rand(1, generator=g) * 2 - 1) / 49).to(dtype)
    return x.to(DEV), w.to(DEV), b.to(DEV)


def _iterate_with_scratch(L, x, w, b, steps):
    from pla_b200 import _lib

    y = torch.empty_like(x)
    scratch = torch.empty_like(x)
    st = L.pla_stencil7x7_iterate(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), scratch.data_ptr(),
                                  x.shape[0], x.shape[1], steps, _lib.DTYPE_CODE[x.dtype],
                                  torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.pla_status_string(st)
    return y


def _iterate_noalloc(L, x, w, b, steps):
    from pla_b200 import _lib

    y = torch.empty_like(x)
    st = L.pla_stencil7x7_iterate_noalloc(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), x.shape[0],
                                          x.shape[1], steps, _lib.DTYPE_CODE[x.dtype],
                                          torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.pla_status_string(st) + b" " + L.pla_last_cuda_error()
    return y


def test_noalloc_iterate_matches_allocating_entry_point_twice():
    from pla_b200 import _lib

    L = _lib.lib()
    # Two calls in a row on the shared static scratch: a large fp32 grid
    # (12 MiB of the 16 MiB scratch), then a smaller bf16 grid whose run
    # starts on the first call's leftovers.
    for seed, (H, W, steps, dtype) in enumerate([(2048, 1536, 11, torch.float32),
                                                 (640, 768, 6, torch.bfloat16)]):
        x, w, b = _inputs(seed, H, W, dtype)
        got = _iterate_noalloc(L, x, w, b, steps)
        ref = _iterate_with_scratch(L, x, w, b, steps)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {seed}: results differ from pla_stencil7x7_iterate"


def test_noalloc_rejects_grids_beyond_the_static_scratch():
    from pla_b200 import _lib

    L = _lib.lib()
    x = torch.empty(1, device=DEV)
    # 2049 x 2048 fp32 is one row more than the 16 MiB scratch holds.
    st = L.pla_stencil7x7_iterate_noalloc(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), 2049, 2048, 3,
                                          _lib.PLA_F32, torch.cuda.current_stream().cuda_stream)
    assert st == 3  # PLA_ERR_TOO_LARGE
    assert b"16777216" in L.pla_last_cuda_error()

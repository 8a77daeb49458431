"""Failure detection without a GPU fault.

The fused multi-GPU band step waits for its neighbours' halo flags with a
bounded spin (about 2 s).  Here a single GPU runs one step whose "neighbour
above" is a local buffer and whose flag nothing ever sets: the wait must run
out, record bit 1 in the device fault word, let the kernel finish, and leave
the context usable.  Nothing traps, faults or hangs; no second kernel waits on
this one."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_halo_wait_times_out_into_fault_word():
    from oracle import oracle
    from pla_b200 import _lib, stencil7x7

    L = _lib.lib()
    dev = torch.device("cuda:0")
    rows, W = 128, 256
    g = torch.Generator().manual_seed(3)
    buf_in = (torch.rand(rows + 6, W, generator=g) * 2 - 1).to(dev)
    buf_out = torch.zeros(rows + 6, W, device=dev)
    fake_up = torch.zeros(rows + 6, W, device=dev)      # stands in for the neighbour's buffer
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    fake_up_flags = torch.zeros(2, dtype=torch.int32, device=dev)
    counters = torch.zeros(2, dtype=torch.int32, device=dev)
    taps, hb = _lib.HostTaps().update(torch.ones(49, device=dev) / 49, None).args()
    assert L.pla_clear_device_faults() == 0

    t0 = time.perf_counter()
    # step 1 needs flags[0] >= 1 ("the neighbour above delivered step 0"); nothing sets it
    st = L.pla_stencil7x7_band_step_halo(buf_in.data_ptr(), taps, hb, buf_out.data_ptr(), rows, W, _lib.PLA_F32,
                                         fake_up.data_ptr(), rows, None, flags.data_ptr(),
                                         fake_up_flags.data_ptr(), None, counters.data_ptr(), 1,
                                         torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    v = ctypes.c_uint(0)
    assert L.pla_read_device_faults(ctypes.byref(v)) == 0
    assert v.value & 2, f"fault word {v.value:#x}: the halo wait did not report its time-out"
    assert 1.0 < waited < 30.0
    assert L.pla_clear_device_faults() == 0
    assert L.pla_read_device_faults(ctypes.byref(v)) == 0 and v.value == 0

    # the context is still usable: a normal launch gives the oracle's answer
    x = torch.rand(1, 1, 64, 64, generator=g)
    w = torch.rand(1, 1, 7, 7, generator=g)
    y = stencil7x7(x.to(dev), w.to(dev))
    assert torch.equal(y.cpu(), oracle.stencil7x7(x, w))

"""Multi-GPU parity: the row-band iterated stencil (one process per GPU; halo
exchange fused into the kernel over peer memory, or over NCCL) must equal the
single-GPU iteration bit for bit.  Needs >= 2 GPUs; ranks never share a GPU."""
import os
import random
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(H, W):
    g = torch.Generator().manual_seed(4)
    x = torch.rand(H, W, generator=g) * 2 - 1
    w = torch.rand(7, 7, generator=g) * 2 - 1
    return x, w / w.sum()


def _second_grid(H, W):
    g = torch.Generator().manual_seed(5)
    return torch.rand(H, W, generator=g) * 2 - 1


def _rank(rank, world, port, H, W, steps, mode, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from pla_b200 import BandedStencil

        x, w = _inputs(H, W)
        bs = BandedStencil(H, W, w.to(dev), device=dev, mode=mode)
        assert bs.mode == mode
        bs.load(x.to(dev))
        bs.run(steps)
        full = bs.gather()
        # Reload a second grid right after the steps (p2p: the neighbours'
        # last halo stores must not land on the new rows), from a host slab
        # that holds only this rank's band and halo rows, and run again.
        x2 = _second_grid(H, W)
        a0, a1 = bs.halo_span()
        bs.load(x2[a0:a1].clone(), row0=a0)
        bs.run(steps + 1)
        full2 = bs.gather()
        torch.cuda.synchronize()
        bs.check_faults()
        if rank == 0:
            q.put((full.cpu(), full2.cpu()))
        bs.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["p2p", "nccl"])
@pytest.mark.parametrize("world,H,W,steps", [(2, 1000, 768, 9), (2, 300, 256, 12), (4, 1000, 768, 9),
                                             (8, 2048, 512, 7)])
def test_banded_multi_gpu_equals_single_gpu(world, H, W, steps, mode):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from pla_b200 import stencil7x7_iterate

    x, w = _inputs(H, W)
    ref = stencil7x7_iterate(x.cuda(), w.cuda(), steps).cpu()
    ref2 = stencil7x7_iterate(_second_grid(H, W).cuda(), w.cuda(), steps + 1).cpu()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, H, W, steps, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    got, got2 = q.get(timeout=180)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert torch.equal(got, ref)
    assert torch.equal(got2, ref2)

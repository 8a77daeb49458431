"""Host-side logic that needs no GPU: the kernels' division-free index
decode, row-band partitioning, and the multi-rank halo exchange of the
iterated stencil on gloo CPU ranks (the band step computed by the oracle)."""
import os
import random

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle


# ---- FastDiv (pla_b200/csrc/pla_common.cuh) restated with the same integers
def _make_fastdiv(d):
    if d <= 1:
        return d, 0, 0
    l = (d - 1).bit_length()  # ceil(log2 d)
    m = ((1 << (31 + l)) + d - 1) // d
    assert m < (1 << 32)
    return d, m, l - 1


def _fdiv(n, f):
    d, m, s = f
    return n if d == 1 else ((n * m) >> 32) >> s


def test_fastdiv_exact_for_all_int31_dividends():
    rng = random.Random(0)
    divisors = list(range(1, 2049)) + [rng.randrange(2, 2 ** 31) for _ in range(2000)] + [2 ** 31 - 1, 2 ** 30,
                                                                                         2 ** 30 + 1, 3 ** 19]
    for d in divisors:
        f = _make_fastdiv(d)
        for n in [0, 1, d - 1, d, d + 1, 2 * d - 1, 2 ** 31 - 1, 2 ** 31 - 2, max(0, 2 ** 31 - d)] + \
                 [rng.randrange(0, 2 ** 31) for _ in range(64)]:
            if 0 <= n < 2 ** 31:
                assert _fdiv(n, f) == n // d, (n, d)


# ---- band partition -----------------------------------------------------------
def test_band_rows_partition():
    from pla_b200.iterate import band_rows

    for H in (1, 7, 32, 100, 32768):
        for world in (1, 2, 3, 4, 8):
            if H < world:
                continue
            bands = [band_rows(H, world, r) for r in range(world)]
            assert bands[0][0] == 0 and bands[-1][1] == H
            for (a0, a1), (b0, b1) in zip(bands, bands[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in bands]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        band_rows(10, 0, 0)


# ---- multi-rank halo exchange on gloo CPU ranks ------------------------------
def _oracle_band_step(w):
    def step(src, dst, rb, re):
        # band row r <-> buffer row r + 3; output rows need buffer rows r .. r+6
        dst[rb + 3:re + 3] = oracle.stencil7x7_rows(src, w, rb + 3, re + 3)
    return step


def _rank_main(rank, world, port, H, W, steps, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pla_b200.iterate import BandedStencil

        g = torch.Generator().manual_seed(4)
        x = torch.rand(H, W, generator=g) * 2 - 1
        w = torch.rand(7, 7, generator=g) * 2 - 1
        w = w / w.sum()
        bs = BandedStencil(H, W, w, device=torch.device("cpu"), step_fn=_oracle_band_step(w))
        bs.load(x)
        bs.run(steps)
        full = bs.gather()
        # Reload a second grid from a slab that holds only this rank's band
        # and halo rows (as the benchmark does), and run again.
        x2 = torch.rand(H, W, generator=g) * 2 - 1
        a0, a1 = bs.halo_span()
        lo, hi = max(0, a0 - 1), min(H, a1 + 2)
        bs.load(x2[lo:hi].clone(), row0=lo)
        bs.run(steps + 1)
        full2 = bs.gather()
        if rank == 0:
            out_q.put((full, full2))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,H,W,steps", [(2, 40, 24, 5), (3, 31, 16, 4), (4, 48, 20, 3)])
def test_banded_iterate_gloo_matches_single_domain(world, H, W, steps):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + random.Random(world * 1000 + H).randrange(0, 5000)
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, H, W, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    full, full2 = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(4)
    x = torch.rand(H, W, generator=g) * 2 - 1
    w = torch.rand(7, 7, generator=g) * 2 - 1
    w = w / w.sum()
    x2 = torch.rand(H, W, generator=g) * 2 - 1
    assert torch.equal(full, oracle.stencil7x7_iterate(x, w, steps))
    assert torch.equal(full2, oracle.stencil7x7_iterate(x2, w, steps + 1))


def test_band_load_rejects_a_slab_that_misses_the_halo():
    from pla_b200.iterate import BandedStencil

    w = torch.rand(7, 7)
    bs = BandedStencil(24, 16, w, device=torch.device("cpu"), step_fn=_oracle_band_step(w))
    x = torch.rand(24, 16)
    with pytest.raises(ValueError):
        bs.load(x[2:], row0=2)  # one rank: its span is the whole grid, rows 0..1 missing
    bs.load(x[:24], row0=0)


# ---- a rank that leaves: the others get an error, not a hang -------------------
def _leaver_main(rank, world, port, out_q):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from pla_b200.iterate import BandedStencil

    g = torch.Generator().manual_seed(4)
    x = torch.rand(24, 16, generator=g)
    w = torch.rand(7, 7, generator=g)
    bs = BandedStencil(24, 16, w, device=torch.device("cpu"), step_fn=_oracle_band_step(w))
    bs.load(x)
    if rank == 1:
        os._exit(0)  # leaves between steps, before any exchange
    try:
        bs.run(3)
        out_q.put("no error")
    except Exception as exc:  # noqa: BLE001
        out_q.put(type(exc).__name__)
    out_q.close()
    out_q.join_thread()  # flush the queue's feeder thread before the hard exit
    os._exit(0)


def test_rank_leaving_raises_on_the_survivor():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + random.Random(77).randrange(5000, 9000)
    procs = [ctx.Process(target=_leaver_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert outcome != "no error"


# ---- the overlapped whole-job schedule of one band ------------------------------
@pytest.mark.parametrize("rows,steps,chunks", [(96, 10, 4), (200, 7, 16), (64, 2, 8), (130, 30, 5), (40, 1, 4)])
def test_job_schedule_covers_every_step_once(rows, steps, chunks):
    from pla_b200.iterate import BandedStencil

    edges, k, launches = BandedStencil.job_schedule(rows, steps, chunks)
    assert edges[-1] == rows and all(a < b for a, b in zip([0] + edges[:-1], edges))
    assert 2 * k <= steps
    covered = {st: [] for st in range(1, steps + 1)}
    arrived = set()
    done_out = set()
    lo_of = [0] + edges[:-1]
    for kind, c, st, lo, hi in launches:
        if kind == "in":
            arrived.add(c)
        elif kind == "step":
            assert 0 <= lo <= hi <= rows
            covered[st].append((lo, hi))
            if hi > lo and st % 2 == 0:  # writes the input buffer: never rows still being copied in
                for p in set(range(len(edges))) - arrived:
                    assert hi <= lo_of[p] or lo >= edges[p]
            if hi > lo and st % 2 == steps % 2:  # writes the output buffer: never rows being copied out
                for p in done_out:
                    assert hi <= lo_of[p] or lo >= edges[p]
            if st == 1:  # the rows read (lo - 3 .. hi + 3) have been copied in
                need = hi + 3
                got = max([edges[a] for a in arrived], default=0)
                assert need <= got or hi == rows and max(arrived) == len(edges) - 1
        else:
            done_out.add(c)
            # chunk c's final rows are complete before they are copied out
            lo_r = 0 if c == 0 else edges[c - 1]
            fin = sorted(covered[steps])
            assert any(a <= lo_r and edges[c] <= b for a, b in fin) or \
                sum(min(b, edges[c]) - max(a, lo_r) for a, b in fin if b > lo_r and a < edges[c]) == edges[c] - lo_r
    assert done_out == set(range(len(edges)))
    for st, regs in covered.items():
        regs = sorted(r for r in regs if r[1] > r[0])
        assert regs[0][0] == 0 and regs[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(regs, regs[1:]))  # contiguous, no overlap


@pytest.mark.parametrize("rows,steps,chunks", [(96, 10, 4), (130, 30, 5), (64, 2, 8), (40, 1, 4)])
def test_run_job_matches_the_oracle_iteration(rows, steps, chunks):
    """run_job (copy in by chunks, skewed first and last steps, copy out by
    chunks) equals the plain oracle iteration bit for bit, and leaves the band
    ready for the next job."""
    from pla_b200.iterate import BandedStencil

    W = 24
    g = torch.Generator().manual_seed(9)
    x = torch.rand(rows, W, generator=g) * 2 - 1
    w = torch.rand(7, 7, generator=g) * 2 - 1
    w = w / w.sum()
    bs = BandedStencil(rows, W, w, device=torch.device("cpu"), step_fn=_oracle_band_step(w))
    bs.load(torch.zeros(rows, W))
    out = torch.empty(rows, W)
    bs.run_job(x, 0, steps, out, chunks=chunks)
    assert torch.equal(out, oracle.stencil7x7_iterate(x, w, steps))
    x2 = torch.rand(rows, W, generator=g)
    bs.run_job(x2, 0, steps + 1, out, chunks=chunks)
    assert torch.equal(out, oracle.stencil7x7_iterate(x2, w, steps + 1))

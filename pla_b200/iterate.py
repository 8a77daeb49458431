"""Iterated 7x7 stencil: u_{t+1} = stencil(u_t), zero Dirichlet boundary.

No reference function exists for the iteration: the reference op is
data/stencil_7x7.py:10-12 applied once.  Iterating it with its zero padding
re-applied every step is the Jacobi scheme with a zero boundary.

* ``stencil7x7_iterate`` — one device, ping-pong between the output and one
  scratch plane (``pla_stencil7x7_iterate``).
* ``BandedStencil`` — the grid split into row bands, one band per rank of a
  process group (one process per GPU).  Each band lives in two
  (rows + 6) x W buffers whose 3 top / 3 bottom rows are halos; bands at the
  top / bottom of the grid keep zero halos (the Dirichlet boundary).  Two
  exchange modes:

  - ``"p2p"`` (default on GPUs): one fused kernel per step
    (``pla_stencil7x7_band_step_halo``).  The buffers of the neighbours are
    mapped into this process with CUDA IPC; the kernel visits the edge tiles
    first, stores their rows straight into the neighbours' halo rows over
    NVLink and raises a flag in the neighbour's memory; a neighbour's edge
    tiles wait on that flag (bounded) before loading their halo.  No
    collective call and no host round trip per step.
  - ``"nccl"``: the 3 edge rows at each end are computed first, handed over
    with NCCL send/recv on a side stream while the interior is computed
    (also the path gloo CPU ranks take in the tests).

  Every point is computed exactly as on one device, so the result is
  bit-identical to ``stencil7x7_iterate`` for any number of ranks.
"""
from __future__ import annotations

from typing import Callable, Optional

import ctypes

import torch
import torch.distributed as dist

from . import _lib


def stencil7x7_iterate(x: torch.Tensor, weight: torch.Tensor, steps: int, bias: torch.Tensor | None = None,
                       out: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
                       host_taps: _lib.HostTaps | None = None) -> torch.Tensor:
    """Apply the 7x7 stencil `steps` times to the CUDA grid x [H, W] (fp32/bf16/fp16).

    Without ``out``, ``scratch`` and ``host_taps`` this is the torch op
    ``torch.ops.pla_b200.stencil7x7_iterate`` (filter read from device
    memory by every step; the op allocates the output and the second
    ping-pong plane).  Otherwise the steps run the constant-operand kernel:
    the filter is copied to the host once per call (a stream sync), or taken
    from ``host_taps``.
    """
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError("stencil7x7_iterate requires a CUDA input")
    if x.dim() != 2 or not x.is_contiguous():
        raise RuntimeError("expected a contiguous [H, W] grid")
    if steps < 0:
        raise ValueError("steps must be >= 0")
    if weight.numel() != 49 or weight.dtype != x.dtype or weight.device != x.device:
        raise RuntimeError("weight must be one 7x7 filter of x's dtype and device")
    if bias is not None and (bias.numel() != 1 or bias.dtype != x.dtype or bias.device != x.device):
        raise RuntimeError("bias device/dtype/shape mismatch")
    H, W = x.shape
    if out is None and scratch is None and host_taps is None:
        return _lib.ops().stencil7x7_iterate(x, weight.detach(), int(steps),
                                             None if bias is None else bias.detach())
    if out is None:
        out = torch.empty_like(x)
    if scratch is None:
        scratch = torch.empty_like(x)
    if host_taps is None:
        host_taps = _lib.HostTaps().update(weight, bias)
    taps, hb = host_taps.args()
    with torch.cuda.device(x.device):
        st = _lib.lib().pla_stencil7x7_iterate_taps(
            x.data_ptr(), taps, hb, out.data_ptr(), scratch.data_ptr(), H, W, steps,
            _lib.DTYPE_CODE[x.dtype], _lib.stream_ptr(x.device))
    _lib.check(st, "pla_stencil7x7_iterate_taps")
    return out


def band_rows(total_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of band `rank` when `total_rows` are split into `world` bands.

    The first total_rows % world bands get one extra row, so band sizes differ
    by at most one.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(total_rows, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


StepFn = Callable[[torch.Tensor, torch.Tensor, int, int], None]


def _cuda_band_step(weight: torch.Tensor, bias: Optional[torch.Tensor]) -> StepFn:
    L = _lib.lib()
    code = _lib.DTYPE_CODE[weight.dtype]
    taps, hb = _lib.HostTaps().update(weight, bias).args()

    def step(src: torch.Tensor, dst: torch.Tensor, row_begin: int, row_end: int) -> None:
        rows, W = src.shape[0] - 6, src.shape[1]
        st = L.pla_stencil7x7_band_step_taps(src.data_ptr(), taps, hb, dst.data_ptr(), rows, W, row_begin,
                                             row_end, code, _lib.stream_ptr(src.device))
        _lib.check(st, "pla_stencil7x7_band_step_taps")

    return step


class BandedStencil:
    """Row-band partitioned iterated stencil over a process group.

    ``step_fn(src, dst, row_begin, row_end)`` computes band rows
    [row_begin, row_end) of one step from band buffer `src` into `dst`; the
    default is the CUDA kernel.  The halo exchange uses the group's P2P
    send/recv (NCCL on GPUs; gloo ranks on the CPU for the tests).
    """

    def __init__(self, H: int, W: int, weight: torch.Tensor, bias: torch.Tensor | None = None,
                 group=None, device: torch.device | None = None, step_fn: StepFn | None = None,
                 overlap: bool = True, mode: str = "auto"):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.H, self.W = H, W
        self.r0, self.r1 = band_rows(H, self.world, self.rank)
        self.rows = self.r1 - self.r0
        if self.world > 1 and H < 3 * self.world:
            raise ValueError("every band needs at least 3 rows (H >= 3 * world size)")
        self.device = device if device is not None else weight.device
        self.dtype = weight.dtype
        self.weight = weight.detach().reshape(49).contiguous()
        self.bias = None if bias is None else bias.detach().reshape(1).contiguous()
        self.up = self.rank - 1 if self.rank > 0 else None
        self.down = self.rank + 1 if self.rank < self.world - 1 else None
        if mode == "auto":
            mode = "p2p" if (self.device.type == "cuda" and self.world > 1 and step_fn is None) else "nccl"
        if mode not in ("p2p", "nccl"):
            raise ValueError("mode must be 'p2p', 'nccl' or 'auto'")
        if mode == "p2p" and (self.device.type != "cuda" or step_fn is not None):
            raise ValueError("the p2p exchange runs the CUDA kernel on CUDA devices")
        self.mode = mode
        self.cur = 0
        self.step_idx = 0
        band = (self.rows + 6) * W
        es = torch.tensor([], dtype=self.dtype).element_size()
        if mode == "p2p":
            # One allocation per rank so that a neighbour maps it with one IPC
            # handle: [buffer 0 | buffer 1 | flags u32[2] | counters u32[2]].
            self._store = torch.zeros(2 * band * es + 16, dtype=torch.uint8, device=self.device)
            self.bufs = [self._store[k * band * es:(k + 1) * band * es].view(self.dtype).view(self.rows + 6, W)
                         for k in range(2)]
            self._flags = self._store[2 * band * es:2 * band * es + 8]
            self._counters = self._store[2 * band * es + 8:2 * band * es + 16]
            self._taps = _lib.HostTaps().update(self.weight, self.bias)
            self._peers = {}
            self._exchange_handles(es)
            self._armed = False
        else:
            self.bufs = [torch.zeros(self.rows + 6, W, dtype=self.dtype, device=self.device) for _ in range(2)]
        self.step_fn = step_fn or (None if mode == "p2p" else _cuda_band_step(self.weight, self.bias))
        self.overlap = overlap and self.device.type == "cuda" and self.rows >= 12
        self.comm_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None

    # -- peer mapping (p2p mode) -------------------------------------------------
    def _exchange_handles(self, es: int) -> None:
        L = _lib.lib()
        h = (ctypes.c_ubyte * 64)()
        off = ctypes.c_uint64()
        with torch.cuda.device(self.device):
            _lib.check(L.pla_ipc_export(self._store.data_ptr(), h, ctypes.byref(off)), "pla_ipc_export")
        info = [None] * self.world
        dist.all_gather_object(info, (bytes(h), off.value, self.rows), group=self.group)
        for name, peer in (("up", self.up), ("down", self.down)):
            if peer is None:
                continue
            hb, poff, prows = info[peer]
            ptr = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(L.pla_ipc_import((ctypes.c_ubyte * 64).from_buffer_copy(hb), poff, ctypes.byref(ptr)),
                           "pla_ipc_import")
            base = ptr.value
            pband = (prows + 6) * self.W * es
            self._peers[name] = {"base": base, "offset": poff, "rows": prows,
                                 "bufs": [base, base + pband], "flags": base + 2 * pband}

    def close(self) -> None:
        """Unmap the neighbours' buffers (p2p mode).  Collective: every rank calls it."""
        if self.mode != "p2p" or not self._peers:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no neighbour still writes into our halos
        L = _lib.lib()
        with torch.cuda.device(self.device):
            for p in self._peers.values():
                L.pla_ipc_close(p["base"], p["offset"])
        self._peers = {}

    def check_faults(self) -> None:
        """Raise if a kernel on this device gave up a bounded wait (synchronises)."""
        v = ctypes.c_uint(0)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().pla_read_device_faults(ctypes.byref(v)), "pla_read_device_faults")
        if v.value:
            raise _lib.PlaError(f"device fault word {v.value:#x}: a bounded wait in a kernel timed out")

    def _global(self, peer: int) -> int:
        return peer if self.group is None else dist.get_global_rank(self.group, peer)

    # -- state -------------------------------------------------------------
    def halo_span(self) -> tuple[int, int]:
        """Grid rows [a0, a1) this rank loads: its band and the halo rows that exist."""
        return max(0, self.r0 - 3), min(self.H, self.r1 + 3)

    def load(self, grid: torch.Tensor, row0: int = 0) -> None:
        """Copy this rank's band and its halo rows out of `grid`.

        ``grid`` holds grid rows [row0, row0 + grid.shape[0]) of the [H, W]
        grid: the whole grid (row0 = 0) or any slab covering ``halo_span()``
        (host or device memory).

        In p2p mode a neighbour's last step may still be storing its edge rows
        into this rank's halo rows over peer memory; once any step has run,
        every rank first drains its stream and meets the others at a barrier,
        so no late store lands on the freshly loaded rows.  Collective then:
        every rank calls it.
        """
        a0, a1 = self.halo_span()
        if grid.dim() != 2 or grid.shape[1] != self.W or row0 > a0 or row0 + grid.shape[0] < a1:
            raise ValueError(f"grid rows [{row0}, {row0 + grid.shape[0]}) do not cover rows [{a0}, {a1})")
        if self.mode == "p2p" and (self._armed or self.step_idx > 0):
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        b = self.bufs[self.cur]
        b.zero_()
        b[3 - (self.r0 - a0):3 + self.rows + (a1 - self.r1)].copy_(grid[a0 - row0:a1 - row0])
        self.bufs[1 - self.cur].zero_()
        if self.mode == "p2p":
            self._armed = False  # neighbours must finish loading before anyone steps

    def load_async(self, host_rows: torch.Tensor, row0: int, stream: torch.cuda.Stream | None = None) -> None:
        """Stream-ordered copy of this rank's band and halo rows from pinned host
        memory into the current buffer, with no barrier and no zeroing.

        For a repeated job on an already loaded band (the halo rows outside
        the grid stay zero from ``load``): the caller has synchronised every
        rank since the last step, and the steps that follow on the same
        stream see the copy.  ``host_rows`` holds grid rows
        [row0, row0 + host_rows.shape[0]).
        """
        a0, a1 = self.halo_span()
        if row0 > a0 or row0 + host_rows.shape[0] < a1:
            raise ValueError("host rows do not cover this rank's band and halo")
        dst = self.bufs[self.cur][3 - (self.r0 - a0):3 + self.rows + (a1 - self.r1)]
        with torch.cuda.stream(stream or torch.cuda.current_stream(self.device)):
            dst.copy_(host_rows[a0 - row0:a1 - row0], non_blocking=True)

    def band(self) -> torch.Tensor:
        """This rank's current band rows [rows, W] (a view)."""
        return self.bufs[self.cur][3:3 + self.rows]

    def gather(self) -> Optional[torch.Tensor]:
        """Full grid on rank 0 (None elsewhere)."""
        band = self.band().contiguous()
        if self.world == 1:
            return band.clone()
        sizes = [band_rows(self.H, self.world, r) for r in range(self.world)]
        if self.rank == 0:
            out = torch.empty(self.H, self.W, dtype=self.dtype, device=self.device)
            out[self.r0:self.r1].copy_(band)
            for r in range(1, self.world):
                a, b = sizes[r]
                if b > a:
                    t = torch.empty(b - a, self.W, dtype=self.dtype, device=self.device)
                    dist.recv(t, self._global(r), group=self.group)
                    out[a:b].copy_(t)
            return out
        if self.rows > 0:
            dist.send(band, self._global(0), group=self.group)
        return None

    # -- one Jacobi step -----------------------------------------------------
    def _exchange_ops(self, dst: torch.Tensor):
        ops = []
        R = self.rows
        if self.up is not None:
            ops.append(dist.P2POp(dist.isend, dst[3:6], self._global(self.up), self.group))
            ops.append(dist.P2POp(dist.irecv, dst[0:3], self._global(self.up), self.group))
        if self.down is not None:
            ops.append(dist.P2POp(dist.isend, dst[R:R + 3], self._global(self.down), self.group))
            ops.append(dist.P2POp(dist.irecv, dst[R + 3:R + 6], self._global(self.down), self.group))
        return ops

    def _step_p2p(self) -> None:
        if not self._armed:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self._armed = True
        L = _lib.lib()
        nxt = 1 - self.cur
        up, down = self._peers.get("up"), self._peers.get("down")
        taps, hb = self._taps.args()
        flags = self._flags.data_ptr()
        st = L.pla_stencil7x7_band_step_halo(
            self.bufs[self.cur].data_ptr(), taps, hb, self.bufs[nxt].data_ptr(), self.rows, self.W,
            _lib.DTYPE_CODE[self.dtype],
            up["bufs"][nxt] if up else None, up["rows"] if up else 0,
            down["bufs"][nxt] if down else None,
            flags, up["flags"] if up else None, down["flags"] if down else None,
            self._counters.data_ptr(), self.step_idx, _lib.stream_ptr(self.device))
        _lib.check(st, "pla_stencil7x7_band_step_halo")
        self.step_idx += 1
        self.cur = nxt

    def step(self) -> None:
        if self.mode == "p2p":
            return self._step_p2p()
        src, dst = self.bufs[self.cur], self.bufs[1 - self.cur]
        R = self.rows
        if self.overlap and self.world > 1:
            compute = torch.cuda.current_stream(self.device)
            # 1) the rows the neighbours need, 2) hand them over on the side
            #    stream while 3) the interior is computed, 4) join.
            self.step_fn(src, dst, 0, 3)
            self.step_fn(src, dst, R - 3, R)
            self.comm_stream.wait_stream(compute)
            with torch.cuda.stream(self.comm_stream):
                for w in dist.batch_isend_irecv(self._exchange_ops(dst)):
                    w.wait()
            self.step_fn(src, dst, 3, R - 3)
            compute.wait_stream(self.comm_stream)
        else:
            self.step_fn(src, dst, 0, R)
            ops = self._exchange_ops(dst)
            if ops:
                for w in dist.batch_isend_irecv(ops):
                    w.wait()
        self.cur = 1 - self.cur

    def run(self, steps: int) -> None:
        for _ in range(steps):
            self.step()

    # -- one whole job with the transfers overlapped (single band) -----------
    @staticmethod
    def job_schedule(rows: int, steps: int, chunks: int, max_skew: int = 48):
        """Row-range launches of ``run_job`` on one band of ``rows`` rows.

        Returns ``(edges, k, launches)``: chunk edges e_0 < ... < e_{C-1} = rows
        (band rows), the number k of skewed steps at each end, and the launch
        list of (kind, chunk, step, row_begin, row_end) with kind "in" (wait for
        chunk c's input copy), "step", "out" (copy chunk c's final rows) in
        issue order.

        Steps 1..k run chunk by chunk as each chunk's input arrives: chunk c
        of step s ends 3 s rows above the chunk's end e_c (its rows' 7x7 cone
        over s steps stays inside the rows already copied; the last chunk
        ends at the band's end).  Steps k+1..steps-k run whole.  Steps
        steps-k+1..steps run chunk by chunk again, chunk c of step s ending
        3 (steps - s) rows past e_c, so chunk c's final rows [e_{c-1}, e_c)
        are done, and copied out, while later chunks still compute.  In both
        skewed phases a launch only overwrites rows that no later launch of
        an earlier step reads (the regions of consecutive steps meet without
        overlapping), so two ping-pong buffers suffice.
        """
        C = max(1, min(chunks, rows // 8))
        edges = [(rows * (c + 1)) // C for c in range(C)]
        height = min(b - a for a, b in zip([0] + edges[:-1], edges))
        k = max(0, min(steps // 2, (height - 1) // 3, max_skew)) if C > 1 else 0
        L = []

        def hi_in(c, st):
            return rows if c == C - 1 else edges[c] - 3 * st

        def hi_out(c, st):
            return rows if c == C - 1 else min(rows, edges[c] + 3 * (steps - st))

        for c in range(C):
            L.append(("in", c, 0, 0, 0))
            for st in range(1, k + 1):
                lo = 0 if c == 0 else hi_in(c - 1, st)
                L.append(("step", c, st, lo, hi_in(c, st)))
        for st in range(k + 1, steps - k + 1):
            L.append(("step", -1, st, 0, rows))
        if k == 0:  # no skew: the output of the last whole step, chunk by chunk
            for c in range(C):
                L.append(("out", c, steps, 0, 0))
            return edges, k, L
        for c in range(C):
            for st in range(steps - k + 1, steps + 1):
                lo = 0 if c == 0 else hi_out(c - 1, st)
                L.append(("step", c, st, lo, hi_out(c, st)))
            L.append(("out", c, steps, 0, 0))
        return edges, k, L

    def run_job(self, host_rows: torch.Tensor, row0: int, steps: int, host_out: torch.Tensor,
                chunks: int = 16) -> None:
        """One whole job through this band: its rows from ``host_rows`` (pinned
        host memory holding grid rows [row0, ...)), ``steps`` steps, the band's
        final rows into ``host_out`` ([rows, W], pinned), stream-ordered on the
        current stream.

        One band (world size 1, zero halos left by ``load``): the copies run on
        a side stream in ``chunks`` row chunks and overlap the steps
        (``job_schedule``): the first steps start on the rows already copied
        in, the last ones finish the top chunks first, which are copied out
        while the rest compute.  Same results bit for bit as copy-in, ``run``,
        copy-out.  Several bands (p2p or NCCL exchange): copy in, ``run``,
        copy out, in order.
        """
        if self.world > 1 or host_out.shape != (self.rows, self.W):
            if host_out.shape != (self.rows, self.W):
                raise ValueError("host_out must be [rows, W]")
            self.load_async(host_rows, row0)
            self.run(steps)
            host_out.copy_(self.band(), non_blocking=True)
            return
        a0, a1 = self.halo_span()
        if row0 > a0 or row0 + host_rows.shape[0] < a1:
            raise ValueError("host rows do not cover the band")
        R = self.rows
        edges, k, launches = self.job_schedule(R, steps, chunks)
        cur0 = self.cur
        cuda = self.device.type == "cuda"
        comp = torch.cuda.current_stream(self.device) if cuda else None
        copy = self.comm_stream
        if cuda:
            copy.wait_stream(comp)
        ev_in, ev_out = {}, {}
        prev = 0
        # every input chunk is queued on the copy stream at once; the steps wait per chunk
        for c, e in enumerate(edges):
            src = host_rows[prev - row0 + self.r0:e - row0 + self.r0]
            dst = self.bufs[cur0][3 + prev:3 + e]
            if cuda:
                with torch.cuda.stream(copy):
                    dst.copy_(src, non_blocking=True)
                    ev_in[c] = torch.cuda.Event()
                    ev_in[c].record(copy)
            else:
                dst.copy_(src)
            prev = e
        for kind, c, st, lo, hi in launches:
            if kind == "in":
                if cuda:
                    comp.wait_event(ev_in[c])
            elif kind == "step":
                if hi > lo:
                    self.step_fn(self.bufs[(cur0 + st - 1) % 2], self.bufs[(cur0 + st) % 2], lo, hi)
            else:  # out: chunk c's final rows
                lo_r = 0 if c == 0 else edges[c - 1]
                src = self.bufs[(cur0 + st) % 2][3 + lo_r:3 + edges[c]]
                if cuda:
                    ev_out[c] = torch.cuda.Event()
                    ev_out[c].record(comp)
                    copy.wait_event(ev_out[c])
                    with torch.cuda.stream(copy):
                        host_out[lo_r:edges[c]].copy_(src, non_blocking=True)
                else:
                    host_out[lo_r:edges[c]].copy_(src)
        if cuda:
            comp.wait_stream(copy)
        self.cur = (cur0 + steps) % 2

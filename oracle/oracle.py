"""CPU oracle for the 7x7 depthwise / stencil path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module, and only as the checker (or as the CPU time that is
reported beside the GPU number).  The product path (``pla_b200``) never
imports it.

It drives ``liboracle.so`` (``oracle/pla_oracle.c``), a C restatement of the
reference's algorithm, torch.nn.Conv2d(C, C, 7, stride=1, padding=3,
groups=C) as built by ``data/depthwise_conv_7x7.py:15-17`` and
``data/stencil_7x7.py:8``, evaluated in the fixed tap order documented in the
C file.  The C routine handles a range of planes and rows per call; this
wrapper splits a tensor over host threads (ctypes releases the GIL).

Parity pin: ``tests/test_oracle.py`` checks this oracle against golden
vectors produced by running the reference modules themselves
(``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

_DTYPE_CODE = {torch.float16: 0, torch.float32: 1, torch.float64: 2, torch.bfloat16: 3}
_NCHW, _NHWC = 0, 1

_lib = None


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc only)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "pla_oracle.c"))
    ):
        subprocess.run(["make", "-C", _HERE, "-B", "liboracle.so"], check=True, capture_output=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB_PATH)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        lib.oracle_depthwise7x7.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i64, i64, i32, i32]
        lib.oracle_depthwise7x7.restype = i32
        lib.oracle_depthwise7x7_f64.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32]
        lib.oracle_depthwise7x7_f64.restype = i32
        lib.oracle_depthwise.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i64, i64, i32, i32]
        lib.oracle_depthwise.restype = i32
        lib.oracle_depthwise_f64.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32]
        lib.oracle_depthwise_f64.restype = i32
        lib.oracle_depthwise7x7_layernorm_nhwc.argtypes = [vp, vp, vp, vp, vp, ctypes.c_float, vp, i32, i32, i32,
                                                           i32, i32, i32, i32]
        lib.oracle_depthwise7x7_layernorm_nhwc.restype = i32
        _lib = lib
    return _lib


def default_threads() -> int:
    return max(1, min(os.cpu_count() or 1, 64))


def _layout_of(x: torch.Tensor):
    if x.is_contiguous():
        return x, _NCHW
    if x.dim() == 4 and x.is_contiguous(memory_format=torch.channels_last):
        return x, _NHWC
    return x.contiguous(), _NCHW


def depthwise7x7(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None,
                 threads: int | None = None, rows: tuple[int, int] | None = None) -> torch.Tensor:
    """Oracle depthwise 7x7 (pad 3, stride 1) of a CPU tensor [N, C, H, W].

    ``w`` is [C, 1, 7, 7] (or anything with C*49 elements), ``b`` [C] or None,
    all of x's dtype.  The result keeps x's memory format (NCHW or
    channels_last).  ``rows=(r0, r1)`` computes only output rows [r0, r1) and
    leaves the other rows of the result zero.
    """
    return depthwise(x, w, b, threads, rows, k=7)


def depthwise(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None,
              threads: int | None = None, rows: tuple[int, int] | None = None, k: int | None = None) -> torch.Tensor:
    """Oracle depthwise k x k (k odd <= 7, pad k // 2, stride 1); k defaults to w.shape[-1].

    Same conventions as depthwise7x7; the k = 3 / 5 cases restate the operator
    of benchmark/MetaSchedule/depthwise_conv.py:32-33.
    """
    lib = _load()
    assert x.device.type == "cpu" and x.dim() == 4
    x, layout = _layout_of(x)
    N, C, H, W = x.shape
    K = int(k if k is not None else w.shape[-1])
    assert K in (1, 3, 5, 7) and w.numel() == C * K * K
    w = w.detach().reshape(C, K * K).to(x.dtype).contiguous()
    b = None if b is None else b.detach().reshape(C).to(x.dtype).contiguous()
    y = torch.zeros_like(x)
    if x.numel() == 0:
        return y
    r0, r1 = (0, H) if rows is None else rows
    bp = None if b is None else b.data_ptr()
    if x.dtype == torch.float64:
        assert rows is None
        lib.oracle_depthwise_f64(x.data_ptr(), w.data_ptr(), bp, y.data_ptr(), N, C, H, W, K, layout)
        return y
    code = _DTYPE_CODE[x.dtype]
    planes = N * C
    nthr = threads or default_threads()
    jobs = []
    if planes >= nthr or (r1 - r0) < 2 * nthr:
        step = max(1, -(-planes // (4 * nthr)))
        for p0 in range(0, planes, step):
            jobs.append((p0, min(planes, p0 + step), r0, r1))
    else:
        step = max(1, -(-(r1 - r0) // (4 * nthr)))
        for p in range(planes):
            for a in range(r0, r1, step):
                jobs.append((p, p + 1, a, min(r1, a + step)))

    def run(job):
        return lib.oracle_depthwise(x.data_ptr(), w.data_ptr(), bp, y.data_ptr(), N, C, H, W, K, code, layout,
                                    job[0], job[1], job[2], job[3])

    if nthr == 1 or len(jobs) == 1:
        for j in jobs:
            run(j)
    else:
        with ThreadPoolExecutor(nthr) as ex:
            list(ex.map(run, jobs))
    return y


def stencil7x7(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None,
               threads: int | None = None) -> torch.Tensor:
    """Oracle of data/stencil_7x7.py's Model on [N,1,H,W] or [1,H,W] input (any strides)."""
    squeeze = x.dim() == 3
    x4 = x.unsqueeze(0) if squeeze else x
    y = depthwise7x7(x4.contiguous(), w.reshape(1, 49), None if b is None else b.reshape(1), threads)
    return y.squeeze(0) if squeeze else y


def stencil7x7_rows(x: torch.Tensor, w: torch.Tensor, r0: int, r1: int, b: torch.Tensor | None = None,
                    threads: int | None = None) -> torch.Tensor:
    """Output rows [r0, r1) of one stencil step of the 2-D grid x [H, W] (fp32).

    Only input rows r0-3 .. r1+2 are read, so a band of a huge grid is cheap.
    """
    H, W = x.shape
    a0, a1 = max(0, r0 - 3), min(H, r1 + 3)
    sub = x[a0:a1].contiguous()
    # Rows outside the grid are zero padding; rows cut off at the band edges
    # are real data that the sub-grid must not pad with zeros, so compute the
    # sub-grid and keep only rows whose window lies inside [a0, a1) or at a
    # true grid edge.
    y = depthwise7x7(sub.view(1, 1, a1 - a0, W), w.reshape(1, 49), None if b is None else b.reshape(1),
                     threads, rows=(r0 - a0, r1 - a0))
    return y.view(a1 - a0, W)[r0 - a0:r1 - a0].clone()


def stencil7x7_iterate(x: torch.Tensor, w: torch.Tensor, steps: int, b: torch.Tensor | None = None,
                       threads: int | None = None) -> torch.Tensor:
    """u_{t+1} = stencil(u_t) for `steps` steps on a 2-D grid (zero Dirichlet boundary)."""
    H, W = x.shape
    u = x.contiguous().view(1, 1, H, W)
    for _ in range(steps):
        u = depthwise7x7(u, w.reshape(1, 49), None if b is None else b.reshape(1), threads)
    return u.view(H, W)


def depthwise7x7_layernorm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, gamma: torch.Tensor | None,
                           beta: torch.Tensor | None, eps: float = 1e-6, threads: int | None = None) -> torch.Tensor:
    """Oracle of depthwise 7x7 followed by LayerNorm over channels (NHWC).

    ``x`` is a CPU tensor [N, C, H, W] (any memory format; computed in
    channels_last), ``w`` [C, 1, 7, 7], ``b``/``gamma``/``beta`` [C] or None,
    all of x's dtype (fp32 / bf16 / fp16).  Returns a channels_last tensor.
    The evaluation order is the one documented in pla_oracle.c.
    """
    lib = _load()
    assert x.device.type == "cpu" and x.dim() == 4 and x.dtype != torch.float64
    x = x.contiguous(memory_format=torch.channels_last)
    N, C, H, W = x.shape
    w = w.detach().reshape(C, 49).to(x.dtype).contiguous()
    vecs = [None if t is None else t.detach().reshape(C).to(x.dtype).contiguous() for t in (b, gamma, beta)]
    ptrs = [None if t is None else t.data_ptr() for t in vecs]
    y = torch.zeros_like(x)
    if x.numel() == 0:
        return y
    code = _DTYPE_CODE[x.dtype]
    nthr = min(threads or default_threads(), N)

    def run(job):
        return lib.oracle_depthwise7x7_layernorm_nhwc(x.data_ptr(), w.data_ptr(), ptrs[0], ptrs[1], ptrs[2],
                                                      float(eps), y.data_ptr(), N, C, H, W, code, job[0], job[1])

    step = max(1, -(-N // nthr))
    jobs = [(n0, min(N, n0 + step)) for n0 in range(0, N, step)]
    if len(jobs) == 1:
        rc = run(jobs[0])
        assert rc == 0, rc
    else:
        with ThreadPoolExecutor(nthr) as ex:
            assert all(rc == 0 for rc in ex.map(run, jobs))
    return y

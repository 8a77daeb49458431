"""The C-ABI library loads without a GPU and exports every declared symbol."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pla_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"PLA_API\s+[\w\s\*]+?\b(pla_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("pla_stencil7x7_forward", "pla_depthwise7x7_forward", "pla_stencil7x7_iterate",
                 "pla_stencil7x7_band_step", "pla_status_string"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from pla_b200 import _lib

    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_status_strings_and_version():
    from pla_b200 import _lib

    L = _lib.lib()
    assert L.pla_status_string(0) == b"ok"
    assert b"unsupported" in L.pla_status_string(2)
    assert L.pla_status_string(12345) == b"unknown status"
    assert L.pla_version() >> 16 == 1


def test_argument_validation_needs_no_device():
    # Invalid enums / negative sizes are rejected before any CUDA call.
    from pla_b200 import _lib

    L = _lib.lib()
    assert L.pla_stencil7x7_forward(None, None, None, None, 1, 1, 1, 1, 1, 1, 99, None) == 2
    assert L.pla_depthwise7x7_forward(None, None, None, None, -1, 1, 1, 1, 1, 0, None) == 1
    assert L.pla_depthwise7x7_forward(None, None, None, None, 1, 1, 1, 1, 1, 7, None) == 1
    assert L.pla_stencil7x7_band_step(None, None, None, None, 4, 8, 3, 2, 1, None) == 1
    # empty problems are a no-op success
    assert L.pla_stencil7x7_forward(None, None, None, None, 0, 5, 5, 25, 5, 1, 1, None) == 0


def test_ops_refuse_cpu_tensors():
    from pla_b200 import depthwise, stencil

    with pytest.raises(ValueError):
        stencil.ModelNew()(torch.rand(1, 1, 8, 8))
    with pytest.raises(ValueError):
        depthwise.ModelNew(4, 7, 1, 3)(torch.rand(1, 4, 8, 8))


def test_module_interfaces_match_reference():
    from pla_b200 import depthwise, stencil

    # data/stencil_direct_cuda_v7/test_stencil.py:23
    assert set(stencil.ModelNew().state_dict()) == {"conv1.weight", "conv1.bias"}
    assert stencil.get_init_inputs() == []
    # data/depthwise_conv_7x7.py:15-17, get_init_inputs() -> [C, 7, 1, 3]
    m = depthwise.ModelNew(*depthwise.get_init_inputs())
    assert set(m.state_dict()) == {"conv2d.weight"}
    assert tuple(m.conv2d.weight.shape) == (8, 1, 7, 7)
    mb = depthwise.ModelNew(16, 7, 1, 3, bias=True)
    assert set(mb.state_dict()) == {"conv2d.weight", "conv2d.bias"}
    # 3x3 with padding 1: the MetaSchedule benchmark's filter
    # (benchmark/MetaSchedule/depthwise_conv.py:7-13)
    assert tuple(depthwise.ModelNew(8, 3, 1, 1).conv2d.weight.shape) == (8, 1, 3, 3)
    with pytest.raises(ValueError):
        depthwise.ModelNew(8, 7, 1, 1)  # the reference default padding=1 is not a 7x7 "same" conv
    with pytest.raises(ValueError):
        depthwise.ModelNew(8, 3, 1, 0)
    with pytest.raises(ValueError):
        depthwise.ModelNew(8, 9, 1, 4)


def test_kxk_entry_validates_without_device():
    from pla_b200 import _lib

    L = _lib.lib()
    # filter sizes other than 3, 5, 7 and bad layouts are refused before any device work
    assert L.pla_depthwise_forward(None, None, None, None, 1, 1, 8, 8, 9, 1, 0, None) == 2
    assert L.pla_depthwise_forward(None, None, None, None, 1, 1, 8, 8, 4, 1, 0, None) == 2
    assert L.pla_depthwise_forward(None, None, None, None, 1, 1, 8, 8, 3, 1, 7, None) == 1
    assert L.pla_depthwise_forward(None, None, None, None, 1, 1, 8, 8, 3, 1, 0, None) == 1  # NULL buffers
    assert L.pla_depthwise_forward(None, None, None, None, 0, 1, 8, 8, 3, 1, 0, None) == 0  # empty


def test_halo_and_ipc_argument_validation_needs_no_device():
    from pla_b200 import _lib

    L = _lib.lib()
    taps = (ctypes.c_float * 49)()
    # bad dtype, missing buffers, neighbour without its flag word
    assert L.pla_stencil7x7_band_step_halo(None, taps, None, None, 64, 128, 2, None, 0, None, None, None, None,
                                           None, 0, None) == 2
    assert L.pla_stencil7x7_band_step_halo(None, taps, None, None, 64, 128, 1, None, 0, None, None, None, None,
                                           None, 0, None) == 1
    assert L.pla_ipc_export(None, None, None) == 1
    assert L.pla_ipc_import(None, 0, None) == 1
    assert L.pla_ipc_close(None, 0) == 1
    # the allocation-free iterate rejects grids beyond its static scratch before touching a device
    assert L.pla_stencil7x7_iterate_noalloc(None, None, None, None, 4096, 4096, 1, 1, None) == 3
    assert b"16777216" in L.pla_last_cuda_error()


def test_bench_reads_profiled_traffic():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    t, src = bench.profiled_traffic("stencil7x7_cfg2_4096x4096_f32")
    assert t and t > 60e6 and src.endswith(".md")
    assert bench.profiled_traffic("no-such-workload") == (None, None)


def test_depthwise_layernorm_validates_without_device():
    from pla_b200 import _lib

    L = _lib.lib()
    f = L.pla_depthwise7x7_layernorm_nhwc
    assert f(None, None, None, None, None, 1e-6, None, 1, 32, 7, 7, 2, None) == 2  # fp64
    assert f(None, None, None, None, None, 1e-6, None, -1, 32, 7, 7, 1, None) == 1  # negative size
    assert f(None, None, None, None, None, -1.0, None, 1, 32, 7, 7, 1, None) == 1  # negative eps
    assert f(None, None, None, None, None, float("nan"), None, 1, 32, 7, 7, 1, None) == 1
    assert f(None, None, None, None, None, 1e-6, None, 1, 32, 7, 7, 1, None) == 1  # NULL buffers
    assert f(None, None, None, None, None, 1e-6, None, 0, 32, 7, 7, 1, None) == 0  # empty


def test_depthwise_layernorm_module_interface():
    from pla_b200 import DepthwiseLayerNorm

    m = DepthwiseLayerNorm(96)
    # ConvNeXt block names: dwconv (7x7 depthwise with bias), norm (LayerNorm over C)
    assert set(m.state_dict()) == {"dwconv.weight", "dwconv.bias", "norm.weight", "norm.bias"}
    assert tuple(m.dwconv.weight.shape) == (96, 1, 7, 7) and m.norm.eps == 1e-6
    with pytest.raises(ValueError):
        m(torch.rand(1, 96, 7, 7).contiguous(memory_format=torch.channels_last))


def test_overlap_check_spans():
    """The ops' out/x overlap guard works on memory spans (CPU tensors stand in for the addresses)."""
    import torch

    from pla_b200 import _lib

    base = torch.zeros(4, 8, 16, 16)
    assert _lib.overlaps(base, base)
    assert _lib.overlaps(base[1:3], base[2:4])
    assert not _lib.overlaps(base[0:2], base[2:4])
    assert _lib.overlaps(base.permute(0, 2, 3, 1), base[3])
    assert not _lib.overlaps(base[:, :, :, :8][0], base[1])
    other = torch.zeros(4, 8, 16, 16)
    assert not _lib.overlaps(base, other)
    assert not _lib.overlaps(base[:0], base)


def test_bench_reference_arm_line_on_cpu():
    """`bench.py --impl reference` (the reference's CPU path) prints one JSON
    line with the contract's keys; it needs no GPU."""
    import json
    import subprocess
    import sys

    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                        "--warmup", "1", "--workload", "dw_cfg1"], capture_output=True, text=True, timeout=300,
                       cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] >= 3
    for key in ("metric", "value", "unit", "n_gpus", "ms_per_step", "higher_is_better", "scaling", "dtype",
                "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "depthwise7x7_cfg1_1x96x56x56_f32"


def test_bench_reference_arm_under_torchrun_uses_every_core():
    """Launched as the scaling run launches it (torch.distributed.run, 2 ranks,
    which export OMP_NUM_THREADS=1): rank 0 alone prints the line, timed with
    every host core; the other rank exits 0 without work."""
    import json
    import socket
    import subprocess
    import sys

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"),
                        "--impl", "reference", "--gpus", "2", "--steps", "2", "--warmup", "1", "--workload", "dw_cfg1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2
    assert d["cpu_baseline"]["cores"] == (os.cpu_count() or 1)
    assert f"{os.cpu_count() or 1} threads (OMP_NUM_THREADS={os.cpu_count() or 1})" in d["cpu_baseline"]["sample"]


def _bench_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    return bench


def test_bench_iterate_parity_leg_on_cpu_bands():
    """The iterated-stencil bench line's parity leg: segments cover the band
    edges and the rows inside them, the slab reaches 6 rows past the band, and
    the check passes on a correct band and names the rows of a planted
    mistake (planted in the oracle's own band step, on the CPU)."""
    from oracle import oracle
    from pla_b200.iterate import BandedStencil

    bench = _bench_module()
    H = 96
    for world, rank in ((1, 0), (3, 1), (3, 2)):
        wl = bench.IterateCfg5(rank, world, None, H=H)
        assert (wl.s0, wl.s1) == (max(0, wl.r0 - 6), min(H, wl.r1 + 6))
        segs = wl.parity_segments()
        rows = sorted(r for a, b in segs for r in range(a, b))
        assert rows[:6] == list(range(6)) and rows[-6:] == list(range(wl.rows - 6, wl.rows))
        assert len(rows) == 12 + 4
    # A single CPU band driven by the oracle's band step, as the kernel would.
    wl = bench.IterateCfg5(0, 1, None, H=H)

    def band_step(src, dst, rb, re):
        dst[rb + 3:re + 3] = oracle.stencil7x7_rows(src, wl.w_cpu, rb + 3, re + 3)

    wl.bs = BandedStencil(H, H, wl.w_cpu, device=torch.device("cpu"), step_fn=band_step)
    res = wl.parity()
    assert res["mismatches"] == [] and res["rows_checked"] == 16

    def planted(src, dst, rb, re):
        band_step(src, dst, rb, re)
        dst[3 + 1, 5] += 1.0  # band row 1 is wrong after every step

    wl.bs = BandedStencil(H, H, wl.w_cpu, device=torch.device("cpu"), step_fn=planted)
    res = wl.parity()
    assert len(res["mismatches"]) == 1 and "grid rows [0, 6)" in res["mismatches"][0]


def test_overlapping_buffers_are_rejected_before_any_device_work():
    """Every single-step entry rejects an output that overlaps its input, and
    the iterate entries a partial x / y overlap or a scratch overlapping
    either (the byte spans are compared before anything touches a device)."""
    from pla_b200 import _lib

    L = _lib.lib()
    F32 = _lib.PLA_F32
    base = 1 << 20  # never dereferenced: the checks return first
    w = base + (1 << 19)
    # 1 x 8 x 8 fp32 stencil: y starts 64 bytes into x
    assert L.pla_stencil7x7_forward(base, w, None, base + 64, 1, 8, 8, 64, 8, 1, F32, None) == 1
    # strided x (row stride 16) reaching into y
    assert L.pla_stencil7x7_forward(base, w, None, base + 8 * 16 * 4 - 64, 1, 8, 8, 128, 16, 1, F32, None) == 1
    taps = (ctypes.c_float * 49)()
    assert L.pla_stencil7x7_forward_taps(base, taps, None, base, 1, 8, 8, 64, 8, 1, F32, None) == 1
    assert L.pla_depthwise7x7_forward(base, w, None, base + 4, 2, 4, 8, 8, F32, _lib.PLA_NCHW, None) == 1
    assert L.pla_depthwise_forward(base, w, None, base, 2, 4, 8, 8, 3, F32, _lib.PLA_NHWC, None) == 1
    assert L.pla_depthwise7x7_layernorm_nhwc(base, w, None, None, None, 1e-6, base + 128, 1, 32, 7, 7, F32,
                                             None) == 1
    # iterate: partial x / y overlap, scratch overlapping x or y
    assert L.pla_stencil7x7_iterate(base, w, None, base + 16, base + (1 << 16), 8, 8, 2, F32, None) == 1
    assert L.pla_stencil7x7_iterate(base, w, None, base, base + 32, 8, 8, 2, F32, None) == 1
    assert L.pla_stencil7x7_iterate_noalloc(base, w, None, base + 16, 8, 8, 2, F32, None) == 1
    # band steps: in / out band buffers of (rows + 6) x width
    assert L.pla_stencil7x7_band_step(base, w, None, base + 256, 64, 32, 0, 64, F32, None) == 1
    flags = (ctypes.c_uint * 2)()
    assert L.pla_stencil7x7_band_step_halo(base, taps, None, base + 256, 64, 32, F32, None, 0, None, flags, None,
                                           None, flags, 0, None) == 1


def test_many_rejects_bad_batches_before_any_device_work():
    """pla_depthwise7x7_forward_many checks every problem, and that no output
    overlaps any problem's input or output, before it touches a device."""
    from pla_b200 import _lib

    L = _lib.lib()
    F32 = _lib.PLA_F32
    P = _lib.DwProblem
    base = 1 << 20
    arr = (P * 2)(P(base, base + (1 << 19), None, base + (1 << 18), 1, 4, 8, 8),
                  P(base + (1 << 17), base + (1 << 19), None, base + (1 << 18) + 64, 1, 4, 8, 8))
    assert L.pla_depthwise7x7_forward_many(arr, 2, F32, _lib.PLA_NCHW, None) == 1   # the two outputs overlap
    arr[1].y = base + (1 << 17) + 16                                               # output 1 inside input 1
    assert L.pla_depthwise7x7_forward_many(arr, 2, F32, _lib.PLA_NCHW, None) == 1
    arr[1].y = base + 32                                                            # output 1 inside input 0
    assert L.pla_depthwise7x7_forward_many(arr, 2, F32, _lib.PLA_NCHW, None) == 1
    arr[1].n = -1
    assert L.pla_depthwise7x7_forward_many(arr, 2, F32, _lib.PLA_NCHW, None) == 1
    assert L.pla_depthwise7x7_forward_many(arr, -1, F32, _lib.PLA_NCHW, None) == 1
    assert L.pla_depthwise7x7_forward_many(None, 2, F32, _lib.PLA_NCHW, None) == 1
    assert L.pla_depthwise7x7_forward_many(arr, 2, 9, _lib.PLA_NCHW, None) == 2
    assert L.pla_depthwise7x7_forward_many(arr, 2, F32, 7, None) == 1
    assert L.pla_depthwise7x7_forward_many(None, 0, F32, _lib.PLA_NCHW, None) == 0

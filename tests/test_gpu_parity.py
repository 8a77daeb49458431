"""GPU parity: the sm_100a kernels (through the C ABI) against the CPU oracle
and against the reference modules' golden vectors.

The CUDA kernels and the oracle evaluate each output point in the same fixed
order (row-major taps, fp32 fma, then + bias, one rounding), so they must agree
bit for bit (``torch.equal``); the golden vectors (reference torch.nn.Conv2d on
the CPU, a different summation order) are matched within the north star's
tolerances: rtol = atol = 1e-5 for fp32, 2e-2 for bf16 (and the reference
tests' 2e-3 for fp16, 1e-10 for fp64,
data/stencil_direct_cuda_v7/test_stencil.py:39-40).
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle
from tests.golden_util import TOL, load_cases

pytestmark = pytest.mark.gpu

CASES = load_cases()
DEV = "cuda:0"


def _gpu_copy(t: torch.Tensor) -> torch.Tensor:
    """Copy a CPU tensor to the GPU keeping its strides (sliced/transposed layouts survive)."""
    g = torch.empty_strided(t.shape, t.stride(), dtype=t.dtype, device=DEV)
    g.copy_(t)
    return g


def _assert_equal(gpu: torch.Tensor, ref: torch.Tensor):
    got = gpu.cpu()
    assert got.shape == ref.shape
    if not torch.equal(got, ref):
        diff = (got.double() - ref.double()).abs()
        raise AssertionError(f"not bit-identical: {int((diff > 0).sum())} of {diff.numel()} differ, "
                             f"max |diff| {diff.max().item():.3e}")


# --------------------------------------------------------------------------
# golden vectors (reference modules) -> GPU, and GPU == oracle bit for bit
# --------------------------------------------------------------------------
@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_golden_cases(case):
    from pla_b200 import depthwise7x7, stencil7x7, stencil7x7_iterate

    x = _gpu_copy(case.x)
    w = case.w.to(DEV)
    b = None if case.b is None else case.b.to(DEV)
    if case.op == "stencil":
        y = stencil7x7(x, w.reshape(1, 1, 7, 7), b)
        ref = oracle.stencil7x7(case.x, case.w, case.b)
    elif case.op == "depthwise":
        C = case.shape[1]
        y = depthwise7x7(x, w.reshape(C, 1, 7, 7), b)
        ref = oracle.depthwise7x7(case.x, case.w.reshape(C, 1, 7, 7), case.b)
        if case.layout == "nhwc":
            assert y.is_contiguous(memory_format=torch.channels_last)
    elif case.op == "depthwise_ms":
        from pla_b200 import depthwise_kxk

        C, k = case.shape[1], case.k
        y = depthwise_kxk(x, w.reshape(C, 1, k, k), b)
        ref = oracle.depthwise(case.x, case.w.reshape(C, 1, k, k), case.b)
    else:
        y = stencil7x7_iterate(x.contiguous(), w, case.steps, b)
        ref = oracle.stencil7x7_iterate(case.x, case.w, case.steps, case.b)
    torch.cuda.synchronize()
    _assert_equal(y, ref)
    if case.op == "iterate":
        scale = case.y.abs().max().item()
        torch.testing.assert_close(y.cpu() / scale, case.y / scale, rtol=1e-5, atol=1e-5)
    else:
        torch.testing.assert_close(y.cpu().float(), case.y.float(), rtol=case.tol, atol=case.tol)


# --------------------------------------------------------------------------
# the reference's own stencil test matrix
# (data/stencil_direct_cuda_v7/test_stencil.py:27-58)
# --------------------------------------------------------------------------
def _v7_cases():
    g = torch.Generator().manual_seed(42)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    return [r(2, 1, 1, 1), r(1, 7, 9), r(2, 1, 17, 257), r(1, 1, 48, 769), r(1, 1, 48, 1536),
            r(1, 1, 35, 10240), r(2, 1, 17, 516), r(1, 1, 2, 4), r(2, 1, 35, 518)[:, :, ::2, ::2],
            r(2, 1, 259, 19).transpose(-1, -2), r(4, 1, 9, 13)[::2], torch.empty(0, 1, 9, 13)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32, torch.float64])
@pytest.mark.parametrize("use_bias", [True, False])
def test_reference_v7_matrix(dtype, use_bias):
    from pla_b200.stencil import ModelNew

    tol = {torch.float16: 2e-3, torch.bfloat16: 2e-2, torch.float32: 2e-5, torch.float64: 1e-10}[dtype]
    torch.manual_seed(0)
    model = ModelNew().to(DEV).to(dtype)
    if not use_bias:
        model.conv1.bias = None
    acc = torch.float64 if dtype == torch.float64 else torch.float32
    for cpu_x in _v7_cases():
        cpu_x = cpu_x.to(dtype)
        x = _gpu_copy(cpu_x)
        with torch.no_grad():
            y = model(x)
            bias = model.conv1.bias
            expected = F.conv2d(cpu_x.to(acc), model.conv1.weight.cpu().to(acc),
                                None if bias is None else bias.cpu().to(acc), padding=3).to(dtype)
        assert y.shape == x.shape and y.is_contiguous()
        torch.testing.assert_close(y.cpu(), expected, atol=tol, rtol=tol)
        if dtype != torch.float64 and cpu_x.numel():
            ref = oracle.stencil7x7(cpu_x, model.conv1.weight.detach().cpu(),
                                    None if bias is None else bias.detach().cpu())
            _assert_equal(y, ref)


def test_updated_weights_side_stream_and_empty():
    # data/stencil_cuda_v2/test_stencil.py:85-96
    from pla_b200.stencil import ModelNew

    for dtype in (torch.float16, torch.float32):
        model = ModelNew().to(DEV).to(dtype)
        with torch.no_grad():
            model.conv1.weight.zero_()
            model.conv1.bias.fill_(0.25)
            x = torch.randn(1, 1, 7, 11, device=DEV, dtype=dtype)
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                y = model(x)
            torch.cuda.current_stream().wait_stream(stream)
            torch.testing.assert_close(y, torch.full_like(y, 0.25), atol=0, rtol=0)
            for shape in [(0, 1, 3, 4), (1, 1, 0, 4), (1, 1, 3, 0)]:
                assert model(torch.empty(shape, device=DEV, dtype=dtype)).shape == shape


# --------------------------------------------------------------------------
# benchmark configurations at full size, bit-exact against the oracle
# --------------------------------------------------------------------------
def _dw_inputs(seed, shape, dtype, bias=True):
    g = torch.Generator().manual_seed(seed)
    N, C, H, W = shape
    x = torch.randn(shape, generator=g).to(dtype)
    w = (torch.randn(C, 1, 7, 7, generator=g) / 7).to(dtype)
    b = (torch.randn(C, generator=g) * 0.1).to(dtype) if bias else None
    return x, w, b


@pytest.mark.parametrize("name,shape,dtype,layout,bias,seed", [
    ("cfg1", (1, 96, 56, 56), torch.float32, "nchw", True, 0),
    ("cfg3_nchw", (128, 384, 14, 14), torch.bfloat16, "nchw", True, 2),
    ("cfg3_nhwc", (128, 384, 14, 14), torch.bfloat16, "nhwc", True, 2),
    ("cfg4_s1", (256, 96, 56, 56), torch.bfloat16, "nchw", False, 3),
    ("cfg4_s2", (256, 192, 28, 28), torch.bfloat16, "nchw", False, 3),
    ("cfg4_s3", (256, 384, 14, 14), torch.bfloat16, "nchw", False, 3),
    ("cfg4_s4", (256, 768, 7, 7), torch.bfloat16, "nchw", False, 3),
    ("cfg4_s1_nhwc", (64, 96, 56, 56), torch.bfloat16, "nhwc", False, 3),
    ("dw_2048_f32", (1, 8, 2048, 2048), torch.float32, "nchw", False, 5),
])
def test_depthwise_configs_full_size(name, shape, dtype, layout, bias, seed):
    from pla_b200.depthwise import ModelNew

    x, w, b = _dw_inputs(seed, shape, dtype, bias)
    if layout == "nhwc":
        x = x.contiguous(memory_format=torch.channels_last)
    m = ModelNew(shape[1], 7, 1, 3, bias=bias).to(DEV).to(dtype)
    with torch.no_grad():
        m.conv2d.weight.copy_(w)
        if bias:
            m.conv2d.bias.copy_(b)
        y = m(x.to(DEV))
    ref = oracle.depthwise7x7(x, w, b)
    _assert_equal(y, ref)
    tol = TOL["bf16" if dtype == torch.bfloat16 else "f32"]
    # and the reference module's arithmetic (fp32 conv, one cast) within tolerance
    if shape[0] * shape[1] <= 128 * 384:
        acc = F.conv2d(x.float(), w.float(), None if b is None else b.float(), padding=3, groups=shape[1])
        torch.testing.assert_close(y.cpu().float(), acc.to(dtype).float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("shape,layout,dtype", [
    ((3, 13, 14, 14), "nchw", torch.bfloat16),   # planes not a multiple of 32: tail stage
    ((2, 40, 14, 14), "nhwc", torch.bfloat16),   # channels not a multiple of 32: clipped TMA box
    ((5, 24, 7, 7), "nhwc", torch.float32),      # 7x7 NHWC, 128-channel stages
    ((3, 50, 7, 7), "nchw", torch.float16),      # 7x7 NCHW, partial 128-plane stage
    ((2, 64, 28, 28), "nhwc", torch.bfloat16),
    ((2, 33, 28, 28), "nchw", torch.bfloat16),
    ((1, 16, 28, 28), "nchw", torch.float32),    # fp32 28x28 falls back to the channel-minor kernel
    ((2, 33, 14, 14), "nhwc", torch.bfloat16),   # C*2 bytes not a multiple of 16: channel-minor kernel
    ((2, 8, 12, 12), "nchw", torch.bfloat16),    # non-stack size
])
def test_depthwise_stack_shapes(shape, layout, dtype):
    from pla_b200 import depthwise7x7

    x, w, b = _dw_inputs(11, shape, dtype, True)
    if layout == "nhwc":
        x = x.contiguous(memory_format=torch.channels_last)
    y = depthwise7x7(x.to(DEV), w.to(DEV), b.to(DEV))
    _assert_equal(y, oracle.depthwise7x7(x, w, b))


def test_stencil_host_taps_equals_device_taps():
    from pla_b200 import _lib, stencil7x7

    g = torch.Generator().manual_seed(9)
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        x = (torch.rand(2, 1, 77, 264, generator=g) * 2 - 1).to(dtype)
        w = ((torch.rand(1, 1, 7, 7, generator=g) * 2 - 1) / 49).to(dtype)
        b = ((torch.rand(1, generator=g) * 2 - 1) / 49).to(dtype)
        xd, wd, bd = x.to(DEV), w.to(DEV), b.to(DEV)
        y_dev = stencil7x7(xd, wd, bd)
        y_host = stencil7x7(xd, wd, bd, host_taps=_lib.HostTaps().update(wd, bd))
        assert torch.equal(y_dev, y_host)
        _assert_equal(y_host, oracle.stencil7x7(x, w, b))


def test_stencil_cfg2_full_size():
    from pla_b200.stencil import ModelNew

    g = torch.Generator().manual_seed(1)
    x = torch.rand(1, 1, 4096, 4096, generator=g) * 2 - 1
    w = (torch.rand(1, 1, 7, 7, generator=g) * 2 - 1) / 49
    b = (torch.rand(1, generator=g) * 2 - 1) / 49
    m = ModelNew().to(DEV)
    with torch.no_grad():
        m.conv1.weight.copy_(w)
        m.conv1.bias.copy_(b)
        y = m(x.to(DEV))
    _assert_equal(y, oracle.stencil7x7(x, w, b))
    ref = F.conv2d(x, w, b, padding=3)
    torch.testing.assert_close(y.cpu(), ref, rtol=1e-5, atol=1e-5)


def test_host_taps_tile_claiming_ragged_planes():
    """Large single fp32 planes with host taps: tens of thousands of 32 x 128
    tiles, so the tile kernel claims the tiles of CTAs not yet started
    (launch control).  The shapes end in a partial tile column (W % 128 != 0)
    and a partial tile row, carry a bias, and include band steps over
    sub-ranges of a band buffer with its 3 halo rows, which must stay
    untouched."""
    from pla_b200 import _lib, stencil7x7

    g = torch.Generator().manual_seed(31)
    H, W = 4001, 40004
    x = torch.rand(1, 1, H, W, generator=g) * 2 - 1
    w = (torch.rand(1, 1, 7, 7, generator=g) * 2 - 1) / 49
    b = (torch.rand(1, generator=g) * 2 - 1) / 49
    xd, wd, bd = x.to(DEV), w.to(DEV), b.to(DEV)
    y = stencil7x7(xd, wd, bd, host_taps=_lib.HostTaps().update(wd, bd))
    _assert_equal(y, oracle.stencil7x7(x, w, b))

    rows, W2 = 8000, 20000
    grid = torch.rand(rows + 6, W2, generator=g) * 2 - 1
    src = grid.to(DEV)
    taps, hb = _lib.HostTaps().update(wd, None).args()
    L = _lib.lib()
    for r_a, r_b in [(0, rows), (3, rows - 3), (1000, 1005 + 218 * 30)]:
        dst = torch.full((rows + 6, W2), 7.0, device=DEV)
        st = L.pla_stencil7x7_band_step_taps(src.data_ptr(), taps, hb, dst.data_ptr(), rows, W2, r_a, r_b, 1,
                                             torch.cuda.current_stream().cuda_stream)
        assert st == 0
        out = dst.cpu()
        # band row r reads buffer rows r .. r + 6 (band rows r - 3 .. r + 3)
        ref = oracle.stencil7x7_rows(grid, w.view(7, 7), r_a + 3, r_b + 3)
        _assert_equal(out[3 + r_a:3 + r_b], ref)
        assert torch.all(out[:3 + r_a] == 7.0) and torch.all(out[3 + r_b:] == 7.0)


# --------------------------------------------------------------------------
# iterated stencil
# --------------------------------------------------------------------------
def _cfg5_inputs(H, W, seed=4):
    g = torch.Generator().manual_seed(seed)
    x = torch.rand(H, W, generator=g) * 2 - 1
    w = torch.rand(7, 7, generator=g) * 2 - 1
    return x, w / w.sum()


@pytest.mark.parametrize("H,W,steps", [(512, 512, 100), (300, 260, 7), (64, 64, 0), (33, 128, 1)])
def test_iterate_matches_oracle_bitwise(H, W, steps):
    from pla_b200 import stencil7x7_iterate

    x, w = _cfg5_inputs(H, W)
    y = stencil7x7_iterate(x.to(DEV), w.to(DEV), steps)
    _assert_equal(y, oracle.stencil7x7_iterate(x, w, steps))


def test_iterate_in_place_and_odd_steps():
    from pla_b200 import stencil7x7_iterate

    x, w = _cfg5_inputs(128, 96)
    ref = oracle.stencil7x7_iterate(x, w, 5)
    xd = x.to(DEV)
    y = stencil7x7_iterate(xd, w.to(DEV), 5, out=xd)
    assert y.data_ptr() == xd.data_ptr()
    _assert_equal(y, ref)


def test_band_step_equals_full_step():
    from pla_b200 import _lib

    x, w = _cfg5_inputs(200, 256)
    full = oracle.stencil7x7(x.view(1, 1, 200, 256), w).view(200, 256)
    r0, r1 = 57, 131
    rows = r1 - r0
    band_in = torch.zeros(rows + 6, 256)
    band_in[:] = x[r0 - 3:r1 + 3]
    src = band_in.to(DEV)
    dst = torch.full((rows + 6, 256), 7.0, device=DEV)
    wd = w.to(DEV).contiguous()
    L = _lib.lib()
    for a, b in [(0, 3), (rows - 3, rows), (3, rows - 3)]:
        st = L.pla_stencil7x7_band_step(src.data_ptr(), wd.data_ptr(), None, dst.data_ptr(), rows, 256, a, b,
                                        1, torch.cuda.current_stream().cuda_stream)
        assert st == 0
    out = dst.cpu()
    _assert_equal(out[3:3 + rows], full[r0:r1])
    assert torch.all(out[:3] == 7.0) and torch.all(out[rows + 3:] == 7.0)  # halos untouched


def test_cfg5_full_size_first_steps():
    """32768^2 grid: two GPU steps against the oracle on three row bands."""
    from pla_b200 import stencil7x7_iterate

    H = W = 32768
    x, w = _cfg5_inputs(H, W)
    xd = x.to(DEV)
    y1 = stencil7x7_iterate(xd, w.to(DEV), 1)
    y2 = stencil7x7_iterate(xd, w.to(DEV), 2)
    for r0, r1 in [(0, 16), (16380, 16420), (H - 16, H)]:
        ref1 = oracle.stencil7x7_rows(x, w, r0, r1)
        _assert_equal(y1[r0:r1], ref1)
        # step 2 on the band needs step-1 rows r0-3 .. r1+2, taken from the GPU
        a0, a1 = max(0, r0 - 3), min(H, r1 + 3)
        u1 = y1[a0:a1].cpu()
        ref2 = oracle.stencil7x7_rows(u1, w, r0 - a0, r1 - a0) if (a0 == 0 or a1 == H) else None
        if ref2 is None:
            sub = oracle.stencil7x7(u1.view(1, 1, a1 - a0, W), w).view(a1 - a0, W)
            ref2 = sub[3:3 + (r1 - r0)]
        _assert_equal(y2[r0:r1], ref2)
    del xd, y1, y2
    torch.cuda.empty_cache()


def test_no_device_faults_recorded():
    import ctypes

    from pla_b200 import _lib

    torch.cuda.synchronize()
    v = ctypes.c_uint(123)
    assert _lib.lib().pla_read_device_faults(ctypes.byref(v)) == 0
    assert v.value == 0


def test_modules_replay_in_cuda_graph():
    """After a warm-up call the launches are capturable: replaying a CUDA graph
    of the modules on new inputs gives the oracle's results."""
    from pla_b200.depthwise import ModelNew as DW
    from pla_b200.stencil import ModelNew as ST

    g = torch.Generator().manual_seed(21)
    st_m = ST().to(DEV)
    dw_m = DW(64, 7, 1, 3, bias=True).to(DEV).bfloat16()
    xs = torch.rand(1, 1, 128, 256, device=DEV)
    xd = torch.rand(4, 64, 14, 14, device=DEV).bfloat16()
    out_s = torch.empty_like(xs)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up: filter caches, kernel attributes
        st_m(xs, out=out_s)
        dw_m(xd)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.no_grad(), torch.cuda.graph(graph):
        st_m(xs, out=out_s)
        out_d = dw_m(xd)
    new_s = torch.rand(1, 1, 128, 256, generator=g)
    new_d = torch.rand(4, 64, 14, 14, generator=g).bfloat16()
    xs.copy_(new_s)
    xd.copy_(new_d)
    graph.replay()
    torch.cuda.synchronize()
    w, b = st_m.conv1.weight.detach().cpu(), st_m.conv1.bias.detach().cpu()
    _assert_equal(out_s, oracle.stencil7x7(new_s, w, b))
    _assert_equal(out_d, oracle.depthwise7x7(new_d, dw_m.conv2d.weight.detach().cpu(),
                                              dw_m.conv2d.bias.detach().cpu()))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape,layout", [((2, 64, 14, 14), "nchw"), ((2, 64, 14, 14), "nhwc"),
                                          ((1, 4, 56, 56), "nchw"), ((1, 2, 40, 256), "nchw")])
def test_misaligned_inputs_take_the_fallbacks(dtype, shape, layout):
    """Inputs whose storage starts one element past a 16-byte boundary cannot be
    read by TMA / bulk copies; the dispatcher must route them elsewhere."""
    from pla_b200 import depthwise7x7, stencil7x7

    x, w, b = _dw_inputs(13, shape, dtype, True)
    if layout == "nhwc":
        x = x.contiguous(memory_format=torch.channels_last)
    flat = torch.empty(x.numel() + 1, dtype=dtype, device=DEV)
    if layout == "nhwc":
        N, C, H, W = shape
        xd = flat[1:].view(N, H, W, C).permute(0, 3, 1, 2)
        xd.copy_(x.to(DEV))
        assert xd.is_contiguous(memory_format=torch.channels_last)
    else:
        xd = flat[1:].view(shape)
        xd.copy_(x.to(DEV))
    assert xd.data_ptr() % 16 != 0
    y = depthwise7x7(xd, w.to(DEV), b.to(DEV))
    _assert_equal(y, oracle.depthwise7x7(x, w, b))
    if shape[1] == 2:  # also as a stencil batch (2 planes of one channel each)
        xs = xd[:, :1]
        ys = stencil7x7(xs, w[0:1].to(DEV), b[0:1].to(DEV))
        _assert_equal(ys, oracle.stencil7x7(x[:, :1].contiguous(), w[0:1], b[0:1]))


def _with_specials(x: torch.Tensor, seed: int) -> torch.Tensor:
    """x with a sprinkling of +-inf, NaN, -0 and subnormals of its own dtype."""
    g = torch.Generator().manual_seed(seed)
    flat = x.clone().reshape(-1)
    n = flat.numel()
    tiny = torch.finfo(x.dtype).tiny
    picks = torch.randint(0, n, (5, max(1, n // 500)), generator=g)
    flat[picks[0]] = float("inf")
    flat[picks[1]] = float("-inf")
    flat[picks[2]] = float("nan")
    flat[picks[3]] = -0.0
    flat[picks[4]] = tiny / 4  # subnormal
    return flat.reshape(x.shape)


def _assert_equal_nan(gpu: torch.Tensor, ref: torch.Tensor):
    got = gpu.cpu()
    assert torch.equal(torch.isnan(got), torch.isnan(ref)), "NaN positions differ"
    keep = ~torch.isnan(ref)
    _assert_equal(got[keep], ref[keep])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape,layout", [((4, 64, 14, 14), "nchw"), ((4, 64, 14, 14), "nhwc"),
                                          ((2, 64, 7, 7), "nchw"), ((2, 64, 28, 28), "nchw"),
                                          ((1, 4, 56, 56), "nchw"), ((1, 2, 100, 300), "nchw")])
def test_16bit_paths_with_special_values(dtype, shape, layout):
    """The 16-bit kernels feed packed x and w into mixed-precision FMAs; infinities,
    NaNs, signed zeros and subnormals must come out where the widened fp32 math
    of the oracle puts them."""
    from pla_b200 import depthwise7x7

    x, w, b = _dw_inputs(21, shape, dtype, True)
    x = _with_specials(x, 22)
    fmt = torch.channels_last if layout == "nhwc" else torch.contiguous_format
    x = x.contiguous(memory_format=fmt)
    y = depthwise7x7(x.to(DEV), w.to(DEV), b.to(DEV))
    _assert_equal_nan(y, oracle.depthwise7x7(x, w, b))


# --------------------------------------------------------------------------
# 3x3 / 5x5 depthwise (the MetaSchedule benchmark's operator,
# benchmark/MetaSchedule/depthwise_conv.py:32-33): every dispatch route
# (TMA tile kernel for dense NCHW planes, the one-thread-per-output kernel
# for the rest) bit-identical to the oracle
# --------------------------------------------------------------------------
@pytest.mark.parametrize("k", [3, 5])
@pytest.mark.parametrize("shape,dtype,layout,bias", [
    ((1, 32, 128, 128), torch.float32, "nchw", False),     # the benchmark's default shape (wide tiles)
    ((2, 8, 200, 260), torch.float16, "nchw", False),      # wide tiles, ragged edges
    ((4, 80, 56, 56), torch.bfloat16, "nchw", True),       # narrow 56 x 64 tiles (320 planes)
    ((1, 4, 40, 40), torch.float32, "nchw", True),         # short tiles (few planes)
    ((2, 16, 14, 14), torch.bfloat16, "nchw", True),       # small planes: generic kernel
    ((2, 24, 17, 9), torch.float32, "nhwc", True),         # NHWC: generic kernel
    ((1, 3, 12, 70), torch.float64, "nchw", True),         # fp64
])
def test_depthwise_kxk_matches_oracle(k, shape, dtype, layout, bias):
    from pla_b200 import depthwise_kxk

    g = torch.Generator().manual_seed(100 + k)
    N, C, H, W = shape
    x = (torch.rand(shape, generator=g) * 2 - 1).to(dtype)
    w = (torch.rand(C, 1, k, k, generator=g) * 2 - 1).to(dtype)
    b = (torch.rand(C, generator=g) * 0.2 - 0.1).to(dtype) if bias else None
    if layout == "nhwc":
        x = x.contiguous(memory_format=torch.channels_last)
    y = depthwise_kxk(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV))
    if layout == "nhwc":
        assert y.is_contiguous(memory_format=torch.channels_last)
    ref = oracle.depthwise(x, w, b)
    _assert_equal(y, ref)
    # and the semantics of torch's grouped conv within the benchmark's tolerance
    tol = 1e-4 if dtype in (torch.float32, torch.float64) else 1e-2
    want = torch.nn.functional.conv2d(x.double(), w.double(), None if b is None else b.double(),
                                      padding=k // 2, groups=C)
    torch.testing.assert_close(y.cpu().double(), want, rtol=tol, atol=tol)


def test_depthwise_kxk_module_and_7x7_route():
    """ModelNew(C, 3, 1, 1) runs the 3x3 path; k = 7 through the k x k entry is the 7x7 path."""
    from pla_b200 import depthwise_kxk
    from pla_b200.depthwise import ModelNew

    m = ModelNew(16, 3, 1, 1).to(DEV)
    x = torch.randn(2, 16, 64, 64, device=DEV)
    with torch.no_grad():
        y = m(x)
    _assert_equal(y, oracle.depthwise(x.cpu(), m.conv2d.weight.detach().cpu(), None))
    w7 = torch.randn(16, 1, 7, 7)
    _assert_equal(depthwise_kxk(x, w7.to(DEV)), oracle.depthwise7x7(x.cpu(), w7))


@pytest.mark.parametrize("k,dtype", [(7, torch.float32), (3, torch.float32), (7, torch.bfloat16)])
def test_tile_claiming_path(k, dtype):
    """8 planes of 2048^2 make 8192 tiles of 32 x 128, more than 8 per resident
    CTA: the tile kernel launches one CTA per tile and the running CTAs claim
    the rest (cluster launch control).  Every tile must be computed exactly once."""
    from pla_b200 import depthwise_kxk

    g = torch.Generator().manual_seed(300 + k)
    x = torch.randn(1, 8, 2048, 2048, generator=g).to(dtype)
    w = (torch.randn(8, 1, k, k, generator=g) / k).to(dtype)
    b = (torch.randn(8, generator=g) * 0.1).to(dtype)
    y = torch.full_like(x, float("nan"), device=DEV)  # a tile left out stays NaN
    depthwise_kxk(x.to(DEV), w.to(DEV), b.to(DEV), out=y)
    assert not torch.isnan(y).any()
    _assert_equal(y, oracle.depthwise(x, w, b))
    assert _lib_faults() == 0


def _lib_faults() -> int:
    import ctypes

    from pla_b200 import _lib

    v = ctypes.c_uint(0)
    _lib.check(_lib.lib().pla_read_device_faults(ctypes.byref(v)), "pla_read_device_faults")
    return v.value


@pytest.mark.parametrize("shape,dtype,bias", [
    ((2, 96, 56, 56), torch.bfloat16, False),   # ConvNeXt stage-1 planes in channels_last
    ((1, 40, 33, 45), torch.float32, True),     # ragged tiles, last channel group partial
    ((2, 64, 20, 9), torch.float16, True),
    ((3, 8, 3, 5), torch.bfloat16, True),       # planes smaller than one tile
    ((1, 32, 100, 30), torch.float32, False),
])
def test_nhwc_spatial_tiles_match_oracle(shape, dtype, bias):
    """channels_last planes outside the plane-stack sizes run 14 x 14 spatial
    tiles of 32 channels (TMA zero fill at the image edge, clipped TMA stores)."""
    from pla_b200 import depthwise7x7

    x, w, b = _dw_inputs(400 + shape[1], shape, dtype, bias)
    x = x.contiguous(memory_format=torch.channels_last)
    y = depthwise7x7(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV))
    assert y.is_contiguous(memory_format=torch.channels_last)
    _assert_equal(y, oracle.depthwise7x7(x, w, b))


@pytest.mark.parametrize("shape,dtype,bias", [
    ((16, 96, 56, 56), torch.bfloat16, True),   # C even: stages walk channel pairs
    ((13, 97, 56, 56), torch.bfloat16, True),   # C odd, odd plane count: last stage half past the end
    ((12, 100, 56, 56), torch.float16, False),
    ((3, 5, 56, 56), torch.bfloat16, True),     # too few planes: the plane-tile kernel instead
])
def test_plane_pair_path_matches_oracle(shape, dtype, bias):
    """Large NCHW stacks of 56 x 56 16-bit planes run two planes per stage
    (224 threads, no column past the plane edge); output == oracle bit for bit,
    no device fault recorded."""
    from pla_b200 import depthwise7x7

    x, w, b = _dw_inputs(500 + shape[1], shape, dtype, bias)
    y = depthwise7x7(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV))
    _assert_equal(y, oracle.depthwise7x7(x, w, b))
    assert _lib_faults() == 0


def test_outputs_overlapping_the_input_are_rejected():
    """Single-step ops read input halos that other CTAs may already have
    overwritten, so an output overlapping the input is refused before launch."""
    from pla_b200 import depthwise7x7, stencil7x7

    x = torch.randn(2, 64, 14, 14, device=DEV)
    w = torch.randn(64, 1, 7, 7, device=DEV)
    with pytest.raises(RuntimeError, match="overlap"):
        depthwise7x7(x, w, None, out=x)
    g = torch.rand(1, 1, 64, 128, device=DEV)
    with pytest.raises(RuntimeError, match="overlap"):
        stencil7x7(g, torch.rand(1, 1, 7, 7, device=DEV), None, out=g)

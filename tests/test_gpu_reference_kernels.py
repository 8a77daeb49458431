"""Head-to-head with the reference's own stencil CUDA kernels on the B200.

oracle/Makefile (`make -C oracle ref REF=<PLA checkout>`, run by
__graft_entry__.build() when the reference tree is next to this repository)
compiles, unmodified and for sm_100a, the kernels behind
``launch_direct`` (data/stencil_direct_cuda_v7/stencil_cuda_kernel.cu:230-244)
and ``launch_stencil`` (data/stencil_cuda_v2/stencil_cuda_kernel.cu:195-209)
into oracle/_ref/.  These tests check this library against them on the
reference harness shape (data/stencil_7x7.py:17-20, 1x1x10240x10240) and on
cfg2's 4096^2, and print both kernels' times (``pytest -s`` shows them).

v7 accumulates in fp32 in (row, column) tap order and adds the bias before
the cast (stencil_cuda_kernel.cu:64-71) — the same arithmetic as this
library — so it must agree bit for bit; v2 uses mma.sync tiles (another
summation order) and rounds to fp16 before adding the bias
(stencil_cuda_kernel.cu:103-106), so it is compared within fp16 tolerance.
"""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")
V7 = os.path.join(REF, "libref_stencil_v7.so")
V2 = os.path.join(REF, "libref_stencil_v2.so")
_vp, _i, _i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64


def _v7():
    lib = ctypes.CDLL(V7)
    f = lib["_Z13launch_directPKvS0_S0_PviiillliP11CUstream_st"]
    f.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i64, _i64, _i64, _i, _vp]
    f.restype = None
    return f


def _v2():
    lib = ctypes.CDLL(V2)
    f = lib["_Z14launch_stencilPKvS0_S0_PviiibP11CUstream_st"]
    f.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, ctypes.c_bool, _vp]
    f.restype = None
    return f


def _record(**kv):
    """Append one timing record (JSON line) to $PLA_HEAD_TO_HEAD_LOG when set."""
    path = os.environ.get("PLA_HEAD_TO_HEAD_LOG")
    if path:
        import json

        with open(path, "a") as f:
            f.write(json.dumps(kv) + "\n")


def _time(fn, iters=20, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _inputs(H, W, dtype):
    g = torch.Generator().manual_seed(1)
    x = (torch.rand(1, 1, H, W, generator=g) * 2 - 1).to(dtype).cuda()
    w = ((torch.rand(1, 1, 7, 7, generator=g) * 2 - 1) / 49).to(dtype).cuda()
    b = ((torch.rand(1, generator=g) * 2 - 1) / 49).to(dtype).cuda()
    return x, w, b


@pytest.mark.skipif(not os.path.exists(V7), reason="reference kernels not built (oracle/_ref)")
@pytest.mark.parametrize("H,W", [(10240, 10240), (4096, 4096)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_against_reference_v7(H, W, dtype):
    from pla_b200.stencil import ModelNew

    x, w, b = _inputs(H, W, dtype)
    code = {torch.float16: 0, torch.float32: 1}[dtype]
    launch = _v7()
    y_ref = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream

    def ref():
        launch(x.data_ptr(), w.data_ptr(), b.data_ptr(), y_ref.data_ptr(), 1, H, W, H * W, W, 1, code, stream)

    m = ModelNew().cuda().to(dtype)
    with torch.no_grad():
        m.conv1.weight.copy_(w)
        m.conv1.bias.copy_(b)
    y = torch.empty_like(x)

    def ours():
        m(x, out=y)

    ref()
    ours()
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    t_ref, t_ours = _time(ref), _time(ours)
    pts = H * W
    print(f"\n[v7 {str(dtype)[6:]} {H}x{W}] reference launch_direct {t_ref * 1e3:.1f} us "
          f"({pts / t_ref / 1e6:.0f} GPt/s), pla_b200 {t_ours * 1e3:.1f} us ({pts / t_ours / 1e6:.0f} GPt/s), "
          f"speed-up {t_ref / t_ours:.2f}x")
    _record(kernel="stencil", reference="v7 launch_direct", dtype=str(dtype)[6:], shape=[H, W],
            reference_us=t_ref * 1e3, pla_b200_us=t_ours * 1e3, speedup=t_ref / t_ours)
    # Same arithmetic, same box: this library's kernel must not be the slower one.
    assert t_ours <= t_ref, f"pla_b200 {t_ours * 1e3:.1f} us slower than v7 {t_ref * 1e3:.1f} us"


@pytest.mark.skipif(not os.path.exists(V2), reason="reference kernels not built (oracle/_ref)")
@pytest.mark.parametrize("H,W", [(10240, 10240), (4096, 4096)])
def test_against_reference_v2_fp16(H, W):
    from pla_b200.stencil import ModelNew

    x, w, b = _inputs(H, W, torch.float16)
    launch = _v2()
    y_ref = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream

    def ref():
        launch(x.data_ptr(), w.data_ptr(), b.data_ptr(), y_ref.data_ptr(), 1, H, W, True, stream)

    m = ModelNew().cuda().half()
    with torch.no_grad():
        m.conv1.weight.copy_(w)
        m.conv1.bias.copy_(b)
    y = torch.empty_like(x)

    def ours():
        m(x, out=y)

    ref()
    ours()
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float(), y_ref.float(), atol=2e-3, rtol=2e-3)
    t_ref, t_ours = _time(ref), _time(ours)
    pts = H * W
    print(f"\n[v2 fp16 {H}x{W}] reference launch_stencil (mma.sync) {t_ref * 1e3:.1f} us "
          f"({pts / t_ref / 1e6:.0f} GPt/s), pla_b200 {t_ours * 1e3:.1f} us ({pts / t_ours / 1e6:.0f} GPt/s), "
          f"speed-up {t_ref / t_ours:.2f}x")
    _record(kernel="stencil", reference="v2 launch_stencil (mma.sync)", dtype="float16", shape=[H, W],
            reference_us=t_ref * 1e3, pla_b200_us=t_ours * 1e3, speedup=t_ref / t_ours)
    assert t_ours <= t_ref, f"pla_b200 {t_ours * 1e3:.1f} us slower than v2 {t_ref * 1e3:.1f} us"


# ---------------------------------------------------------------------------
# the reference's CUTLASS depthwise kernels (its generated fp16 Toeplitz-GEMM variants):
# data/depthwise_conv_7x7_cuda/model_cutlass.py (v1), model_cutlass_autotune_v5.py,
# model_cutlass_autotune_v6.py, launch_depthwise_7x7_cutlass(x, packed_w, y,
# n, c, h, w, fp16, stream); CUDA source strings compiled unmodified for
# sm_100a against CUTLASS headers (oracle/Makefile, target `ref`).
# ---------------------------------------------------------------------------
def _dw(tag):
    lib = ctypes.CDLL(os.path.join(REF, f"libref_dw_{tag}.so"))
    f = lib["_Z28launch_depthwise_7x7_cutlassPKvS0_PviiiibP11CUstream_st"]
    f.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i, ctypes.c_bool, _vp]
    f.restype = None
    return f


def _pack_weight(w: torch.Tensor) -> torch.Tensor:
    """The reference's [C,1,7,7] -> [C,8,80] packing (model_cutlass_autotune_v6.py:484-492,
    identical in model_cutlass.py:305-313 and model_cutlass_autotune_v5.py:445-453):
    row m = 2x4 output position (m // 2, m % 2), column k = input offset (k // 8, k % 8)."""
    m = torch.arange(8, device=w.device)[:, None]
    k = torch.arange(80, device=w.device)[None, :]
    ky = k // 8 - m // 2
    kx = k % 8 - m % 2
    valid = (ky >= 0) & (ky < 7) & (kx >= 0) & (kx < 7)
    vals = w[:, 0, ky.clamp(0, 6), kx.clamp(0, 6)]
    return torch.where(valid[None], vals, torch.zeros_like(vals)).contiguous()


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "libref_dw_v6.so")),
                    reason="reference CUTLASS depthwise kernels not built (oracle/_ref)")
@pytest.mark.parametrize("shape", [(1, 8, 2048, 2048), (1, 32, 1024, 1024)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_against_reference_cutlass_depthwise(shape, dtype):
    from pla_b200.depthwise import ModelNew

    N, C, H, W = shape
    g = torch.Generator().manual_seed(2)
    x = torch.rand(shape, generator=g).to(dtype).cuda()               # harness draw: torch.rand
    w = ((torch.rand(C, 1, 7, 7, generator=g) * 2 - 1) / 7).to(dtype).cuda()  # Conv2d default-init range
    packed = _pack_weight(w)
    stream = torch.cuda.current_stream().cuda_stream
    m = ModelNew(C, 7, 1, 3).cuda().to(dtype)
    with torch.no_grad():
        m.conv2d.weight.copy_(w)
    y = torch.empty_like(x)

    from pla_b200.depthwise import depthwise7x7

    def ours():
        depthwise7x7(x, m.conv2d.weight, None, out=y)

    ours()
    want = torch.nn.functional.conv2d(x.float().cpu(), w.float().cpu(), padding=3, groups=C)
    # 1e-2 for low precision, as the reference's own checks (benchmark/MetaSchedule/common.py:181-191)
    tol = 1e-2 if dtype == torch.float16 else 1e-5
    torch.testing.assert_close(y.float().cpu(), want.to(dtype).float(), atol=tol, rtol=tol)
    pts = N * C * H * W
    t_ours = _time(ours)
    line = f"\n[depthwise {str(dtype)[6:]} {N}x{C}x{H}x{W}] pla_b200 {t_ours * 1e3:.1f} us ({pts / t_ours / 1e6:.0f} GPt/s)"
    refs = {}
    for tag in ("v1", "v5", "v6"):
        launch = _dw(tag)
        y_ref = torch.empty_like(x)

        def ref():
            launch(x.data_ptr(), packed.data_ptr(), y_ref.data_ptr(), N, C, H, W, dtype == torch.float16, stream)

        ref()
        torch.cuda.synchronize()
        torch.testing.assert_close(y_ref.float().cpu(), want.to(dtype).float(), atol=tol, rtol=tol)
        t_ref = _time(ref)
        refs[tag] = t_ref * 1e3
        line += f"; ref {tag} {t_ref * 1e3:.1f} us ({t_ref / t_ours:.2f}x)"
    print(line)
    _record(kernel="depthwise", reference="CUTLASS v1/v5/v6 launch_depthwise_7x7_cutlass", dtype=str(dtype)[6:],
            shape=list(shape), reference_us=refs, pla_b200_us=t_ours * 1e3,
            speedup=min(refs.values()) / (t_ours * 1e3))
    assert t_ours * 1e3 <= min(refs.values()), f"pla_b200 {t_ours * 1e3:.1f} us slower than {refs}"

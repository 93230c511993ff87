"""Parity of the sibling gathers (grid_sample, ROI-Align) with the operators
they replace -- torch.nn.functional.grid_sample and torchvision.ops.roi_align
run on the CPU in float64 on the same (dtype-rounded) inputs -- and with the
restated oracle (oracle/gather_oracle.py), forward and backward (GPU only).

Tolerances: the strict bar of the MSDA suite (cases.STRICT_TOL) on outputs
and input gradients; grid gradients in pixel units with the bilinear kinks
excluded for fp32 grids (as for the MSDA location gradients).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import cases
from cases import REF_BWD_TOL, STRICT_TOL
from msda_triton_b200 import grid_sample, roi_align
from oracle import gather_oracle as go

torchvision = pytest.importorskip("torchvision")

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = [torch.float32, torch.float16, torch.bfloat16]


@pytest.fixture(autouse=True)
def _lib_loaded(cuda_lib):
    yield


def close(actual, expected, tol, what=""):
    torch.testing.assert_close(actual.double().cpu(), expected.double().cpu(), **tol,
                               msg=lambda m: f"{what}: {m}")


def _bitwise_equal(a, b):
    as_int = {2: torch.int16, 4: torch.int32}[a.element_size()]
    return torch.equal(a.contiguous().view(as_int), b.contiguous().view(as_int))


# ---------------------------------------------------------------------------
# grid_sample
# ---------------------------------------------------------------------------
GS_CASES = [
    ("c32", dict(N=2, C=32, H=24, W=31, Ho=20, Wo=17)),
    ("c3_scalar", dict(N=2, C=3, H=16, W=16, Ho=9, Wo=11)),
    ("c256", dict(N=1, C=256, H=12, W=10, Ho=8, Wo=8)),
    ("c96", dict(N=2, C=96, H=9, W=13, Ho=7, Wo=5)),
    ("c512_cpl2", dict(N=1, C=512, H=6, W=7, Ho=5, Wo=4)),
]


def _gs_inputs(kw, dtype, seed=0, lo=-1.15, hi=1.15):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(kw["N"], kw["C"], kw["H"], kw["W"], generator=g)
    grid = lo + (hi - lo) * torch.rand(kw["N"], kw["Ho"], kw["Wo"], 2, generator=g)
    gout = torch.randn(kw["N"], kw["C"], kw["Ho"], kw["Wo"], generator=g)
    return (x.to(DEV, dtype), grid.to(DEV, dtype), gout.to(DEV, dtype))


def _gs_reference(x, grid, gout, padding, align, mode="bilinear"):
    """torch's CPU grid_sample in float64 on the same rounded inputs, with autograd."""
    xr = x.detach().double().cpu().requires_grad_(True)
    gr = grid.detach().double().cpu().requires_grad_(True)
    out = F.grid_sample(xr, gr, mode=mode, padding_mode=padding, align_corners=align)
    out.backward(gout.double().cpu())
    return out.detach(), xr.grad, gr.grad


def _gs_kinks(grid, H, W, align, eps):
    """Grid points whose pixel coordinate lies within eps of an integer."""
    g = grid.detach().double().cpu()
    size = torch.tensor([W, H], dtype=torch.float64)
    px = ((g + 1) / 2) * (size - 1) if align else ((g + 1) * size - 1) / 2
    return ((px - px.round()).abs() < eps).any(-1)


def _run_gs(x, grid, gout, padding, align, **kw):
    xl = x.clone().requires_grad_(True)
    gl = grid.clone().requires_grad_(True)
    out = grid_sample(xl, gl, mode="bilinear", padding_mode=padding, align_corners=align, **kw)
    out.backward(gout)
    return out.detach(), xl.grad, gl.grad


@pytest.mark.parametrize("align", [False, True], ids=["ac0", "ac1"])
@pytest.mark.parametrize("padding", ["zeros", "border", "reflection"])
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw", GS_CASES, ids=[c[0] for c in GS_CASES])
def test_grid_sample_matches_torch(name, kw, dtype, padding, align):
    # Reflection: grids reaching well past the borders (several folds).
    span = 2.6 if padding == "reflection" else 1.15
    x, grid, gout = _gs_inputs(kw, dtype, lo=-span, hi=span)
    out, gx, gg = _run_gs(x, grid, gout, padding, align)
    assert out.shape == (kw["N"], kw["C"], kw["Ho"], kw["Wo"]) and out.dtype == dtype
    ref, gx_r, gg_r = _gs_reference(x, grid, gout, padding, align)
    tol = STRICT_TOL[dtype]
    close(out, ref, tol, "out")
    close(gx, gx_r, tol, "grad_input")
    # grad_grid in pixel units. fp32 grids: points within 1e-3 px of a
    # bilinear kink are excluded (the fp32 and float64 pixel coordinates may
    # floor differently there). 16-bit grids give pixel coordinates that are
    # exact in fp32, so both sides take the same one-sided derivative and
    # nothing is excluded.
    scale = torch.tensor([kw["W"], kw["H"]], dtype=torch.float64) / 2
    if dtype == torch.float32:
        keep = ~_gs_kinks(grid, kw["H"], kw["W"], align, 1e-3)
        assert keep.double().mean() > 0.98
    else:
        keep = torch.ones(grid.shape[:-1], dtype=torch.bool)
    torch.testing.assert_close((gg.double().cpu() / scale)[keep], (gg_r / scale)[keep], **tol)


@pytest.mark.parametrize("align", [False, True], ids=["ac0", "ac1"])
@pytest.mark.parametrize("padding", ["zeros", "border", "reflection"])
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw", GS_CASES[:3], ids=[c[0] for c in GS_CASES[:3]])
def test_grid_sample_nearest_matches_torch(name, kw, dtype, padding, align):
    """mode="nearest": the pixel at the coordinate rounded half to even.
    Grid values are bf16-representable for every dtype, so the pixel
    coordinate is exact in fp32 and ties round the same way on both sides."""
    x, grid, gout = _gs_inputs(kw, dtype, seed=2, lo=-1.6, hi=1.6)
    grid = grid.to(torch.bfloat16).to(dtype)
    xl = x.clone().requires_grad_(True)
    gl = grid.clone().requires_grad_(True)
    out = grid_sample(xl, gl, mode="nearest", padding_mode=padding, align_corners=align)
    out.backward(gout)
    ref, gx_r, _ = _gs_reference(x, grid, gout, padding, align, mode="nearest")
    tol = STRICT_TOL[dtype]
    close(out, ref, tol, "out")
    close(xl.grad, gx_r, tol, "grad_input")
    assert (gl.grad == 0).all()
    # The deterministic accumulation gives the same input gradient.
    xd = x.clone().requires_grad_(True)
    grid_sample(xd, grid, mode="nearest", padding_mode=padding, align_corners=align,
                deterministic=True).backward(gout)
    close(xd.grad, gx_r, tol, "grad_input (deterministic)")


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_grid_sample_matches_the_oracle(dtype):
    x, grid, gout = _gs_inputs(GS_CASES[0][1], dtype, seed=3)
    out, gx, _ = _run_gs(x, grid, gout, "zeros", False)
    xr = x.double().cpu().requires_grad_(True)
    ref = go.grid_sample(xr, grid.double().cpu(), "bilinear", "zeros", False)
    ref.backward(gout.double().cpu())
    close(out, ref.detach(), STRICT_TOL[dtype], "out")
    close(gx, xr.grad, STRICT_TOL[dtype], "grad_input")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=str)
def test_grid_sample_native_accumulation(dtype):
    x, grid, gout = _gs_inputs(GS_CASES[0][1], dtype, seed=4)
    _, gx, _ = _run_gs(x, grid, gout, "zeros", False, fp32_grad_accum=False)
    _, gx_r, _ = _gs_reference(x, grid, gout, "zeros", False)
    close(gx, gx_r, REF_BWD_TOL[dtype], "grad_input (native atomics)")


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw", GS_CASES[:3], ids=[c[0] for c in GS_CASES[:3]])
def test_grid_sample_deterministic(name, kw, dtype):
    """The fixed-point input gradient is bitwise invariant to the order of
    the output pixels (a permutation of the grid reorders every atomic)."""
    # A zoomed-out grid: many output pixels share input pixels.
    x, grid, gout = _gs_inputs(kw, dtype, seed=5, lo=-0.3, hi=0.3)
    _, gx, gg = _run_gs(x, grid, gout, "zeros", False, deterministic=True)
    _, gx2, _ = _run_gs(x, grid, gout, "zeros", False, deterministic=True)
    assert _bitwise_equal(gx, gx2)
    N, Ho, Wo = kw["N"], kw["Ho"], kw["Wo"]
    perm = torch.randperm(Ho * Wo, generator=torch.Generator().manual_seed(1)).to(DEV)
    gridp = grid.reshape(N, Ho * Wo, 2)[:, perm].reshape(N, Ho, Wo, 2)
    goutp = gout.reshape(N, -1, Ho * Wo)[:, :, perm].reshape(N, -1, Ho, Wo)
    _, gxp, ggp = _run_gs(x, gridp, goutp, "zeros", False, deterministic=True)
    assert _bitwise_equal(gx, gxp)
    assert _bitwise_equal(gg.reshape(N, Ho * Wo, 2)[:, perm], ggp.reshape(N, Ho * Wo, 2))
    _, gx_r, _ = _gs_reference(x, grid, gout, "zeros", False)
    close(gx, gx_r, STRICT_TOL[dtype], "grad_input (deterministic)")


def test_grid_sample_channels_last_input_and_edges():
    kw = GS_CASES[0][1]
    x, grid, gout = _gs_inputs(kw, torch.bfloat16, seed=6)
    a = grid_sample(x, grid, align_corners=False)
    b = grid_sample(x.contiguous(memory_format=torch.channels_last), grid, align_corners=False)
    assert torch.equal(a, b)
    assert a.is_contiguous(memory_format=torch.channels_last)
    # Empty output grid; grid points far outside (zeros padding) give zeros.
    empty = grid_sample(x, grid[:, :0], align_corners=False)
    assert empty.shape == (kw["N"], kw["C"], 0, kw["Wo"])
    far = torch.full_like(grid, 7.0)
    assert (grid_sample(x, far) == 0).all()
    nan = torch.full_like(grid, float("nan"))
    assert torch.isfinite(grid_sample(x, nan)).all()


# ---------------------------------------------------------------------------
# ROI-Align
# ---------------------------------------------------------------------------
def _roi_inputs(dtype, C, seed=0, N=2, H=28, W=33, K=12, scale=0.25):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, C, H, W, generator=g)
    xy = torch.rand(K, 2, generator=g) * torch.tensor([W, H]) / scale
    wh = (0.05 + torch.rand(K, 2, generator=g)) * torch.tensor([W, H]) / scale * 0.5
    idx = torch.randint(0, N, (K, 1), generator=g).float()
    boxes = torch.cat([idx, xy - 0.3 * wh, xy + wh], 1)  # some boxes cross the border
    return x.to(DEV, dtype), boxes, scale


ROI_CASES = [("c32", 32), ("c3_scalar", 3), ("c256", 256), ("c64", 64)]


@pytest.mark.parametrize("aligned", [False, True], ids=["unaligned", "aligned"])
@pytest.mark.parametrize("sampling_ratio", [-1, 2], ids=["adaptive", "sr2"])
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,C", ROI_CASES, ids=[c[0] for c in ROI_CASES])
def test_roi_align_matches_torchvision(name, C, dtype, sampling_ratio, aligned):
    x, boxes, scale = _roi_inputs(dtype, C)
    xl = x.clone().requires_grad_(True)
    out = roi_align(xl, boxes.to(DEV), (7, 6), scale, sampling_ratio, aligned)
    assert out.shape == (boxes.shape[0], C, 7, 6) and out.dtype == dtype
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(9)).to(DEV, dtype)
    out.backward(gout)
    # The kernels compute box geometry in fp32: the oracle with fp32 box
    # arithmetic is the tight reference, torchvision (float64 boxes) the
    # public one (sample positions differ by ~1e-6 px).
    xr = x.double().cpu().requires_grad_(True)
    ref = go.roi_align(xr, boxes, (7, 6), scale, sampling_ratio, aligned)
    ref.backward(gout.double().cpu())
    close(out, ref.detach(), STRICT_TOL[dtype], "out")
    close(xl.grad, xr.grad, STRICT_TOL[dtype], "grad_input")
    tv = torchvision.ops.roi_align(x.double().cpu(), boxes.double(), (7, 6), scale, sampling_ratio, aligned)
    close(out, tv, REF_BWD_TOL[dtype] if dtype != torch.float32 else dict(rtol=1e-4, atol=1e-4), "out vs torchvision")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=str)
def test_roi_align_native_accumulation_and_box_lists(dtype):
    x, boxes, scale = _roi_inputs(dtype, 32, seed=2)
    # torchvision's list-of-boxes format gives the same result as (K, 5).
    per_image = [boxes[boxes[:, 0] == i, 1:].to(DEV) for i in range(x.shape[0])]
    order = torch.cat([torch.nonzero(boxes[:, 0] == i).flatten() for i in range(x.shape[0])])
    a = roi_align(x, boxes.to(DEV), 5, scale, 2)
    b = roi_align(x, per_image, 5, scale, 2)
    assert torch.equal(a[order.to(DEV)], b)
    xl = x.clone().requires_grad_(True)
    out = roi_align(xl, boxes.to(DEV), 5, scale, 2, fp32_grad_accum=False)
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(3)).to(DEV, dtype)
    out.backward(gout)
    xr = x.double().cpu().requires_grad_(True)
    go.roi_align(xr, boxes, 5, scale, 2).backward(gout.double().cpu())
    close(xl.grad, xr.grad, REF_BWD_TOL[dtype], "grad_input (native atomics)")


def test_roi_align_edges():
    x, boxes, scale = _roi_inputs(torch.float32, 32, seed=5)
    # No boxes; a box on a missing batch item; a degenerate aligned box.
    assert roi_align(x, torch.zeros(0, 5, device=DEV), 3, scale).shape == (0, 32, 3, 3)
    bad = torch.tensor([[7.0, 1.0, 1.0, 20.0, 20.0], [0.0, 5.0, 5.0, 5.0, 5.0]], device=DEV)
    out = roi_align(x, bad, 3, 1.0, -1, True)
    assert (out[0] == 0).all()
    ref = torchvision.ops.roi_align(x.double().cpu(), bad[1:].double().cpu(), 3, 1.0, -1, True)
    close(out[1:], ref, dict(rtol=1e-5, atol=1e-6), "degenerate box")


@pytest.mark.parametrize("deterministic", [False, True], ids=["fp32", "fixed"])
@pytest.mark.parametrize("sampling_ratio", [-1, 2, 5], ids=["adaptive", "sr2", "sr5"])
def test_roi_align_reversed_and_tiny_boxes(sampling_ratio, deterministic):
    """Boxes with x2 < x1 or y2 < y1 (aligned=True keeps the negative bin
    size, so the samples run backwards), sub-pixel boxes whose samples share
    pixels, and boxes hanging over the border, forward and backward."""
    x, boxes, scale = _roi_inputs(torch.float32, 64, seed=11, K=16)
    rev = boxes.clone()
    rev[:8, [1, 3]] = boxes[:8, [3, 1]]        # x reversed
    rev[4:12, [2, 4]] = boxes[4:12, [4, 2]]    # y reversed (4 boxes both)
    rev[12:, 3:] = rev[12:, 1:3] + 0.7 / scale  # under one pixel per side
    rev[15, 1:] = torch.tensor([-3.0, -2.0, 0.5, 0.8]) / scale  # mostly outside
    xl = x.clone().requires_grad_(True)
    out = roi_align(xl, rev.to(DEV), (4, 3), scale, sampling_ratio, True, deterministic=deterministic)
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(12)).to(DEV)
    out.backward(gout)
    xr = x.double().cpu().requires_grad_(True)
    ref = go.roi_align(xr, rev, (4, 3), scale, sampling_ratio, True)
    ref.backward(gout.double().cpu())
    close(out, ref.detach(), STRICT_TOL[torch.float32], "out")
    close(xl.grad, xr.grad, STRICT_TOL[torch.float32], "grad_input")
    if sampling_ratio > 0:  # torchvision's CPU kernel rejects an adaptive grid on a reversed box
        tv = torchvision.ops.roi_align(x.double().cpu(), rev.double(), (4, 3), scale, sampling_ratio, True)
        close(out, tv, dict(rtol=1e-4, atol=1e-4), "out vs torchvision")


@pytest.mark.parametrize("sampling_ratio", [-1, 2], ids=["adaptive", "sr2"])
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_roi_align_deterministic(dtype, sampling_ratio):
    """The fixed-point input gradient: within the strict bar of the oracle,
    bitwise equal across runs, under a permutation of the boxes (which
    reorders every atomic), and under torch.use_deterministic_algorithms
    (where torchvision's backward raises)."""
    x, boxes, scale = _roi_inputs(dtype, 32, seed=6, K=24)
    gout = torch.randn(24, 32, 5, 4, generator=torch.Generator().manual_seed(4)).to(DEV, dtype)

    def grad(b, g, **kw):
        xl = x.clone().requires_grad_(True)
        roi_align(xl, b.to(DEV), (5, 4), scale, sampling_ratio, True, **kw).backward(g)
        return xl.grad

    g1 = grad(boxes, gout, deterministic=True)
    assert _bitwise_equal(g1, grad(boxes, gout, deterministic=True))
    perm = torch.randperm(24, generator=torch.Generator().manual_seed(8))
    assert _bitwise_equal(g1, grad(boxes[perm], gout[perm.to(DEV)], deterministic=True))
    before = torch.are_deterministic_algorithms_enabled()
    try:
        torch.use_deterministic_algorithms(True)
        assert _bitwise_equal(g1, grad(boxes, gout))
    finally:
        torch.use_deterministic_algorithms(before)
    xr = x.double().cpu().requires_grad_(True)
    go.roi_align(xr, boxes, (5, 4), scale, sampling_ratio, True).backward(gout.double().cpu())
    close(g1, xr.grad, STRICT_TOL[dtype], "grad_input (deterministic)")


# ---------------------------------------------------------------------------
# Layout conversion (msda_transpose) and the layouts of inputs and gradients
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("N,R,C", [(1, 1, 1), (2, 3, 130), (3, 64, 64), (2, 200, 77), (1, 4096, 33),
                                   (2, 100, 132), (1, 256, 4096),
                                   # more than 65535 row tiles (an NHWC image above 2048 x 2048)
                                   (1, 64 * 65536 + 5, 3), (1, 64 * 65536 + 4, 8)])
def test_transpose_is_exact(N, R, C, dtype):
    """Both kernels: the scalar one (ragged sizes) and the 4-element vector
    one (R and C multiples of 4)."""
    from msda_triton_b200.gather import _transpose
    x = torch.randn(N, R, C, generator=torch.Generator().manual_seed(R * C)).to(DEV, dtype)
    y = _transpose(x, N, R, C)
    assert torch.equal(y, x.transpose(1, 2).contiguous())
    assert torch.equal(_transpose(y, N, C, R), x)


@pytest.mark.parametrize("kind", ["f32", "bf16_native", "bf16_fp32", "f16_fixed", "f32_fixed"])
@pytest.mark.parametrize("name,kw", GS_CASES[:2], ids=[c[0] for c in GS_CASES[:2]])
def test_nchw_gradient_flag_through_the_abi(name, kw, kind):
    """MSDA_BWD_GRAD_INPUT_NCHW for every accumulator (data type, fp32,
    fixed point): the NCHW input gradient equals the NHWC one transposed --
    bitwise where the accumulation is order-independent (fixed point),
    within the bar of its accumulation otherwise -- and grad_grid is
    unchanged."""
    import ctypes

    from msda_triton_b200 import _lib
    from msda_triton_b200.ops import _DTYPE_CODE
    dtype = {"f32": torch.float32, "f32_fixed": torch.float32, "f16_fixed": torch.float16}.get(kind, torch.bfloat16)
    flags = {"bf16_fp32": _lib.MSDA_BWD_FP32_ACCUM, "f16_fixed": _lib.MSDA_BWD_DETERMINISTIC,
             "f32_fixed": _lib.MSDA_BWD_DETERMINISTIC}.get(kind, 0)
    x, grid, gout = _gs_inputs(kw, dtype, seed=13)
    N, C, H, W = x.shape
    Ho, Wo = grid.shape[1:3]
    xn = x.permute(0, 2, 3, 1).contiguous()
    gn = gout.permute(0, 2, 3, 1).contiguous()
    lib = _lib.load()
    code = _DTYPE_CODE[dtype]
    p = lambda t: ctypes.c_void_p(t.data_ptr() if t is not None else 0)  # noqa: E731

    def run(f, gi_shape):
        nbytes = lib.msda_grid_sample_backward_workspace_size(N, H, W, C, Ho, Wo, code, f)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV) if nbytes else None
        gi = torch.full(gi_shape, float("nan"), dtype=dtype, device=DEV)
        gg = torch.empty_like(grid)
        rc = lib.msda_grid_sample_backward(p(xn), p(grid), p(gn), p(gi), p(gg), p(ws), nbytes, N, H, W, C, Ho, Wo,
                                           0, 0, 0, code, f, ctypes.c_void_p(0))
        assert rc == _lib.MSDA_OK, lib.msda_last_error()
        return gi, gg

    gi_hwc, gg_a = run(flags, (N, H, W, C))
    gi_chw, gg_b = run(flags | _lib.MSDA_BWD_GRAD_INPUT_NCHW, (N, C, H, W))
    torch.cuda.synchronize()
    if "fixed" in kind:
        assert _bitwise_equal(gi_chw, gi_hwc.permute(0, 3, 1, 2))
    else:
        tol = REF_BWD_TOL[dtype] if kind == "bf16_native" else STRICT_TOL[dtype]  # native: rounded per add
        close(gi_chw, gi_hwc.permute(0, 3, 1, 2), tol, "grad_input (NCHW)")
    assert torch.equal(gg_a, gg_b)


@pytest.mark.parametrize("channels_last", [False, True], ids=["nchw", "channels_last"])
def test_gather_ops_keep_the_input_layout(channels_last):
    """An NCHW input gets an NCHW-contiguous gradient (and a channels_last one
    a channels_last gradient), for NCHW and channels_last output gradients
    alike; values match the references."""
    kw = GS_CASES[0][1]
    x, grid, gout = _gs_inputs(kw, torch.bfloat16, seed=8)
    fmt = torch.channels_last if channels_last else torch.contiguous_format
    xl = x.detach().contiguous(memory_format=fmt).requires_grad_(True)
    _, gx_r, _ = _gs_reference(x, grid, gout, "zeros", False)
    for g in (gout, gout.contiguous(memory_format=torch.channels_last)):
        xl.grad = None
        out = grid_sample(xl, grid, align_corners=False)
        out.backward(g)
        assert xl.grad.is_contiguous(memory_format=fmt)
        close(xl.grad, gx_r, STRICT_TOL[torch.bfloat16], "grad_input")
    xr, boxes, scale = _roi_inputs(torch.float32, 32, seed=4)
    xl = xr.detach().contiguous(memory_format=fmt).requires_grad_(True)
    out = roi_align(xl, boxes.to(DEV), 4, scale, 2)
    out.backward(torch.ones_like(out))
    assert xl.grad.is_contiguous(memory_format=fmt)
    xd = xr.detach().double().cpu().requires_grad_(True)
    go.roi_align(xd, boxes, 4, scale, 2).backward(torch.ones(out.shape, dtype=torch.float64))
    close(xl.grad, xd.grad, STRICT_TOL[torch.float32], "roi grad_input")

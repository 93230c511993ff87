"""The sibling-gather oracle (oracle/gather_oracle.py) pinned to the public
operators it restates -- torch.nn.functional.grid_sample and
torchvision.ops.roi_align -- on CPU in float64, forward and backward (CPU
only: no GPU needed)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import gather_oracle as go

torchvision = pytest.importorskip("torchvision")


def _grid_inputs(seed, N=2, C=5, H=7, W=9, Ho=6, Wo=8, lo=-1.2, hi=1.2):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, C, H, W, generator=g, dtype=torch.float64)
    grid = lo + (hi - lo) * torch.rand(N, Ho, Wo, 2, generator=g, dtype=torch.float64)
    return x, grid


@pytest.mark.parametrize("align", [False, True])
@pytest.mark.parametrize("padding", ["zeros", "border", "reflection"])
@pytest.mark.parametrize("mode", ["bilinear", "nearest"])
def test_grid_sample_restatement_matches_torch(mode, padding, align):
    # Grids reaching well past the borders, so that reflection folds more than once.
    x, grid = _grid_inputs(0, lo=-3.2, hi=3.2)
    a = [t.clone().requires_grad_(True) for t in (x, grid)]
    b = [t.clone().requires_grad_(True) for t in (x, grid)]
    out = go.grid_sample(*a, mode=mode, padding_mode=padding, align_corners=align)
    ref = F.grid_sample(*b, mode=mode, padding_mode=padding, align_corners=align)
    torch.testing.assert_close(out, ref, rtol=1e-12, atol=1e-12)
    g = torch.randn_like(ref)
    out.backward(g)
    ref.backward(g)
    torch.testing.assert_close(a[0].grad, b[0].grad, rtol=1e-12, atol=1e-12)
    # "nearest" is piecewise constant in the grid: no gradient (torch: zeros).
    ga = a[1].grad if a[1].grad is not None else torch.zeros_like(grid)
    torch.testing.assert_close(ga, b[1].grad, rtol=1e-10, atol=1e-10)


def _boxes(seed, K=6, N=2, H=20, W=24, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    xy = torch.rand(K, 2, generator=g) * torch.tensor([W, H]) / scale
    wh = torch.rand(K, 2, generator=g) * torch.tensor([W, H]) / scale * 0.6
    idx = torch.randint(0, N, (K, 1), generator=g).float()
    boxes = torch.cat([idx, xy - 0.2 * wh, xy + wh], 1)  # some boxes cross the border
    return boxes


@pytest.mark.parametrize("aligned", [False, True])
@pytest.mark.parametrize("sampling_ratio", [-1, 2])
def test_roi_align_restatement_matches_torchvision(sampling_ratio, aligned):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 4, 20, 24, generator=g, dtype=torch.float64)
    boxes = _boxes(4)
    a = x.clone().requires_grad_(True)
    b = x.clone().requires_grad_(True)
    out = go.roi_align(a, boxes.double(), (5, 4), 0.5, sampling_ratio, aligned, box_dtype=torch.float64)
    ref = torchvision.ops.roi_align(b, boxes.double(), (5, 4), 0.5, sampling_ratio, aligned)
    torch.testing.assert_close(out, ref, rtol=1e-12, atol=1e-12)
    gout = torch.randn_like(ref)
    out.backward(gout)
    ref.backward(gout)
    torch.testing.assert_close(a.grad, b.grad, rtol=1e-12, atol=1e-12)
    # fp32 box arithmetic (the kernels') moves sample positions by ~1e-6 px.
    out32 = go.roi_align(x, boxes, (5, 4), 0.5, sampling_ratio, aligned)
    torch.testing.assert_close(out32, ref.detach(), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("sampling_ratio", [2, 5])
def test_roi_align_restatement_on_reversed_and_tiny_boxes(sampling_ratio):
    """Boxes with x2 < x1 and/or y2 < y1 (aligned=True keeps the negative bin
    size), boxes under one pixel, and a box mostly outside the image: the
    restatement agrees with torchvision in float64, forward and backward.
    (torchvision's CPU kernel rejects an adaptive sampling grid on a reversed
    box, so the ratio is fixed here.)"""
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 3, 14, 17, generator=g, dtype=torch.float64)
    boxes = torch.tensor([
        [0, 20.0, 4.0, 6.0, 22.0],    # x reversed
        [1, 3.0, 25.0, 30.0, 5.0],    # y reversed
        [0, 28.0, 24.0, 2.0, 1.0],    # both reversed
        [1, 9.3, 7.1, 9.9, 7.6],      # under one pixel
        [0, -12.0, -8.0, 2.0, 3.2],   # mostly outside
    ], dtype=torch.float64)
    a = x.clone().requires_grad_(True)
    b = x.clone().requires_grad_(True)
    out = go.roi_align(a, boxes, (4, 3), 0.5, sampling_ratio, True, box_dtype=torch.float64)
    ref = torchvision.ops.roi_align(b, boxes, (4, 3), 0.5, sampling_ratio, True)
    torch.testing.assert_close(out, ref, rtol=1e-12, atol=1e-12)
    gout = torch.randn(ref.shape, generator=g, dtype=torch.float64)
    out.backward(gout)
    ref.backward(gout)
    torch.testing.assert_close(a.grad, b.grad, rtol=1e-12, atol=1e-12)

"""Sibling-gather oracle -- TEST INFRASTRUCTURE ONLY.

CPU restatements of the two operators the reference names as siblings of
MSDA (docs/course/08-exercises.md:39), used as the checkers of the sm_100a
grid_sample and ROI-Align kernels. Only ``tests/`` may import this module;
the product path (``msda_triton_b200``) never does.

Neither operator is part of the reference; their published definitions are
those of the third-party operators the B200 versions replace, installed in
this image and used to pin the restatements (tests/test_gather_oracle.py):

* :func:`grid_sample` restates ``torch.nn.functional.grid_sample``
  (torch 2.11.0; mode "bilinear" / "nearest", padding_mode "zeros" /
  "border" / "reflection", align_corners): source index
  ((g + 1) * size - 1) / 2 or (g + 1) / 2 * (size - 1), clipped to
  [0, size - 1] for "border", reflected about the borders (at -0.5 and
  size - 0.5, or 0 and size - 1 with align_corners) and then clipped for
  "reflection"; bilinear weights of the four neighbours, or the neighbour at
  the coordinate rounded half to even for "nearest"; zero outside the map.
* :func:`roi_align` restates ``torchvision.ops.roi_align`` (torchvision
  0.26.0; the RoIAlign of Mask R-CNN, He et al. 2017): per output bin, the
  mean over a grid of sampling points (sampling_ratio per side, or
  ceil(roi size / bins)) of a bilinear interpolation that is zero more than
  one pixel outside the map and clamps to the edge otherwise; `aligned`
  shifts the box by half a pixel.

Both are written with differentiable torch operations, so autograd gives
their backward passes.
"""

from __future__ import annotations

import math

import torch


def _reflect(x: torch.Tensor, twice_lo: int, twice_hi: int) -> torch.Tensor:
    """x reflected about twice_lo / 2 and twice_hi / 2 until it lies between them."""
    if twice_lo == twice_hi:
        return torch.zeros_like(x)
    lo, span = twice_lo / 2, (twice_hi - twice_lo) / 2
    d = (x - lo).abs()
    extra = torch.fmod(d, span)
    flips = torch.floor(d / span)
    return torch.where(torch.fmod(flips, 2) == 0, extra + lo, span - extra + lo)


def grid_sample(input: torch.Tensor, grid: torch.Tensor, mode: str = "bilinear",
                padding_mode: str = "zeros", align_corners: bool = False) -> torch.Tensor:
    """(N, C, H, W), (N, Ho, Wo, 2) -> (N, C, Ho, Wo)."""
    N, C, H, W = input.shape

    def source(g, size):
        if align_corners:
            x = ((g + 1) / 2) * (size - 1)
        else:
            x = ((g + 1) * size - 1) / 2
        if padding_mode == "reflection":
            x = _reflect(x, 0, 2 * (size - 1)) if align_corners else _reflect(x, -1, 2 * size - 1)
        if padding_mode in ("border", "reflection"):
            x = x.clamp(0, size - 1)
        return x

    x = source(grid[..., 0], W)
    y = source(grid[..., 1], H)
    img = input.permute(0, 2, 3, 1)  # (N, H, W, C)
    if mode == "nearest":
        xi, yi = x.detach().round(), y.detach().round()  # half to even
        valid = (xi >= 0) & (xi < W) & (yi >= 0) & (yi < H)
        n = torch.arange(N).view(N, 1, 1).expand_as(xi)
        v = img[n, yi.clamp(0, H - 1).long(), xi.clamp(0, W - 1).long()]
        return (v * valid[..., None]).permute(0, 3, 1, 2)
    x0, y0 = x.detach().floor(), y.detach().floor()
    lx, ly = x - x0, y - y0
    n = torch.arange(N).view(N, 1, 1).expand_as(x0)
    out = 0
    for dy, dx, w in ((0, 0, (1 - lx) * (1 - ly)), (0, 1, lx * (1 - ly)),
                      (1, 0, (1 - lx) * ly), (1, 1, lx * ly)):
        xi, yi = x0 + dx, y0 + dy
        valid = (xi >= 0) & (xi < W) & (yi >= 0) & (yi < H)
        v = img[n, yi.clamp(0, H - 1).long(), xi.clamp(0, W - 1).long()]  # (N, Ho, Wo, C)
        out = out + (w * valid)[..., None] * v
    return out.permute(0, 3, 1, 2)


def _bilinear_roi(img: torch.Tensor, y: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """img (H, W, C); y, x sample positions (any shape, detached) -> (..., C)."""
    H, W, _ = img.shape
    inside = (y >= -1.0) & (y <= H) & (x >= -1.0) & (x <= W)
    y = y.clamp(min=0)
    x = x.clamp(min=0)
    ylo, xlo = y.floor().long(), x.floor().long()
    ytop, xtop = ylo >= H - 1, xlo >= W - 1
    ylo = torch.where(ytop, torch.full_like(ylo, H - 1), ylo)
    xlo = torch.where(xtop, torch.full_like(xlo, W - 1), xlo)
    yhi = torch.where(ytop, ylo, ylo + 1)
    xhi = torch.where(xtop, xlo, xlo + 1)
    y = torch.where(ytop, ylo.to(y.dtype), y)
    x = torch.where(xtop, xlo.to(x.dtype), x)
    ly, lx = y - ylo, x - xlo
    hy, hx = 1 - ly, 1 - lx
    val = ((hy * hx)[..., None] * img[ylo, xlo] + (hy * lx)[..., None] * img[ylo, xhi]
           + (ly * hx)[..., None] * img[yhi, xlo] + (ly * lx)[..., None] * img[yhi, xhi])
    return val * inside[..., None]


def roi_align(input: torch.Tensor, rois: torch.Tensor, output_size, spatial_scale: float = 1.0,
              sampling_ratio: int = -1, aligned: bool = False,
              box_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """(N, C, H, W), (K, 5) -> (K, C, PH, PW). Box and sample-position
    arithmetic in `box_dtype` (fp32: the kernels' precision; float64: the
    precision torchvision uses for float64 boxes); interpolation in the
    input's dtype."""
    PH, PW = (output_size, output_size) if isinstance(output_size, int) else output_size
    img_all = input.permute(0, 2, 3, 1)  # (N, H, W, C)
    N = input.shape[0]
    outs = []
    r32 = rois.detach().to(box_dtype)
    for k in range(rois.shape[0]):
        b = int(r32[k, 0])
        off = 0.5 if aligned else 0.0
        x1 = r32[k, 1] * spatial_scale - off
        y1 = r32[k, 2] * spatial_scale - off
        x2 = r32[k, 3] * spatial_scale - off
        y2 = r32[k, 4] * spatial_scale - off
        rw, rh = x2 - x1, y2 - y1
        if not aligned:
            rw, rh = rw.clamp(min=1.0), rh.clamp(min=1.0)
        bh, bw = rh / PH, rw / PW
        gh = sampling_ratio if sampling_ratio > 0 else int(math.ceil(float(rh / PH)))
        gw = sampling_ratio if sampling_ratio > 0 else int(math.ceil(float(rw / PW)))
        count = max(gh * gw, 1)
        if gh <= 0 or gw <= 0 or not 0 <= b < N:
            outs.append(input.new_zeros(PH, PW, input.shape[1]))
            continue
        ph = torch.arange(PH, dtype=box_dtype).view(PH, 1, 1, 1)
        pw = torch.arange(PW, dtype=box_dtype).view(1, PW, 1, 1)
        iy = torch.arange(gh, dtype=box_dtype).view(1, 1, gh, 1)
        ix = torch.arange(gw, dtype=box_dtype).view(1, 1, 1, gw)
        y = (y1 + ph * bh) + (iy + 0.5) * bh / gh  # (PH, 1, gh, 1)
        x = (x1 + pw * bw) + (ix + 0.5) * bw / gw  # (1, PW, 1, gw)
        y, x = torch.broadcast_tensors(y, x)
        img = img_all[b]
        val = _bilinear_roi(img, y.to(img.dtype), x.to(img.dtype))  # (PH, PW, gh, gw, C)
        outs.append(val.sum((2, 3)) / count)
    if not outs:
        return input.new_zeros(0, input.shape[1], PH, PW)
    return torch.stack(outs).permute(0, 3, 1, 2)

"""Sibling gathers on the B200 kernels: ``grid_sample`` and ``roi_align``.

The reference names these as the operators its recipe transfers to
(docs/course/08-exercises.md:39: "ROI-Align, grid_sample itself ... share
MSDA's anatomy: data-dependent bilinear gathers forward, atomic scatters
backward"). Both run on the MSDA kernel skeleton in channels-last layout
(csrc/msda_gather.cuh) through the C ABI of include/msda_b200.h, and are
drop-ins for the public operators they replace:

* :func:`grid_sample` for ``torch.nn.functional.grid_sample`` (4-D input,
  ``mode`` "bilinear" or "nearest", ``padding_mode`` "zeros", "border" or
  "reflection");
* :func:`roi_align` for ``torchvision.ops.roi_align``.

The kernels read and write NHWC. An input already in ``torch.channels_last``
memory format is used as is; an NCHW input (and an NCHW output gradient) is
converted by the library's tiled transpose kernel (``msda_transpose``), and
the input gradient is returned in the input's layout: for an NCHW input the
backward writes it NCHW directly (``MSDA_BWD_GRAD_INPUT_NCHW``: the
accumulator is rounded and transposed in one pass, no separate transpose).
The outputs are channels-last NCHW tensors (same shape and values as the
replaced operators, a different memory format). There is no CPU path.
"""

from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from . import _lib
from .ops import _DTYPE_CODE, _FLOAT_DTYPES, _device_guard, _ptr, _stream, _use_deterministic

_PADDING = {"zeros": 0, "border": 1, "reflection": 2}
_MODE = {"bilinear": 0, "nearest": 1}


def _transpose(src: torch.Tensor, N: int, R: int, C: int) -> torch.Tensor:
    """(N, R, C) contiguous -> (N, C, R) contiguous, on the device."""
    dst = src.new_empty(N, C, R)
    lib = _lib.load()
    with _device_guard(src.device):
        rc = lib.msda_transpose(_ptr(src), _ptr(dst), N, R, C, _DTYPE_CODE[src.dtype], _stream(src.device))
    _lib.check("msda_transpose", rc)
    return dst


class _ToNHWC(torch.autograd.Function):
    """NCHW -> contiguous NHWC with the transpose kernel. The gathers'
    backward writes the input gradient NCHW (MSDA_BWD_GRAD_INPUT_NCHW) and
    hands it back as an (N, H, W, C)-shaped view, which passes through here
    as is; any other gradient goes back to NCHW with the transpose kernel."""

    @staticmethod
    def forward(ctx, x):
        N, C, H, W = x.shape
        return _transpose(x.contiguous(), N, C, H * W).view(N, H, W, C)

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        nchw = g.permute(0, 3, 1, 2)
        if nchw.is_contiguous():
            return nchw
        N, H, W, C = g.shape
        return _transpose(_nhwc_contiguous(g), N, H * W, C).view(N, C, H, W)


def _backward_rounds(dtype: torch.dtype, flags: int) -> bool:
    """Whether the gather backward ends with a rounding pass over its
    accumulator (fixed point, or fp32 accumulation of 16-bit data)."""
    return bool(flags & _lib.MSDA_BWD_DETERMINISTIC) or (
        bool(flags & _lib.MSDA_BWD_FP32_ACCUM) and dtype != torch.float32)


def _nhwc(x: torch.Tensor, flags: int) -> tuple[torch.Tensor, bool]:
    """(N, C, H, W) -> (contiguous (N, H, W, C), whether the backward writes
    the input gradient NCHW): a view of a channels_last tensor, else one
    transpose kernel. The NCHW gradient is asked for where the backward has
    a rounding pass anyway, which then transposes for free; elsewhere it
    would only move the transpose into the library."""
    v = x.permute(0, 2, 3, 1)
    if v.is_contiguous():
        return v, False
    return _ToNHWC.apply(x), _backward_rounds(x.dtype, flags)


def _grad_input(like: torch.Tensor, nhwc_shape, nchw: bool) -> torch.Tensor:
    """The input gradient's buffer (dtype and device of `like`) as an
    (N, H, W, C)-shaped tensor: NHWC memory, or NCHW memory seen through a
    permute (the layout MSDA_BWD_GRAD_INPUT_NCHW writes)."""
    N, H, W, C = nhwc_shape
    if nchw:
        return like.new_empty(N, C, H, W).permute(0, 2, 3, 1)
    return like.new_empty(N, H, W, C)


def _nhwc_contiguous(t: torch.Tensor) -> torch.Tensor:
    """An (N, H, W, C)-shaped tensor as contiguous NHWC: itself, one
    transpose kernel when it is an NCHW-contiguous tensor seen through a
    permute (an output gradient from an NCHW consumer), else a copy."""
    if t.is_contiguous():
        return t
    N, H, W, C = t.shape
    nchw = t.permute(0, 3, 1, 2)
    if nchw.is_contiguous() and t.dtype in _DTYPE_CODE:
        return _transpose(nchw, N, C, H * W).view(N, H, W, C)
    return t.contiguous()


def _bwd_flags(dtype, fp32_grad_accum, deterministic):
    if fp32_grad_accum is None:
        fp32_grad_accum = dtype != torch.float32
    return ((_lib.MSDA_BWD_FP32_ACCUM if fp32_grad_accum else 0)
            | (_lib.MSDA_BWD_DETERMINISTIC if deterministic else 0))


def _workspace(nbytes, device):
    return torch.empty(nbytes, dtype=torch.uint8, device=device) if nbytes else None


# ---------------------------------------------------------------------------
# grid_sample
# ---------------------------------------------------------------------------
class _GridSampleFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, grid, mode, padding, align, flags, nchw):
        N, H, W, C = x.shape
        _, Ho, Wo, _ = grid.shape
        out = x.new_empty(N, Ho, Wo, C)
        lib = _lib.load()
        with _device_guard(x.device):
            rc = lib.msda_grid_sample_forward(_ptr(x), _ptr(grid), _ptr(out), N, H, W, C, Ho, Wo,
                                              mode, padding, int(align), _DTYPE_CODE[x.dtype],
                                              _stream(x.device))
        _lib.check("msda_grid_sample_forward", rc)
        ctx.save_for_backward(x, grid)
        ctx.cfg = (mode, padding, align, flags | (_lib.MSDA_BWD_GRAD_INPUT_NCHW if nchw else 0), nchw)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out):
        x, grid = ctx.saved_tensors
        mode, padding, align, flags, nchw = ctx.cfg
        N, H, W, C = x.shape
        _, Ho, Wo, _ = grid.shape
        grad_out = _nhwc_contiguous(grad_out.to(x.dtype))
        grad_in = _grad_input(x, x.shape, nchw)
        grad_grid = torch.empty_like(grid)
        lib = _lib.load()
        code = _DTYPE_CODE[x.dtype]
        nbytes = lib.msda_grid_sample_backward_workspace_size(N, H, W, C, Ho, Wo, code, flags)
        ws = _workspace(nbytes, x.device)
        with _device_guard(x.device):
            rc = lib.msda_grid_sample_backward(
                _ptr(x), _ptr(grid), _ptr(grad_out), _ptr(grad_in), _ptr(grad_grid), _ptr(ws), nbytes,
                N, H, W, C, Ho, Wo, mode, padding, int(align), code, flags, _stream(x.device))
        _lib.check("msda_grid_sample_backward", rc)
        return grad_in, grad_grid, None, None, None, None, None


def grid_sample(
    input: torch.Tensor,
    grid: torch.Tensor,
    mode: str = "bilinear",
    padding_mode: str = "zeros",
    align_corners: bool | None = None,
    *,
    fp32_grad_accum: bool | None = None,
    deterministic: bool | None = None,
) -> torch.Tensor:
    """``torch.nn.functional.grid_sample`` for 4-D input on B200.

    Args:
        input: ``(N, C, H, W)``; channels-last memory avoids a copy.
        grid: ``(N, H_out, W_out, 2)`` normalised ``(x, y)`` in ``[-1, 1]``.
        mode: ``"bilinear"`` or ``"nearest"`` (``"bicubic"`` is not built).
        padding_mode: ``"zeros"``, ``"border"`` or ``"reflection"``.
        align_corners: as in torch; ``None`` means ``False``.
        fp32_grad_accum: accumulate the input gradient in fp32 (default for
            fp16/bf16) or with native half-precision atomics.
        deterministic: bitwise-reproducible input gradient (64-bit
            fixed-point accumulation); ``None`` follows
            ``torch.are_deterministic_algorithms_enabled()``.

    Returns:
        ``(N, C, H_out, W_out)`` in ``input.dtype``, channels-last memory.
    """
    if input.dim() != 4:
        raise ValueError(f"grid_sample: only 4-D input (N, C, H, W) is supported, got {input.dim()}-D")
    if grid.dim() != 4 or grid.shape[-1] != 2 or grid.shape[0] != input.shape[0]:
        raise ValueError(f"grid_sample: grid must be (N, H_out, W_out, 2) with N={input.shape[0]}, "
                         f"got {tuple(grid.shape)}")
    if mode not in ("bilinear", "nearest", "bicubic"):
        raise ValueError(f"grid_sample: expected mode to be 'bilinear', 'nearest' or 'bicubic', got '{mode}'")
    if mode == "bicubic":
        raise NotImplementedError("grid_sample: mode='bicubic' is not built (bilinear and nearest are)")
    if padding_mode not in ("zeros", "border", "reflection"):
        raise ValueError("grid_sample: expected padding_mode to be 'zeros', 'border' or 'reflection', "
                         f"got '{padding_mode}'")
    if input.dtype != grid.dtype:
        raise ValueError(f"grid_sample: input and grid dtypes must match, got {input.dtype}/{grid.dtype}")
    if input.dtype not in _FLOAT_DTYPES:
        raise ValueError(f"grid_sample: unsupported dtype {input.dtype}; use fp32, fp16 or bf16")
    if input.device.type != "cuda" or grid.device != input.device:
        raise ValueError("grid_sample: input and grid must be CUDA tensors on the same device")
    if input.shape[2] < 1 or input.shape[3] < 1 or input.shape[1] < 1:
        raise ValueError(f"grid_sample: empty input {tuple(input.shape)}")
    _lib.load()
    flags = _bwd_flags(input.dtype, fp32_grad_accum, _use_deterministic(deterministic))
    x, nchw = _nhwc(input, flags)
    out = _GridSampleFunction.apply(x, grid.contiguous(), _MODE[mode], _PADDING[padding_mode],
                                    bool(align_corners), flags, nchw)
    return out.permute(0, 3, 1, 2)


# ---------------------------------------------------------------------------
# roi_align
# ---------------------------------------------------------------------------
def _check_boxes(boxes) -> None:
    if isinstance(boxes, (list, tuple)):
        for b in boxes:
            if b.dim() != 2 or b.shape[1] != 4:
                raise ValueError(f"roi_align: each box tensor must be (L, 4), got {tuple(b.shape)}")
    elif boxes.dim() != 2 or boxes.shape[1] != 5:
        raise ValueError(f"roi_align: boxes must be a (K, 5) tensor or a list of (L, 4) tensors, "
                         f"got {tuple(boxes.shape)}")


def _rois(boxes, device) -> torch.Tensor:
    """torchvision's box formats -> (K, 5) fp32 (batch index, x1, y1, x2, y2)."""
    if isinstance(boxes, (list, tuple)):
        parts = [torch.cat([torch.full((b.shape[0], 1), float(i), dtype=torch.float32, device=b.device),
                            b.float()], 1) for i, b in enumerate(boxes)]
        rois = torch.cat(parts, 0) if parts else torch.zeros(0, 5)
    else:
        rois = boxes.float()
    return rois.to(device).contiguous()


class _RoiAlignFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, rois, out_hw, spatial_scale, sampling_ratio, aligned, flags, nchw):
        N, H, W, C = x.shape
        K = rois.shape[0]
        PH, PW = out_hw
        out = x.new_empty(K, PH, PW, C)
        lib = _lib.load()
        with _device_guard(x.device):
            rc = lib.msda_roi_align_forward(_ptr(x), _ptr(rois), _ptr(out), N, H, W, C, K, PH, PW,
                                            float(spatial_scale), int(sampling_ratio), int(aligned),
                                            _DTYPE_CODE[x.dtype], _stream(x.device))
        _lib.check("msda_roi_align_forward", rc)
        ctx.save_for_backward(rois)
        ctx.cfg = (tuple(x.shape), x.dtype, out_hw, spatial_scale, sampling_ratio, aligned,
                   flags | (_lib.MSDA_BWD_GRAD_INPUT_NCHW if nchw else 0), nchw)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out):
        (rois,) = ctx.saved_tensors
        shape, dtype, (PH, PW), spatial_scale, sampling_ratio, aligned, flags, nchw = ctx.cfg
        N, H, W, C = shape
        grad_out = _nhwc_contiguous(grad_out.to(dtype))
        grad_in = _grad_input(grad_out, shape, nchw)
        lib = _lib.load()
        code = _DTYPE_CODE[dtype]
        nbytes = lib.msda_roi_align_backward_workspace_size(N, H, W, C, code, flags)
        ws = _workspace(nbytes, grad_out.device)
        with _device_guard(grad_out.device):
            rc = lib.msda_roi_align_backward(
                _ptr(rois), _ptr(grad_out), _ptr(grad_in), _ptr(ws), nbytes, N, H, W, C, rois.shape[0],
                PH, PW, float(spatial_scale), int(sampling_ratio), int(aligned), code, flags,
                _stream(grad_out.device))
        _lib.check("msda_roi_align_backward", rc)
        return grad_in, None, None, None, None, None, None, None


def roi_align(
    input: torch.Tensor,
    boxes,
    output_size,
    spatial_scale: float = 1.0,
    sampling_ratio: int = -1,
    aligned: bool = False,
    *,
    fp32_grad_accum: bool | None = None,
    deterministic: bool | None = None,
) -> torch.Tensor:
    """``torchvision.ops.roi_align`` on B200.

    Args:
        input: ``(N, C, H, W)``; channels-last memory avoids a copy.
        boxes: ``(K, 5)`` tensor of ``(batch index, x1, y1, x2, y2)`` or a
            list of per-image ``(L, 4)`` tensors (torchvision's formats);
            coordinates are used in fp32.
        output_size: ``int`` or ``(height, width)`` of the pooled output.
        spatial_scale, sampling_ratio, aligned: as in torchvision.
        fp32_grad_accum: accumulate the input gradient in fp32 (default for
            fp16/bf16) or with native half-precision atomics.
        deterministic: bitwise-reproducible input gradient (64-bit
            fixed-point accumulation; torchvision's backward has none);
            ``None`` follows ``torch.are_deterministic_algorithms_enabled()``.

    Returns:
        ``(K, C, height, width)`` in ``input.dtype``, channels-last memory.
        Differentiable with respect to ``input`` only.
    """
    if input.dim() != 4:
        raise ValueError(f"roi_align: input must be (N, C, H, W), got {input.dim()}-D")
    _check_boxes(boxes)
    if input.dtype not in _FLOAT_DTYPES:
        raise ValueError(f"roi_align: unsupported dtype {input.dtype}; use fp32, fp16 or bf16")
    if input.device.type != "cuda":
        raise ValueError("roi_align: input must be a CUDA tensor")
    out_hw = (output_size, output_size) if isinstance(output_size, int) else tuple(int(v) for v in output_size)
    if len(out_hw) != 2 or min(out_hw) < 1:
        raise ValueError(f"roi_align: output_size must be an int or (height, width) >= 1, got {output_size}")
    _lib.load()
    rois = _rois(boxes, input.device)
    flags = _bwd_flags(input.dtype, fp32_grad_accum, _use_deterministic(deterministic))
    x, nchw = _nhwc(input, flags)
    out = _RoiAlignFunction.apply(x, rois, out_hw, float(spatial_scale), int(sampling_ratio),
                                  bool(aligned), flags, nchw)
    return out.permute(0, 3, 1, 2)

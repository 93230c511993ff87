"""Public MSDA operator on B200: the reference's Python surface
(src/msda_triton/ops.py:96-199) over the sm_100a kernels of libmsda_b200.

The signature, validation order, error types and messages, dtype handling and
return conventions follow the reference; the Triton launches and the
Metal/MPS dispatch are replaced by calls through the C ABI
(include/msda_b200.h). There is no CPU path and no fallback: a non-CUDA
tensor raises ``ValueError`` and a missing library raises ``RuntimeError``.
"""

from __future__ import annotations

import contextlib
import ctypes

import torch
from torch.autograd.function import once_differentiable

from . import _lib

_FLOAT_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
_DTYPE_CODE = {
    torch.float32: _lib.MSDA_DTYPE_F32,
    torch.float16: _lib.MSDA_DTYPE_F16,
    torch.bfloat16: _lib.MSDA_DTYPE_BF16,
}


def _use_fp32_grad_accum(value: torch.Tensor) -> bool:
    """Default accumulator precision for grad_value (reference: ops.py:21-33).

    The reference picks native half-precision atomics on SM >= 9.0. On B200
    (SM 10.0) this build instead accumulates fp16/bf16 gradients in fp32 by
    default: a native bf16/fp16 add rounds the running sum at every hit, and
    at encoder density (about 1300 hits per coarse-level element) that error
    exceeds 1e-2 relative. fp32 inputs always accumulate in fp32, so the flag
    only matters for fp16/bf16. ``fp32_grad_accum=False`` selects the native
    packed f16x2/bf16x2 `red` path. With fp32 accumulation and sparse
    sampling (Q*L*K <= 2*S per head, e.g. a DETR decoder) the library uses
    its hit-counted backward, which writes rows hit once directly and keeps
    fp32 rows only where a row is hit more than once.
    """
    return value.dtype != torch.float32


def _use_deterministic(deterministic: bool | None) -> bool:
    """``deterministic=None`` follows ``torch.use_deterministic_algorithms``:
    when PyTorch is asked for deterministic algorithms the backward takes the
    library's order-independent grad_value accumulation (integer sums:
    bitwise reproducible) instead of raising or silently using atomics."""
    if deterministic is None:
        return torch.are_deterministic_algorithms_enabled()
    return bool(deterministic)


def _bwd_flags(fp32_grad_accum: bool, deterministic: bool, algo_flags: int) -> int:
    return ((_lib.MSDA_BWD_FP32_ACCUM if fp32_grad_accum else 0)
            | (_lib.MSDA_BWD_DETERMINISTIC if deterministic else 0) | algo_flags)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _device_guard(device: torch.device):
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _forward(value, spatial_shapes, level_start_index, sampling_locations, attention_weights):
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_locations.shape
    out = value.new_empty(B, Q, M, D)
    lib = _lib.load()
    with _device_guard(value.device):
        rc = lib.msda_forward(
            _ptr(value), _ptr(spatial_shapes), _ptr(level_start_index),
            _ptr(sampling_locations), _ptr(attention_weights), _ptr(out),
            B, S, Q, M, D, L, K, _DTYPE_CODE[value.dtype], _stream(value.device),
        )
    _lib.check("msda_forward", rc)
    return out


def _backward(value, spatial_shapes, level_start_index, sampling_locations, attention_weights,
              grad_out, fp32_grad_accum, algo_flags=0, deterministic=False):
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_locations.shape
    grad_value = torch.empty_like(value)
    grad_loc = torch.empty_like(sampling_locations)
    grad_attn = torch.empty_like(attention_weights)
    lib = _lib.load()
    code = _DTYPE_CODE[value.dtype]
    flags = _bwd_flags(fp32_grad_accum, deterministic, algo_flags)
    ws_bytes = lib.msda_backward_workspace_size(B, S, Q, M, D, L, K, code, flags)
    workspace = (
        torch.empty(ws_bytes, dtype=torch.uint8, device=value.device) if ws_bytes else None
    )
    with _device_guard(value.device):
        rc = lib.msda_backward(
            _ptr(value), _ptr(spatial_shapes), _ptr(level_start_index),
            _ptr(sampling_locations), _ptr(attention_weights), _ptr(grad_out),
            _ptr(grad_value), _ptr(grad_loc), _ptr(grad_attn),
            _ptr(workspace), ws_bytes,
            B, S, Q, M, D, L, K, code, flags, _stream(value.device),
        )
    _lib.check("msda_backward", rc)
    return grad_value, grad_loc, grad_attn


class _MSDAFunction(torch.autograd.Function):
    """Autograd Function with the reference's ``apply`` contract
    (src/msda_triton/ops.py:36-93): ``apply(value, spatial_shapes,
    level_start_index, sampling_locations, attention_weights, fp32_grad_accum)``
    on contiguous CUDA tensors with int64 shapes on the same device, returning
    ``(B, Q, M*D)``; backward returns gradients for value, sampling_locations
    and attention_weights only. An optional 7th argument ``deterministic``
    (default False) selects the bitwise-reproducible grad_value accumulation."""

    @staticmethod
    def forward(ctx, value, spatial_shapes, level_start_index, sampling_locations,
                attention_weights, fp32_grad_accum, deterministic=False):
        B, S, M, D = value.shape
        Q = sampling_locations.shape[1]
        out = _forward(value, spatial_shapes, level_start_index, sampling_locations,
                       attention_weights)
        ctx.save_for_backward(value, spatial_shapes, level_start_index,
                              sampling_locations, attention_weights)
        ctx.fp32_grad_accum = bool(fp32_grad_accum)
        ctx.deterministic = bool(deterministic)
        return out.view(B, Q, M * D)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out):
        value, spatial_shapes, level_start_index, sampling_locations, attention_weights = (
            ctx.saved_tensors
        )
        B, S, M, D = value.shape
        Q = sampling_locations.shape[1]
        grad_out = grad_out.reshape(B, Q, M, D).to(value.dtype).contiguous()
        grad_value, grad_loc, grad_attn = _backward(
            value, spatial_shapes, level_start_index, sampling_locations, attention_weights,
            grad_out, ctx.fp32_grad_accum, deterministic=ctx.deterministic,
        )
        return grad_value, None, None, grad_loc, grad_attn, None, None


class MultiScaleDeformableAttnFunction(torch.autograd.Function):
    """mmcv-compatible Function: ``apply(value, value_spatial_shapes,
    value_level_start_index, sampling_locations, attention_weights,
    im2col_step)`` (the call made at benchmarks/modal_benchmark.py:231-233 of
    the reference). ``im2col_step`` is accepted for signature compatibility
    and ignored: the kernels need no batch chunking. grad_value uses the
    default accumulator policy of :func:`_use_fp32_grad_accum`, deterministic
    when ``torch.use_deterministic_algorithms(True)`` is in effect."""

    @staticmethod
    def forward(ctx, value, value_spatial_shapes, value_level_start_index,
                sampling_locations, attention_weights, im2col_step=64):
        value = value.contiguous()
        sampling_locations = sampling_locations.contiguous()
        attention_weights = attention_weights.contiguous()
        shapes = value_spatial_shapes.to(device=value.device, dtype=torch.int64).contiguous()
        starts = value_level_start_index.to(device=value.device, dtype=torch.int64).contiguous()
        B, S, M, D = value.shape
        Q = sampling_locations.shape[1]
        out = _forward(value, shapes, starts, sampling_locations, attention_weights)
        ctx.save_for_backward(value, shapes, starts, sampling_locations, attention_weights)
        ctx.fp32_grad_accum = _use_fp32_grad_accum(value)
        ctx.deterministic = _use_deterministic(None)
        return out.view(B, Q, M * D)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out):
        value, shapes, starts, sampling_locations, attention_weights = ctx.saved_tensors
        B, S, M, D = value.shape
        Q = sampling_locations.shape[1]
        grad_out = grad_out.reshape(B, Q, M, D).to(value.dtype).contiguous()
        grad_value, grad_loc, grad_attn = _backward(
            value, shapes, starts, sampling_locations, attention_weights, grad_out,
            ctx.fp32_grad_accum, deterministic=ctx.deterministic,
        )
        return grad_value, None, None, grad_loc, grad_attn, None


def multi_scale_deformable_attention(
    value: torch.Tensor,
    spatial_shapes: torch.Tensor,
    level_start_index: torch.Tensor | None,
    sampling_locations: torch.Tensor,
    attention_weights: torch.Tensor,
    *,
    fp32_grad_accum: bool | None = None,
    deterministic: bool | None = None,
) -> torch.Tensor:
    """Multi-scale deformable attention (Zhu et al. 2021, Eq. 1) on B200.

    Drop-in for ``msda_triton.multi_scale_deformable_attention``
    (src/msda_triton/ops.py:96-199): same arguments, same validation and error
    messages, same output.

    For each query, head, feature level l and sampling point k, bilinearly
    samples ``value`` at ``sampling_locations`` and sums the samples weighted
    by ``attention_weights``. Sampling uses ``x_im = x * W_l - 0.5`` (==
    ``grid_sample(align_corners=False, padding_mode="zeros")``).

    Args:
        value: ``(B, S, M, D)`` flattened multi-scale feature maps,
            ``S = sum_l H_l * W_l``.
        spatial_shapes: ``(L, 2)`` integer ``(H_l, W_l)`` per level.
        level_start_index: ``(L,)`` offset of each level along ``S``, or
            ``None`` to derive it from ``spatial_shapes``.
        sampling_locations: ``(B, Q, M, L, K, 2)`` normalised ``(x, y)``;
            locations outside ``[0, 1]`` sample zeros.
        attention_weights: ``(B, Q, M, L, K)``.
        fp32_grad_accum: accumulate ``grad_value`` in fp32 and downcast once
            (``True``) or with native packed half-precision atomics
            (``False``). ``None`` picks fp32 for fp16/bf16 (see
            :func:`_use_fp32_grad_accum`); fp32 inputs always accumulate in
            fp32.
        deterministic: accumulate ``grad_value`` as exact integer sums
            (integer-valued fp32 rows, or 64-bit fixed point) so the backward
            is bitwise reproducible (no counterpart in the
            reference; ``fp32_grad_accum`` is then moot). ``None`` follows
            ``torch.are_deterministic_algorithms_enabled()``.

    Returns:
        ``(B, Q, M * D)`` output in ``value.dtype``.

    Note:
        Unless ``deterministic``, ``grad_value`` is accumulated with fp32 (or
        native) atomics, so the backward is not bitwise deterministic from
        run to run (as in the reference).
    """
    if value.dim() != 4:
        raise ValueError(f"value must be (B, S, M, D), got {tuple(value.shape)}")
    if sampling_locations.dim() != 6 or sampling_locations.shape[-1] != 2:
        raise ValueError(
            f"sampling_locations must be (B, Q, M, L, K, 2), got {tuple(sampling_locations.shape)}"
        )
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_locations.shape
    if sampling_locations.shape[0] != B or sampling_locations.shape[2] != M:
        raise ValueError(
            f"sampling_locations {tuple(sampling_locations.shape)} inconsistent with value "
            f"{tuple(value.shape)}"
        )
    if attention_weights.shape != (B, Q, M, L, K):
        raise ValueError(
            f"attention_weights must be {(B, Q, M, L, K)}, got {tuple(attention_weights.shape)}"
        )
    if spatial_shapes.shape != (L, 2):
        raise ValueError(f"spatial_shapes must be ({L}, 2), got {tuple(spatial_shapes.shape)}")
    if not (value.dtype == sampling_locations.dtype == attention_weights.dtype):
        raise ValueError(
            f"value/sampling_locations/attention_weights dtypes must match, got "
            f"{value.dtype}/{sampling_locations.dtype}/{attention_weights.dtype}"
        )
    if value.dtype not in _FLOAT_DTYPES:
        raise ValueError(f"unsupported dtype {value.dtype}; use fp32, fp16 or bf16")
    if value.device.type != "cuda":
        raise ValueError(
            "the operator requires CUDA tensors on a B200 (sm_100a) GPU; MPS (Apple GPU) "
            "and CPU tensors are not supported -- on CPU use a grid_sample-based "
            "implementation"
        )
    if sampling_locations.device != value.device or attention_weights.device != value.device:
        raise ValueError(
            f"value, sampling_locations and attention_weights must be on the same CUDA device, "
            f"got {value.device}/{sampling_locations.device}/{attention_weights.device}"
        )
    _lib.load()  # RuntimeError if the CUDA library is missing

    spatial_shapes, level_start_index = _level_tables(spatial_shapes, level_start_index, value, L, S)

    if B == 0 or Q == 0:
        return value.new_zeros(B, Q, M * D)

    if fp32_grad_accum is None:
        fp32_grad_accum = _use_fp32_grad_accum(value)

    return _MSDAFunction.apply(
        value.contiguous(),
        spatial_shapes,
        level_start_index,
        sampling_locations.contiguous(),
        attention_weights.contiguous(),
        fp32_grad_accum,
        _use_deterministic(deterministic),
    )


def _level_tables(spatial_shapes, level_start_index, value, L, S):
    """int64 (L, 2) shapes and (L,) level starts on value's device (starts
    derived from the shapes when None), checked against S when on the host."""
    shapes_host = spatial_shapes if spatial_shapes.device.type == "cpu" else None
    spatial_shapes = spatial_shapes.to(device=value.device, dtype=torch.int64).contiguous()
    if level_start_index is None:
        hw = spatial_shapes.prod(-1)
        level_start_index = torch.cat([hw.new_zeros(1), hw.cumsum(0)[:-1]])
        starts_host = None
        if shapes_host is not None:
            hw_h = shapes_host.to(torch.int64).prod(-1)
            starts_host = torch.cat([hw_h.new_zeros(1), hw_h.cumsum(0)[:-1]])
    else:
        if level_start_index.shape != (L,):
            raise ValueError(
                f"level_start_index must be ({L},), got {tuple(level_start_index.shape)}"
            )
        starts_host = level_start_index if level_start_index.device.type == "cpu" else None
        level_start_index = level_start_index.to(
            device=value.device, dtype=torch.int64
        ).contiguous()
    # The reference reads out of bounds when a level extends past S; here the
    # kernels treat such a level as empty, and when the shapes are on the host
    # (no device sync needed) the mismatch is reported up front.
    if shapes_host is not None and starts_host is not None and L > 0:
        ends = starts_host.to(torch.int64) + shapes_host.to(torch.int64).prod(-1)
        if int(ends.max()) > S:
            raise ValueError(
                f"spatial_shapes/level_start_index address {int(ends.max())} value rows but "
                f"value has S={S}"
            )
    return spatial_shapes, level_start_index


# ---------------------------------------------------------------------------
# Fused prologue: reference points + offsets and attention logits
# ---------------------------------------------------------------------------
def _forward_fused(value, spatial_shapes, level_start_index, reference_points, sampling_offsets,
                   attention_logits):
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_offsets.shape
    out = value.new_empty(B, Q, M, D)
    lib = _lib.load()
    with _device_guard(value.device):
        rc = lib.msda_forward_fused(
            _ptr(value), _ptr(spatial_shapes), _ptr(level_start_index), _ptr(reference_points),
            _ptr(sampling_offsets), _ptr(attention_logits), _ptr(out),
            B, S, Q, M, D, L, K, _DTYPE_CODE[value.dtype], _stream(value.device),
        )
    _lib.check("msda_forward_fused", rc)
    return out


def _backward_fused(value, spatial_shapes, level_start_index, reference_points, sampling_offsets,
                    attention_logits, grad_out, fp32_grad_accum, algo_flags=0, deterministic=False):
    """(grad_value, grad_offsets, grad_logits) of the fused forward."""
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_offsets.shape
    grad_value = torch.empty_like(value)
    grad_off = torch.empty_like(sampling_offsets)
    grad_logits = torch.empty_like(attention_logits)
    lib = _lib.load()
    code = _DTYPE_CODE[value.dtype]
    flags = _bwd_flags(fp32_grad_accum, deterministic, algo_flags)
    ws_bytes = lib.msda_backward_workspace_size(B, S, Q, M, D, L, K, code, flags)
    workspace = (
        torch.empty(ws_bytes, dtype=torch.uint8, device=value.device) if ws_bytes else None
    )
    with _device_guard(value.device):
        rc = lib.msda_backward_fused(
            _ptr(value), _ptr(spatial_shapes), _ptr(level_start_index), _ptr(reference_points),
            _ptr(sampling_offsets), _ptr(attention_logits), _ptr(grad_out),
            _ptr(grad_value), _ptr(grad_off), _ptr(grad_logits), _ptr(workspace), ws_bytes,
            B, S, Q, M, D, L, K, code, flags, _stream(value.device),
        )
    _lib.check("msda_backward_fused", rc)
    return grad_value, grad_off, grad_logits


class _MSDAFusedFunction(torch.autograd.Function):
    """Autograd Function of :func:`multi_scale_deformable_attention_fused`."""

    @staticmethod
    def forward(ctx, value, spatial_shapes, level_start_index, reference_points, sampling_offsets,
                attention_logits, fp32_grad_accum, deterministic=False):
        B, S, M, D = value.shape
        Q = sampling_offsets.shape[1]
        out = _forward_fused(value, spatial_shapes, level_start_index, reference_points,
                             sampling_offsets, attention_logits)
        ctx.save_for_backward(value, spatial_shapes, level_start_index, reference_points,
                              sampling_offsets, attention_logits)
        ctx.fp32_grad_accum = bool(fp32_grad_accum)
        ctx.deterministic = bool(deterministic)
        return out.view(B, Q, M * D)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out):
        value, shapes, starts, ref, off, logits = ctx.saved_tensors
        B, S, M, D = value.shape
        Q = off.shape[1]
        grad_out = grad_out.reshape(B, Q, M, D).to(value.dtype).contiguous()
        if grad_out.data_ptr() % 16:  # the fused kernels read 16-byte vectors
            grad_out = grad_out.clone()
        grad_value, grad_off, grad_logits = _backward_fused(
            value, shapes, starts, ref, off, logits, grad_out, ctx.fp32_grad_accum,
            deterministic=ctx.deterministic)
        grad_ref = None
        if ctx.needs_input_grad[3]:
            # location = ref + offset / (W_l, H_l): d/dref = sum over (m, l, k)
            # of d/doffset * (W_l, H_l).
            wh = shapes.flip(-1).to(torch.float32)  # (L, 2)
            grad_ref = (grad_off.float() * wh[:, None, :]).sum(dim=(2, 3, 4)).to(ref.dtype)
        return grad_value, None, None, grad_ref, grad_off, grad_logits, None, None


def multi_scale_deformable_attention_fused(
    value: torch.Tensor,
    spatial_shapes: torch.Tensor,
    level_start_index: torch.Tensor | None,
    reference_points: torch.Tensor,
    sampling_offsets: torch.Tensor,
    attention_logits: torch.Tensor,
    *,
    fp32_grad_accum: bool | None = None,
    deterministic: bool | None = None,
) -> torch.Tensor:
    """Multi-scale deformable attention with the Deformable-DETR layer's
    prologue fused in (the prologue of the reference's layer,
    labs/solutions/lab00.py:199-208, followed by the operator).

    Equivalent to ``multi_scale_deformable_attention(value, spatial_shapes,
    level_start_index, reference_points[:, :, None, None, None, :] +
    sampling_offsets / (W_l, H_l), attention_logits.softmax over (L, K))``
    without materialising the locations and weights.

    Args:
        value: ``(B, S, M, D)``.
        spatial_shapes: ``(L, 2)`` ``(H_l, W_l)``; level_start_index as in
            :func:`multi_scale_deformable_attention`.
        reference_points: ``(B, Q, 2)`` normalised ``(x, y)``.
        sampling_offsets: ``(B, Q, M, L, K, 2)`` in pixels of each level.
        attention_logits: ``(B, Q, M, L, K)``, softmaxed jointly over
            ``(L, K)`` per query and head.
        fp32_grad_accum, deterministic: as in
            :func:`multi_scale_deformable_attention`.

    Returns:
        ``(B, Q, M * D)`` in ``value.dtype``; differentiable with respect to
        value, reference_points, sampling_offsets and attention_logits.
    """
    if value.dim() != 4:
        raise ValueError(f"value must be (B, S, M, D), got {tuple(value.shape)}")
    if sampling_offsets.dim() != 6 or sampling_offsets.shape[-1] != 2:
        raise ValueError(
            f"sampling_offsets must be (B, Q, M, L, K, 2), got {tuple(sampling_offsets.shape)}")
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_offsets.shape
    if sampling_offsets.shape[0] != B or sampling_offsets.shape[2] != M:
        raise ValueError(f"sampling_offsets {tuple(sampling_offsets.shape)} inconsistent with value "
                         f"{tuple(value.shape)}")
    if reference_points.shape != (B, Q, 2):
        raise ValueError(f"reference_points must be {(B, Q, 2)}, got {tuple(reference_points.shape)}")
    if attention_logits.shape != (B, Q, M, L, K):
        raise ValueError(
            f"attention_logits must be {(B, Q, M, L, K)}, got {tuple(attention_logits.shape)}")
    if spatial_shapes.shape != (L, 2):
        raise ValueError(f"spatial_shapes must be ({L}, 2), got {tuple(spatial_shapes.shape)}")
    if not (value.dtype == reference_points.dtype == sampling_offsets.dtype == attention_logits.dtype):
        raise ValueError("value/reference_points/sampling_offsets/attention_logits dtypes must match, "
                         f"got {value.dtype}/{reference_points.dtype}/{sampling_offsets.dtype}/"
                         f"{attention_logits.dtype}")
    if value.dtype not in _FLOAT_DTYPES:
        raise ValueError(f"unsupported dtype {value.dtype}; use fp32, fp16 or bf16")
    if value.device.type != "cuda":
        raise ValueError("the operator requires CUDA tensors on a B200 (sm_100a) GPU; MPS (Apple GPU) "
                         "and CPU tensors are not supported")
    if any(t.device != value.device for t in (reference_points, sampling_offsets, attention_logits)):
        raise ValueError("value, reference_points, sampling_offsets and attention_logits must be on "
                         "the same CUDA device")
    _lib.load()
    spatial_shapes, level_start_index = _level_tables(spatial_shapes, level_start_index, value, L, S)
    if B == 0 or Q == 0:
        return value.new_zeros(B, Q, M * D)
    if fp32_grad_accum is None:
        fp32_grad_accum = _use_fp32_grad_accum(value)
    if D % (16 // value.element_size()) or value.data_ptr() % 16:
        # The fused kernels run on the 16-byte vector path only; otherwise the
        # prologue is formed with tensor operations before the operator.
        wh = spatial_shapes.flip(-1).to(value.dtype)
        locations = reference_points[:, :, None, None, None, :] + sampling_offsets / wh[:, None, :]
        weights = attention_logits.reshape(B, Q, M, L * K).softmax(-1).view(B, Q, M, L, K)
        return multi_scale_deformable_attention(value, spatial_shapes, level_start_index,
                                                locations, weights, fp32_grad_accum=fp32_grad_accum,
                                                deterministic=deterministic)
    return _MSDAFusedFunction.apply(
        value.contiguous(), spatial_shapes, level_start_index, reference_points.contiguous(),
        sampling_offsets.contiguous(), attention_logits.contiguous(), fp32_grad_accum,
        _use_deterministic(deterministic),
    )

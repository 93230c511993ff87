"""MSDA oracle -- TEST INFRASTRUCTURE ONLY.

A CPU restatement of the reference operator roulbac/msda-triton, used as the
checker for the sm_100a kernels. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU legs (``cpu_baseline`` and ``--impl reference``) may
import this module; the product path (``msda_triton_b200``) never does.

Contents, each restating one reference function:

* :func:`msda_grid_sample` -- per-level ``F.grid_sample`` formulation of the
  reference's CPU implementation ``msda_reference``
  (tests/reference_impls.py:12-45); differentiable through autograd, so its
  backward is torch's grid_sample backward.
* :func:`msda_loops` -- pure-Python loop specification ``msda_naive``
  (tests/reference_impls.py:48-87); tiny inputs only.
* :func:`msda_backward_analytic` -- hand-derived gradients with an
  ``index_add_`` scatter (labs/solutions/lab07.py:12-104), following the
  backward maths of src/msda_triton/kernels.py:205-291.
* :func:`reference_fp32` -- fp32 CPU forward/backward on detached copies
  (tests/test_msda.py:80-93), the comparison target of the parity tests.

Pinning: tests/test_oracle.py checks every function here against golden
vectors produced by the reference's own code (its grid_sample implementation
and its Triton kernels run under ``TRITON_INTERPRET=1``), committed under
tests/golden/ together with tests/golden/make_golden.py.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def level_starts(spatial_shapes: torch.Tensor) -> torch.Tensor:
    """Exclusive prefix sum of H_l * W_l (reference: src/msda_triton/ops.py:174-176)."""
    hw = spatial_shapes.to(torch.int64).prod(-1)
    return torch.cat([hw.new_zeros(1), hw.cumsum(0)[:-1]])


def msda_grid_sample(value, spatial_shapes, sampling_locations, attention_weights):
    """Forward via one ``grid_sample`` per level (tests/reference_impls.py:12-45).

    ``grid_sample(align_corners=False)`` maps a grid coordinate g in [-1, 1] to
    the pixel coordinate ((g + 1) * W - 1) / 2, which for g = 2x - 1 is
    x * W - 0.5: the operator's convention. Returns ``(B, Q, M * D)``.
    """
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_locations.shape
    hw = [(int(h), int(w)) for h, w in spatial_shapes.tolist()]
    start = 0
    total = None
    for lvl, (h, w) in enumerate(hw):
        # (B, H*W, M, D) -> (B*M, D, H, W)
        img = value[:, start:start + h * w].permute(0, 2, 3, 1).reshape(B * M, D, h, w)
        start += h * w
        # (B, Q, M, K, 2) -> (B*M, Q, K, 2), [0, 1] -> [-1, 1]
        grid = sampling_locations[:, :, :, lvl].permute(0, 2, 1, 3, 4).reshape(B * M, Q, K, 2)
        samples = F.grid_sample(img, grid * 2 - 1, mode="bilinear", padding_mode="zeros",
                                align_corners=False)  # (B*M, D, Q, K)
        weights = attention_weights[:, :, :, lvl].permute(0, 2, 1, 3).reshape(B * M, 1, Q, K)
        part = (samples * weights).sum(-1)  # (B*M, D, Q)
        total = part if total is None else total + part
    # (B*M, D, Q) -> (B, Q, M*D)
    return total.reshape(B, M, D, Q).permute(0, 3, 1, 2).reshape(B, Q, M * D)


def msda_loops(value, spatial_shapes, sampling_locations, attention_weights):
    """Scalar loop specification (tests/reference_impls.py:48-87): hand-rolled
    bilinear interpolation with zero padding. O(B*Q*M*L*K*D) Python work:
    tiny inputs only. Returns ``(B, Q, M * D)`` in value's dtype."""
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_locations.shape
    hw = [(int(h), int(w)) for h, w in spatial_shapes.tolist()]
    starts = [0]
    for h, w in hw[:-1]:
        starts.append(starts[-1] + h * w)
    v = value.tolist()
    loc = sampling_locations.tolist()
    att = attention_weights.tolist()
    out = [[[[0.0] * D for _ in range(M)] for _ in range(Q)] for _ in range(B)]
    for b in range(B):
        for q in range(Q):
            for m in range(M):
                acc = out[b][q][m]
                for lvl in range(L):
                    h, w = hw[lvl]
                    for k in range(K):
                        px = loc[b][q][m][lvl][k][0] * w - 0.5
                        py = loc[b][q][m][lvl][k][1] * h - 0.5
                        a = att[b][q][m][lvl][k]
                        x0, y0 = math.floor(px), math.floor(py)
                        fx, fy = px - x0, py - y0
                        for yy, xx, wt in ((y0, x0, (1 - fx) * (1 - fy)),
                                           (y0, x0 + 1, fx * (1 - fy)),
                                           (y0 + 1, x0, (1 - fx) * fy),
                                           (y0 + 1, x0 + 1, fx * fy)):
                            if 0 <= xx < w and 0 <= yy < h:
                                row = v[b][starts[lvl] + yy * w + xx][m]
                                for d in range(D):
                                    acc[d] += a * wt * row[d]
    return torch.tensor(out, dtype=value.dtype).reshape(B, Q, M * D)


def msda_backward_analytic(value, spatial_shapes, level_start_index, sampling_locations,
                           attention_weights, grad_out, coord_dtype=None):
    """Hand-derived gradients (labs/solutions/lab07.py:12-104; maths of
    src/msda_triton/kernels.py:253-291), vectorised over (B, Q, M) and looped
    over (l, k), computed in the dtype of ``value`` (pass float64 for a
    high-precision check). ``coord_dtype=torch.float32`` rounds the pixel
    coordinates x = loc*W - 0.5 to fp32 once, as the reference's fp32 kernel
    arithmetic does (src/msda_triton/kernels.py:112-113, one fused
    multiply-add), and keeps everything after that in the working dtype.
    Returns (grad_value (B,S,M,D), grad_loc (B,Q,M,L,K,2), grad_attn
    (B,Q,M,L,K)) on the device of ``value`` (a test may run this checker on
    the GPU in float64 when the CPU would take minutes)."""
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = sampling_locations.shape
    dt = value.dtype
    dev = value.device
    flat = value.reshape(-1)
    loc = sampling_locations.to(device=dev, dtype=dt)
    att = attention_weights.to(device=dev, dtype=dt)
    g = grad_out.reshape(B, Q, M, D).to(device=dev, dtype=dt)
    grad_value = torch.zeros(B * S * M * D, dtype=dt, device=dev)
    grad_loc = torch.zeros(B, Q, M, L, K, 2, dtype=dt, device=dev)
    grad_attn = torch.zeros(B, Q, M, L, K, dtype=dt, device=dev)
    bi = torch.arange(B, device=dev).view(B, 1, 1)
    mi = torch.arange(M, device=dev).view(1, 1, M)
    di = torch.arange(D, device=dev)
    for lvl in range(L):
        h = int(spatial_shapes[lvl, 0])
        w = int(spatial_shapes[lvl, 1])
        st = int(level_start_index[lvl])
        for k in range(K):
            px = loc[:, :, :, lvl, k, 0] * w - 0.5
            py = loc[:, :, :, lvl, k, 1] * h - 0.5
            if coord_dtype is not None:
                px = px.to(coord_dtype).to(dt)
                py = py.to(coord_dtype).to(dt)
            a = att[:, :, :, lvl, k]
            x0f, y0f = torch.floor(px), torch.floor(py)
            fx, fy = px - x0f, py - y0f
            x0, y0 = x0f.long(), y0f.long()
            corners = []
            for dy, dx, wt in ((0, 0, (1 - fx) * (1 - fy)), (0, 1, fx * (1 - fy)),
                               (1, 0, (1 - fx) * fy), (1, 1, fx * fy)):
                xx, yy = x0 + dx, y0 + dy
                ok = (xx >= 0) & (xx < w) & (yy >= 0) & (yy < h)
                pix = st + yy.clamp(0, h - 1) * w + xx.clamp(0, w - 1)
                idx = ((bi * S + pix) * M + mi) * D  # (B, Q, M) element offset of channel 0
                gidx = idx.unsqueeze(-1) + di
                vals = flat[gidx] * ok.unsqueeze(-1).to(dt)
                corners.append((gidx, ok, wt, vals))
            (_, _, w00, v00), (_, _, w01, v01), (_, _, w10, v10), (_, _, w11, v11) = corners
            sampled = (v00 * w00[..., None] + v01 * w01[..., None]
                       + v10 * w10[..., None] + v11 * w11[..., None])
            grad_attn[:, :, :, lvl, k] = (g * sampled).sum(-1)
            ddx = (v01 - v00) * (1 - fy)[..., None] + (v11 - v10) * fy[..., None]
            ddy = (v10 - v00) * (1 - fx)[..., None] + (v11 - v01) * fx[..., None]
            grad_loc[:, :, :, lvl, k, 0] = a * w * (g * ddx).sum(-1)
            grad_loc[:, :, :, lvl, k, 1] = a * h * (g * ddy).sum(-1)
            ga = g * a[..., None]
            for gidx, ok, wt, _ in corners:
                contrib = ga * (wt * ok.to(dt))[..., None]
                grad_value.index_add_(0, gidx.reshape(-1), contrib.reshape(-1))
    return grad_value.view(B, S, M, D), grad_loc, grad_attn


def reference_fp32(value, spatial_shapes, sampling_locations, attention_weights, grad_out=None):
    """fp32 CPU forward (and backward when ``grad_out`` is given) on detached
    fp32 copies, whatever device/dtype the inputs have (tests/test_msda.py:80-93).
    Returns CPU ``(out, (grad_value, grad_loc, grad_attn) or None)``."""
    shapes = spatial_shapes.detach().cpu()
    v = value.detach().float().cpu().requires_grad_(grad_out is not None)
    l = sampling_locations.detach().float().cpu().requires_grad_(grad_out is not None)
    a = attention_weights.detach().float().cpu().requires_grad_(grad_out is not None)
    out = msda_grid_sample(v, shapes, l, a)
    if grad_out is None:
        return out.detach(), None
    out.backward(grad_out.detach().float().cpu())
    return out.detach(), (v.grad, l.grad, a.grad)

"""Shared test inputs: the reference suite's seeded generator, its cases and
its tolerances (tests/test_msda.py:43-77 of roulbac/msda-triton), restated."""

from __future__ import annotations

import hashlib

import numpy as np
import torch

# Forward tolerances vs the fp32 reference (tests/test_msda.py:43-48) ...
REF_FWD_TOL = {
    torch.float32: dict(rtol=1e-5, atol=1e-5),
    torch.float16: dict(rtol=5e-3, atol=5e-3),
    torch.bfloat16: dict(rtol=3e-2, atol=3e-2),
}
# ... and backward tolerances (tests/test_msda.py:49-55).
REF_BWD_TOL = {
    torch.float32: dict(rtol=1e-4, atol=1e-4),
    torch.float16: dict(rtol=3e-2, atol=3e-2),
    torch.bfloat16: dict(rtol=8e-2, atol=8e-2),
}
# The stricter bar this build is held to (forward output and all three
# gradients): fp32 atol 1e-5 / rtol 1e-4; fp16/bf16 within 1e-2 relative to
# the fp32 reference. The half-precision atol only absorbs fp32 reordering
# noise on results that cancel to ~0; every non-tiny element is held to 1%.
STRICT_TOL = {
    torch.float32: dict(rtol=1e-4, atol=1e-5),
    torch.float16: dict(rtol=1e-2, atol=1e-4),
    torch.bfloat16: dict(rtol=1e-2, atol=1e-4),
}

# tests/test_msda.py:57-62
CASES = [
    dict(id="decoder", B=2, Q=100, M=4, D=32, K=4, shapes=[(24, 32), (12, 16), (6, 8)]),
    dict(id="single_level_point", B=1, Q=17, M=1, D=16, K=1, shapes=[(13, 9)]),
    dict(id="nonpow2_D", B=2, Q=33, M=2, D=24, K=3, shapes=[(10, 14), (5, 7)]),
    dict(id="wide", B=1, Q=64, M=8, D=64, K=4, shapes=[(16, 16), (8, 8)]),
]

# labs/common/checks.py:71-75
LAB_CASES = [
    dict(B=2, Q=5, M=2, D=4, shapes=[(5, 7), (3, 4)], K=3),
    dict(B=1, Q=7, M=1, D=3, shapes=[(4, 6)], K=1),
    dict(B=1, Q=4, M=2, D=5, shapes=[(6, 5), (3, 3)], K=2, loc_lo=-0.4, loc_hi=1.4),
]


def case_kwargs(case: dict) -> dict:
    return {k: v for k, v in case.items() if k != "id"}


def make_inputs(B, Q, M, D, shapes, K, dtype, device, loc_lo=0.0, loc_hi=1.0, seed=0):
    """Seeded inputs exactly as tests/test_msda.py:65-77 draws them: one CPU
    generator, value ~ N(0,1), loc ~ U[lo,hi), attn = softmax of U[0,1)
    logits over L*K; then cast/moved. Returns (value, shapes, starts, loc, attn)."""
    gen = torch.Generator().manual_seed(seed)
    L = len(shapes)
    S = sum(h * w for h, w in shapes)
    value = torch.randn(B, S, M, D, generator=gen).to(device, dtype)
    loc = loc_lo + (loc_hi - loc_lo) * torch.rand(B, Q, M, L, K, 2, generator=gen)
    loc = loc.to(device, dtype)
    attn = torch.rand(B, Q, M, L, K, generator=gen)
    attn = attn.flatten(3).softmax(-1).view(B, Q, M, L, K).to(device, dtype)
    spatial_shapes = torch.tensor(shapes, dtype=torch.long, device=device)
    hw = spatial_shapes.prod(-1)
    starts = torch.cat([hw.new_zeros(1), hw.cumsum(0)[:-1]])
    return value, spatial_shapes, starts, loc, attn


def exact_corner_locations(shape, dtype=torch.float64):
    """Locations drawn from {0, 0.5, 1} (tests/test_msda.py:116-117)."""
    grid_vals = torch.tensor([0.0, 0.5, 1.0], dtype=dtype)
    return grid_vals[torch.randint(0, 3, shape, generator=torch.Generator().manual_seed(1))]


def grad_output_like(out: torch.Tensor, seed: int = 7) -> torch.Tensor:
    """grad_out as tests/test_msda.py:193-195 draws it (CPU generator, seed 7)."""
    return torch.randn(out.shape, generator=torch.Generator().manual_seed(seed)).to(
        out.device, out.dtype)


def digest(t: torch.Tensor) -> str:
    """sha256 of a tensor's bytes (contiguous CPU copy; bf16 viewed as int16)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def unpack_golden(npz, name: str):
    """Golden arrays are stored in full (``name``) or as a seeded sample of
    flat indices (``name__idx`` / ``name__val``) plus ``name__sum`` and
    ``name__sumsq``. Returns (kind, payload)."""
    if name in npz:
        return "full", np.asarray(npz[name])
    return "sampled", (np.asarray(npz[name + "__idx"]), np.asarray(npz[name + "__val"]),
                       float(npz[name + "__sum"]), float(npz[name + "__sumsq"]),
                       tuple(int(x) for x in npz[name + "__shape"]))


def assert_matches_golden(actual: torch.Tensor, npz, name: str, rtol: float, atol: float):
    kind, payload = unpack_golden(npz, name)
    a = actual.detach().cpu().double()
    if kind == "full":
        torch.testing.assert_close(a, torch.from_numpy(payload).double(), rtol=rtol, atol=atol,
                                   msg=lambda m: f"{name}: {m}")
        return
    idx, val, s, ss, shape = payload
    assert tuple(a.shape) == shape, f"{name}: shape {tuple(a.shape)} != {shape}"
    flat = a.reshape(-1)
    torch.testing.assert_close(flat[torch.from_numpy(idx)], torch.from_numpy(val).double(),
                               rtol=rtol, atol=atol, msg=lambda m: f"{name} (sampled): {m}")
    n = flat.numel()
    tol_sum = atol * n ** 0.5 + rtol * abs(s) + 1e-9
    assert abs(float(flat.sum()) - s) <= tol_sum * 10, f"{name}: sum {float(flat.sum())} != {s}"
    assert abs(float((flat * flat).sum()) - ss) <= (rtol * 4 + 1e-9) * ss + atol * n, (
        f"{name}: sum of squares {float((flat * flat).sum())} != {ss}")


# ---------------------------------------------------------------------------
# Gradient comparison helpers
# ---------------------------------------------------------------------------
def pixel_scale(shapes: torch.Tensor, K: int) -> torch.Tensor:
    """(L, K, 2) float64 factors (W_l, H_l): grad_loc / pixel_scale is the
    gradient with respect to pixel coordinates. grad_loc itself grows with the
    level resolution (tests/test_msda.py:49-51 of the reference makes the same
    point), so absolute tolerances are applied in pixel units."""
    s = shapes.detach().cpu().to(torch.float64)
    wh = torch.stack([s[:, 1], s[:, 0]], -1)  # (L, 2) = (W, H)
    return wh[:, None, :].expand(s.shape[0], K, 2)


def kink_mask(loc: torch.Tensor, shapes: torch.Tensor, eps: float = 1e-3) -> torch.Tensor:
    """(B, Q, M, L, K) True where a sampling point's pixel coordinate
    x = loc*W - 0.5 (or y) lies within eps of an integer. There the bilinear
    interpolant has a kink: grad_loc jumps between two one-sided derivatives,
    and implementations whose coordinate arithmetic rounds differently by an
    ulp (grid_sample vs loc*W - 0.5, fma vs mul+sub) legitimately disagree."""
    l = loc.detach().cpu().double()
    K = l.shape[-2]
    px = l * pixel_scale(shapes, K) - 0.5
    return ((px - px.round()).abs() < eps).any(-1)


def assert_native_grad_value_close(gv, ref, what=""):
    """grad_value accumulated with native fp16/bf16 reductions. Each hit
    rounds the running sum to 16 bits, in the order the atomics land, so an
    element whose contributions cancel can sit far from the exact sum relative
    to itself (the reason fp32 accumulation is the default). Held normwise
    instead: ||gv - ref|| <= 3e-2 ||ref|| (bf16 measured 1.7e-2 at the
    encoder point and up to 2.6e-2 on clustered sampling), and every element
    within 8e-2 of max|ref| (the reference suite's bf16 tolerance, relative
    to the tensor's scale)."""
    d = (gv.double().cpu() - ref.double().cpu())
    scale = ref.double().abs().max().item()
    norm_err = d.norm().item() / max(ref.double().norm().item(), 1e-30)
    assert norm_err <= 3e-2, f"{what} grad_value (native): normwise error {norm_err:.3g} > 3e-2"
    worst = d.abs().max().item()
    assert worst <= 8e-2 * scale, f"{what} grad_value (native): max error {worst:.3g} > 8e-2 * {scale:.3g}"


def assert_grads_close(got, ref, loc, shapes, tol, gl_tol=None, gv_tol=None, what="", native_gv=False):
    """Compare (grad_value, grad_loc, grad_attn): grad_loc in pixel units. For
    fp32 locations, kink points are excluded from the grad_loc comparison (at
    most 1% of points may be); fp16/bf16 locations make x = loc*W - 0.5 exact
    in fp32 for every implementation, so nothing is excluded for them."""
    gv, gl, ga = got
    gv_r, gl_r, ga_r = ref
    kw = lambda t: dict(rtol=t["rtol"], atol=t["atol"])  # noqa: E731
    if native_gv:
        assert_native_grad_value_close(gv, gv_r, what)
    else:
        torch.testing.assert_close(gv.double().cpu(), gv_r.double().cpu(), **kw(gv_tol or tol),
                                   msg=lambda m: f"{what} grad_value: {m}")
    torch.testing.assert_close(ga.double().cpu(), ga_r.double().cpu(), **kw(tol),
                               msg=lambda m: f"{what} grad_attn: {m}")
    K = loc.shape[-2]
    scale = pixel_scale(shapes, K)
    if loc.dtype == torch.float32:
        keep = ~kink_mask(loc, shapes)
    else:
        keep = torch.ones(loc.shape[:-1], dtype=torch.bool)
    assert keep.double().mean() > 0.99, f"{what}: too many kink points ({(~keep).sum()})"
    a = (gl.double().cpu() / scale)[keep]
    b = (gl_r.double().cpu() / scale)[keep]
    torch.testing.assert_close(a, b, **kw(gl_tol or tol), msg=lambda m: f"{what} grad_loc (px): {m}")

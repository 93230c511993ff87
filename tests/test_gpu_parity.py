"""Parity of the sm_100a kernels with the reference, through the public op and
the C ABI (GPU only). Mirrors tests/test_msda.py of roulbac/msda-triton
(forward :128-150, backward :179-227, options :153-170 and :230-246,
validation :254-271) and adds the benchmark operating points (small,
decoder, encoder, Mask2Former and the scaling sweep's shapes) at full size,
the reference Triton kernels' own outputs (golden vectors), and edge cases.

Tolerances: the reference suite's (tests/cases.py REF_*_TOL) and the
stricter bar of this build (STRICT_TOL: fp32 rtol 1e-4 / atol 1e-5; fp16 and
bf16 within 1e-2 relative of the fp32 reference, on the forward output and
all three gradients).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from cases import CASES, REF_BWD_TOL, REF_FWD_TOL, STRICT_TOL
from msda_triton_b200 import MultiScaleDeformableAttnFunction, multi_scale_deformable_attention, presets
from oracle import msda_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = [torch.float32, torch.float16, torch.bfloat16]
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _lib_loaded(cuda_lib):
    yield


def run_op(value, shapes, starts, loc, attn, grad_out=None, **kw):
    v = value.detach().clone().requires_grad_(grad_out is not None)
    l = loc.detach().clone().requires_grad_(grad_out is not None)
    a = attn.detach().clone().requires_grad_(grad_out is not None)
    out = multi_scale_deformable_attention(v, shapes, starts, l, a, **kw)
    if grad_out is None:
        return out.detach(), None
    out.backward(grad_out)
    return out.detach(), (v.grad, l.grad, a.grad)


def close(actual, expected, tol, what=""):
    torch.testing.assert_close(actual.double().cpu(), expected.double().cpu(), **tol,
                               msg=lambda m: f"{what}: {m}")


def fp32_rounded_locations(loc, shapes):
    """float64 locations whose pixel coordinates are the reference's fp32
    ones: x = fma(loc, W, -0.5) rounded once to fp32
    (src/msda_triton/kernels.py:112-113), mapped back as (x + 0.5) / W, so
    grid_sample's x = loc * W - 0.5 in float64 reproduces them. fp16/bf16
    locations give exact coordinates either way and are returned as they are."""
    loc64 = loc.detach().cpu().double()
    if loc.dtype != torch.float32:
        return loc64
    wh = shapes.cpu().flip(-1).double().view(1, 1, 1, -1, 1, 2)  # (W, H) per level
    px = (loc64 * wh - 0.5).float().double()  # one rounding, as fmaf
    return (px + 0.5) / wh


def oracle64(value, shapes, starts, loc, attn, g):
    """float64 oracle on the same (possibly half-precision) inputs: the
    grid_sample forward and the analytic backward, in float64. For fp32
    locations the backward uses the reference's fp32-rounded pixel
    coordinates (x = fma(loc, W, -0.5) in fp32, src/msda_triton/kernels.py:112-113):
    at W ~ 167 that rounding alone moves grad_attn by ~1e-4, more than the
    strict fp32 atol, for every fp32 implementation of the reference's maths.
    fp16/bf16 locations give exact coordinates either way."""
    cpu = lambda t: t.detach().cpu().double()  # noqa: E731
    out = orc.msda_grid_sample(cpu(value), shapes.cpu(), fp32_rounded_locations(loc, shapes), cpu(attn))
    coord = torch.float32 if loc.dtype == torch.float32 else None
    grads = orc.msda_backward_analytic(cpu(value), shapes.cpu(), starts.cpu(), cpu(loc), cpu(attn),
                                       cpu(g), coord_dtype=coord)
    return out, grads


# ---------------------------------------------------------------------------
# The reference suite's cases
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_forward_matches_reference(case, dtype):
    value, shapes, starts, loc, attn = cases.make_inputs(**cases.case_kwargs(case), dtype=dtype,
                                                         device=DEV)
    out, _ = run_op(value, shapes, starts, loc, attn)
    ref, _ = orc.reference_fp32(value, shapes, loc, attn)
    assert out.dtype == dtype and out.shape == ref.shape
    close(out, ref, STRICT_TOL[dtype], "out")


@pytest.mark.parametrize("fp32_grad_accum", [False, True], ids=["native_acc", "fp32_acc"])
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("case", [CASES[0], CASES[2]], ids=[CASES[0]["id"], CASES[2]["id"]])
def test_backward_matches_reference(case, dtype, fp32_grad_accum):
    value, shapes, starts, loc, attn = cases.make_inputs(**cases.case_kwargs(case), dtype=dtype,
                                                         device=DEV)
    B, Q, M, D = value.shape[0], loc.shape[1], value.shape[2], value.shape[3]
    g = cases.grad_output_like(torch.empty(B, Q, M * D, device=DEV, dtype=dtype))
    _, got = run_op(value, shapes, starts, loc, attn, g, fp32_grad_accum=fp32_grad_accum)
    assert all(t.dtype == dtype for t in got)
    _, ref = oracle64(value, shapes, starts, loc, attn, g)
    # Native half-precision atomics round at every add: held to the
    # reference suite's tolerance; every fp32-accumulated path to the strict bar.
    gv_tol = STRICT_TOL[dtype] if (fp32_grad_accum or dtype == torch.float32) else REF_BWD_TOL[dtype]
    cases.assert_grads_close(got, ref, loc, shapes, STRICT_TOL[dtype], gv_tol=gv_tol)
    # ... and the reference suite's own comparison (tests/test_msda.py:199-205):
    # every gradient in raw units, no point excluded, against its fp32
    # grid_sample path at its backward tolerance.
    _, ref32 = orc.reference_fp32(value, shapes, loc, attn, g)
    for name, a, b in zip(("grad_value", "grad_loc", "grad_attn"), got, ref32):
        torch.testing.assert_close(a.float().cpu(), b, **REF_BWD_TOL[dtype],
                                   msg=lambda m, n=name: f"{n} (raw units): {m}")


def test_forward_out_of_bounds_locations():
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=2, Q=64, M=4, D=32, shapes=[(14, 20), (7, 10)], K=4, dtype=torch.float32, device=DEV,
        loc_lo=-0.5, loc_hi=1.5)
    out, _ = run_op(value, shapes, starts, loc, attn)
    ref, _ = orc.reference_fp32(value, shapes, loc, attn)
    close(out, ref, REF_FWD_TOL[torch.float32], "out")


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_backward_out_of_bounds_locations(dtype):
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=2, Q=64, M=4, D=32, shapes=[(14, 20), (7, 10)], K=4, dtype=dtype, device=DEV,
        loc_lo=-0.5, loc_hi=1.5)
    g = cases.grad_output_like(torch.empty(2, 64, 128, device=DEV, dtype=dtype))
    out, got = run_op(value, shapes, starts, loc, attn, g)
    ref, grads = oracle64(value, shapes, starts, loc, attn, g)
    close(out, ref, STRICT_TOL[dtype], "out")
    cases.assert_grads_close(got, grads, loc, shapes, STRICT_TOL[dtype])


def test_forward_level_start_index_optional_and_noncontiguous():
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=2, Q=50, M=4, D=32, shapes=[(12, 16), (6, 8)], K=4, dtype=torch.float32, device=DEV)
    out, _ = run_op(value, shapes, starts, loc, attn)
    out_nostarts, _ = run_op(value, shapes, None, loc, attn)
    torch.testing.assert_close(out, out_nostarts)
    value_nc = value.transpose(1, 2).contiguous().transpose(1, 2)
    assert not value_nc.is_contiguous()
    out_nc = multi_scale_deformable_attention(value_nc, shapes, starts, loc, attn)
    torch.testing.assert_close(out, out_nc)
    # Host-side spatial_shapes / level_start_index are accepted too.
    out_host = multi_scale_deformable_attention(value, shapes.cpu(), starts.cpu(), loc, attn)
    torch.testing.assert_close(out, out_host)


def test_fp32_accum_paths_agree_at_fp32():
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=2, Q=100, M=4, D=32, shapes=[(24, 32), (12, 16)], K=4, dtype=torch.float32, device=DEV)
    grads = []
    for acc in (False, True):
        v = value.clone().requires_grad_(True)
        out = multi_scale_deformable_attention(v, shapes, starts, loc, attn, fp32_grad_accum=acc)
        out.backward(torch.ones_like(out))
        grads.append(v.grad)
    torch.testing.assert_close(grads[0], grads[1], rtol=1e-5, atol=1e-5)


def test_rejects_mismatched_shapes_and_dtypes():
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=1, Q=8, M=2, D=16, shapes=[(6, 6)], K=2, dtype=torch.float32, device=DEV)
    with pytest.raises(ValueError, match="attention_weights"):
        multi_scale_deformable_attention(value, shapes, starts, loc, attn[:, :, :, :, :1])
    with pytest.raises(ValueError, match="dtypes"):
        multi_scale_deformable_attention(value, shapes, starts, loc.half(), attn)
    with pytest.raises(ValueError, match="CUDA"):
        multi_scale_deformable_attention(value.cpu(), shapes.cpu(), starts.cpu(), loc.cpu(),
                                         attn.cpu())
    with pytest.raises(ValueError, match="level_start_index"):
        multi_scale_deformable_attention(value, shapes, starts[:0], loc, attn)
    with pytest.raises(ValueError, match="same CUDA device"):
        multi_scale_deformable_attention(value, shapes, starts, loc.cpu(), attn)
    # Host-side shapes that address more rows than value holds are rejected.
    with pytest.raises(ValueError, match="value has S"):
        multi_scale_deformable_attention(value, torch.tensor([[7, 6]]), None, loc, attn)


# ---------------------------------------------------------------------------
# The reference's own Triton kernels (golden vectors from the interpreter)
# ---------------------------------------------------------------------------

GOLDEN_TRITON = sorted(p.stem for p in GOLDEN.glob("*.npz") if p.stem.startswith(("case_", "preset_")))


@pytest.mark.parametrize("name", GOLDEN_TRITON)
def test_matches_reference_triton_kernels(name):
    npz = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(npz["meta"]))
    if meta["kind"] == "preset":
        x = presets.make_inputs(presets.get(meta["preset"]), seed=meta["seed"])
        value, shapes, starts = x["value"], x["spatial_shapes"], x["level_start_index"]
        loc, attn, g = x["sampling_locations"], x["attention_weights"], x["grad_output"]
    else:
        kw = dict(meta["kwargs"])
        kw["shapes"] = [tuple(s) for s in kw["shapes"]]
        value, shapes, starts, loc, attn = cases.make_inputs(
            **kw, dtype=torch.float32, device="cpu", loc_lo=meta["loc_lo"], loc_hi=meta["loc_hi"])
        g = cases.grad_output_like(torch.empty(loc.shape[0], loc.shape[1], loc.shape[2] * kw["D"]))
    assert cases.digest(value) == str(npz["digest_value"])
    assert cases.digest(loc) == str(npz["digest_loc"])
    dev = [t.to(DEV) for t in (value, shapes, starts, loc, attn, g)]
    out, (gv, gl, ga) = run_op(*dev[:5], dev[5])
    cases.assert_matches_golden(out, npz, "triton_out", rtol=1e-5, atol=1e-5)
    # The reference suite's fp32 backward tolerance (tests/test_msda.py:52).
    cases.assert_matches_golden(gv, npz, "triton_grad_value", rtol=1e-4, atol=1e-4)
    cases.assert_matches_golden(gl, npz, "triton_grad_loc", rtol=1e-4, atol=1e-4)
    cases.assert_matches_golden(ga, npz, "triton_grad_attn", rtol=1e-4, atol=1e-4)


# ---------------------------------------------------------------------------
# The benchmark operating points at full size
# ---------------------------------------------------------------------------

OPERATING_POINTS = [("small", None), ("decoder", None), ("encoder", None), ("m2f", torch.float16),
                   ("m2f", torch.float32), ("decoder", torch.float16), ("decoder", torch.float32)]


@pytest.mark.parametrize("name,dtype", OPERATING_POINTS,
                         ids=[f"{n}-{d if d else 'default'}" for n, d in OPERATING_POINTS])
def test_baseline_operating_point_full_parity(name, dtype):
    """Full-size parity. small/decoder: against the float64 oracle at the
    strict bar. encoder/m2f (CPU float64 would take minutes): against the
    fp32 grid_sample reference -- strict for fp16/bf16, the reference suite's
    fp32 backward tolerance for fp32 (whose error there is the reference's own
    fp32 coordinate rounding, amplified by W ~ 128-167)."""
    p = presets.get(name)
    x = presets.make_inputs(p, dtype=dtype, device=DEV, seed=0)
    v, s, st = x["value"], x["spatial_shapes"], x["level_start_index"]
    l, a, g = x["sampling_locations"], x["attention_weights"], x["grad_output"]
    dt = v.dtype
    out, got = run_op(v, s, st, l, a, g)
    if name in ("small", "decoder"):
        ref, grads = oracle64(v, s, st, l, a, g)
        close(out, ref, STRICT_TOL[dt], "out")
        cases.assert_grads_close(got, grads, l, s, STRICT_TOL[dt], what=name)
    else:
        ref, grads = orc.reference_fp32(v, s, l, a, g)
        close(out, ref, STRICT_TOL[dt], "out")
        tol = STRICT_TOL[dt] if dt != torch.float32 else REF_BWD_TOL[dt]
        cases.assert_grads_close(got, grads, l, s, tol, what=name)


@pytest.mark.parametrize("name", ["encoder", "m2f"])
def test_dense_operating_points_fp32_at_the_strict_bar(name):
    """encoder / m2f in fp32 at full size (one batch item, every query)
    against float64 checkers at fp32's strict bar (rtol 1e-4, atol 1e-5), all
    three gradients in raw units with no point excluded. The checkers run on
    the GPU in float64 (a CPU run would take minutes), on the reference's
    fp32-rounded pixel coordinates: the oracle's grid_sample forward
    (fp32_rounded_locations) and its analytic backward (coord_dtype fp32),
    which keeps the exact coordinates -- a location whose fp32 coordinate is
    an integer sits on a kink of the bilinear interpolant, and only the exact
    coordinate picks the same one-sided derivative as the kernel."""
    p = presets.get(name)
    x = presets.make_inputs(p, dtype=torch.float32, device=DEV, seed=0, batch=1)
    v, s, st = x["value"], x["spatial_shapes"], x["level_start_index"]
    l, a, g = x["sampling_locations"], x["attention_weights"], x["grad_output"]
    out, got = run_op(v, s, st, l, a, g)
    tol = STRICT_TOL[torch.float32]
    out64 = orc.msda_grid_sample(v.double(), s, fp32_rounded_locations(l, s).to(DEV), a.double())
    close(out, out64, tol, f"{name} out")
    refs = orc.msda_backward_analytic(v.double(), s.cpu(), st.cpu(), l, a, g, coord_dtype=torch.float32)
    close(got[0], refs[0], tol, f"{name} grad_value")
    close(got[2], refs[2], tol, f"{name} grad_attn")
    # grad_loc = a * W_l * d/dx_pixel: an fp32 implementation's absolute error
    # there is its dot products' rounding (32 products of N(0, 1) values)
    # times a * W_l, so the absolute bar is 1e-5 per pixel of level width
    # (rtol 1e-4 as everywhere, raw units, no point excluded) ...
    wl = s.cpu().double()[:, 1].view(1, 1, 1, -1, 1, 1).to(DEV)
    err = (got[1].double() - refs[1]).abs()
    bound = 1e-5 * wl + 1e-4 * refs[1].abs()
    assert bool((err <= bound).all()), f"{name} grad_loc: {int((err > bound).sum())} elements past 1e-5*W + 1e-4*|ref|"
    # ... and it is no larger than the same maths restated in fp32 makes.
    refs32 = orc.msda_backward_analytic(v, s.cpu(), st.cpu(), l, a, g, coord_dtype=torch.float32)
    err32 = (refs32[1].double() - refs[1]).abs()
    assert err.max().item() <= 2.0 * err32.max().item() + 1e-6, (err.max().item(), err32.max().item())


def test_native_accumulation_error_at_encoder_density():
    """The default accumulator policy's evidence: bf16 grad_value at the
    encoder point (one batch item, ~1300 corner hits per coarse-level row)
    with native bf16 reductions and with fp32 accumulation, against a float64
    checker (the oracle's grid_sample on the GPU). fp32 accumulation meets the
    strict bf16 bar (1e-2 relative, 1e-4 absolute) on every element; native
    reductions do not. Prints the measured errors."""
    import json as _json

    p = presets.get("encoder")
    x = presets.make_inputs(p, dtype=torch.bfloat16, device=DEV, seed=0, batch=1)
    v, s, st = x["value"], x["spatial_shapes"], x["level_start_index"]
    l, a, g = x["sampling_locations"], x["attention_weights"], x["grad_output"]
    v64 = v.double().requires_grad_(True)
    out64 = orc.msda_grid_sample(v64, s, l.double(), a.double())
    out64.backward(g.double())
    ref = v64.grad
    stats = {}
    for name, fp32 in (("native", False), ("fp32", True)):
        _, (gv, _, _) = run_op(v, s, st, l, a, g, fp32_grad_accum=fp32)
        err = (gv.double() - ref).abs()
        bad = err > 1e-2 * ref.abs() + 1e-4
        stats[name] = {"normwise": (err.norm() / ref.norm()).item(),
                       "max_err_over_max_ref": (err.max() / ref.abs().max()).item(),
                       "frac_outside_strict": bad.double().mean().item(),
                       "elements_outside_strict": int(bad.sum())}
    print("native-accumulation error at encoder density:", _json.dumps(stats))
    assert stats["fp32"]["elements_outside_strict"] == 0
    assert stats["native"]["elements_outside_strict"] > 0


def test_scale_d64_variant_parity():
    p = presets.get("scale_d64")
    x = presets.make_inputs(p, device=DEV, seed=3, batch=2)
    v, s, st = x["value"], x["spatial_shapes"], x["level_start_index"]
    l, a, g = x["sampling_locations"], x["attention_weights"], x["grad_output"]
    out, got = run_op(v, s, st, l, a, g)
    ref, grads = orc.reference_fp32(v, s, l, a, g)
    tol = STRICT_TOL[torch.bfloat16]
    close(out, ref, tol, "out")
    cases.assert_grads_close(got, grads, l, s, tol, what="scale_d64")


def test_encoder_properties_at_full_size():
    """Size-independent properties at the encoder point (fp32): the forward
    is linear in value and in attention_weights, grad_value is linear in
    grad_output, and sum(grad_attn * attn) == <grad_output, output>."""
    p = presets.get("encoder")
    x = presets.make_inputs(p, dtype=torch.float32, device=DEV, seed=1)
    v, s, st, l, a, g = (x["value"], x["spatial_shapes"], x["level_start_index"],
                         x["sampling_locations"], x["attention_weights"], x["grad_output"])
    f = lambda vv, aa: multi_scale_deformable_attention(vv, s, st, l, aa)  # noqa: E731
    v2 = torch.randn_like(v)
    torch.testing.assert_close(f(2.5 * v + v2, a), 2.5 * f(v, a) + f(v2, a), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(f(v, 3.0 * a), 3.0 * f(v, a), rtol=1e-5, atol=1e-5)
    _, (gv1, _, ga1) = run_op(v, s, st, l, a, g)
    _, (gv2, _, _) = run_op(v, s, st, l, a, -2.0 * g)
    torch.testing.assert_close(gv2, -2.0 * gv1, rtol=1e-5, atol=1e-5)
    out = f(v, a)
    lhs = (ga1.double() * a.double()).sum()
    rhs = (g.double() * out.double()).sum()
    torch.testing.assert_close(lhs, rhs, rtol=1e-5, atol=1e-3)


# ---------------------------------------------------------------------------
# Edge cases
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("D,dtype", [(3, torch.float32), (5, torch.float16), (24, torch.bfloat16),
                                     (8, torch.bfloat16), (4, torch.float32), (128, torch.bfloat16),
                                     (256, torch.float32), (96, torch.float16), (40, torch.float32)])
def test_head_dims(D, dtype):
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=2, Q=19, M=3, D=D, shapes=[(7, 9), (4, 5)], K=3, dtype=dtype, device=DEV,
        loc_lo=-0.2, loc_hi=1.2)
    g = cases.grad_output_like(torch.empty(2, 19, 3 * D, device=DEV, dtype=dtype))
    out, got = run_op(value, shapes, starts, loc, attn, g)
    ref, grads = oracle64(value, shapes, starts, loc, attn, g)
    close(out, ref, STRICT_TOL[dtype], "out")
    cases.assert_grads_close(got, grads, loc, shapes, STRICT_TOL[dtype], what=f"D={D}")


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_misaligned_buffers_take_the_scalar_path(dtype):
    """A value tensor whose data pointer is not 16-byte aligned (a view with a
    storage offset) is served by the scalar-load kernels, with equal results."""
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=1, Q=21, M=2, D=32, shapes=[(9, 8), (5, 4)], K=4, dtype=dtype, device=DEV)
    base = torch.empty(value.numel() + 1, device=DEV, dtype=dtype)
    shifted = base[1:].view_as(value)
    shifted.copy_(value)
    assert shifted.data_ptr() % 16 != 0
    g = cases.grad_output_like(torch.empty(1, 21, 64, device=DEV, dtype=dtype))
    out_a, (gv_a, gl_a, ga_a) = run_op(value, shapes, starts, loc, attn, g)
    v = shifted.requires_grad_(True)
    out_b = multi_scale_deformable_attention(v, shapes, starts, loc, attn)
    out_b.backward(g)
    tol = dict(rtol=1e-6, atol=1e-6) if dtype == torch.float32 else STRICT_TOL[dtype]
    close(out_b.detach(), out_a, tol, "out")
    close(v.grad, gv_a, tol, "grad_value")


def test_exact_corner_locations():
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=1, Q=4, M=1, D=3, shapes=[(4, 6)], K=2, dtype=torch.float32, device=DEV)
    loc = cases.exact_corner_locations(loc.shape, torch.float32).to(DEV)
    g = cases.grad_output_like(torch.empty(1, 4, 3, device=DEV))
    out, got = run_op(value, shapes, starts, loc, attn, g)
    ref, grads = oracle64(value, shapes, starts, loc, attn, g)
    close(out, ref, STRICT_TOL[torch.float32], "out")
    cases.assert_grads_close(got, grads, loc, shapes, STRICT_TOL[torch.float32], what="corners")


def test_zero_sized_batch_and_queries():
    for B, Q in ((0, 5), (2, 0)):
        value = torch.randn(B, 20, 2, 8, device=DEV)
        loc = torch.rand(B, Q, 2, 1, 2, 2, device=DEV)
        attn = torch.rand(B, Q, 2, 1, 2, device=DEV)
        out = multi_scale_deformable_attention(value, torch.tensor([[4, 5]], device=DEV), None,
                                               loc, attn)
        assert out.shape == (B, Q, 16) and out.abs().sum() == 0


def test_non_finite_and_huge_locations_stay_in_bounds():
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=1, Q=8, M=2, D=16, shapes=[(6, 7), (3, 4)], K=2, dtype=torch.float32, device=DEV)
    bad = torch.tensor([float("nan"), float("inf"), -float("inf"), 1e30, -1e30, 3e9],
                       device=DEV)
    flat = loc.view(-1)
    flat[: bad.numel() * 4] = bad.repeat(4)
    g = torch.ones(1, 8, 32, device=DEV)
    out, (gv, gl, ga) = run_op(value, shapes, starts, loc, attn, g)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all() and torch.isfinite(gv).all()
    assert torch.isfinite(ga).all() and torch.isfinite(gl).all()
    # Queries whose locations are all finite and in range still match the oracle.
    ok = torch.isfinite(loc).all(-1).all(-1).all(-1).all(-1)[0]
    ref, _ = orc.reference_fp32(value, shapes, loc.nan_to_num(0.0, 5.0, -5.0), attn)
    close(out[0, ok], ref[0, ok.cpu()], STRICT_TOL[torch.float32], "out")


def test_device_shapes_beyond_value_rows_are_treated_as_empty():
    """Device-side spatial_shapes that claim more rows than value holds cannot
    be checked without a sync; the kernels treat such a level as empty instead
    of reading out of bounds."""
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=1, Q=16, M=2, D=16, shapes=[(6, 7), (3, 4)], K=2, dtype=torch.float32, device=DEV)
    bad_shapes = torch.tensor([[6, 7], [30, 40]], device=DEV)
    out = multi_scale_deformable_attention(value, bad_shapes, starts, loc, attn)
    attn0 = attn.clone()
    attn0[:, :, :, 1] = 0
    ref, _ = orc.reference_fp32(value, shapes, loc, attn0)
    close(out, ref, STRICT_TOL[torch.float32], "out")


def test_mmcv_style_function():
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=2, Q=30, M=4, D=32, shapes=[(12, 16), (6, 8)], K=4, dtype=torch.float32, device=DEV)
    v = value.clone().requires_grad_(True)
    out = MultiScaleDeformableAttnFunction.apply(v, shapes, starts, loc, attn, 64)
    out.backward(torch.ones_like(out))
    ref, (gv_r, _, _) = oracle64(value, shapes, starts, loc, attn, torch.ones(2, 30, 128))
    close(out.detach(), ref, STRICT_TOL[torch.float32], "out")
    close(v.grad, gv_r, STRICT_TOL[torch.float32], "grad_value")


def test_side_stream_and_graph_capture():
    """Calls enqueue on the caller's current stream and can be captured in a
    CUDA graph (no host synchronisation inside the op)."""
    x = presets.make_inputs(presets.get("decoder"), device=DEV, seed=5)
    args = (x["value"], x["spatial_shapes"], x["level_start_index"], x["sampling_locations"],
            x["attention_weights"])
    ref_out = multi_scale_deformable_attention(*args)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out_side = multi_scale_deformable_attention(*args)
    torch.cuda.current_stream().wait_stream(side)
    torch.testing.assert_close(out_side, ref_out)

    static_g = x["grad_output"].clone()
    warm = torch.cuda.Stream()
    warm.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(warm):  # warm up on a side stream, as torch's graph recipe asks
        for _ in range(2):
            vw = x["value"].clone().requires_grad_(True)
            multi_scale_deformable_attention(vw, *args[1:]).backward(static_g)
    torch.cuda.current_stream().wait_stream(warm)
    torch.cuda.synchronize()
    v = x["value"].clone().requires_grad_(True)  # fresh leaf: its AccumulateGrad is captured
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = multi_scale_deformable_attention(v, *args[1:])
        static_out.backward(static_g)
    graph.replay()
    torch.cuda.synchronize()
    _, (gv_ref, _, _) = run_op(*args, static_g)
    torch.testing.assert_close(static_out.detach(), ref_out)
    close(v.grad, gv_ref, STRICT_TOL[torch.bfloat16], "grad_value (graph)")


# ---------------------------------------------------------------------------
# Every grad_value algorithm, forced through the C ABI flags
# ---------------------------------------------------------------------------
from msda_triton_b200 import _lib as _clib  # noqa: E402
from msda_triton_b200 import ops as _ops  # noqa: E402

ALGOS = {
    "scatter_fp32": (_clib.MSDA_BWD_FORCE_SCATTER, True),
    "scatter_native": (_clib.MSDA_BWD_FORCE_SCATTER, False),
    "counted": (_clib.MSDA_BWD_FORCE_COUNTED, True),
}
ALGO_CASES = [
    ("decoder_case", dict(B=2, Q=100, M=4, D=32, K=4, shapes=[(24, 32), (12, 16), (6, 8)]), 0.0, 1.0),
    ("nonpow2", dict(B=2, Q=33, M=2, D=24, K=3, shapes=[(10, 14), (5, 7)]), 0.0, 1.0),
    ("wide_oob", dict(B=1, Q=64, M=8, D=64, K=4, shapes=[(16, 16), (8, 8)]), -0.5, 1.5),
    ("odd_d", dict(B=2, Q=9, M=3, D=5, K=2, shapes=[(7, 9), (4, 5)]), -0.2, 1.2),
    ("d128", dict(B=1, Q=40, M=2, D=128, K=4, shapes=[(20, 30), (10, 15)]), 0.0, 1.0),
    ("one_pixel_levels", dict(B=2, Q=50, M=2, D=32, K=4, shapes=[(1, 1), (2, 1), (1, 3)]), -0.3, 1.3),
    # Dense sampling clustered in a few rows (Q*L*K > 2*S): the scatter merges
    # a warp's same-row contributions before reducing them.
    ("dense_local", dict(B=2, Q=64, M=4, D=32, K=4, shapes=[(8, 8), (4, 4)]), 0.45, 0.55),
    ("dense_local_d64", dict(B=1, Q=96, M=2, D=64, K=4, shapes=[(6, 10), (3, 5)]), 0.4, 0.6),
]


@pytest.mark.parametrize("algo", list(ALGOS))
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw,lo,hi", ALGO_CASES, ids=[c[0] for c in ALGO_CASES])
def test_backward_algorithms(name, kw, lo, hi, dtype, algo):
    flags, fp32 = ALGOS[algo]
    value, shapes, starts, loc, attn = cases.make_inputs(**kw, dtype=dtype, device=DEV, loc_lo=lo,
                                                         loc_hi=hi)
    B, Q, M, D = value.shape[0], loc.shape[1], value.shape[2], value.shape[3]
    g = cases.grad_output_like(torch.empty(B, Q, M, D, device=DEV, dtype=dtype))
    got = _ops._backward(value, shapes, starts, loc, attn, g, fp32, flags)
    _, ref = oracle64(value, shapes, starts, loc, attn, g)
    native = algo == "scatter_native" and dtype != torch.float32
    cases.assert_grads_close(got, ref, loc, shapes, STRICT_TOL[dtype], native_gv=native, what=algo)


# ---------------------------------------------------------------------------
# Long grids (more query-heads than a few waves of one-query warps) take the
# multi-query launch shapes: 2 queries per warp, rounds of consecutive
# queries per CTA, and -- when the warp's queries have at most 32 points --
# one point resolved per lane and shared with the lane groups. Ragged query
# counts leave partially live warps and CTAs.
# ---------------------------------------------------------------------------
LONG_CASES = [
    ("dense_l2k4", dict(B=1, Q=3001, M=8, D=32, K=4, shapes=[(30, 40), (15, 20)]), 0.3, 0.7),
    ("dense_l3k4_oob", dict(B=1, Q=2999, M=8, D=32, K=4, shapes=[(32, 32), (16, 16), (8, 8)]), -0.1, 1.1),
    ("d64_k3", dict(B=2, Q=1203, M=8, D=64, K=3, shapes=[(20, 30), (10, 15)]), 0.0, 1.0),
    ("sparse", dict(B=1, Q=3001, M=8, D=32, K=4, shapes=[(100, 200)]), 0.0, 1.0),
    # 24 points per query: 2 queries exceed a warp's 32 lanes, so the long
    # shape resolves points per lane group instead of sharing them.
    ("many_points", dict(B=1, Q=2501, M=8, D=32, K=8, shapes=[(30, 40), (15, 20), (8, 10)]), -0.05, 1.05),
]
_LONG_CACHE: dict = {}


def _long_case(name, kw, lo, hi, dtype):
    key = (name, dtype)
    if key not in _LONG_CACHE:
        value, shapes, starts, loc, attn = cases.make_inputs(**kw, dtype=dtype, device=DEV, loc_lo=lo,
                                                             loc_hi=hi, seed=5)
        B, Q, M, D = value.shape[0], loc.shape[1], value.shape[2], value.shape[3]
        g = cases.grad_output_like(torch.empty(B, Q, M, D, device=DEV, dtype=dtype))
        _LONG_CACHE.clear()
        _LONG_CACHE[key] = (value, shapes, starts, loc, attn, g, oracle64(value, shapes, starts, loc, attn, g))
    return _LONG_CACHE[key]


@pytest.mark.parametrize("acc", ["fp32", "native", "deterministic"])
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw,lo,hi", LONG_CASES, ids=[c[0] for c in LONG_CASES])
def test_long_grid_launch_shapes(name, kw, lo, hi, dtype, acc):
    value, shapes, starts, loc, attn, g, (out_ref, grads_ref) = _long_case(name, kw, lo, hi, dtype)
    out = _ops._forward(value, shapes, starts, loc, attn)
    close(out, out_ref.view_as(out), STRICT_TOL[dtype], f"{name} forward")
    got = _ops._backward(value, shapes, starts, loc, attn, g, acc != "native", deterministic=acc == "deterministic")
    native = acc == "native" and dtype != torch.float32
    cases.assert_grads_close(got, grads_ref, loc, shapes, STRICT_TOL[dtype], native_gv=native,
                             what=f"{name}/{acc}")


@pytest.mark.parametrize("algo", ["scatter_fp32", "counted"])
@pytest.mark.parametrize("name", ["decoder", "small"])
def test_backward_algorithms_at_baseline_points(name, algo):
    flags, fp32 = ALGOS[algo]
    x = presets.make_inputs(presets.get(name), device=DEV, seed=2)
    v, s, st = x["value"], x["spatial_shapes"], x["level_start_index"]
    l, a = x["sampling_locations"], x["attention_weights"]
    g = x["grad_output"].view(v.shape[0], l.shape[1], v.shape[2], v.shape[3])
    got = _ops._backward(v, s, st, l, a, g, fp32, flags)
    _, ref = oracle64(v, s, st, l, a, g)
    cases.assert_grads_close(got, ref, l, s, STRICT_TOL[v.dtype], what=f"{name}/{algo}")


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_counted_scatter_matches_fp32_accumulation(dtype):
    """The hit-counted scatter stores one-hit rows and reduces multi-hit rows in
    fp32: its grad_value must equal the fp32-workspace scatter's up to fp32
    summation order, and untouched rows (here: a padding tail) must be zeros
    even when grad_value starts as garbage."""
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=2, Q=40, M=4, D=32, K=4, shapes=[(20, 30), (10, 15), (5, 8)], dtype=dtype, device=DEV,
        loc_lo=-0.1, loc_hi=1.1, seed=4)
    value = torch.cat([value, torch.randn(2, 9, 4, 32, device=DEV).to(dtype)], 1)  # 9 unused rows
    g = cases.grad_output_like(torch.empty(2, 40, 4, 32, device=DEV, dtype=dtype))
    ref = _ops._backward(value, shapes, starts, loc, attn, g, True, _clib.MSDA_BWD_FORCE_SCATTER)
    torch.empty(value.numel() * 8, device=DEV).fill_(float("nan"))  # dirty the allocator
    got = _ops._backward(value, shapes, starts, loc, attn, g, True, _clib.MSDA_BWD_FORCE_COUNTED)
    assert (got[0][:, -9:] == 0).all()
    tol = dict(rtol=1e-6, atol=1e-6) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-5)
    torch.testing.assert_close(got[0].float(), ref[0].float(), **tol)
    torch.testing.assert_close(got[1], ref[1])
    torch.testing.assert_close(got[2], ref[2])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=str)
def test_counted_backward_repeated_calls(dtype):
    """The hit-counted backward's passes (count, backward, finalize) overlap
    their predecessors' tails; each reads the counts and accumulator rows
    that the passes before it wrote. Many back-to-back calls must all stay
    at the strict bar (a stale count would store a row instead of reducing
    it, or skip a zero fill)."""
    kw, lo, hi = ALGO_CASES[0][1], ALGO_CASES[0][2], ALGO_CASES[0][3]
    value, shapes, starts, loc, attn = cases.make_inputs(**kw, dtype=dtype, device=DEV, loc_lo=lo, loc_hi=hi)
    B, Q, M, D = value.shape[0], loc.shape[1], value.shape[2], value.shape[3]
    g = cases.grad_output_like(torch.empty(B, Q, M, D, device=DEV, dtype=dtype))
    _, ref = oracle64(value, shapes, starts, loc, attn, g)
    runs = [_ops._backward(value, shapes, starts, loc, attn, g, True, _clib.MSDA_BWD_FORCE_COUNTED)
            for _ in range(16)]
    for got in runs:
        cases.assert_grads_close(got, ref, loc, shapes, STRICT_TOL[dtype], what="counted/repeated")


# ---------------------------------------------------------------------------
# Fused prologue: reference points + offsets (level pixels), attention logits
# ---------------------------------------------------------------------------
from msda_triton_b200 import multi_scale_deformable_attention_fused  # noqa: E402
from oracle import msda_oracle as _orc  # noqa: E402

FUSED_CASES = [
    ("sparse", dict(B=2, Q=40, M=4, D=32, K=4, shapes=[(24, 32), (12, 16), (6, 8)])),
    ("dense", dict(B=1, Q=160, M=2, D=32, K=2, shapes=[(8, 10), (4, 5)])),
    ("d64_oob", dict(B=1, Q=24, M=2, D=64, K=3, shapes=[(10, 14), (5, 7)])),
]
FUSED_ALGOS = {
    "auto_fp32": (0, True),
    "native": (0, False),
    "scatter_fp32": (_clib.MSDA_BWD_FORCE_SCATTER, True),
    "counted": (_clib.MSDA_BWD_FORCE_COUNTED, True),
}


def _fused_inputs(kw, dtype, seed=11):
    value, shapes, starts, _, _ = cases.make_inputs(**kw, dtype=dtype, device=DEV, seed=seed)
    B, Q, M, K, L = kw["B"], kw["Q"], kw["M"], kw["K"], len(kw["shapes"])
    gen = torch.Generator().manual_seed(seed + 1)
    ref = torch.rand(B, Q, 2, generator=gen)
    off = 3.0 * torch.randn(B, Q, M, L, K, 2, generator=gen)  # pixels; some corners fall outside
    logits = torch.randn(B, Q, M, L, K, generator=gen)
    return value, shapes, starts, ref.to(DEV, dtype), off.to(DEV, dtype), logits.to(DEV, dtype)


def _kink_eps(dtype):
    return 1e-3 if dtype == torch.float32 else 1e-6


def _fused_reference(value, shapes, ref, off, logits, g):
    """float64 composition on the CPU (the layer's prologue, then the
    grid_sample oracle), differentiated by autograd."""
    v, r, o, lg = (t.detach().double().cpu().requires_grad_(True) for t in (value, ref, off, logits))
    B, Q, M, L, K, _ = o.shape
    wh = shapes.detach().cpu().flip(-1).double()
    loc = r[:, :, None, None, None, :] + o / wh[:, None, :]
    attn = lg.reshape(B, Q, M, L * K).softmax(-1).view(B, Q, M, L, K)
    out = _orc.msda_grid_sample(v, shapes.cpu(), loc, attn)
    out.backward(g.detach().double().cpu().reshape(out.shape))
    return out.detach(), v.grad, r.grad, o.grad, lg.grad, loc.detach()


@pytest.mark.parametrize("algo", list(FUSED_ALGOS))
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw", FUSED_CASES, ids=[c[0] for c in FUSED_CASES])
def test_fused_prologue_matches_the_composition(name, kw, dtype, algo):
    flags, fp32 = FUSED_ALGOS[algo]
    value, shapes, starts, ref, off, logits = _fused_inputs(kw, dtype)
    B, Q, M, D = kw["B"], kw["Q"], kw["M"], kw["D"]
    out = _ops._forward_fused(value, shapes, starts, ref, off, logits)
    g = cases.grad_output_like(out)
    gv, goff, glog = _ops._backward_fused(value, shapes, starts, ref, off, logits, g, fp32, flags)
    out_r, gv_r, _, goff_r, glog_r, loc = _fused_reference(value, shapes, ref, off, logits, g)
    tol = STRICT_TOL[dtype]
    close(out.reshape(B, Q, M * D), out_r, tol, "out")
    gv_tol = REF_BWD_TOL[dtype] if (algo == "native" and dtype != torch.float32) else tol
    close(gv, gv_r, gv_tol, "grad_value")
    close(glog, glog_r, tol, "grad_logits")
    # Kinks of the bilinear interpolant are excluded for every dtype here:
    # reference + offset lands exactly on integers often with 16-bit inputs,
    # where the float64 composition (divide by W, then multiply) may round to
    # the other side. For 16-bit inputs the kernel's pixel coordinate is
    # exact, so only points within float64 rounding of an integer go.
    keep = ~cases.kink_mask(loc, shapes, _kink_eps(dtype))
    assert keep.double().mean() > 0.95
    torch.testing.assert_close(goff.double().cpu()[keep], goff_r[keep], **tol, msg=lambda m: f"grad_offsets: {m}")


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_fused_public_op_gradients_including_reference_points(dtype):
    value, shapes, starts, ref, off, logits = _fused_inputs(FUSED_CASES[0][1], dtype, seed=21)
    leaves = [t.clone().requires_grad_(True) for t in (value, ref, off, logits)]
    out = multi_scale_deformable_attention_fused(leaves[0], shapes, None, *leaves[1:])
    g = cases.grad_output_like(out.detach())
    out.backward(g)
    out_r, gv_r, gr_r, goff_r, glog_r, loc = _fused_reference(value, shapes, ref, off, logits, g)
    tol = STRICT_TOL[dtype]
    close(out, out_r, tol, "out")
    close(leaves[0].grad, gv_r, tol, "grad_value")
    close(leaves[3].grad, glog_r, tol, "grad_logits")
    # Kink points excluded (see above); the reference points' gradient sums
    # over a query's points, so queries with any kink point are excluded.
    keep = ~cases.kink_mask(loc, shapes, _kink_eps(dtype))
    torch.testing.assert_close(leaves[2].grad.double().cpu()[keep], goff_r[keep], **tol)
    q_keep = keep.all(-1).all(-1).all(-1)
    assert q_keep.double().mean() > (0.5 if dtype == torch.float32 else 0.3)
    got_r = leaves[1].grad.double().cpu()[q_keep]
    if dtype == torch.float32:
        torch.testing.assert_close(got_r, gr_r[q_keep], rtol=1e-3, atol=1e-3)
    else:  # a sum of M*L*K 16-bit offset gradients
        assert (got_r - gr_r[q_keep]).abs().max() <= 2e-2 * gr_r.abs().max()




def test_fused_op_falls_back_off_the_vector_path():
    """Head dims that are not a multiple of the 16-byte vector (and
    misaligned value buffers) take the tensor-op prologue + the operator."""
    kw = dict(B=1, Q=12, M=2, D=6, K=2, shapes=[(5, 7), (3, 4)])
    value, shapes, starts, ref, off, logits = _fused_inputs(kw, torch.bfloat16, seed=31)
    lib = _clib.load()
    out = torch.empty(1, 12, 2, 6, device=DEV, dtype=torch.bfloat16)
    rc = lib.msda_forward_fused(_ops._ptr(value), _ops._ptr(shapes), _ops._ptr(starts), _ops._ptr(ref),
                                _ops._ptr(off), _ops._ptr(logits), _ops._ptr(out), 1, value.shape[1], 12,
                                2, 6, 2, 2, _clib.MSDA_DTYPE_BF16, None)
    assert rc == _clib.MSDA_ERR_UNSUPPORTED
    leaves = [t.clone().requires_grad_(True) for t in (value, ref, off, logits)]
    out = multi_scale_deformable_attention_fused(leaves[0], shapes, None, *leaves[1:])
    g = cases.grad_output_like(out.detach())
    out.backward(g)
    # The fallback feeds the operator bf16 locations and weights (formed
    # with bf16 tensor ops, as the reference layer does): check it against
    # the float64 oracle on those same inputs.
    wh = shapes.flip(-1).to(torch.bfloat16)
    loc = ref[:, :, None, None, None, :] + off / wh[:, None, :]
    attn = logits.reshape(1, 12, 2, 4).softmax(-1).view(1, 12, 2, 2, 2)
    _, (gv_r, _, _) = oracle64(value, shapes, starts, loc, attn, g.view(1, 12, 2, 6))
    out_r = _orc.msda_grid_sample(value.double().cpu(), shapes.cpu(), loc.double().cpu(), attn.double().cpu())
    close(out, out_r, STRICT_TOL[torch.bfloat16], "out")
    close(leaves[0].grad, gv_r, STRICT_TOL[torch.bfloat16], "grad_value")
    assert leaves[1].grad is not None and leaves[3].grad is not None

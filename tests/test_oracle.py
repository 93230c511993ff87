"""Pin the oracle (CPU, no GPU): every oracle function against the golden
vectors that the reference's own code produced (tests/golden/make_golden.py:
the reference's grid_sample implementation, its loop specification, and its
Triton kernels run by Triton's interpreter)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from oracle import msda_oracle as orc
from msda_triton_b200 import presets

GOLDEN = Path(__file__).resolve().parent / "golden"
ALL = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def _load(name):
    npz = np.load(GOLDEN / f"{name}.npz")
    return npz, json.loads(str(npz["meta"]))


def _regenerate(meta):
    """Rebuild a golden case's inputs and check them against the stored digests."""
    dt = {"float64": torch.float64, "float32": torch.float32}[meta["dtype"]]
    if meta["kind"] == "preset":
        x = presets.make_inputs(presets.get(meta["preset"]), seed=meta["seed"])
        return (x["value"], x["spatial_shapes"], x["level_start_index"], x["sampling_locations"],
                x["attention_weights"], x["grad_output"])
    kw = dict(meta["kwargs"])
    kw["shapes"] = [tuple(s) for s in kw["shapes"]]
    value, shapes, starts, loc, attn = cases.make_inputs(
        **kw, dtype=dt, device="cpu", loc_lo=meta.get("loc_lo", 0.0), loc_hi=meta.get("loc_hi", 1.0),
        seed=meta["seed"])
    if meta["kind"] == "ref_naive_corners":
        loc = cases.exact_corner_locations(loc.shape)
    B, Q, M = loc.shape[0], loc.shape[1], loc.shape[2]
    g = cases.grad_output_like(torch.empty(B, Q, M * kw["D"], dtype=dt), seed=meta["grad_seed"])
    return value, shapes, starts, loc, attn, g


def _tols(meta):
    if meta["dtype"] == "float64":
        return dict(rtol=1e-10, atol=1e-12), dict(rtol=1e-9, atol=1e-10)
    return dict(rtol=1e-5, atol=1e-5), dict(rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("name", ALL)
def test_inputs_regenerate_bit_exactly(name):
    npz, meta = _load(name)
    value, shapes, starts, loc, attn, g = _regenerate(meta)
    for key, t in dict(value=value, loc=loc, attn=attn, grad_out=g).items():
        assert cases.digest(t) == str(npz[f"digest_{key}"]), f"{name}: input {key} differs"


@pytest.mark.parametrize("name", ALL)
def test_grid_sample_oracle_matches_reference(name):
    npz, meta = _load(name)
    value, shapes, starts, loc, attn, g = _regenerate(meta)
    fwd_tol, bwd_tol = _tols(meta)
    v = value.clone().requires_grad_(True)
    l = loc.clone().requires_grad_(True)
    a = attn.clone().requires_grad_(True)
    out = orc.msda_grid_sample(v, shapes, l, a)
    out.backward(g)
    cases.assert_matches_golden(out, npz, "out", **fwd_tol)
    cases.assert_matches_golden(v.grad, npz, "grad_value", **bwd_tol)
    cases.assert_matches_golden(l.grad, npz, "grad_loc", **bwd_tol)
    cases.assert_matches_golden(a.grad, npz, "grad_attn", **bwd_tol)


@pytest.mark.parametrize("name", ALL)
def test_analytic_backward_oracle_matches_reference(name):
    npz, meta = _load(name)
    value, shapes, starts, loc, attn, g = _regenerate(meta)
    _, bwd_tol = _tols(meta)
    gv, gl, ga = orc.msda_backward_analytic(value, shapes, starts, loc, attn, g)
    cases.assert_matches_golden(gv, npz, "grad_value", **bwd_tol)
    cases.assert_matches_golden(gl, npz, "grad_loc", **bwd_tol)
    cases.assert_matches_golden(ga, npz, "grad_attn", **bwd_tol)


@pytest.mark.parametrize("name", [n for n in ALL if n.startswith(("naive", "lab"))])
def test_loop_oracle_matches_reference(name):
    npz, meta = _load(name)
    value, shapes, starts, loc, attn, g = _regenerate(meta)
    out = orc.msda_loops(value, shapes, loc, attn)
    cases.assert_matches_golden(out, npz, "out", rtol=1e-10, atol=1e-12)
    if "naive" in npz:
        cases.assert_matches_golden(out, npz, "naive", rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("name", [n for n in ALL if n.startswith(("case_", "preset_"))])
def test_reference_triton_kernels_agree_with_reference_cpu(name):
    """The two reference implementations recorded in the fixtures (grid_sample
    and the Triton kernels) agree: the golden vectors are self-consistent."""
    npz, meta = _load(name)
    for key in ("out", "grad_value", "grad_loc", "grad_attn"):
        kind, ref = cases.unpack_golden(npz, key)
        kind_t, tri = cases.unpack_golden(npz, "triton_" + key)
        assert kind == kind_t
        if kind == "full":
            np.testing.assert_allclose(tri, ref, rtol=1e-4, atol=1e-4)
        else:
            np.testing.assert_array_equal(tri[0], ref[0])
            np.testing.assert_allclose(tri[1], ref[1], rtol=1e-4, atol=1e-4)


def test_reference_fp32_helper_matches_grid_sample():
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=1, Q=6, M=2, D=8, shapes=[(5, 6), (3, 3)], K=2, dtype=torch.bfloat16, device="cpu")
    g = cases.grad_output_like(torch.empty(1, 6, 16, dtype=torch.bfloat16))
    out, (gv, gl, ga) = orc.reference_fp32(value, shapes, loc, attn, g)
    assert out.dtype == torch.float32 and gv.dtype == torch.float32
    gv2, gl2, ga2 = orc.msda_backward_analytic(value.double(), shapes, starts, loc.double(),
                                               attn.double(), g.double())
    torch.testing.assert_close(gv.double(), gv2, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(gl.double(), gl2, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(ga.double(), ga2, rtol=1e-5, atol=1e-5)

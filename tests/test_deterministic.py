"""Deterministic grad_value (MSDA_BWD_DETERMINISTIC; GPU only).

The reference documents its backward as nondeterministic (grad_value is
accumulated with atomics; README.md:179, src/msda_triton/ops.py:135-138).
This build adds an opt-in mode that accumulates in 64-bit fixed point, so
the sum does not depend on the order the reductions land in. Checked here:

* parity with the float64 oracle at the same strict bar as fp32
  accumulation, for every algorithm (scatter, merged scatter, hit-counted),
  dtype and the fused prologue;
* bitwise reproducibility -- across repeated runs and, the stronger check,
  under a permutation of the queries, which reorders every atomic (with fp32
  atomics the rounding of the sums would change);
* the scale at extreme input magnitudes, all-zero gradients, non-finite
  inputs (fp32 fallback: Inf / NaN where fp32 accumulation puts them), CUDA
  graph capture, and the public op under torch.use_deterministic_algorithms.
"""

from __future__ import annotations

import pytest
import torch

import cases
from cases import STRICT_TOL
from msda_triton_b200 import _lib as _clib
from msda_triton_b200 import multi_scale_deformable_attention, multi_scale_deformable_attention_fused, presets
from msda_triton_b200 import ops as _ops
from test_gpu_parity import ALGO_CASES, FUSED_CASES, _fused_inputs, _fused_reference, _kink_eps, close, oracle64

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = [torch.float32, torch.float16, torch.bfloat16]
DET = _clib.MSDA_BWD_DETERMINISTIC
DET_ALGOS = {
    "auto": DET,
    "scatter": DET | _clib.MSDA_BWD_FORCE_SCATTER,
    "counted": DET | _clib.MSDA_BWD_FORCE_COUNTED,
}


@pytest.fixture(autouse=True)
def _lib_loaded(cuda_lib):
    yield


def _inputs(kw, lo, hi, dtype, seed=0):
    value, shapes, starts, loc, attn = cases.make_inputs(**kw, dtype=dtype, device=DEV, loc_lo=lo,
                                                         loc_hi=hi, seed=seed)
    B, Q, M, D = value.shape[0], loc.shape[1], value.shape[2], value.shape[3]
    g = cases.grad_output_like(torch.empty(B, Q, M, D, device=DEV, dtype=dtype))
    return value, shapes, starts, loc, attn, g


def _bitwise_equal(a, b):
    """Same bits (NaN payloads and signed zeros included)."""
    as_int = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[a.element_size()]
    return a.dtype == b.dtype and torch.equal(a.contiguous().view(as_int), b.contiguous().view(as_int))


@pytest.mark.parametrize("algo", list(DET_ALGOS))
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw,lo,hi", ALGO_CASES, ids=[c[0] for c in ALGO_CASES])
def test_deterministic_matches_the_oracle(name, kw, lo, hi, dtype, algo):
    value, shapes, starts, loc, attn, g = _inputs(kw, lo, hi, dtype)
    got = _ops._backward(value, shapes, starts, loc, attn, g, True, DET_ALGOS[algo])
    _, ref = oracle64(value, shapes, starts, loc, attn, g)
    cases.assert_grads_close(got, ref, loc, shapes, STRICT_TOL[dtype], what=f"deterministic/{algo}")


@pytest.mark.parametrize("algo", list(DET_ALGOS))
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw,lo,hi", ALGO_CASES, ids=[c[0] for c in ALGO_CASES])
def test_deterministic_is_bitwise_invariant_to_query_order(name, kw, lo, hi, dtype, algo):
    """grad_value sums over queries: permuting them (with their locations,
    weights and output gradients) reorders every contribution across warps
    and CTAs. The fixed-point sum is exact, so grad_value must not change in
    a single bit; grad_loc / grad_attn permute along."""
    value, shapes, starts, loc, attn, g = _inputs(kw, lo, hi, dtype, seed=3)
    flags = DET_ALGOS[algo]
    gv, gl, ga = _ops._backward(value, shapes, starts, loc, attn, g, True, flags)
    gv2, _, _ = _ops._backward(value, shapes, starts, loc, attn, g, True, flags)
    assert _bitwise_equal(gv, gv2), "repeated run differs"
    Q = loc.shape[1]
    perm = torch.randperm(Q, generator=torch.Generator().manual_seed(5)).to(DEV)
    gvp, glp, gap = _ops._backward(value, shapes, starts, loc[:, perm].contiguous(), attn[:, perm].contiguous(),
                                   g[:, perm].contiguous(), True, flags)
    assert _bitwise_equal(gv, gvp), "query permutation changed grad_value"
    assert _bitwise_equal(gl[:, perm], glp)
    assert _bitwise_equal(ga[:, perm], gap)


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_deterministic_at_the_decoder_operating_point(dtype):
    """Full-size decoder (B4 Q300 M8 D32 L4 K4, S = 22223): oracle parity,
    and bitwise equality under a query permutation."""
    x = presets.make_inputs(presets.get("decoder"), dtype=dtype, device=DEV, seed=2)
    v, s, st = (x[k] for k in ("value", "spatial_shapes", "level_start_index"))
    l, a = x["sampling_locations"], x["attention_weights"]
    g = x["grad_output"].view(v.shape[0], l.shape[1], v.shape[2], v.shape[3])
    got = _ops._backward(v, s, st, l, a, g, True, DET)
    _, ref = oracle64(v, s, st, l, a, g)
    cases.assert_grads_close(got, ref, l, s, STRICT_TOL[dtype], what="decoder/deterministic")
    perm = torch.randperm(l.shape[1], generator=torch.Generator().manual_seed(9)).to(DEV)
    gvp, _, _ = _ops._backward(v, s, st, l[:, perm].contiguous(), a[:, perm].contiguous(),
                               g[:, perm].contiguous(), True, DET)
    assert _bitwise_equal(got[0], gvp)


@pytest.mark.parametrize("name,kw,lo,hi", ALGO_CASES[:1] + [c for c in ALGO_CASES if c[0] == "dense_local_d64"],
                         ids=["decoder_case", "dense_local_d64"])
def test_deterministic_repeated_calls(name, kw, lo, hi):
    """Many back-to-back calls on one stream: every kernel of a call starts
    while the one before it still runs (programmatic dependent launch), so
    each must read what its predecessors wrote through coherent loads. A
    stale read shows as an occasional run with different bits (it did, about
    one run in ten, before the counts and row bounds were read that way)."""
    value, shapes, starts, loc, attn, g = _inputs(kw, lo, hi, torch.bfloat16, seed=3)
    first = _ops._backward(value, shapes, starts, loc, attn, g, True, DET)[0]
    for _ in range(24):
        assert _bitwise_equal(first, _ops._backward(value, shapes, starts, loc, attn, g, True, DET)[0])


def test_deterministic_at_the_encoder_operating_point():
    """Full-size encoder (Q = S = 22223 per item, dense local sampling; the
    merged fixed-point scatter): bitwise equal across runs and under a query
    permutation, and within bf16 rounding of the fp32-accumulated scatter
    (both sum far more precisely than bf16 resolves)."""
    x = presets.make_inputs(presets.get("encoder"), device=DEV, seed=1, batch=1)
    v, s, st = (x[k] for k in ("value", "spatial_shapes", "level_start_index"))
    l, a = x["sampling_locations"], x["attention_weights"]
    g = x["grad_output"].view(v.shape[0], l.shape[1], v.shape[2], v.shape[3])
    det = _ops._backward(v, s, st, l, a, g, True, DET)
    det2 = _ops._backward(v, s, st, l, a, g, True, DET)
    assert _bitwise_equal(det[0], det2[0])
    perm = torch.randperm(l.shape[1], generator=torch.Generator().manual_seed(4)).to(DEV)
    detp = _ops._backward(v, s, st, l[:, perm].contiguous(), a[:, perm].contiguous(),
                          g[:, perm].contiguous(), True, DET)
    assert _bitwise_equal(det[0], detp[0])
    f32 = _ops._backward(v, s, st, l, a, g, True, 0)
    d, r = det[0].float(), f32[0].float()
    assert ((d - r).abs() <= 1e-2 * r.abs() + 1e-3).float().mean() > 0.999
    assert (d - r).norm() <= 4e-3 * r.norm()
    assert _bitwise_equal(det[1], f32[1]) and _bitwise_equal(det[2], f32[2])


@pytest.mark.parametrize("algo", list(DET_ALGOS))
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("scale_a,scale_g", [(2.0 ** 40, 2.0 ** -60), (2.0 ** -50, 2.0 ** 30),
                                              (1e-30, 1e-6)], ids=["big_a", "big_g", "tiny"])
def test_deterministic_scale_follows_the_input_magnitudes(scale_a, scale_g, dtype, algo):
    """The fixed-point scale is set from max|a| and max|g| on the device:
    results stay at the strict relative bar far from unit magnitudes."""
    if dtype == torch.float16 and (max(scale_a, scale_g) > 6e4 or min(scale_a, scale_g) < 1e-4):
        pytest.skip("outside the fp16 range")
    kw, lo, hi = ALGO_CASES[0][1], 0.0, 1.0
    value, shapes, starts, loc, attn, g = _inputs(kw, lo, hi, torch.float32, seed=6)
    attn = (attn * scale_a).to(dtype)
    g = (g * scale_g).to(dtype)
    value, loc = value.to(dtype), loc.to(dtype)
    gv, _, _ = _ops._backward(value, shapes, starts, loc, attn, g, True, DET_ALGOS[algo])
    _, ref = oracle64(value, shapes, starts, loc, attn, g)
    scale = ref[0].abs().max()
    assert scale > 0
    tol = STRICT_TOL[dtype]
    torch.testing.assert_close((gv.double().cpu() / scale), ref[0] / scale, rtol=tol["rtol"],
                               atol=tol["atol"])


@pytest.mark.parametrize("algo", list(DET_ALGOS))
def test_deterministic_zero_gradient(algo):
    kw, lo, hi = ALGO_CASES[0][1], 0.0, 1.0
    value, shapes, starts, loc, attn, g = _inputs(kw, lo, hi, torch.bfloat16)
    gv, gl, ga = _ops._backward(value, shapes, starts, loc, attn, torch.zeros_like(g), True, DET_ALGOS[algo])
    assert (gv == 0).all() and (gl == 0).all() and (ga == 0).all()


@pytest.mark.parametrize("algo", list(DET_ALGOS))
@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_deterministic_non_finite_inputs_fall_back_to_fp32(dtype, algo):
    """A non-finite grad_out element: the fixed-point range is undefined, so
    the scatter falls back to fp32 atomics -- Inf / NaN land in the same
    elements as with fp32 accumulation, finite elements match it."""
    kw, lo, hi = ALGO_CASES[0][1], 0.0, 1.0
    value, shapes, starts, loc, attn, g = _inputs(kw, lo, hi, dtype, seed=8)
    g = g.clone()
    g[0, 3, 1, 5] = float("inf")
    g[1, 7, 2, 0] = float("nan")
    gv, _, _ = _ops._backward(value, shapes, starts, loc, attn, g, True, DET_ALGOS[algo])
    gr, _, _ = _ops._backward(value, shapes, starts, loc, attn, g, True, _clib.MSDA_BWD_FORCE_SCATTER)
    assert torch.equal(torch.isnan(gv), torch.isnan(gr))
    assert torch.equal(torch.isinf(gv), torch.isinf(gr))
    fin = torch.isfinite(gr)
    assert (~fin).any() and fin.float().mean() > 0.9
    torch.testing.assert_close(gv[fin].float(), gr[fin].float(), **STRICT_TOL[dtype])


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("name,kw", FUSED_CASES, ids=[c[0] for c in FUSED_CASES])
def test_deterministic_fused_prologue(name, kw, dtype):
    value, shapes, starts, ref, off, logits = _fused_inputs(kw, dtype)
    B, Q, M, D = kw["B"], kw["Q"], kw["M"], kw["D"]
    out = _ops._forward_fused(value, shapes, starts, ref, off, logits)
    g = cases.grad_output_like(out)
    gv, goff, glog = _ops._backward_fused(value, shapes, starts, ref, off, logits, g, True, 0,
                                          deterministic=True)
    out_r, gv_r, _, goff_r, glog_r, loc = _fused_reference(value, shapes, ref, off, logits, g)
    tol = STRICT_TOL[dtype]
    close(gv, gv_r, tol, "grad_value")
    close(glog, glog_r, tol, "grad_logits")
    keep = ~cases.kink_mask(loc, shapes, _kink_eps(dtype))
    torch.testing.assert_close(goff.double().cpu()[keep], goff_r[keep], **tol)
    perm = torch.randperm(Q, generator=torch.Generator().manual_seed(2)).to(DEV)
    gvp, _, _ = _ops._backward_fused(value, shapes, starts, ref[:, perm].contiguous(), off[:, perm].contiguous(),
                                     logits[:, perm].contiguous(), g.view(B, Q, M, D)[:, perm].contiguous(),
                                     True, 0, deterministic=True)
    assert _bitwise_equal(gv, gvp)


def test_public_op_under_torch_deterministic_algorithms():
    """With torch.use_deterministic_algorithms(True) the op's backward takes
    the fixed-point path: identical bits to deterministic=True, and to the
    run on permuted queries; the flag is restored afterwards."""
    kw, lo, hi = ALGO_CASES[0][1], 0.0, 1.0
    value, shapes, starts, loc, attn, g = _inputs(kw, lo, hi, torch.bfloat16, seed=12)
    B, Q, M, D = g.shape

    def grads(loc_, attn_, g_, **kw_):
        v = value.clone().requires_grad_(True)
        l_ = loc_.clone().requires_grad_(True)
        a_ = attn_.clone().requires_grad_(True)
        multi_scale_deformable_attention(v, shapes, starts, l_, a_, **kw_).backward(g_.reshape(B, Q, M * D))
        return v.grad

    explicit = grads(loc, attn, g, deterministic=True)
    before = torch.are_deterministic_algorithms_enabled()
    try:
        torch.use_deterministic_algorithms(True)
        implicit = grads(loc, attn, g)
        perm = torch.randperm(Q, generator=torch.Generator().manual_seed(1)).to(DEV)
        permuted = grads(loc[:, perm], attn[:, perm], g[:, perm])
    finally:
        torch.use_deterministic_algorithms(before)
    assert _bitwise_equal(explicit, implicit)
    assert _bitwise_equal(explicit, permuted)
    _, ref = oracle64(value, shapes, starts, loc, attn, g)
    close(explicit, ref[0], STRICT_TOL[torch.bfloat16], "grad_value")
    # The fused op follows the same switch.
    value2, shapes2, starts2, ref2, off2, logits2 = _fused_inputs(FUSED_CASES[0][1], torch.bfloat16)
    outs = []
    for det in (True, None):
        leaves = [t.clone().requires_grad_(True) for t in (value2, ref2, off2, logits2)]
        try:
            torch.use_deterministic_algorithms(det is None)
            out = multi_scale_deformable_attention_fused(leaves[0], shapes2, None, *leaves[1:],
                                                         deterministic=det)
            out.backward(cases.grad_output_like(out.detach()))
        finally:
            torch.use_deterministic_algorithms(before)
        outs.append(leaves[0].grad)
    assert _bitwise_equal(outs[0], outs[1])


def test_deterministic_backward_in_a_cuda_graph():
    kw, lo, hi = ALGO_CASES[0][1], 0.0, 1.0
    value, shapes, starts, loc, attn, g = _inputs(kw, lo, hi, torch.bfloat16, seed=13)
    eager = _ops._backward(value, shapes, starts, loc, attn, g, True, DET)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            _ops._backward(value, shapes, starts, loc, attn, g, True, DET)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static = _ops._backward(value, shapes, starts, loc, attn, g, True, DET)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert all(_bitwise_equal(a, b) for a, b in zip(static, eager))

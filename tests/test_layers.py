"""MSDACrossAttention (the layer around the operator, reference
labs/solutions/lab00.py:169-208): parameter layout on CPU; forward and
training-gradient parity on the GPU against the same layer whose attention
is the CPU oracle's grid_sample restatement (test infrastructure)."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(REPO), str(REPO / "msda-triton_b200")]

from msda_triton_b200 import MSDACrossAttention  # noqa: E402
from msda_triton_b200 import layers as msda_layers  # noqa: E402
from oracle import msda_oracle as orc  # noqa: E402

SHAPES = [(16, 20), (8, 10), (4, 5), (2, 3)]


def test_parameters_match_the_reference_layer():
    layer = MSDACrossAttention(64, 8, 4, 4)
    got = {k: tuple(v.shape) for k, v in layer.state_dict().items()}
    assert got == {
        "value_proj.weight": (64, 64), "value_proj.bias": (64,),
        "offset_proj.weight": (256, 64), "offset_proj.bias": (256,),
        "weight_proj.weight": (128, 64), "weight_proj.bias": (128,),
        "out_proj.weight": (64, 64), "out_proj.bias": (64,),
    }
    with pytest.raises(ValueError):
        MSDACrossAttention(60, 8, 4, 4)


def test_sampling_locations_and_weights():
    torch.manual_seed(0)
    layer = MSDACrossAttention(32, 4, 4, 2)
    q = torch.randn(2, 5, 32)
    ref = torch.rand(2, 5, 2)
    shapes = torch.tensor(SHAPES)
    loc, w = layer.sampling(q, ref, shapes)
    assert loc.shape == (2, 5, 4, 4, 2, 2) and w.shape == (2, 5, 4, 4, 2)
    torch.testing.assert_close(w.sum((-1, -2)), torch.ones(2, 5, 4))
    off = layer.offset_proj(q).view(2, 5, 4, 4, 2, 2)
    for lvl, (h, wd) in enumerate(SHAPES):
        torch.testing.assert_close(loc[:, :, :, lvl, :, 0],
                                   ref[:, :, None, None, 0] + off[:, :, :, lvl, :, 0] / wd)
        torch.testing.assert_close(loc[:, :, :, lvl, :, 1],
                                   ref[:, :, None, None, 1] + off[:, :, :, lvl, :, 1] / h)


def _oracle_layer_forward(layer, query, ref, value, shapes):
    """The same layer with the oracle's grid_sample attention (fp32, CPU)."""
    B, Q, C = query.shape
    S = value.shape[1]
    v = layer.value_proj(value).view(B, S, layer.num_heads, layer.head_dim)
    loc, w = layer.sampling(query, ref, shapes)
    return layer.out_proj(orc.msda_grid_sample(v, shapes, loc, w))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=str)
def test_layer_forward_and_training_gradients_match_the_oracle(dtype):
    torch.manual_seed(3)
    C, M, L, K = 64, 8, 4, 4
    layer = MSDACrossAttention(C, M, L, K)
    with torch.no_grad():  # larger offsets so points spread over each level
        layer.offset_proj.weight.mul_(8.0)
    ref_layer = MSDACrossAttention(C, M, L, K)
    ref_layer.load_state_dict(layer.state_dict())
    shapes = torch.tensor(SHAPES)
    S = sum(h * w for h, w in SHAPES)
    query = torch.randn(2, 30, C)
    ref = torch.rand(2, 30, 2)
    value = torch.randn(2, S, C)
    g = torch.randn(2, 30, C)

    dev = torch.device("cuda")
    layer = layer.to(dev, dtype)
    out = layer(query.to(dev, dtype), ref.to(dev, dtype), value.to(dev, dtype), shapes.to(dev))
    out.backward(g.to(dev, dtype))

    ref_out = _oracle_layer_forward(ref_layer, query, ref, value, shapes)
    ref_out.backward(g)
    # fp32: relative Frobenius-norm errors at fp32 rounding. bf16: the layer
    # rounds its GEMMs, offsets and gradients to bf16, and bf16 offsets put a
    # sizeable share of sampling points exactly on integer pixel coordinates,
    # where the bilinear derivative is one-sided and the fp32 oracle (whose
    # offsets are not rounded) takes the other side: those points dominate
    # offset_proj's summed gradient. The bf16 check is therefore the output
    # and the direction of every parameter gradient (the operator itself is
    # held to the strict bar in test_gpu_parity.py).
    if dtype == torch.float32:
        assert _rel(out.float().cpu(), ref_out) < 1e-4
        for (name, p), (_, rp) in zip(layer.named_parameters(), ref_layer.named_parameters()):
            assert _rel(p.grad.float().cpu(), rp.grad) < 1e-4, (name, _rel(p.grad.float().cpu(), rp.grad))
    else:
        assert _rel(out.float().cpu(), ref_out) < 3e-2
        for (name, p), (_, rp) in zip(layer.named_parameters(), ref_layer.named_parameters()):
            a, b = p.grad.double().cpu().flatten(), rp.grad.double().flatten()
            cos = float(a @ b / (a.norm() * b.norm()))
            assert cos > 0.95, (name, cos)


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-12))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=str)
def test_fused_layer_matches_unfused_layer(dtype):
    """fp32: the fused and unfused layers agree to fp32 rounding. bf16: the
    unfused prologue rounds the sampling locations themselves to bf16 (up to
    ~0.3 px on the finest level), the fused one works from the offsets in
    fp32, so the fused layer must be at least as close to the fp32 oracle."""
    torch.manual_seed(5)
    dev = torch.device("cuda")
    base = MSDACrossAttention(64, 8, 4, 4)
    with torch.no_grad():
        base.offset_proj.weight.mul_(8.0)
    shapes = torch.tensor(SHAPES)
    S = sum(h * w for h, w in SHAPES)
    q, ref, v, g = torch.randn(2, 30, 64), torch.rand(2, 30, 2), torch.randn(2, S, 64), torch.randn(2, 30, 64)
    oracle = MSDACrossAttention(64, 8, 4, 4)
    oracle.load_state_dict(base.state_dict())
    ref_out = _oracle_layer_forward(oracle, q, ref, v, shapes)
    ref_out.backward(g)
    results = {}
    for fused in (True, False):
        layer = MSDACrossAttention(64, 8, 4, 4, fused=fused)
        layer.load_state_dict(base.state_dict())
        layer = layer.to(dev, dtype)
        out = layer(*(t.to(dev, dtype) for t in (q, ref, v)), shapes.to(dev))
        out.backward(g.to(dev, dtype))
        results[fused] = (out.float().cpu(), {n: p.grad.float().cpu() for n, p in layer.named_parameters()})
    if dtype == torch.float32:
        torch.testing.assert_close(results[True][0], results[False][0], rtol=1e-4, atol=1e-4)
        for n in results[True][1]:
            assert _rel(results[True][1][n], results[False][1][n]) < 1e-4, n
    else:
        err = {f: _rel(results[f][0], ref_out) for f in (True, False)}
        assert err[True] <= err[False] * 1.1 + 1e-3, err
        assert err[True] < 3e-2

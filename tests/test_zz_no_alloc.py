"""The backward entry point for callers that cannot allocate device memory.

msda_backward_noalloc exists for callers that may not call cudaMalloc while
they run -- a runtime that plans all device memory ahead of time (a
TensorRT-style plugin's enqueue), an embedder without a device allocator of
its own. Instead of
a caller-provided fp32 workspace it uses a static device array inside the
library (16 MiB). These tests call it through the C ABI and check it against
msda_backward, the regular entry point, on two calls in a row: the shared
scratch keeps the previous call's contents, so the second call proves it is
cleared before use.

The file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import cases
from msda_triton_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
FLAGS = _lib.MSDA_BWD_FP32_ACCUM | _lib.MSDA_BWD_FORCE_SCATTER
CODE = {torch.float32: _lib.MSDA_DTYPE_F32, torch.float16: _lib.MSDA_DTYPE_F16,
        torch.bfloat16: _lib.MSDA_DTYPE_BF16}
TOL = {torch.float32: dict(rtol=1e-5, atol=1e-5), torch.float16: dict(rtol=1e-2, atol=1e-4),
       torch.bfloat16: dict(rtol=1e-2, atol=1e-4)}


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _inputs(dtype, seed):
    value, shapes, starts, loc, attn = cases.make_inputs(
        B=2, Q=100, M=4, D=32, K=4, shapes=[(24, 32), (12, 16), (6, 8)], dtype=dtype, device=DEV,
        loc_lo=-0.1, loc_hi=1.1, seed=seed)
    g = torch.randn(2, 100, 4, 32, generator=torch.Generator().manual_seed(seed + 7)).to(DEV, dtype)
    return value, shapes, starts, loc, attn, g


def _dims(value, loc):
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = loc.shape
    return B, S, Q, M, D, L, K


def _regular(lib, value, shapes, starts, loc, attn, g):
    """msda_backward with a workspace the caller allocated (torch)."""
    gv, gl, ga = torch.empty_like(value), torch.empty_like(loc), torch.empty_like(attn)
    B, S, Q, M, D, L, K = _dims(value, loc)
    code = CODE[value.dtype]
    nbytes = lib.msda_backward_workspace_size(B, S, Q, M, D, L, K, code, FLAGS)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=DEV)
    rc = lib.msda_backward(_p(value), _p(shapes), _p(starts), _p(loc), _p(attn), _p(g), _p(gv),
                           _p(gl), _p(ga), _p(ws), nbytes, B, S, Q, M, D, L, K, code, FLAGS,
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check("msda_backward", rc)
    return gv, gl, ga


def _no_alloc(lib, value, shapes, starts, loc, attn, g, outs):
    """msda_backward_noalloc into caller-provided outputs; no workspace."""
    gv, gl, ga = outs
    B, S, Q, M, D, L, K = _dims(value, loc)
    rc = lib.msda_backward_noalloc(_p(value), _p(shapes), _p(starts), _p(loc), _p(attn), _p(g),
                                   _p(gv), _p(gl), _p(ga), B, S, Q, M, D, L, K, CODE[value.dtype],
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check("msda_backward_noalloc", rc)
    return gv, gl, ga


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=str)
def test_no_alloc_backward_matches_regular_backward_twice(dtype):
    lib = _lib.load()
    # Two calls in a row on different inputs: the second must not see the
    # first call's partial sums left in the shared static scratch.
    for seed in (0, 1):
        args = _inputs(dtype, seed)
        want = _regular(lib, *args)
        # Outputs pre-filled with NaN: every element must be written.
        outs = tuple(torch.full_like(t, float("nan")) for t in want)
        got = _no_alloc(lib, *args, outs)
        torch.cuda.synchronize()
        for name, a, b in zip(("grad_value", "grad_loc", "grad_attn"), got, want):
            torch.testing.assert_close(a.float(), b.float(), **TOL[dtype],
                                       msg=lambda m, n=name: f"seed {seed} {n}: {m}")


def test_no_alloc_backward_rejects_sizes_beyond_the_static_scratch():
    lib = _lib.load()
    # 2 * 8192 * 8 * 32 fp32 elements = 16 MiB + (one row more than fits).
    B, S, Q, M, D, L, K = 2, 8193, 10, 8, 32, 1, 4
    need = lib.msda_backward_workspace_size(B, S, Q, M, D, L, K, _lib.MSDA_DTYPE_BF16, FLAGS)
    assert need > _lib.MSDA_NOALLOC_SCRATCH_BYTES
    vp = ctypes.c_void_p
    rc = lib.msda_backward_noalloc(vp(256), vp(256), vp(256), vp(256), vp(256), vp(256), vp(256),
                                   vp(256), vp(256), B, S, Q, M, D, L, K, _lib.MSDA_DTYPE_BF16,
                                   vp(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert b"static scratch" in lib.msda_last_error()

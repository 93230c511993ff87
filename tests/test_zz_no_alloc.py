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
    # Null buffers: the scratch limit is checked first; were that check ever
    # to move behind the launch, msda_backward would still refuse the nulls
    # on the host (and the message would not name the static scratch).
    vp = ctypes.c_void_p
    rc = lib.msda_backward_noalloc(vp(0), vp(0), vp(0), vp(0), vp(0), vp(0), vp(0), vp(0), vp(0),
                                   B, S, Q, M, D, L, K, _lib.MSDA_DTYPE_BF16,
                                   vp(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert b"static scratch" in lib.msda_last_error()
    # Sizes msda_backward does not support fail as they fail there, before
    # the scratch limit is considered.
    rc = lib.msda_backward_noalloc(vp(0), vp(0), vp(0), vp(0), vp(0), vp(0), vp(0), vp(0), vp(0),
                                   1, 1 << 28, 1, 8, 1, 1, 1, _lib.MSDA_DTYPE_BF16,
                                   vp(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.MSDA_ERR_UNSUPPORTED and b"2^31" in lib.msda_last_error()


def test_no_alloc_backward_on_a_side_stream():
    """On a non-default stream of the current device: the same gradients as
    msda_backward, twice in a row."""
    lib = _lib.load()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for seed in (2, 3):
            args = _inputs(torch.bfloat16, seed)
            want = _regular(lib, *args)
            outs = tuple(torch.full_like(t, float("nan")) for t in want)
            got = _no_alloc(lib, *args, outs)
            side.synchronize()
            for a, b in zip(got, want):
                torch.testing.assert_close(a.float(), b.float(), **TOL[torch.bfloat16])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_no_alloc_backward_refuses_a_stream_of_another_device():
    lib = _lib.load()
    args = _inputs(torch.bfloat16, 4)
    outs = tuple(torch.empty_like(t) for t in (args[0], args[3], args[4]))
    other = torch.cuda.Stream(device=1)
    B, S, Q, M, D, L, K = _dims(args[0], args[3])
    rc = lib.msda_backward_noalloc(*(_p(t) for t in args), *(_p(t) for t in outs), B, S, Q, M, D, L, K,
                                   CODE[torch.bfloat16], ctypes.c_void_p(other.cuda_stream))
    assert rc == _lib.MSDA_ERR_INVALID_ARGUMENT and b"belongs to device" in lib.msda_last_error()

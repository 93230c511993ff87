"""Host-side checks that need no GPU: the C ABI library loads and exports
every symbol include/msda_b200.h declares, its argument checks reject bad
calls before touching the device, and the Python op validates like the
reference (src/msda_triton/ops.py:140-171; tests/test_msda.py:254-271)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

import cases
from hostonly import host_only
from msda_triton_b200 import MultiScaleDeformableAttnFunction, _lib, multi_scale_deformable_attention
from msda_triton_b200.ops import _use_fp32_grad_accum

HEADER = Path(__file__).resolve().parent.parent / "include" / "msda_b200.h"


def _declared():
    text = HEADER.read_text()
    return re.findall(r"MSDA_API\s+[\w\s\*]+?\b(msda_\w+)\s*\(", text)


def test_header_declares_the_abi():
    assert set(_declared()) == {"msda_version", "msda_last_error", "msda_forward",
                                "msda_backward_workspace_size", "msda_backward",
                                "msda_backward_noalloc", "msda_forward_fused",
                                "msda_backward_fused", "msda_grid_sample_forward",
                                "msda_grid_sample_backward_workspace_size",
                                "msda_grid_sample_backward", "msda_roi_align_forward",
                                "msda_roi_align_backward_workspace_size",
                                "msda_roi_align_backward", "msda_transpose"}


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name
    assert _lib.version().startswith("msda_b200 ")
    assert "sm_100a" in _lib.version()


def _fwd(lib, **over):
    args = dict(value=1, shapes=8, starts=8, loc=8, attn=8, out=8, B=1, S=4, Q=1, M=1, D=4, L=1,
                K=1, dtype=0)
    args.update(over)
    vp = ctypes.c_void_p
    return lib.msda_forward(vp(args["value"]), vp(args["shapes"]), vp(args["starts"]),
                            vp(args["loc"]), vp(args["attn"]), vp(args["out"]), args["B"],
                            args["S"], args["Q"], args["M"], args["D"], args["L"], args["K"],
                            args["dtype"], vp(0))


@host_only
def test_abi_rejects_bad_arguments_before_any_device_work():
    lib = _lib.load()
    assert _fwd(lib, dtype=7) == _lib.MSDA_ERR_UNSUPPORTED
    assert b"dtype" in lib.msda_last_error()
    assert _fwd(lib, L=0) == _lib.MSDA_ERR_UNSUPPORTED
    assert _fwd(lib, L=17) == _lib.MSDA_ERR_UNSUPPORTED
    assert _fwd(lib, S=0) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert _fwd(lib, S=(1 << 30) + 1) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert _fwd(lib, D=0) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert _fwd(lib, B=-1) == _lib.MSDA_ERR_INVALID_ARGUMENT
    # A batch item's value slice is addressed with 32-bit offsets.
    assert _fwd(lib, S=1 << 28, M=8, D=1) == _lib.MSDA_ERR_UNSUPPORTED
    assert b"2^31" in lib.msda_last_error()
    # Null pointers and misaligned sampling locations are caught on the host.
    assert _fwd(lib, value=0) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert b"null" in lib.msda_last_error()
    assert _fwd(lib, loc=6) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert b"misaligned" in lib.msda_last_error()
    # Empty work (B == 0 or Q == 0) succeeds without launching anything.
    assert _fwd(lib, B=0, value=0, out=0) == _lib.MSDA_OK
    assert _fwd(lib, Q=0) == _lib.MSDA_OK
    assert lib.msda_last_error() == b""


def test_abi_workspace_size():
    lib = _lib.load()
    f = _lib.MSDA_BWD_FP32_ACCUM
    ws = lambda B, S, Q, M, D, L, K, dt, fl: lib.msda_backward_workspace_size(  # noqa: E731
        B, S, Q, M, D, L, K, dt, fl)
    full = 2 * 10 * 3 * 8 * 4
    # Dense sampling (Q*L*K per value row > 1) takes the scatter path: fp32
    # accumulation of fp16/bf16 needs the workspace, fp32 and native do not.
    assert ws(2, 10, 50, 3, 8, 1, 4, _lib.MSDA_DTYPE_BF16, f) == full
    assert ws(2, 10, 50, 3, 8, 1, 4, _lib.MSDA_DTYPE_F16, f) == full
    assert ws(2, 10, 50, 3, 8, 1, 4, _lib.MSDA_DTYPE_F32, f) == 0
    assert ws(2, 10, 50, 3, 8, 1, 4, _lib.MSDA_DTYPE_BF16, 0) == 0
    # Sparse sampling takes the hit-counted scatter: per-row counts (padded to
    # 256 bytes) plus fp32 rows for fp16/bf16, counts only for fp32.
    counted = 256 + 2 * 10 * 3 * 8 * 4
    assert ws(2, 10, 2, 3, 8, 1, 4, _lib.MSDA_DTYPE_BF16, f) == counted
    assert ws(2, 10, 2, 3, 8, 1, 4, _lib.MSDA_DTYPE_F32, 0) == 256
    assert ws(2, 10, 50, 3, 8, 1, 4, _lib.MSDA_DTYPE_BF16, f | _lib.MSDA_BWD_FORCE_COUNTED) == counted
    # Forcing the plain scatter keeps the full fp32 workspace.
    assert ws(2, 10, 2, 3, 8, 1, 4, _lib.MSDA_DTYPE_BF16, f | _lib.MSDA_BWD_FORCE_SCATTER) == full
    # Unknown flag bits (4 was the removed owner algorithm's) size nothing.
    assert ws(2, 10, 50, 3, 8, 1, 4, _lib.MSDA_DTYPE_BF16, f | 4) == 0


def test_abi_workspace_size_deterministic():
    """Deterministic grad_value: the scatter (dense sampling) takes a 256-byte
    absmax header, then a 64-bit fixed-point element per grad_value element;
    the hit-counted algorithm (sparse sampling) takes per-row counts and
    64-bit rows, with the header before the counts (fp32 values) or per-row
    bounds after them (fp16 / bf16); whatever fp32_grad_accum says."""
    lib = _lib.load()
    d = _lib.MSDA_BWD_DETERMINISTIC
    ws = lambda Q, dt, fl: lib.msda_backward_workspace_size(2, 10, Q, 3, 8, 1, 4, dt, fl)  # noqa: E731
    elems = 2 * 10 * 3 * 8
    scatter = 256 + elems * 8
    for dt in (_lib.MSDA_DTYPE_F32, _lib.MSDA_DTYPE_F16, _lib.MSDA_DTYPE_BF16):
        counted = 256 + 256 + elems * 8  # header + counts (fp32) or (count, bound) pairs (fp16 / bf16)
        for f in (0, _lib.MSDA_BWD_FP32_ACCUM):
            assert ws(50, dt, d | f) == scatter
            assert ws(2, dt, d | f) == counted
            assert ws(2, dt, d | f | _lib.MSDA_BWD_FORCE_SCATTER) == scatter
            assert ws(50, dt, d | f | _lib.MSDA_BWD_FORCE_COUNTED) == counted


@host_only
def test_abi_deterministic_flag_checks():
    text = HEADER.read_text()
    assert re.search(r"#define MSDA_BWD_DETERMINISTIC (\d+)u", text).group(1) == str(_lib.MSDA_BWD_DETERMINISTIC)
    lib = _lib.load()
    vp = ctypes.c_void_p
    call = lambda flags, ws=0: lib.msda_backward(  # noqa: E731
        vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16),
        vp(ws), 0, 1, 4, 1, 1, 8, 1, 1, _lib.MSDA_DTYPE_BF16, flags, vp(0))
    # Flag bits the library does not know are refused.
    assert call(_lib.MSDA_BWD_DETERMINISTIC | 4) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert b"unknown flag" in lib.msda_last_error()
    # The fixed-point accumulator lives in the workspace.
    assert call(_lib.MSDA_BWD_DETERMINISTIC) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert b"deterministic" in lib.msda_last_error()


def test_deterministic_option_follows_torch_flag():
    from msda_triton_b200.ops import _use_deterministic
    assert _use_deterministic(True) and not _use_deterministic(False)
    before = torch.are_deterministic_algorithms_enabled()
    try:
        torch.use_deterministic_algorithms(True)
        assert _use_deterministic(None)
        torch.use_deterministic_algorithms(False)
        assert not _use_deterministic(None)
    finally:
        torch.use_deterministic_algorithms(before)


@host_only
def test_gather_abi_checks_before_any_device_work():
    """grid_sample / roi_align entry points: argument checks on the host,
    workspace sizes, and empty work as a no-op (no device touched)."""
    lib = _lib.load()
    vp = ctypes.c_void_p
    gs = lambda **o: lib.msda_grid_sample_forward(  # noqa: E731
        vp(o.get("x", 16)), vp(o.get("g", 16)), vp(o.get("y", 16)), o.get("N", 1), o.get("H", 4),
        o.get("W", 4), o.get("C", 8), o.get("Ho", 2), o.get("Wo", 2), o.get("mode", 0), o.get("pad", 0), 0,
        o.get("dtype", 0), vp(0))
    assert gs(dtype=9) == _lib.MSDA_ERR_UNSUPPORTED
    assert gs(pad=3) == _lib.MSDA_ERR_UNSUPPORTED
    assert b"padding_mode" in lib.msda_last_error()
    assert gs(mode=2) == _lib.MSDA_ERR_UNSUPPORTED  # bicubic is not built
    assert b"mode" in lib.msda_last_error()
    assert gs(H=0) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert gs(C=0) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert gs(x=0) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert gs(g=6, dtype=0) == _lib.MSDA_ERR_INVALID_ARGUMENT  # grid needs 8-byte alignment for fp32
    assert gs(Ho=0) == _lib.MSDA_OK and gs(N=0, x=0, g=0, y=0) == _lib.MSDA_OK
    ws = lib.msda_grid_sample_backward_workspace_size
    n = 2 * 5 * 6 * 8
    assert ws(2, 5, 6, 8, 3, 3, _lib.MSDA_DTYPE_BF16, _lib.MSDA_BWD_FP32_ACCUM) == n * 4
    assert ws(2, 5, 6, 8, 3, 3, _lib.MSDA_DTYPE_F32, _lib.MSDA_BWD_FP32_ACCUM) == 0
    assert ws(2, 5, 6, 8, 3, 3, _lib.MSDA_DTYPE_BF16, 0) == 0
    assert ws(2, 5, 6, 8, 3, 3, _lib.MSDA_DTYPE_F32, _lib.MSDA_BWD_DETERMINISTIC) == 256 + n * 8
    rws = lib.msda_roi_align_backward_workspace_size
    assert rws(2, 5, 6, 8, _lib.MSDA_DTYPE_F16, _lib.MSDA_BWD_FP32_ACCUM) == n * 4
    assert rws(2, 5, 6, 8, _lib.MSDA_DTYPE_F16, _lib.MSDA_BWD_DETERMINISTIC) == 256 + n * 8
    ra = lambda **o: lib.msda_roi_align_forward(  # noqa: E731
        vp(16), vp(16), vp(16), 1, 4, 4, 8, o.get("K", 3), o.get("ph", 2), 2, 1.0, -1, 0, 0, vp(0))
    assert ra(ph=0) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert ra(K=0) == _lib.MSDA_OK
    # An explicit sampling ratio beyond the kernels' 1024 samples per bin side
    # would be clamped (torchvision honours it): refused instead.
    rc = lib.msda_roi_align_forward(vp(16), vp(16), vp(16), 1, 4, 4, 8, 3, 2, 2, 1.0, 1025, 0, 0, vp(0))
    assert rc == _lib.MSDA_ERR_UNSUPPORTED and b"sampling_ratio" in lib.msda_last_error()
    # The deterministic backward needs its fixed-point workspace.
    rc = lib.msda_roi_align_backward(vp(16), vp(16), vp(16), vp(0), 0, 1, 4, 4, 8, 3, 2, 2, 1.0, -1, 0,
                                     0, _lib.MSDA_BWD_DETERMINISTIC, vp(0))
    assert rc == _lib.MSDA_ERR_INVALID_ARGUMENT and b"workspace" in lib.msda_last_error()


@host_only
def test_transpose_abi_checks_before_any_device_work():
    """msda_transpose: dtype, sizes, pointers and alignment are checked on
    the host, empty work is a no-op, and sizes no grid can cover are refused
    (N past gridDim.z; both tile counts past gridDim.y) -- all without a
    device (the pointers below are never dereferenced)."""
    lib = _lib.load()
    vp = ctypes.c_void_p
    t = lambda N=1, R=64, C=64, dtype=0, src=256, dst=512: lib.msda_transpose(  # noqa: E731
        vp(src), vp(dst), N, R, C, dtype, vp(0))
    assert t(dtype=7) == _lib.MSDA_ERR_UNSUPPORTED
    assert t(R=-1) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert t(N=0, src=0, dst=0) == _lib.MSDA_OK and t(C=0) == _lib.MSDA_OK
    assert t(src=0) == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert t(dst=514) == _lib.MSDA_ERR_INVALID_ARGUMENT  # fp32 needs 4-byte alignment
    assert t(N=70000) == _lib.MSDA_ERR_UNSUPPORTED
    assert t(R=64 * 65536, C=64 * 65536) == _lib.MSDA_ERR_UNSUPPORTED
    assert b"too large" in lib.msda_last_error()


def test_gather_nchw_gradient_is_asked_for_where_the_backward_rounds():
    """The host asks for MSDA_BWD_GRAD_INPUT_NCHW only where the backward
    has a rounding pass to fold the transpose into."""
    from msda_triton_b200.gather import _backward_rounds, _bwd_flags
    for dtype in (torch.float16, torch.bfloat16):
        assert _backward_rounds(dtype, _bwd_flags(dtype, None, False))       # fp32 accumulation by default
        assert not _backward_rounds(dtype, _bwd_flags(dtype, False, False))  # native atomics: no pass
        assert _backward_rounds(dtype, _bwd_flags(dtype, False, True))
    assert not _backward_rounds(torch.float32, _bwd_flags(torch.float32, None, False))
    assert not _backward_rounds(torch.float32, _bwd_flags(torch.float32, True, False))
    assert _backward_rounds(torch.float32, _bwd_flags(torch.float32, None, True))


@host_only
def test_gather_nchw_gradient_flag():
    """MSDA_BWD_GRAD_INPUT_NCHW: the header value, the workspace it adds
    (the accumulator in the data type when no other flag asks for one), its
    refusal by the MSDA backward, and its size checks before any launch."""
    text = HEADER.read_text()
    assert re.search(r"#define MSDA_BWD_GRAD_INPUT_NCHW (\d+)u", text).group(1) == str(_lib.MSDA_BWD_GRAD_INPUT_NCHW)
    lib = _lib.load()
    vp = ctypes.c_void_p
    NCHW = _lib.MSDA_BWD_GRAD_INPUT_NCHW
    ws = lib.msda_grid_sample_backward_workspace_size
    rws = lib.msda_roi_align_backward_workspace_size
    n = 2 * 5 * 6 * 8
    assert ws(2, 5, 6, 8, 3, 3, _lib.MSDA_DTYPE_F32, NCHW) == n * 4
    assert ws(2, 5, 6, 8, 3, 3, _lib.MSDA_DTYPE_BF16, NCHW) == n * 2
    assert ws(2, 5, 6, 8, 3, 3, _lib.MSDA_DTYPE_BF16, NCHW | _lib.MSDA_BWD_FP32_ACCUM) == n * 4
    assert rws(2, 5, 6, 8, _lib.MSDA_DTYPE_F16, NCHW | _lib.MSDA_BWD_DETERMINISTIC) == 256 + n * 8
    assert rws(2, 5, 6, 8, _lib.MSDA_DTYPE_F32, NCHW) == n * 4
    # The flag belongs to the gathers: the MSDA backward refuses it.
    rc = lib.msda_backward(vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16),
                           vp(16), 1 << 20, 1, 4, 1, 1, 8, 1, 1, _lib.MSDA_DTYPE_BF16, NCHW, vp(0))
    assert rc == _lib.MSDA_ERR_UNSUPPORTED and b"GRAD_INPUT_NCHW" in lib.msda_last_error()
    # Without its workspace the call fails on the host.
    rc = lib.msda_roi_align_backward(vp(16), vp(16), vp(16), vp(0), 0, 1, 4, 4, 8, 3, 2, 2, 1.0, -1, 0,
                                     _lib.MSDA_DTYPE_F32, NCHW, vp(0))
    assert rc == _lib.MSDA_ERR_INVALID_ARGUMENT and b"workspace" in lib.msda_last_error()
    # N beyond the transpose grid's z limit is refused before any launch.
    big = 70000
    rc = lib.msda_roi_align_backward(vp(16), vp(16), vp(16), vp(256), 1 << 40, big, 1, 1, 4, 0, 2, 2, 1.0,
                                     -1, 0, _lib.MSDA_DTYPE_F32, NCHW, vp(0))
    assert rc == _lib.MSDA_ERR_UNSUPPORTED and b"NCHW" in lib.msda_last_error()


def test_gather_op_validation():
    from msda_triton_b200 import grid_sample, roi_align
    x = torch.zeros(1, 4, 5, 5)
    g = torch.zeros(1, 3, 3, 2)
    with pytest.raises(ValueError, match="mode"):
        grid_sample(x, g, mode="linear")
    with pytest.raises(NotImplementedError, match="bicubic"):
        grid_sample(x, g, mode="bicubic")
    with pytest.raises(ValueError, match="padding_mode"):
        grid_sample(x, g, padding_mode="wrap")
    with pytest.raises(ValueError, match="grid"):
        grid_sample(x, torch.zeros(2, 3, 3, 2))
    with pytest.raises(ValueError, match="CUDA"):
        grid_sample(x, g)
    with pytest.raises(ValueError, match="boxes"):
        roi_align(x, torch.zeros(3, 4), 2)
    with pytest.raises(ValueError, match="CUDA"):
        roi_align(x, torch.zeros(3, 5), 2)


@host_only
def test_abi_backward_needs_workspace_for_fp32_accumulation():
    lib = _lib.load()
    vp = ctypes.c_void_p
    rc = lib.msda_backward(vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16), vp(16),
                           vp(0), 0, 1, 4, 1, 1, 8, 1, 1, _lib.MSDA_DTYPE_BF16,
                           _lib.MSDA_BWD_FP32_ACCUM | _lib.MSDA_BWD_FORCE_SCATTER, vp(0))
    assert rc == _lib.MSDA_ERR_INVALID_ARGUMENT
    assert b"workspace" in lib.msda_last_error()


def _small(dtype=torch.float32, device="cpu"):
    return cases.make_inputs(B=1, Q=8, M=2, D=16, shapes=[(6, 6)], K=2, dtype=dtype, device=device)


def test_op_validation_messages_match_reference():
    value, shapes, starts, loc, attn = _small()
    with pytest.raises(ValueError, match="attention_weights"):
        multi_scale_deformable_attention(value, shapes, starts, loc, attn[:, :, :, :, :1])
    with pytest.raises(ValueError, match="dtypes"):
        multi_scale_deformable_attention(value, shapes, starts, loc.half(), attn)
    with pytest.raises(ValueError, match="CUDA"):
        multi_scale_deformable_attention(value, shapes, starts, loc, attn)
    with pytest.raises(ValueError, match="CUDA .*MPS"):
        multi_scale_deformable_attention(torch.zeros(1, 1, 1, 1), torch.tensor([[1, 1]]), None,
                                         torch.zeros(1, 1, 1, 1, 1, 2), torch.zeros(1, 1, 1, 1, 1))
    with pytest.raises(ValueError, match="value must be"):
        multi_scale_deformable_attention(value[0], shapes, starts, loc, attn)
    with pytest.raises(ValueError, match="sampling_locations must be"):
        multi_scale_deformable_attention(value, shapes, starts, loc[..., :1], attn)
    with pytest.raises(ValueError, match="inconsistent"):
        multi_scale_deformable_attention(value, shapes, starts, loc[:, :, :1], attn)
    with pytest.raises(ValueError, match="spatial_shapes"):
        multi_scale_deformable_attention(value, shapes[:, :1], starts, loc, attn)
    with pytest.raises(ValueError, match="unsupported dtype"):
        multi_scale_deformable_attention(value.double(), shapes, starts, loc.double(), attn.double())


def test_default_accumulator_policy():
    assert _use_fp32_grad_accum(torch.zeros(1, dtype=torch.bfloat16)) is True
    assert _use_fp32_grad_accum(torch.zeros(1, dtype=torch.float16)) is True
    assert _use_fp32_grad_accum(torch.zeros(1, dtype=torch.float32)) is False


def test_package_surface():
    import msda_triton_b200 as pkg

    # The reference's export (src/msda_triton/__init__.py:9-12) plus the
    # mmcv-style Function, the layer around the operator and the sibling gathers.
    assert pkg.__all__[0] == "multi_scale_deformable_attention"
    assert set(pkg.__all__) == {"multi_scale_deformable_attention", "MultiScaleDeformableAttnFunction",
                                "MSDACrossAttention", "multi_scale_deformable_attention_fused",
                                "grid_sample", "roi_align"}
    assert callable(MultiScaleDeformableAttnFunction.apply)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "libmsda_b200.so")
    with pytest.raises(RuntimeError, match="not built"):
        _lib.load()

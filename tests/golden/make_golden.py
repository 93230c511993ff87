"""Generate the golden vectors under tests/golden/ from the REFERENCE's own code.

Runs only where the reference checkout is present; its path must be given
in MSDA_REFERENCE (``MSDA_REFERENCE=<checkout> python tests/golden/make_golden.py``).
It imports, by file path:

* tests/reference_impls.py -- ``msda_reference`` (grid_sample) and
  ``msda_naive`` (loops), the reference's CPU implementations;
* src/msda_triton/kernels.py -- the reference's Triton forward/backward
  kernels, executed on the CPU by Triton's interpreter (TRITON_INTERPRET=1),
  launched exactly as src/msda_triton/ops.py:46-52 and :81-89 launch them
  (BLOCK_Q=16 for the forward instead of the autotuner, which needs a GPU).

Inputs come from the reference suite's own generator
(tests/test_msda.py:65-77, imported from the reference) and, for the
``small`` operating point (B=1 Q=100 M=8 D=32 L=4 K=4, fp32), from ``msda_triton_b200.presets``. Each
case is written as ``<case>.npz``: input sha256 digests (the tests regenerate
the inputs and check the digests), the reference outputs, and the Triton
interpreter outputs. Tensors above 65536 elements are stored as 8192 seeded
samples plus their sum and sum of squares, to keep the fixtures small.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
import time
import zlib
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"  # before triton is imported

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
if not os.environ.get("MSDA_REFERENCE"):
    raise SystemExit("set MSDA_REFERENCE to the roulbac/msda-triton checkout the vectors are made from")
REF = Path(os.environ["MSDA_REFERENCE"])
FULL_LIMIT = 65536
N_SAMPLES = 8192

sys.path.insert(0, str(REPO / "tests"))
sys.path.insert(0, str(REPO / "msda-triton_b200"))
import cases as my_cases  # noqa: E402
from msda_triton_b200 import presets  # noqa: E402


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ref_modules():
    sys.path.insert(0, str(REF / "tests"))  # test_msda does `from reference_impls import ...`
    impls = _load("ref_reference_impls", REF / "tests" / "reference_impls.py")
    suite = _load("ref_test_msda", REF / "tests" / "test_msda.py")
    kernels = _load("ref_msda_kernels", REF / "src" / "msda_triton" / "kernels.py")
    return impls, suite, kernels


def _next_pow2(x: int) -> int:
    return 1 << (x - 1).bit_length()


def triton_forward(kernels, value, shapes, starts, loc, attn):
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = loc.shape
    out = value.new_empty(B, Q, M, D)
    block_q = 16
    grid = ((Q + block_q - 1) // block_q, B * M)
    kernels._msda_forward_kernel.fn[grid](
        value, shapes, starts, loc, attn, out, Q, S, M=M, D=D, L=L, K=K,
        BLOCK_Q=block_q, BLOCK_D=_next_pow2(D))
    return out.view(B, Q, M * D)


def triton_backward(kernels, value, shapes, starts, loc, attn, grad_out):
    B, S, M, D = value.shape
    _, Q, _, L, K, _ = loc.shape
    grad_out = grad_out.reshape(B, Q, M, D).contiguous()
    gv = torch.zeros_like(value)
    gl = torch.empty_like(loc)
    ga = torch.empty_like(attn)
    grid = ((Q + kernels.BWD_BLOCK_Q - 1) // kernels.BWD_BLOCK_Q, B * M)
    kernels._msda_backward_kernel[grid](
        value, shapes, starts, loc, attn, grad_out, gv, gl, ga, Q, S, M=M, D=D, L=L, K=K,
        BLOCK_Q=kernels.BWD_BLOCK_Q, BLOCK_D=_next_pow2(D), num_warps=kernels.BWD_NUM_WARPS)
    return gv, gl, ga


def reference_fwd_bwd(impls, value, shapes, loc, attn, grad_out):
    v = value.detach().clone().requires_grad_(True)
    l = loc.detach().clone().requires_grad_(True)
    a = attn.detach().clone().requires_grad_(True)
    out = impls.msda_reference(v, shapes, l, a)
    out.backward(grad_out)
    return out.detach(), v.grad, l.grad, a.grad


def _store(arrays: dict, case: str, name: str, t: torch.Tensor):
    # The sample indices depend only on (case, tensor role), so a reference
    # output and its Triton twin ("triton_<name>") are sampled at the same places.
    role = name.removeprefix("triton_")
    rng = np.random.default_rng(zlib.crc32(f"{case}/{role}".encode()))
    t = t.detach().cpu()
    x = (t if t.dtype in (torch.float32, torch.float64) else t.double()).numpy()
    if x.size <= FULL_LIMIT:
        arrays[name] = x
        return
    flat = x.reshape(-1)
    idx = np.sort(rng.choice(flat.size, size=N_SAMPLES, replace=False)).astype(np.int64)
    arrays[name + "__idx"] = idx
    arrays[name + "__val"] = flat[idx]
    f64 = flat.astype(np.float64)
    arrays[name + "__sum"] = np.float64(f64.sum())
    arrays[name + "__sumsq"] = np.float64((f64 * f64).sum())
    arrays[name + "__shape"] = np.asarray(x.shape, dtype=np.int64)


def write_case(name: str, meta: dict, inputs: dict, outputs: dict):
    arrays = {"meta": np.asarray(json.dumps(meta))}
    for k, t in inputs.items():
        arrays[f"digest_{k}"] = np.asarray(my_cases.digest(t))
    for k, t in outputs.items():
        _store(arrays, name, k, t)
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"  wrote {name}.npz ({(HERE / f'{name}.npz').stat().st_size / 1024:.0f} KiB)")


def main() -> int:
    if not REF.exists():
        print(f"reference checkout not found at {REF}", file=sys.stderr)
        return 1
    impls, suite, kernels = _ref_modules()
    t0 = time.time()

    # 1. reference-vs-naive known-answer cases (tests/test_msda.py:101-120), float64.
    kw = dict(B=2, Q=5, M=2, D=4, shapes=[(5, 7), (3, 4)], K=3)
    value, shapes, starts, loc, attn = suite.make_inputs(
        **kw, dtype=torch.float64, device="cpu", loc_lo=-0.3, loc_hi=1.3)
    g = my_cases.grad_output_like(impls.msda_reference(value, shapes, loc, attn))
    out, gv, gl, ga = reference_fwd_bwd(impls, value, shapes, loc, attn, g)
    naive = impls.msda_naive(value, shapes, loc, attn)
    write_case("naive_random", dict(kind="ref_naive", kwargs=kw, dtype="float64", loc_lo=-0.3,
                                    loc_hi=1.3, seed=0, grad_seed=7),
               dict(value=value, loc=loc, attn=attn, grad_out=g),
               dict(out=out, naive=naive, grad_value=gv, grad_loc=gl, grad_attn=ga))

    kw = dict(B=1, Q=4, M=1, D=3, shapes=[(4, 6)], K=2)
    value, shapes, starts, loc, attn = suite.make_inputs(**kw, dtype=torch.float64, device="cpu")
    grid_vals = torch.tensor([0.0, 0.5, 1.0], dtype=torch.float64)
    loc = grid_vals[torch.randint(0, 3, loc.shape, generator=torch.Generator().manual_seed(1))]
    g = my_cases.grad_output_like(impls.msda_reference(value, shapes, loc, attn))
    out, gv, gl, ga = reference_fwd_bwd(impls, value, shapes, loc, attn, g)
    naive = impls.msda_naive(value, shapes, loc, attn)
    write_case("naive_exact_corners", dict(kind="ref_naive_corners", kwargs=kw, dtype="float64",
                                           seed=0, grad_seed=7),
               dict(value=value, loc=loc, attn=attn, grad_out=g),
               dict(out=out, naive=naive, grad_value=gv, grad_loc=gl, grad_attn=ga))

    # 2. the suite's GPU cases (tests/test_msda.py:57-62) and its out-of-bounds case
    #    (:142-150, :208-227), fp32: grid_sample reference + Triton kernels.
    case_list = [(c["id"], my_cases.case_kwargs(c), 0.0, 1.0) for c in suite.CASES]
    case_list.append(("oob", dict(B=2, Q=64, M=4, D=32, shapes=[(14, 20), (7, 10)], K=4), -0.5, 1.5))
    for cid, kw, lo, hi in case_list:
        value, shapes, starts, loc, attn = suite.make_inputs(
            **kw, dtype=torch.float32, device="cpu", loc_lo=lo, loc_hi=hi)
        g = my_cases.grad_output_like(impls.msda_reference(value, shapes, loc, attn))
        out, gv, gl, ga = reference_fwd_bwd(impls, value, shapes, loc, attn, g)
        t_out = triton_forward(kernels, value, shapes, starts, loc, attn)
        t_gv, t_gl, t_ga = triton_backward(kernels, value, shapes, starts, loc, attn, g)
        write_case(f"case_{cid}", dict(kind="suite_case", kwargs=kw, dtype="float32", loc_lo=lo,
                                       loc_hi=hi, seed=0, grad_seed=7),
                   dict(value=value, loc=loc, attn=attn, grad_out=g),
                   dict(out=out, grad_value=gv, grad_loc=gl, grad_attn=ga,
                        triton_out=t_out, triton_grad_value=t_gv, triton_grad_loc=t_gl,
                        triton_grad_attn=t_ga))
        print(f"  {cid}: {time.time() - t0:.1f}s")

    # 3. lab edge cases (labs/common/checks.py:71-75), float64 reference only.
    for i, c in enumerate(my_cases.LAB_CASES):
        kw = {k: v for k, v in c.items() if k not in ("loc_lo", "loc_hi")}
        lo, hi = c.get("loc_lo", 0.0), c.get("loc_hi", 1.0)
        value, shapes, starts, loc, attn = suite.make_inputs(
            **kw, dtype=torch.float64, device="cpu", loc_lo=lo, loc_hi=hi)
        g = my_cases.grad_output_like(impls.msda_reference(value, shapes, loc, attn))
        out, gv, gl, ga = reference_fwd_bwd(impls, value, shapes, loc, attn, g)
        write_case(f"lab_{i}", dict(kind="lab_case", kwargs=kw, dtype="float64", loc_lo=lo,
                                    loc_hi=hi, seed=0, grad_seed=7),
                   dict(value=value, loc=loc, attn=attn, grad_out=g),
                   dict(out=out, grad_value=gv, grad_loc=gl, grad_attn=ga))

    # 4. the ``small`` operating point (fp32), inputs from msda_triton_b200.presets.
    p = presets.get("small")
    x = presets.make_inputs(p, seed=0)
    value, shapes, starts = x["value"], x["spatial_shapes"], x["level_start_index"]
    loc, attn, g = x["sampling_locations"], x["attention_weights"], x["grad_output"]
    out, gv, gl, ga = reference_fwd_bwd(impls, value, shapes, loc, attn, g)
    t_out = triton_forward(kernels, value, shapes, starts, loc, attn)
    t_gv, t_gl, t_ga = triton_backward(kernels, value, shapes, starts, loc, attn, g)
    write_case("preset_small", dict(kind="preset", preset="small", dtype="float32", seed=0),
               dict(value=value, loc=loc, attn=attn, grad_out=g),
               dict(out=out, grad_value=gv, grad_loc=gl, grad_attn=ga, triton_out=t_out,
                    triton_grad_value=t_gv, triton_grad_loc=t_gl, triton_grad_attn=t_ga))
    print(f"done in {time.time() - t0:.1f}s")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

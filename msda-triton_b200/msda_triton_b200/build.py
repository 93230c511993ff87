"""Build ``libmsda_b200.so`` (the sm_100a kernels behind the C ABI of
``include/msda_b200.h``) in-tree with nvcc.

Each ``csrc/*.cu`` translation unit is compiled in parallel to an object file
under ``_build/``, then linked into ``msda_triton_b200/libmsda_b200.so`` with
the CUDA runtime linked statically and only the ``msda_*`` symbols exported.

Run as ``python -m msda_triton_b200.build`` (from ``msda-triton_b200/``) or
call :func:`build`.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
PROJECT_DIR = PKG_DIR.parent
REPO_DIR = PROJECT_DIR.parent
CSRC = PROJECT_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PROJECT_DIR / "_build"
LIB_NAME = "libmsda_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXX_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden"]


def _nvcc() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile and link the library if any source is newer than it; return its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    deps = _deps()
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]

    def compile_one(src: Path, obj: Path) -> str:
        if not force and not _stale(obj, [src, *deps]):
            return ""
        cmd = [nvcc, *ARCH_FLAGS, *CXX_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        return res.stderr

    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as ex:
        logs = list(ex.map(compile_one, srcs, objs))
    if ptxas_verbose or verbose:
        for log in logs:
            if log:
                print(log, file=sys.stderr)

    if force or _stale(LIB_PATH, objs):
        vscript = BUILD_DIR / "exports.map"
        vscript.write_text("{ global: msda_*; local: *; };\n")
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
               "-Xlinker", f"--version-script={vscript}"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true", help="rebuild everything")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills per kernel")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

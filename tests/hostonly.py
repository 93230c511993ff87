"""Run a test that hands the library fabricated device addresses without a
visible GPU.

Several C-ABI tests pass made-up pointers to check that a call is refused on
the host before any launch. On a machine without a GPU a regression that let
such a call through would fail with a CUDA error; on a machine with one it
could make a kernel dereference the fabricated addresses. ``host_only`` runs
the test body in a child pytest process with ``CUDA_VISIBLE_DEVICES=""``
whenever this process can see a GPU, so the refusal is always tested where
no device can be touched.
"""

from __future__ import annotations

import functools
import inspect
import os
import subprocess
import sys


def _gpu_visible() -> bool:
    if os.environ.get("CUDA_VISIBLE_DEVICES") == "":
        return False
    import torch

    return torch.cuda.is_available()


def host_only(fn):
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        if not _gpu_visible():
            return fn(*args, **kwargs)
        path = inspect.getfile(fn)
        env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
        res = subprocess.run(
            [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-m", "not gpu",
             f"{path}::{fn.__name__}"],
            env=env, capture_output=True, text=True, cwd=os.path.dirname(os.path.dirname(path)),
            timeout=600)
        assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-2000:]
        return None

    return wrapper

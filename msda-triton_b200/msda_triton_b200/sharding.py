"""Batch sharding of the operator across ranks (one process per GPU).

value[b] is read, and grad_value[b] written, only by the queries of batch b
(src/msda_triton/kernels.py:96 and :199), so ranks own disjoint batch slices
and the operator needs no collective: a rank calls the op on its own slice.
This module holds the host-side pieces of that path:

* ``rank_batch``: the slice of the global batch a rank owns. Presets with
  ``scaling == "weak"`` give every rank ``preset.B`` items of its own (the
  global batch grows with the world); ``"strong"`` presets split
  ``preset.B`` evenly (the scaling sweep: global B = 64 at encoder shapes over
  1..8 GPUs).
* ``init_ranks``: process-group setup from the torchrun environment.
* ``max_over_ranks`` / ``barrier``: the only collectives, used for timing.

Everything here runs with the ``gloo`` backend on CPU as well as ``nccl``.
"""

from __future__ import annotations

import datetime
import os

import torch

from .presets import Preset


def rank_batch(preset: Preset, world: int, rank: int) -> tuple[int, int]:
    """(first global batch index, number of items) owned by ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if preset.scaling == "strong":
        if preset.B % world:
            raise ValueError(f"global batch {preset.B} does not split evenly over {world} ranks")
        n = preset.B // world
        return rank * n, n
    return rank * preset.B, preset.B


def global_batch(preset: Preset, world: int) -> int:
    return preset.B if preset.scaling == "strong" else preset.B * world


def init_ranks(backend: str = "nccl", timeout_s: float = 120.0) -> tuple[int, int, int]:
    """(rank, world, local rank) from the torchrun environment; initialises the
    default process group when the world has more than one rank (for
    ``nccl`` the local rank's GPU becomes current first)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        kwargs = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return rank, world, local


def _device():
    import torch.distributed as dist

    return torch.device("cuda") if dist.get_backend() == "nccl" else torch.device("cpu")


def max_over_ranks(x: float, world: int) -> float:
    """Maximum of ``x`` over all ranks (identity for a world of one)."""
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    """All ranks meet here; with a GPU, also wait for this rank's device work."""
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()

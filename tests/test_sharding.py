"""Multi-rank host path on CPU: world_size-2 ``gloo`` process groups.

The op shards over the batch with no collective (a rank runs the op on its
own batch slice); these tests check the host-side pieces of that path with
real ranks: the slices the ranks own, the per-item seeded inputs a rank
builds for its slice, that the per-rank results of the (batch-independent)
computation reassemble into the full-batch result, and the max-over-ranks
timing reduction. The computation stand-in is the CPU oracle (test
infrastructure); the CUDA op itself runs on the GPU tests.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(REPO), str(REPO / "msda-triton_b200")]

from msda_triton_b200 import presets, sharding  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, preset_name, overrides, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path[:0] = [str(REPO), str(REPO / "msda-triton_b200")]
    from oracle import msda_oracle as orc

    r, w, _ = sharding.init_ranks("gloo", timeout_s=60)
    try:
        assert (r, w) == (rank, world)
        preset = presets.get(preset_name, **overrides)
        b0, nb = sharding.rank_batch(preset, w, r)
        x = presets.make_inputs(preset, batch=nb, batch_offset=b0)
        out = orc.msda_grid_sample(x["value"], x["spatial_shapes"], x["sampling_locations"],
                                   x["attention_weights"])
        # Gather every rank's slice bounds and output on every rank.
        bounds = [None] * w
        dist.all_gather_object(bounds, (b0, nb))
        outs = [torch.empty_like(out) for _ in range(w)]
        dist.all_gather(outs, out)
        worst = sharding.max_over_ranks(float(r + 1) * 0.25, w)
        sharding.barrier(w)
        if r == 0:
            torch.save({"bounds": bounds, "outs": outs, "worst": worst}, Path(out_dir) / "result.pt")
    finally:
        dist.destroy_process_group()


def _run(world, preset_name, overrides, tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, preset_name, overrides, str(tmp_path)),
                       nprocs=world,
                       join=True, start_method="spawn")
    return torch.load(tmp_path / "result.pt")


def test_rank_batch_weak_and_strong():
    dec = presets.get("decoder")
    assert [sharding.rank_batch(dec, 4, r) for r in range(4)] == [(0, 4), (4, 4), (8, 4), (12, 4)]
    assert sharding.global_batch(dec, 4) == 16
    sc = presets.get("scale")
    for n in (1, 2, 4, 8):
        sl = [sharding.rank_batch(sc, n, r) for r in range(n)]
        assert sum(k for _, k in sl) == 64
        assert [b for b, _ in sl] == [i * (64 // n) for i in range(n)]
        assert sharding.global_batch(sc, n) == 64
    with pytest.raises(ValueError):
        sharding.rank_batch(sc, 3, 0)
    with pytest.raises(ValueError):
        sharding.rank_batch(sc, 2, 2)


def test_slice_inputs_equal_full_batch_slice():
    p = presets.get("small", B=4)
    full = presets.make_inputs(p)
    part = presets.make_inputs(p, batch=2, batch_offset=1)
    for k in ("value", "sampling_locations", "attention_weights", "grad_output"):
        assert torch.equal(part[k], full[k][1:3]), k


def test_two_gloo_ranks_strong_split(tmp_path):
    """Global batch 4 split over 2 ranks: slices are disjoint and cover the
    batch, and the per-rank outputs reassemble into the full-batch output."""
    strong = {"B": 4, "scaling": "strong"}
    res = _run(2, "small", strong, tmp_path)
    assert res["bounds"] == [(0, 2), (2, 2)]
    assert res["worst"] == 0.5
    p = presets.get("small", **strong)
    sys.path.insert(0, str(REPO))
    from oracle import msda_oracle as orc

    x = presets.make_inputs(p)
    full = orc.msda_grid_sample(x["value"], x["spatial_shapes"], x["sampling_locations"],
                                x["attention_weights"])
    torch.testing.assert_close(torch.cat(res["outs"]), full, rtol=0, atol=0)


def test_two_gloo_ranks_weak(tmp_path):
    """Weak scaling: each rank owns preset.B items of its own."""
    res = _run(2, "small", {}, tmp_path)
    assert res["bounds"] == [(0, 1), (1, 1)]
    p = presets.get("small", B=2)
    sys.path.insert(0, str(REPO))
    from oracle import msda_oracle as orc

    x = presets.make_inputs(p)
    full = orc.msda_grid_sample(x["value"], x["spatial_shapes"], x["sampling_locations"],
                                x["attention_weights"])
    torch.testing.assert_close(torch.cat(res["outs"]), full, rtol=0, atol=0)

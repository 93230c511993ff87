"""Deformable-DETR / Mask2Former operating points and seeded synthetic inputs.

The pyramid shapes follow the reference benchmark's presets
(benchmarks/modal_benchmark.py:73-98: strides 8..64 with ceil division on an
800x1333 image, 8 heads x 32 channels, 4 levels x 4 points). Inputs are
generated on the CPU, batch item by batch item, each item from its own
``torch.Generator`` seeded by (seed, global item index) in a fixed draw order,
so every process (test, bench rank, CPU baseline) builds identical tensors and
a rank can build just its own slice of a global batch:

* value ~ N(0, 1);
* attention_weights = softmax over the L*K axis of N(0, 1) logits;
* grad_output ~ N(0, 1);
* sampling_locations: U[lo, hi) for ``small``/``decoder``/``m2f``; for
  ``encoder``/``scale``, the normalised centre of the query's own pixel
  ((x + 0.5) / W, (y + 0.5) / H) on its own level, broadcast over (m, l, k),
  plus N(0, 0.02) offsets, clamped to [-0.05, 1.05].
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace

import torch


def pyramid(height: int, width: int, levels: int = 4, stride0: int = 8) -> list[tuple[int, int]]:
    """Feature-pyramid shapes at strides stride0 * 2**i (ceil division)."""
    out = []
    for i in range(levels):
        s = stride0 << i
        out.append(((height + s - 1) // s, (width + s - 1) // s))
    return out


@dataclass(frozen=True)
class Preset:
    name: str
    B: int
    M: int
    D: int
    K: int
    shapes: tuple[tuple[int, int], ...]
    Q: int | None  # None: one query per value row (Q = S)
    dtype: torch.dtype
    loc_mode: str = "uniform"  # "uniform" or "pixel_centre"
    loc_lo: float = 0.0
    loc_hi: float = 1.0
    scaling: str = "weak"  # "weak": B per rank; "strong": B is the global batch, split over ranks
    note: str = field(default="", compare=False)

    @property
    def L(self) -> int:
        return len(self.shapes)

    @property
    def S(self) -> int:
        return sum(h * w for h, w in self.shapes)

    @property
    def num_queries(self) -> int:
        return self.S if self.Q is None else self.Q


_DETR = tuple(pyramid(800, 1333))

PRESETS: dict[str, Preset] = {
    "small": Preset("small", B=1, M=8, D=32, K=4, shapes=((32, 32), (16, 16), (8, 8), (4, 4)),
                    Q=100, dtype=torch.float32, note="CPU-runnable small case"),
    "decoder": Preset("decoder", B=4, M=8, D=32, K=4, shapes=_DETR, Q=300, dtype=torch.bfloat16,
                      note="Deformable-DETR decoder, 800x1333"),
    "encoder": Preset("encoder", B=4, M=8, D=32, K=4, shapes=_DETR, Q=None, dtype=torch.bfloat16,
                      loc_mode="pixel_centre", note="Deformable-DETR encoder, Q = S"),
    "m2f": Preset("m2f", B=2, M=8, D=32, K=4, shapes=((128, 128), (64, 64), (32, 32)), Q=None,
                  dtype=torch.float16, loc_lo=-0.1, loc_hi=1.1,
                  note="Mask2Former pixel decoder; out-of-bounds corners"),
    "scale": Preset("scale", B=64, M=8, D=32, K=4, shapes=_DETR, Q=None, dtype=torch.bfloat16,
                    loc_mode="pixel_centre", scaling="strong",
                    note="global batch 64 split over the ranks, encoder shapes"),
    "scale_d64": Preset("scale_d64", B=64, M=4, D=64, K=4, shapes=_DETR, Q=None,
                        dtype=torch.bfloat16, loc_mode="pixel_centre", scaling="strong",
                        note="global batch 64 split over the ranks, 256 channels as 4 heads x 64"),
}


def get(name: str, **overrides) -> Preset:
    p = PRESETS[name]
    return replace(p, **overrides) if overrides else p


def _pixel_centres(shapes) -> torch.Tensor:
    """(S, 2) normalised centre of every value row, level by level."""
    parts = []
    for h, w in shapes:
        ys, xs = torch.meshgrid(torch.arange(h, dtype=torch.float32),
                                torch.arange(w, dtype=torch.float32), indexing="ij")
        parts.append(torch.stack([(xs + 0.5) / w, (ys + 0.5) / h], -1).reshape(-1, 2))
    return torch.cat(parts)


def _item_generator(seed: int, item: int) -> torch.Generator:
    return torch.Generator().manual_seed((seed * 1_000_003 + item) & 0x7FFF_FFFF_FFFF_FFFF)


def make_inputs(preset: Preset, *, dtype: torch.dtype | None = None, device="cpu", seed: int = 0,
                batch: int | None = None, batch_offset: int = 0,
                with_grad: bool = True) -> dict[str, torch.Tensor]:
    """Seeded synthetic inputs for ``preset``: global batch items
    ``batch_offset .. batch_offset + batch - 1`` (``batch`` defaults to B)."""
    dtype = dtype or preset.dtype
    B = preset.B if batch is None else batch
    M, D, K, L, S, Q = preset.M, preset.D, preset.K, preset.L, preset.S, preset.num_queries
    centre = None
    if preset.loc_mode == "pixel_centre":
        if Q != S:
            raise ValueError("pixel_centre locations need one query per value row")
        centre = _pixel_centres(preset.shapes).view(Q, 1, 1, 1, 2)
    value = torch.empty(B, S, M, D)
    loc = torch.empty(B, Q, M, L, K, 2)
    logits = torch.empty(B, Q, M, L * K)
    grad = torch.empty(B, Q, M * D) if with_grad else None
    for b in range(B):
        gen = _item_generator(seed, batch_offset + b)
        value[b] = torch.randn(S, M, D, generator=gen)
        if centre is not None:
            loc[b] = (centre + 0.02 * torch.randn(Q, M, L, K, 2, generator=gen)).clamp_(-0.05, 1.05)
        else:
            loc[b] = preset.loc_lo + (preset.loc_hi - preset.loc_lo) * torch.rand(
                Q, M, L, K, 2, generator=gen)
        logits[b] = torch.randn(Q, M, L * K, generator=gen)
        if with_grad:
            grad[b] = torch.randn(Q, M * D, generator=gen)
    attn = logits.softmax(-1).view(B, Q, M, L, K)
    out = {
        "value": value.to(device=device, dtype=dtype),
        "spatial_shapes": torch.tensor(preset.shapes, dtype=torch.int64, device=device),
        "sampling_locations": loc.to(device=device, dtype=dtype),
        "attention_weights": attn.to(device=device, dtype=dtype),
    }
    hw = out["spatial_shapes"].prod(-1)
    out["level_start_index"] = torch.cat([hw.new_zeros(1), hw.cumsum(0)[:-1]])
    if with_grad:
        out["grad_output"] = grad.to(device=device, dtype=dtype)
    return out

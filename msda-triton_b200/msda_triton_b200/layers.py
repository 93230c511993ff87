"""The Deformable-DETR cross-attention layer around the operator.

``MSDACrossAttention`` is the caller the operator exists for
(labs/solutions/lab00.py:169-208 of the reference): it projects the value
pyramid, predicts per (head, level, point) sampling offsets and attention
logits from the query, turns them into normalised sampling locations and
softmax weights, runs multi-scale deformable attention and projects the
result. The four projections are ``torch.nn.Linear`` (cuBLAS GEMMs); the
attention itself is this package's operator, so the layer trains through the
B200 kernels. Parameter names and shapes match the reference layer, so its
``state_dict`` loads unchanged.

With ``fused=True`` the prologue -- reference point plus offsets over
(W_l, H_l), softmax of the logits -- runs inside the kernels
(``multi_scale_deformable_attention_fused``) instead of as separate tensor
operations that write and re-read the sampling locations and weights. The
default ``fused="auto"`` fuses when sampling is sparse (Q*L*K <= 2*S, a
DETR decoder: 332 vs 344 us per bf16 forward+backward of the layer on B200)
and keeps the tensor-op prologue when it is dense (an encoder with a query
per pixel: the issue-bound kernels pay more for the in-kernel prologue than
the bandwidth-bound tensor operations cost, 2.52 vs 2.30 ms).

Shapes: ``query`` (B, Q, C); ``reference_points`` (B, Q, 2), normalised
(x, y) in [0, 1]; ``value`` (B, S, C), the pyramid flattened level by level;
``spatial_shapes`` (L, 2) as (H_l, W_l). Returns (B, Q, C).
"""

from __future__ import annotations

import torch
from torch import nn

from .ops import multi_scale_deformable_attention, multi_scale_deformable_attention_fused


class MSDACrossAttention(nn.Module):
    def __init__(self, embed_dim: int, num_heads: int, num_levels: int, num_points: int,
                 fused: bool | str = "auto"):
        super().__init__()
        self.fused = fused
        if embed_dim % num_heads:
            raise ValueError(f"embed_dim={embed_dim} is not a multiple of num_heads={num_heads}")
        self.num_heads = num_heads
        self.num_levels = num_levels
        self.num_points = num_points
        self.head_dim = embed_dim // num_heads
        n_pts = num_heads * num_levels * num_points
        self.value_proj = nn.Linear(embed_dim, embed_dim)
        self.offset_proj = nn.Linear(embed_dim, 2 * n_pts)  # (x, y) offset per point, level pixels
        self.weight_proj = nn.Linear(embed_dim, n_pts)      # attention logit per point
        self.out_proj = nn.Linear(embed_dim, embed_dim)

    def sampling(self, query: torch.Tensor, reference_points: torch.Tensor,
                 spatial_shapes: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Sampling locations (B, Q, M, L, K, 2) and attention weights
        (B, Q, M, L, K) for ``query``: offsets in each level's pixels are
        divided by that level's (W_l, H_l) and added to the reference point;
        the logits of a (query, head) are softmaxed over all L*K points."""
        B, Q, _ = query.shape
        M, L, K = self.num_heads, self.num_levels, self.num_points
        offsets = self.offset_proj(query).view(B, Q, M, L, K, 2)
        logits = self.weight_proj(query).view(B, Q, M, L * K)
        weights = logits.softmax(dim=-1).view(B, Q, M, L, K)
        wh = spatial_shapes.flip(-1).to(device=query.device, dtype=query.dtype)  # (L, 2): (W_l, H_l)
        locations = reference_points[:, :, None, None, None, :] + offsets / wh[:, None, :]
        return locations, weights

    def forward(self, query: torch.Tensor, reference_points: torch.Tensor, value: torch.Tensor,
                spatial_shapes: torch.Tensor,
                level_start_index: torch.Tensor | None = None) -> torch.Tensor:
        B, Q, C = query.shape
        S = value.shape[1]
        v = self.value_proj(value).view(B, S, self.num_heads, self.head_dim)
        fused = self.fused
        if fused == "auto":
            fused = Q * self.num_levels * self.num_points <= 2 * S
        if fused:
            M, L, K = self.num_heads, self.num_levels, self.num_points
            offsets = self.offset_proj(query).view(B, Q, M, L, K, 2)
            logits = self.weight_proj(query).view(B, Q, M, L, K)
            out = multi_scale_deformable_attention_fused(v, spatial_shapes, level_start_index,
                                                         reference_points, offsets, logits)
        else:
            locations, weights = self.sampling(query, reference_points, spatial_shapes)
            out = multi_scale_deformable_attention(v, spatial_shapes, level_start_index,
                                                   locations.contiguous(), weights.contiguous())
        return self.out_proj(out)

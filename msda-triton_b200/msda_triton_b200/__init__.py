"""B200-native (sm_100a) multi-scale deformable attention.

Drop-in for the public surface of roulbac/msda-triton
(src/msda_triton/__init__.py:9-12): ``multi_scale_deformable_attention``,
plus the mmcv-style ``MultiScaleDeformableAttnFunction`` and the
Deformable-DETR cross-attention layer ``MSDACrossAttention`` that calls it
(layers.py), whose prologue (reference point + offsets, softmax of the
attention logits) the kernels can take fused
(``multi_scale_deformable_attention_fused``). The sibling gathers
``grid_sample`` and ``roi_align`` (gather.py) run on the same kernel
skeleton. The kernels live in ``libmsda_b200.so`` behind the C ABI of
include/msda_b200.h.
"""

from .gather import grid_sample, roi_align
from .layers import MSDACrossAttention
from .ops import (MultiScaleDeformableAttnFunction, multi_scale_deformable_attention,
                  multi_scale_deformable_attention_fused)

__all__ = ["multi_scale_deformable_attention", "MultiScaleDeformableAttnFunction",
           "MSDACrossAttention", "multi_scale_deformable_attention_fused", "grid_sample", "roi_align"]
__version__ = "0.1.0"

"""B200-native (sm_100a) multi-scale deformable attention.

Drop-in for the public surface of roulbac/msda-triton
(src/msda_triton/__init__.py:9-12): ``multi_scale_deformable_attention``,
plus the mmcv-style ``MultiScaleDeformableAttnFunction``. The kernels live in
``libmsda_b200.so`` behind the C ABI of include/msda_b200.h.
"""

from .ops import MultiScaleDeformableAttnFunction, multi_scale_deformable_attention

__all__ = ["multi_scale_deformable_attention", "MultiScaleDeformableAttnFunction"]
__version__ = "0.1.0"

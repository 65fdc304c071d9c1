"""ress_b200 -- ReSS/HeSS block-sparse global attention on NVIDIA B200 (sm_100a).

A drop-in for libary753/ReSS's sparse attention path: the same public API

    import ress_b200 as ress
    ress.apply_ress(model, sparse_ratio=0.5)

with the scoring, budget, restore-swap selection and block-sparse attention
running as hand-written sm_100a kernels behind the C ABI in
include/ress_sm100.h (library ress_b200/libress_sm100.so).
"""

from .api import apply_dense, apply_hess, apply_ress, apply_sparse_vggt, load_backbone  # noqa: F401
from .backbones import BACKBONES, get_backbone  # noqa: F401

__all__ = ["BACKBONES", "apply_dense", "apply_hess", "apply_ress", "apply_sparse_vggt", "get_backbone",
           "load_backbone"]

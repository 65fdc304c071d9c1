"""Public entry points: load a backbone, then install one attention mode.

Same functions, arguments and behaviour as the reference's ``api.py``
(``load_backbone`` :47, ``apply_dense`` :95, ``apply_sparse_vggt`` :103,
``apply_hess`` :117, ``apply_ress`` :130): every ``apply_*`` fully resets the
previous mode; ``apply_dense`` is the uniform budget at sparse_ratio 0 (every
candidate kept, the sparse kernel still runs); ``apply_ress`` uses the
restore-swap criterion ``restore_swap_iter{n}_bf16_trackbest``.
"""

from __future__ import annotations

from .backbones import get_backbone, infer_backbone
from .budget import HessBudget, UniformBudget
from .projected import bake_and_attach_M
from .static import set_static_budget

RESS_CRITERION = "restore_swap_iter{n_iters}_bf16_trackbest"


def load_backbone(name, device="cuda", **kwargs):
    backbone = get_backbone(name)
    model = backbone.load(device=device, **kwargs)
    model._ress_backbone = backbone.name
    return model


def _budgets(model, backbone, lam=None):
    key = ("_ress_budgets", lam)
    cached = getattr(model, "_ress_budget_cache", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    if not getattr(model, "_ress_M_baked", False):
        bake_and_attach_M(model)
        model._ress_M_baked = True
    uniform = UniformBudget(n_blocks=backbone.n_global_blocks, n_heads=backbone.n_heads)
    score_pcd, score_cam_pos = backbone.calibration_paths()
    hess = HessBudget(score_cam_pos, score_pcd, lam=backbone.hess_lam if lam is None else lam, qkv_idx=0)
    model._ress_budget_cache = (key, (uniform, hess))
    return uniform, hess


def _resolve(model, backbone):
    return get_backbone(backbone) if backbone is not None else infer_backbone(model)


def apply_dense(model, backbone=None):
    spec = _resolve(model, backbone)
    uniform, _ = _budgets(model, spec)
    set_static_budget(model, uniform, 0.0, None, beta=1.0)
    return model


def apply_sparse_vggt(model, sparse_ratio, cdf_threshold=None, backbone=None):
    spec = _resolve(model, backbone)
    uniform, _ = _budgets(model, spec)
    set_static_budget(model, uniform, sparse_ratio, cdf_threshold, beta=1.0)
    return model


def apply_hess(model, sparse_ratio, cdf_threshold=None, lam=None, backbone=None):
    spec = _resolve(model, backbone)
    _, hess = _budgets(model, spec, lam=lam)
    set_static_budget(model, hess, sparse_ratio, cdf_threshold, beta=1.0)
    return model


def apply_ress(model, sparse_ratio, n_iters=5, lam=None, backbone=None):
    spec = _resolve(model, backbone)
    _, hess = _budgets(model, spec, lam=lam)
    set_static_budget(model, hess, sparse_ratio, None, beta=1.0,
                      block_criterion=RESS_CRITERION.format(n_iters=n_iters))
    return model

"""Backbone registry: the per-backbone constants the method needs.

Same entries and meaning as the reference's ``backbones.py`` (``Backbone``
:24-44, ``BACKBONES`` :130-174): number of sparsifiable global blocks, heads
per block, and the HeSS lambda each backbone was tuned at.  Loading a
pretrained checkpoint needs the backbone's own source tree and network
access; when those are absent ``load`` raises with the reason (Pi3 and DA3
wiring of a model the caller has built: ``ress_b200.pi3`` / ``ress_b200.da3``).  The Fisher
tables are read from ``RESS_CALIBRATION_DIR`` (default: ``calibration/``
beside this file), file names ``fisher_scores_<name>_{pcd,cam_pos}.pt`` as in
the reference.
"""

from __future__ import annotations

import os
from collections.abc import Callable
from dataclasses import dataclass


def calibration_dir() -> str:
    return os.environ.get("RESS_CALIBRATION_DIR",
                          os.path.join(os.path.dirname(os.path.abspath(__file__)), "calibration"))


@dataclass(frozen=True)
class Backbone:
    name: str
    n_global_blocks: int
    n_heads: int
    hess_lam: float
    load: Callable

    def calibration_paths(self):
        """(pcd, cam_pos) table paths, in the reference's order."""
        d = calibration_dir()
        return (os.path.join(d, f"fisher_scores_{self.name}_pcd.pt"),
                os.path.join(d, f"fisher_scores_{self.name}_cam_pos.pt"))


def _unavailable(name, pkg):
    def load(**kw):
        raise RuntimeError(f"loading the pretrained {name} backbone needs the `{pkg}` source tree and its "
                           "checkpoint (network); build the model yourself, wire it with "
                           "ress_b200.wiring.wire_ress_attention and tag it with model._ress_backbone")
    return load


def _load_pi3(**kw):
    from .pi3 import load_pi3
    return load_pi3(**kw)


def _load_da3(**kw):
    from .da3 import load_da3
    return load_da3(**kw)


BACKBONES = {
    "vggt": Backbone("vggt", n_global_blocks=24, n_heads=16, hess_lam=0.5, load=_unavailable("vggt", "vggt")),
    "pi3": Backbone("pi3", n_global_blocks=18, n_heads=16, hess_lam=0.0, load=_load_pi3),
    "da3": Backbone("da3", n_global_blocks=14, n_heads=24, hess_lam=1.0, load=_load_da3),
}


def get_backbone(name):
    try:
        return BACKBONES[name]
    except KeyError:
        raise ValueError(f"no backbone is registered as {name!r}; the registry holds "
                         f"{', '.join(sorted(BACKBONES))}") from None


def infer_backbone(model):
    name = getattr(model, "_ress_backbone", None)
    if name is None:
        raise ValueError("this model has no _ress_backbone tag: name its backbone with the backbone= "
                         "argument, or create it with load_backbone(), which sets the tag")
    return get_backbone(name)

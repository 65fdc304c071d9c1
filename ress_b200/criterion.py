"""The ``block_criterion`` name grammar of the restore-swap family.

Same grammar and field meanings as the reference's ``scoring/criterion.py``
(``RestoreSwapSpec`` :54-77, ``parse_restore_swap`` :96-124), so criterion
strings written for the reference parse identically here:

    base    := ["damage_"] "restore_swap" ["_iter" N]
    suffix  := "_nowo" | "_wo" | "_bf16" | "_trackbest" | "_rf" NN | "_dc" NN
             | "_antiswap" | "_anti"        (any order, stripped from the end)
"""

from __future__ import annotations

import re
from dataclasses import dataclass

import torch

_SUFFIX = re.compile(r"_(nowo|wo|bf16|trackbest|rf\d+|dc\d+|antiswap|anti)$")
_BASE = re.compile(r"^(?P<damage>damage_)?restore_swap(?:_iter(?P<iters>\d+))?$")


@dataclass
class RestoreSwapSpec:
    n_iters: int = 1
    use_wo: bool = True            # M = W_O^T W_O per head; False -> identity
    track_best: bool = False
    big_dtype: torch.dtype | None = None
    restore_frac: float = 0.5
    maximize: bool = False
    invert_cut: bool = False
    decay: float = 0.5


def _split(name: str):
    core, found = name, []
    while True:
        m = _SUFFIX.search(core)
        if m is None:
            return core, found
        found.append(m.group(1))
        core = core[: m.start()]


def is_restore_swap(block_criterion: str) -> bool:
    return _BASE.match(_split(block_criterion)[0]) is not None


def parse_restore_swap(block_criterion: str) -> RestoreSwapSpec:
    core, suffixes = _split(block_criterion)
    m = _BASE.match(core)
    if m is None:
        raise ValueError(f"not a restore-swap block_criterion: {block_criterion!r}")
    spec = RestoreSwapSpec(n_iters=int(m.group("iters")) if m.group("iters") else 1,
                           use_wo=m.group("damage") is None)
    for sfx in suffixes:
        if sfx == "nowo":
            spec.use_wo = False
        elif sfx == "wo":
            spec.use_wo = True
        elif sfx == "trackbest":
            spec.track_best = True
        elif sfx == "antiswap":
            spec.maximize = True
        elif sfx == "anti":
            spec.maximize, spec.invert_cut = True, True
        elif sfx.startswith("rf"):
            spec.restore_frac = int(sfx[2:]) / 100.0
        elif sfx.startswith("dc"):
            spec.decay = int(sfx[2:]) / 100.0
        else:
            spec.big_dtype = torch.bfloat16
    return spec

"""Loading helpers for the golden vectors produced by tests/golden/make_golden.py."""
from __future__ import annotations

import glob
import os

import numpy as np

from oracle.ska_oracle import SkaParams

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def core_cases() -> list[str]:
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "core_*.npz")))


def load(name: str) -> dict:
    with np.load(os.path.join(GOLDEN_DIR, name + ".npz")) as d:
        return {k: d[k] for k in d.files}


def params_of(d: dict) -> SkaParams:
    a = float(d["meta_decay_alpha"])
    return SkaParams(chunk_size=int(d["meta_CS"]), ridge_eps=float(d["meta_ridge"]),
                     power_K=int(d["meta_K"]), decay_alpha=None if a < 0 else a)


def strategy_kwargs(d: dict) -> dict:
    a = float(d["meta_decay_alpha"])
    return dict(chunk_size=int(d["meta_CS"]), ridge_eps=float(d["meta_ridge"]), power_K=int(d["meta_K"]),
                chunk_strategy="standard" if a < 0 else "decay", decay_alpha=0.95 if a < 0 else a)

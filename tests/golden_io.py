"""Loader for the committed golden vectors (``tests/golden/*.npz``)."""

from __future__ import annotations

import json
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_cases(family: str):
    """Return a list of ``(meta, arrays)`` for ``tests/golden/<family>.npz``."""
    with np.load(os.path.join(GOLDEN_DIR, f"{family}.npz")) as z:
        metas = json.loads(str(z["meta"]))
        files = {k: z[k] for k in z.files if k != "meta"}
    cases = []
    for meta in metas:
        prefix = f"c{meta['id']}_"
        arrays = {k[len(prefix):]: v for k, v in files.items() if k.startswith(prefix)}
        cases.append((meta, arrays))
    return cases


def case_id(meta) -> str:
    keys = ("kind", "x_dtype", "w_dtype", "width", "silu", "has_init", "final", "circular",
            "mode", "state_len", "padded")
    return "-".join(f"{meta[k]}" for k in keys if k in meta) + f"-{meta['id']}"

"""Loader for the golden vectors under tests/golden (made by make_golden.py)."""

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict:
    """{case: {key: array}} for multi-case files, {key: array} otherwise."""
    z = np.load(GOLDEN / f"{name}.npz")
    keys = list(z.keys())
    if all("__" in k for k in keys):
        out: dict = {}
        for k in keys:
            case, field = k.split("__", 1)
            out.setdefault(case, {})[field] = z[k]
        return out
    return {k: z[k] for k in keys}

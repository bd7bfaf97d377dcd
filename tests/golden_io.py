"""Reader for the golden-vector fixtures written by ``tests/golden/make_golden.py``."""

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


class Case(dict):
    def __init__(self, name, meta, arrays):
        super().__init__(arrays)
        self.name = name
        self.meta = meta


def load_cases(fname="golden_unit.npz"):
    z = np.load(os.path.join(GOLDEN, fname))
    groups = {}
    for key in z.files:
        case, field = key.split("__", 1)
        groups.setdefault(case, {})[field] = z[key]
    out = {}
    for case, arrays in groups.items():
        meta = json.loads(str(arrays.pop("meta")))
        out[case] = Case(case, meta, arrays)
    return out


def cases_of_kind(kind, fname="golden_unit.npz"):
    return {k: v for k, v in load_cases(fname).items() if v.meta.get("kind") == kind}

"""Loading helpers for the golden vectors in ``tests/golden`` (made by make_golden.py)."""

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    """Returns {case_key: {field: array}} for ``golden/<name>.npz``."""
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    out = {}
    for k in z.files:
        case, field = k.split("/", 1)
        out.setdefault(case, {})[field] = z[k]
    return out


def spec_of(case):
    from oracle import fixtures as F

    d = json.loads(str(case["spec"]))
    d["hash_pattern"] = tuple(d.get("hash_pattern") or ())
    return F.LayerSpec(**d)


LAYER_FILES = ("mini_sigmoid", "mini_sqrtsoftplus_clamp", "mini_softmax", "mini_hash_dups",
               "mini_hash_random", "mini_fp32scale", "cfg1", "cfg2", "cfg2_batch", "cfg4")

"""Loader for the committed golden fixtures in tests/golden/*.npz."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(family):
    """Returns {case_name: (params, {field: array})} for one fixture file."""
    data = np.load(os.path.join(GOLDEN, f"{family}.npz"))
    meta = json.loads(str(data["__meta__"]))
    cases = {}
    for name, params in meta.items():
        prefix = f"{name}__"
        arrays = {k[len(prefix):]: data[k] for k in data.files if k.startswith(prefix)}
        cases[name] = (params, arrays)
    return cases


def case_ids(family):
    return sorted(load(family).keys())

"""Loading helpers for the golden fixtures in tests/golden/."""
import glob
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def case_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    d = {k: z[k] for k in z.files}
    d["dtype"] = str(d["dtype"])
    d["orig_shape"] = tuple(int(v) for v in d["orig_shape"])
    d["padded_shape"] = tuple(int(v) for v in d["padded_shape"])
    d["count"] = int(d["count"])
    d["threshold"] = float(d["threshold"])
    d["value"] = d["value_bits"].view(np.float16)
    xs = []
    i = 0
    while f"X{i}" in d:
        xs.append((d[f"X{i}"], str(d[f"X{i}_dtype"]), d[f"Y{i}"]))
        i += 1
    d["xs"] = xs
    return d


def fullsize():
    with open(os.path.join(GOLDEN, "fullsize.json")) as f:
        return json.load(f)

"""Loads the reference's MatMulNBits / GatherBlockQuantized fixtures from tests/golden/*.npz
(extracted from test/fixtures/ops by tests/golden/make_golden.py)."""

import glob
import os

import numpy as np

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cases(prefix):
    out = []
    for path in sorted(glob.glob(os.path.join(HERE, prefix + "*.npz"))):
        z = np.load(path)
        case = {"name": os.path.basename(path)[:-4]}
        case["attrs"] = {k[5:]: int(z[k]) for k in z.files if k.startswith("attr_")}
        names = [str(x) for x in z["inputs"]]
        case["input_names"] = names

        def get(i):
            if i < len(names) and names[i] and "init_" + names[i] in z.files:
                return z["init_" + names[i]]
            if i < len(names) and names[i] and "in_" + names[i] in z.files:
                return z["in_" + names[i]]
            return None

        case["inputs"] = [get(i) for i in range(len(names))]
        case["Y"] = z["out_Y"]
        out.append(case)
    return out


def matmul_nbits_cases():
    return cases("MatMulNBits_")


def gather_cases():
    return cases("GatherBlockQuantized_")

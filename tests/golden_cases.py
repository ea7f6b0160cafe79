"""Loads the golden fixtures of tests/golden/ (made by make_golden.py)."""
import ast
import glob
import os

import numpy as np

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def case_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "mm_*.npz")))


def load(name):
    d = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    P = O.Params(**ast.literal_eval(str(d.pop("params"))))
    return d, P

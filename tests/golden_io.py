"""Readers for the reference golden vectors copied under tests/golden/."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name, fname, shape=None):
    a = np.fromfile(os.path.join(GOLDEN, name, fname), dtype="<f4")
    return a.reshape(shape) if shape is not None else a

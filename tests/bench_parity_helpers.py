"""Paths for the bench parity tests: bench.py (repository root) and
tests/golden/make_bench_parity.py importable, the fixture loader."""
import os
import sys

import numpy as np

from conftest import GOLDEN, ROOT

sys.path.insert(0, ROOT)
sys.path.insert(0, GOLDEN)


def load():
    return np.load(os.path.join(GOLDEN, "bench_parity.npz"))

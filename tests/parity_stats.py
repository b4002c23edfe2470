"""Measured error of every tolerance check in the GPU parity tests, printed in pytest's summary.

Each entry: (test, what, max-abs, mean-abs, max-abs bar, mean-abs bar). The tests append; the
terminal-summary hook in conftest.py prints the table, so a `pytest -q -m gpu` run shows the
achieved figures next to the bars."""
import os

import numpy as np

RECORDS = []


def record(what: str, got, ref, max_abs: float, mean_abs: float):
    """Appends the error of `got` against `ref` and returns (max-abs, mean-abs)."""
    err = np.abs(np.asarray(got, dtype=np.float64) - np.asarray(ref, dtype=np.float64))
    mx, mn = (float(err.max()), float(err.mean())) if err.size else (0.0, 0.0)
    test = os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0].split("::")[-1]
    RECORDS.append((test, what, mx, mn, max_abs, mean_abs))
    return mx, mn

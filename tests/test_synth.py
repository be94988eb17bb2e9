"""The seeded generator shared by the bench's two arms (mini-llama_b200/synth.py):
the torch form draws the numpy form's numbers bit for bit on the CPU, and a
row range drawn at an offset equals those rows of the whole matrix."""
from __future__ import annotations

import numpy as np
import pytest


def test_torch_form_equals_numpy_form(pkg):
    pytest.importorskip("torch")
    for seed, std, shape in [(1, 1.0, (3, 33)), (1000, 0.02, (17, 1024)), ((1 << 63) + 3, 2.0, (5,))]:
        a = pkg.synth.normal(shape, seed=seed, std=std)
        b = pkg.synth.normal_torch(shape, seed=seed, std=std).numpy()
        np.testing.assert_array_equal(a, b)


def test_row_range_at_offset(pkg):
    pytest.importorskip("torch")
    full = pkg.synth.normal((40, 96), seed=2000, std=0.02)
    part = pkg.synth.normal_torch((13, 96), seed=2000, std=0.02, offset=21 * 96).numpy()
    np.testing.assert_array_equal(full[21:34], part)
    with pytest.raises(ValueError):
        pkg.synth.normal_torch((2, 3), seed=1, offset=3)

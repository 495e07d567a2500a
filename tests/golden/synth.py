"""Seeded synthetic weights and inputs shared by the fixture generator and the tests.

Everything is drawn from ``numpy.random.default_rng(seed)``, which is bit-reproducible
across machines, so large weight sets never need to be stored as fixtures: a fixture
stores the seed and the shapes and the test regenerates the same arrays.
"""
from __future__ import annotations

import numpy as np


def normal(seed: int, shape, std: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(shape) * std).astype(np.float32)


def xavier_normal(seed: int, shape) -> np.ndarray:
    """Xavier/Glorot normal for an ``nn.Linear`` weight of shape [..., fan_out, fan_in]."""
    fan_out, fan_in = shape[-2], shape[-1]
    return normal(seed, shape, float(np.sqrt(2.0 / (fan_in + fan_out))))


def swiglu_weights(seed: int, E: int, d: int, F: int, init: str = "xavier", std: float = 0.02):
    """w1, w3: [E, F, d]; w2: [E, d, F] (nn.Linear layouts), independent streams."""
    if init == "xavier":
        return (xavier_normal(seed * 10 + 1, (E, F, d)), xavier_normal(seed * 10 + 3, (E, F, d)),
                xavier_normal(seed * 10 + 2, (E, d, F)))
    return (normal(seed * 10 + 1, (E, F, d), std), normal(seed * 10 + 3, (E, F, d), std),
            normal(seed * 10 + 2, (E, d, F), std))

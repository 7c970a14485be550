"""Seeded synthetic inputs on the host, bit-identical to the library's device
generator and to the oracle: splitmix64 output i of state `seed`."""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1


def hash64(seed: int, i: int) -> int:
    z = (seed + (i + 1) * 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def uniform_ids(seed: int, vocab: int, n: int) -> np.ndarray:
    """n ids in [0, vocab): hash64(seed, i) % vocab (BASELINE config 1 prompt)."""
    return np.array([hash64(seed, i) % vocab for i in range(n)], np.uint32)


def prompt_for(cfg: dict, n: int = 16) -> np.ndarray:
    """The config-1 prompt of a model: seed = hash64(model seed, 2)."""
    return uniform_ids(hash64(cfg["seed"], 2), cfg["vocab"], n)

"""Shared fixtures. `-m gpu` tests need a B200; everything else runs on CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "gemma4.c_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def g4():
    import g4cuda
    g4cuda.load()
    return g4cuda


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import Reference
    try:
        return Reference()
    except FileNotFoundError as e:
        pytest.skip(str(e))


@pytest.fixture(scope="session")
def image(g4):
    """Seed-0 synthetic E2B image with per-group scales and random norms (the
    variations make indexing mistakes visible)."""
    return g4.synth_image(seed=0, flags=g4.SYN_GROUP_SCALES | g4.SYN_RANDOM_NORMS)


def packed_case(rng, N, K, scale_lo=1e-4, scale_hi=1e-2, per_group=True):
    """Random int8 weights in [-127, 127] with FP16 scales, packed as in the .bin."""
    import g4cuda
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int16).astype(np.int8)
    G = K // 64
    if per_group:
        s = rng.uniform(scale_lo, scale_hi, size=(N, G)).astype(np.float16)
    else:
        s = np.repeat(rng.uniform(scale_lo, scale_hi, size=(N, 1)), G, axis=1).astype(np.float16)
    wp, sp = g4cuda.pack_matrix(w, s.view(np.uint16))
    return w, s, wp, sp


def activations(rng, T, K, outliers=True):
    x = rng.standard_normal((T, K)).astype(np.float32)
    if outliers and T >= 4:
        rows = rng.choice(T, size=max(1, T // 100), replace=False)
        x[rows] *= 50.0
    return x

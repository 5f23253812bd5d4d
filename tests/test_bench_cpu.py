"""Host logic of bench.py that needs no GPU: the config-5 bin packing."""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_pack_sequences_balanced_and_complete():
    b = _bench()
    for world in (1, 2, 4, 8):
        rng = np.random.default_rng(2)
        plen = np.exp(rng.uniform(np.log(128), np.log(8192), 64 * world)).astype(np.int64)
        members = b.pack_sequences(plen, world, 64)
        assert all(len(m) == 64 for m in members)
        flat = sorted(i for m in members for i in m)
        assert flat == list(range(64 * world))          # every sequence exactly once
        loads = [int(plen[m].sum()) for m in members]
        assert max(loads) - min(loads) <= int(plen.max())  # within one prompt of each other
    # one replica keeps the draw order
    rng = np.random.default_rng(2)
    plen = np.exp(rng.uniform(np.log(128), np.log(8192), 64)).astype(np.int64)
    assert b.pack_sequences(plen, 1, 64) == [list(range(64))]

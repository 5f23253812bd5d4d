"""g4_open_file (the .bin streamed to the device through page-locked buffers,
repacked from the device image) builds the same model as g4_open on the
mapped image: identical logits after a prefill and a decode step."""
import os
import shutil
import tempfile
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_open_file_equals_open(g4, image):
    d = tempfile.gettempdir()
    if shutil.disk_usage(d).free < image.nbytes + (1 << 30):
        pytest.skip("not enough temporary disk space for the 5 GB model file")
    path = os.path.join(d, "g4_open_file_test.bin")
    try:
        with open(path, "wb") as f:
            f.write(memoryview(image))
        rng = np.random.default_rng(13)
        toks = rng.integers(0, 262144, size=9).astype(np.int32)
        outs = []
        for kw in ({"image": image}, {"path": path}):
            t0 = time.perf_counter()
            with g4.Model(**kw) as m:
                t1 = time.perf_counter()
                m.forward(toks[:8], 0)
                m.forward(toks[8:], 8)
                outs.append(m.logits(0)[0])
            print(f"open {list(kw)[0]}: {t1 - t0:.2f} s")
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    finally:
        if os.path.exists(path):
            os.remove(path)

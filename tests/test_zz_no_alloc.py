"""g4_topk_noalloc: the top-k entry point that allocates nothing.

Some hosts cannot call cudaMalloc where they sample the next token: a
framework that owns all device memory through its own pool, a decode loop
captured into a CUDA graph (allocation is refused during stream capture), or
a latency-bound loop that must not stall in the allocator. For them the
library keeps the selection's only scratch in a fixed device array and takes
device pointers for input and output. This test drives it through the C ABI
with device buffers the test owns (allocated by torch, which here is only a
device-memory helper), and checks two calls in a row against the existing
entry point g4_topk on the same logits: identical ids and values (the same
selection, exact). It runs last (file name) so that a failure here cannot
hide another test's, and it needs nothing from earlier tests.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_topk_noalloc_matches_g4_topk(g4, image):
    torch = pytest.importorskip("torch")
    L = g4.load()
    rng = np.random.default_rng(21)
    toks = rng.integers(0, g4.VOCAB, size=6).astype(np.int32)
    with g4.Model(image) as m:
        m.forward(toks, 0)
        for row, k in ((5, 64), (2, 17)):            # two calls in a row
            ref_vals, ref_ids = m.topk(row, k)       # existing entry point
            logits, _ = m.logits(row)
            d_logits = torch.from_numpy(logits).to("cuda:0")
            d_vals = torch.empty(k, dtype=torch.float32, device="cuda:0")
            d_ids = torch.empty(k, dtype=torch.int32, device="cuda:0")
            torch.cuda.synchronize()
            rc = L.g4_topk_noalloc(C.c_void_p(d_logits.data_ptr()), g4.VOCAB, k, C.c_void_p(d_vals.data_ptr()),
                                   C.c_void_p(d_ids.data_ptr()), None)
            assert rc == 0
            torch.cuda.synchronize()
            assert np.array_equal(d_ids.cpu().numpy(), ref_ids)
            assert np.array_equal(d_vals.cpu().numpy().view(np.uint32), ref_vals.view(np.uint32))
        # sizes beyond the fixed scratch are refused before any GPU work
        big = C.c_void_p(d_logits.data_ptr())
        assert L.g4_topk_noalloc(big, 262145, 8, C.c_void_p(d_vals.data_ptr()), C.c_void_p(d_ids.data_ptr()),
                                 None) == -1
        assert L.g4_topk_noalloc(big, g4.VOCAB, 65, C.c_void_p(d_vals.data_ptr()), C.c_void_p(d_ids.data_ptr()),
                                 None) == -1


def test_topk_noalloc_ragged_sizes(g4):
    """Sizes that are not whole 4096-value slices (a short last slice padded
    inside the selection, a single slice, k close to n), two calls in a row
    per size, against a stable host sort: value descending, ties to the lower
    index (the reference's candidate order, gemma4.c:544-551)."""
    torch = pytest.importorskip("torch")
    L = g4.load()
    rng = np.random.default_rng(22)
    for n in (64, 4097, 5000):
        x = rng.standard_normal(n).astype(np.float32)
        x[rng.integers(0, n, size=8)] = x[0]          # a few exact ties
        d_x = torch.from_numpy(x).to("cuda:0")
        order = np.lexsort((np.arange(n), -x.astype(np.float64)))
        for k in (1, min(64, n)):
            for _ in range(2):
                d_vals = torch.empty(k, dtype=torch.float32, device="cuda:0")
                d_ids = torch.empty(k, dtype=torch.int32, device="cuda:0")
                torch.cuda.synchronize()
                rc = L.g4_topk_noalloc(C.c_void_p(d_x.data_ptr()), n, k, C.c_void_p(d_vals.data_ptr()),
                                       C.c_void_p(d_ids.data_ptr()), None)
                assert rc == 0
                torch.cuda.synchronize()
                assert np.array_equal(d_ids.cpu().numpy(), order[:k].astype(np.int32)), (n, k)
                assert np.array_equal(d_vals.cpu().numpy(), x[order[:k]]), (n, k)

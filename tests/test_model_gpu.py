"""Whole-model checks of the fast path on the GPU.

The fast path differs from the reference only in the order of floating-point
reductions (RMSNorm sums of squares, softmax max/sum, value sums) and in the
device expf. On the random-weight model those one-ulp differences flip int8
quantisation steps that the layers amplify (see test_strict_gpu.py), so after
35 layers logits are not comparable position by position — the reference
itself diverges the same way when only its summation order changes. What is
checked here instead:
  - after ONE layer the residual stays within the size of a few quantisation
    flips of the reference's (a layout/indexing error would be O(1));
  - the fast decode path (CUDA graph + PDL), the eager path and the T = 3 and
    prefill paths are self-consistent: greedy argmax equals the first maximum
    of the returned logits, logits are finite and within the soft-cap;
  - the graph replay and an eager launch of the same step agree exactly;
  - API errors: out-of-range tokens / rows / positions.
Bit-exact whole-model parity is test_strict_gpu.py.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu(g4, image):
    m = g4.Model(image)
    yield m
    m.close()


def test_one_layer_tracks_reference(g4, oracle, image, gpu):
    o = oracle
    o.lib.or_forward_layers.argtypes = [C.c_void_p, C.c_void_p, np.ctypeslib.ndpointer(np.int32), C.c_size_t,
                                        C.c_int, C.c_int]
    rng = np.random.default_rng(7)
    toks = rng.integers(0, 262144, size=9).astype(np.int32)
    om = o.open_model(image)
    try:
        gpu.set_option(4, 1)        # G4_OPT_LAYERS = 1
        gpu.forward(toks[:8], 0)
        o.lib.or_forward_layers(om.h, om.state, toks[:8], 8, 0, 1)
        a, e = gpu.residual(8), om.residual(8)
        assert np.abs(a - e).max() / np.abs(e).max() < 2e-2
        gpu.forward(toks[8:9], 8)
        o.lib.or_forward_layers(om.h, om.state, toks[8:9], 1, 8, 1)
        a, e = gpu.residual(1), om.residual(1)
        assert np.abs(a - e).max() / np.abs(e).max() < 2e-2
    finally:
        gpu.set_option(4, 35)
        om.close()


def test_paths_self_consistent(gpu):
    rng = np.random.default_rng(8)
    toks = rng.integers(0, 262144, size=600).astype(np.int32)
    gpu.forward(toks[:512], 0)
    for row in (0, 511):
        lg, am = gpu.logits(row)
        assert np.isfinite(lg).all() and np.abs(lg).max() <= 30.0
        assert am == int(np.argmax(lg))
    pos = 512
    for _ in range(3):                       # graph path (first call eager, then capture + replay)
        gpu.forward(toks[pos:pos + 1], pos)
        lg, am = gpu.logits(0)
        assert am == int(np.argmax(lg)) and np.isfinite(lg).all()
        pos += 1
    gpu.forward(toks[pos:pos + 3], pos)      # small batch
    for r in range(3):
        lg, am = gpu.logits(r)
        assert am == int(np.argmax(lg))
    vals, ids = gpu.topk(2, 64)
    lg, _ = gpu.logits(2)
    order = np.lexsort((np.arange(lg.size), -lg))[:64]   # value desc, id asc
    assert np.array_equal(ids, order.astype(np.int32))
    assert np.array_equal(vals, lg[order])


def test_graph_replay_equals_eager(g4, image):
    rng = np.random.default_rng(9)
    toks = rng.integers(0, 262144, size=16).astype(np.int32)
    outs = []
    for graphs in (1, 0):
        with g4.Model(image) as m:
            m.set_option(g4.OPT_PERSISTENT, 0)
            m.set_option(1, graphs)
            m.forward(toks[:8], 0)
            for p in range(8, 12):
                m.forward(toks[p:p + 1], p)
            outs.append(m.logits(0)[0])
    assert np.array_equal(outs[0], outs[1])


def test_prefill_gemm_paths_bitidentical(g4, image):
    """The tensor-core GEMM (store, GEGLU-pair and PLE-gate epilogues) and the
    SIMT dp4a GEMM run the same per-group fp32 chain, so a whole prefill gives
    the same bits on either path."""
    rng = np.random.default_rng(10)
    toks = rng.integers(0, 262144, size=300).astype(np.int32)
    res, lgs = [], []
    for path in (2, 1):
        with g4.Model(image) as m:
            m.set_option(g4.OPT_GEMM_PATH, path)
            m.forward(toks, 0)
            res.append(m.residual(300))
            lgs.append(m.logits(299)[0])
    assert np.array_equal(res[0].view(np.uint32), res[1].view(np.uint32))
    assert np.array_equal(lgs[0].view(np.uint32), lgs[1].view(np.uint32))


def test_prefill_pdl_on_off_bitidentical(g4, image):
    """Programmatic dependent launch only lets a kernel start before the
    previous one ends: each waits for its predecessor before it reads or
    writes anything the predecessor touches, so three 512-token chunks
    (tcgen05 GEMMs; tensor-core attention in its whole-pair and split
    schedules, with and without the K/V split reused) give the same bits with
    it on and off."""
    rng = np.random.default_rng(12)
    toks = rng.integers(0, 262144, size=1536).astype(np.int32)
    res, lgs = [], []
    for pdl in (1, 0):
        with g4.Model(image) as m:
            m.set_option(g4.OPT_PDL, pdl)
            for c in range(0, 1536, 512):
                m.forward(toks[c:c + 512], c)
            res.append(m.residual(512))
            lgs.append(m.logits(511)[0])
    assert np.array_equal(res[0].view(np.uint32), res[1].view(np.uint32))
    assert np.array_equal(lgs[0].view(np.uint32), lgs[1].view(np.uint32))


@pytest.mark.parametrize("T", [20, 64])
def test_small_batch_gemm_paths_bitidentical(g4, image, T):
    """A chunk of at most 64 rows takes the small-batch mma GEMM by default;
    its store, GEGLU-pair and PLE-gate epilogues give the bits of the
    tensor-core and SIMT paths."""
    rng = np.random.default_rng(20 + T)
    toks = rng.integers(0, 262144, size=T).astype(np.int32)
    res, lgs = [], []
    for path in (3, 2, 1):
        with g4.Model(image) as m:
            m.set_option(g4.OPT_GEMM_PATH, path)
            m.forward(toks, 0)
            res.append(m.residual(T))
            lgs.append(m.logits(T - 1)[0])
    for i in (1, 2):
        assert np.array_equal(res[0].view(np.uint32), res[i].view(np.uint32))
        assert np.array_equal(lgs[0].view(np.uint32), lgs[i].view(np.uint32))


def test_logits_rows_equal_logits(g4, image):
    """g4_logits_rows (the --dump-logits loop: lm_head GEMM over 64-row chunks,
    copies overlapped) gives every row the same bits as g4_logits."""
    rng = np.random.default_rng(12)
    toks = rng.integers(0, 262144, size=300).astype(np.int32)
    with g4.Model(image) as m:
        m.forward(toks, 0)
        allrows = m.logits_rows(0, 300)
        part = m.logits_rows(100, 37)
        for r in (0, 63, 64, 150, 299):
            lg, _ = m.logits(r)
            assert np.array_equal(allrows[r].view(np.uint32), lg.view(np.uint32))
        assert np.array_equal(part.view(np.uint32), allrows[100:137].view(np.uint32))
        with pytest.raises(g4.G4Error):
            m.logits_rows(290, 20)


def test_api_errors(g4, gpu):
    with pytest.raises(g4.G4Error) as e:
        gpu.forward(np.array([262144], np.int32), 0)
    assert e.value.code == -1
    with pytest.raises(g4.G4Error):
        gpu.forward(np.zeros(513, np.int32), 0)
    with pytest.raises(g4.G4Error):
        gpu.forward(np.zeros(1, np.int32), 131072)
    gpu.forward(np.zeros(2, np.int32), 0)
    with pytest.raises(g4.G4Error) as e:
        gpu.logits(2)
    assert e.value.code == -6

"""The persistent single-token decode kernel against the multi-kernel path.

With G4_OPT_PERSISTENT (the default) a one-token g4_forward is one cooperative
kernel per step: every GEMV, the split attention, the split combine and the
per-layer-input preparation run back to back inside it, separated by grid
barriers, while one warp per SM streams the step's weights. It computes the
same per-row integer dots, the same ordered dequantisation chains, the same
block reductions and the same attention tiles as the standalone kernels, so
its results must equal the multi-kernel path's bit for bit: residual stream,
every KV-cache slot written, logits and argmax. Covered: the fused
forward+logits launch, the forward-only launch (flushed by the next forward,
by a residual read, by a cache read), sliding-window wrap and global layers
at a long context (many attention splits), and a reduced layer count.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(g4, image, persistent, toks, prefill, steps, layers=35, read_every=0):
    """Prefill `prefill` tokens in 512-token chunks, then `steps` single-token
    steps; returns per-step (logits, argmax) plus final residual and caches."""
    out = {"logits": [], "argmax": [], "res": []}
    with g4.Model(image) as m:
        m.set_option(g4.OPT_PERSISTENT, persistent)
        m.set_option(g4.OPT_LAYERS, layers)
        for p0 in range(0, prefill, 512):
            m.forward(toks[p0:min(prefill, p0 + 512)], p0)
        pos = prefill
        for s in range(steps):
            m.forward(toks[pos:pos + 1], pos)
            if read_every and s % read_every == 1:
                out["res"].append(m.residual(1))       # flushes a forward-only launch
                m.forward(toks[pos + 1:pos + 2], pos + 1)  # another step without logits in between
                pos += 1
            lg, am = m.logits(0)
            out["logits"].append(lg)
            out["argmax"].append(am)
            pos += 1
        out["res"].append(m.residual(1))
        out["caches"] = []
        for layer in (0, 4, 13, 14, min(layers, 35) - 1):
            glob = layer % 5 == 4
            hd = 512 if glob else 256
            lo, n = (max(0, pos - 600), pos - max(0, pos - 600)) if glob else (0, 1024)
            k = m.cache(layer, 0, lo, n, hd)
            v = m.cache(layer, 1, lo, n, hd)
            out["caches"].append((k, v))
    return out


def _same(a, b):
    for la, lb in zip(a["logits"], b["logits"]):
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    assert a["argmax"] == b["argmax"]
    for ra, rb in zip(a["res"], b["res"]):
        assert np.array_equal(ra.view(np.uint32), rb.view(np.uint32))
    for (ka, va), (kb, vb) in zip(a["caches"], b["caches"]):
        assert np.array_equal(ka.view(np.uint32), kb.view(np.uint32))
        assert np.array_equal(va.view(np.uint32), vb.view(np.uint32))


def test_persistent_equals_kernels_short(g4, image):
    rng = np.random.default_rng(31)
    toks = rng.integers(0, g4.VOCAB, size=64).astype(np.int32)
    a = _run(g4, image, 1, toks, 8, 6, read_every=3)
    b = _run(g4, image, 0, toks, 8, 6, read_every=3)
    _same(a, b)


def test_persistent_equals_kernels_long_context(g4, image):
    # 2100 positions: the sliding ring has wrapped twice, global layers attend
    # to all keys with every split active
    rng = np.random.default_rng(32)
    toks = rng.integers(0, g4.VOCAB, size=2200).astype(np.int32)
    a = _run(g4, image, 1, toks, 2100, 3)
    b = _run(g4, image, 0, toks, 2100, 3)
    _same(a, b)


def test_persistent_reduced_layers(g4, image):
    rng = np.random.default_rng(33)
    toks = rng.integers(0, g4.VOCAB, size=32).astype(np.int32)
    a = _run(g4, image, 1, toks, 5, 3, layers=7)
    b = _run(g4, image, 0, toks, 5, 3, layers=7)
    _same(a, b)


def test_persistent_one_launch_per_token(g4, image):
    with g4.Model(image) as m:
        m.set_option(g4.OPT_PERSISTENT, 1)
        assert m.launches_per_token() == 1
        m.set_option(g4.OPT_PERSISTENT, 0)
        assert m.launches_per_token() == 2 + 8 * 35 + 2


def test_trace_timeline(g4, image):
    with g4.Model(image) as m:
        m.set_option(g4.OPT_PERSISTENT, 1)
        m.forward(np.arange(4, dtype=np.int32), 0)
        types, t = m.trace_decode(5, 4)
        assert len(types) == 2 + 8 * 35 + 1            # embed GEMV, PLE prep, 8 ops per layer, lm_head
        assert types[0] == 0 and types[1] == 3 and types[-1] == 0
        ends = t[:, 2]
        assert (np.diff(ends) >= 0).all() and ends[-1] > 0
        gemv = types == 0
        assert (t[gemv, 0] >= 0).all() and (t[gemv, 0] <= t[gemv, 1]).all()
        lg, am = m.logits(0)                            # the traced step computed row 0's logits
        assert am == int(np.argmax(lg))
        m.set_option(g4.OPT_PERSISTENT, 0)
        with pytest.raises(g4.G4Error):
            m.trace_decode(5, 5)

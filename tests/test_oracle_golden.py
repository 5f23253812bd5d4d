"""The oracle restatement against the reference's own outputs (CPU).

tests/golden/*.npz were produced by running the unmodified reference
gemma4.c (tests/golden/make_golden.py); every comparison here is bit-exact.
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def gk():
    return np.load(os.path.join(GOLD, "kernels.npz"))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_quantize(oracle, gk):
    q, s = oracle.quantize(gk["quant_x"])
    assert np.array_equal(q, gk["quant_q"])
    assert np.array_equal(bits(s), bits(gk["quant_s"]))


@pytest.mark.parametrize("tag", ["mm_a", "mm_b"])
def test_matmul(oracle, gk, tag):
    N, K, T = (int(v) for v in gk[f"{tag}_shape"])
    out = oracle.linear(gk[f"{tag}_xq"], gk[f"{tag}_xs"], gk[f"{tag}_wp"], gk[f"{tag}_sp"], N, K)
    assert np.array_equal(bits(out), bits(gk[f"{tag}_out"]))


def test_rmsnorm(oracle, gk):
    assert np.array_equal(bits(oracle.rmsnorm(gk["rms_x"], gk["rms_w"])), bits(gk["rms_y"]))
    assert np.array_equal(bits(oracle.rmsnorm(gk["rms2_x"], None)), bits(gk["rms2_y"]))


@pytest.mark.parametrize("tag", ["rope_s", "rope_g"])
def test_rope(oracle, gk, tag):
    hd, pairs = (int(v) for v in gk[f"{tag}_cfg"])
    # the fixture holds table rows 1001..1002; run at start_pos 0 on those rows
    y = oracle.rope(gk[f"{tag}_v"], gk[f"{tag}_cos"], gk[f"{tag}_sin"], 8, hd, 0)
    assert np.array_equal(bits(y), bits(gk[f"{tag}_y"]))


def test_geglu_edges(oracle, gk):
    y = oracle.geglu(gk["geglu_gate"], gk["geglu_up"], 256, 512, gk["geglu_table"])
    assert np.array_equal(bits(y), bits(gk["geglu_y"]))


def test_embedding(oracle, gk):
    mult = np.float32(np.sqrt(np.float32(1536)))
    y = oracle.embedding(gk["emb_wp"], gk["emb_sp"], 1536, gk["emb_tokens"], mult)
    assert np.array_equal(bits(y), bits(gk["emb_y"]))


def test_softmax(oracle, gk):
    x = np.array(gk["softmax_x"], np.float32)
    oracle.lib.or_softmax.argtypes = [np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS"), __import__("ctypes").c_int]
    oracle.lib.or_softmax(x, x.size)
    assert np.array_equal(bits(x), bits(gk["softmax_y"]))


def test_whole_model(oracle, image):
    """6-token prefill + 1 decode step on the seed-0 image: residuals and the
    logits' top-32 and float64 checksums equal the reference's."""
    g = np.load(os.path.join(GOLD, "model.npz"))
    m = oracle.open_model(image)
    try:
        toks = g["tokens"]
        m.forward(toks[:6], 0)
        assert np.array_equal(bits(m.residual(6)), bits(g["prefill_residual"]))
        for tag, row in (("prefill_row5", 5), ("prefill_row0", 0)):
            lg = m.logits(row)
            top = np.argsort(-lg, kind="stable")[:32]
            assert np.array_equal(top, g[f"{tag}_top_ids"])
            assert np.array_equal(bits(lg[top]), bits(g[f"{tag}_top_vals"]))
            assert lg.astype(np.float64).sum() == g[f"{tag}_sum"][0]
        m.forward(toks[6:7], 6)
        assert np.array_equal(bits(m.residual(1)), bits(g["decode_residual"]))
        lg = m.logits(0)
        top = np.argsort(-lg, kind="stable")[:32]
        assert np.array_equal(top, g["decode_top_ids"])
        assert (lg.astype(np.float64) ** 2).sum() == g["decode_sum"][1]
    finally:
        m.close()


def test_sample(oracle):
    """sample() (gemma4.c:536-561) with the generator state chained through the rows."""
    g = np.load(os.path.join(GOLD, "sample.npz"))
    state = 42
    for lg, t, tok, st in zip(g["logits"], g["temperature"], g["token"], g["state"]):
        got, state = oracle.sample(lg, float(t), state)
        assert got == int(tok) and state == int(st)

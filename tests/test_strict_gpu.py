"""Whole-model parity in strict mode: bit-exact with the reference.

The synthetic random-weight model is chaotic: a one-ulp difference anywhere
(for example a different RMSNorm summation order) flips an int8 quantisation
step, and the random layers amplify the flip until, after 35 layers, logits
decorrelate. Reordering only the reference's own sums on the CPU already
produces that (the oracle with a blocked sum of squares diverges from the
reference by ~1 in relative residual after 35 layers). So a tolerance check
of the fast path on this model cannot pass, and whole-model parity is shown
in strict mode instead: RMSNorm sums, attention scores, softmax and value sums
run in the reference's sequential order with the host library's expf
(G4_OPT_STRICT). Everything else (embedding, quantisation, every int8 dot
product and its dequant chain, RoPE, GeGLU, residual updates) runs on the same
kernels as the fast path. The residual stream must then equal the reference
bit for bit after every call, and the logits differ only through the final
30*tanh(x/30) (device tanhf vs the host's), i.e. by a few ulp.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-5   # tanhf ulp differences on |logit| <= 30


@pytest.fixture(scope="module")
def strict_pair(g4, reference, image):
    gpu = g4.Model(image)
    gpu.set_option(5, 1)   # G4_OPT_STRICT
    ref = reference.open_model(image)
    yield gpu, ref
    gpu.close()
    ref.close()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def check(pair, tokens, start_pos, rows):
    gpu, ref = pair
    gpu.forward(tokens, start_pos)
    ref.forward(tokens, start_pos)
    n = len(tokens)
    a, e = gpu.residual(n), ref.residual(n)
    mism = int((bits(a) != bits(e)).sum())
    assert mism == 0, f"residual differs in {mism} values (max abs {np.abs(a - e).max():.3e})"
    for r in rows:
        lg, am = gpu.logits(r)
        le = ref.logits(r)
        assert np.abs(lg - le).max() <= LOGIT_ATOL
        assert am == int(np.argmax(le))


def test_strict_sequence_bitexact(strict_pair):
    rng = np.random.default_rng(4)
    toks = rng.integers(0, 262144, size=700).astype(np.int32)
    check(strict_pair, toks[0:6], 0, [0, 5])                 # prefill chunk (GEMM path)
    check(strict_pair, toks[6:7], 6, [0])                    # single-token decode
    check(strict_pair, toks[7:10], 7, [0, 2])                # small batch (GEMV path, T=3)
    check(strict_pair, toks[10:522], 10, [0, 255, 511])      # 512-token chunk across the window
    check(strict_pair, toks[522:523], 522, [0])              # decode with a full sliding window
    check(strict_pair, toks[523:524], 523, [0])

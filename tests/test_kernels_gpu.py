"""Kernel-level parity on the GPU, through the C ABI, against the oracle.

Bar: the int8 dot products (int32 per token, row and
64-group) and the quantised activations are bit-exact; the dequantised fp32
GEMV/GEMM outputs are bit-exact too, because the kernels reproduce the
reference's per-group FMA chain (gemma4.c:218); RMSNorm outputs are within
fp32 tolerance (parallel sum of squares).
"""
import numpy as np
import pytest

from conftest import activations, packed_case

pytestmark = pytest.mark.gpu

# every projection shape of one layer (both head widths / MLP widths), the PLE
# projections and the model-level per_layer_model_projection (config 2)
LAYER_SHAPES = [
    (2048, 1536), (4096, 1536),      # q_proj sliding / global
    (256, 1536), (512, 1536),        # k/v_proj sliding / global
    (1536, 2048), (1536, 4096),      # o_proj
    (6144, 1536), (12288, 1536),     # gate/up (L0-14 / L15-34)
    (1536, 6144), (1536, 12288),     # down
    (1536, 256),                     # per_layer_projection (K=256)
    (8960, 1536),                    # per_layer_model_projection
]


def test_quantize_bitexact(g4, oracle):
    rng = np.random.default_rng(11)
    for rows, width in [(1, 1536), (7, 2048), (64, 12288), (3, 256)]:
        x = activations(rng, rows, width)
        x[0, :64] = 0.0                                   # zero group -> scale 0, q 0
        x[0, 64:128] = np.arange(64, dtype=np.float32) - 32.0
        x[0, 64 + 31] = 127.0                             # scale exactly 1: halves round to even
        x[0, 64:70] = [2.5, 3.5, -2.5, -3.5, 0.5, -0.5]
        q, s = g4.quantize(x)
        qo, so = oracle.quantize(x)
        assert np.array_equal(s.view(np.uint32), so.view(np.uint32)), (rows, width)
        assert np.array_equal(q, qo), (rows, width)
        assert list(q[0, 64:70]) == [2, 4, -2, -4, 0, 0]


@pytest.mark.parametrize("N,K", LAYER_SHAPES)
def test_gemv_decode_bitexact(g4, oracle, N, K):
    rng = np.random.default_rng(N * 7 + K)
    # config 2: one FP16 scale per row in [1e-4, 1e-2], replicated across groups
    _, _, wp, sp = packed_case(rng, N, K, per_group=False)
    xq, xs = oracle.quantize(rng.standard_normal((1, K)).astype(np.float32))
    out, dots = g4.linear(wp, sp, N, K, xq, xs, path=1, want_dots=True)
    ref_dots = oracle.linear_dots(xq, wp, N, K)
    ref = oracle.linear(xq, xs, wp, sp, N, K)
    assert np.array_equal(dots, ref_dots)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_gemv_lm_head_bitexact(g4, oracle):
    N, K = 262144, 1536
    rng = np.random.default_rng(5)
    _, _, wp, sp = packed_case(rng, N, K, per_group=True)
    xq, xs = oracle.quantize(rng.standard_normal((1, K)).astype(np.float32))
    out, _ = g4.linear(wp, sp, N, K, xq, xs, path=1)
    ref = oracle.linear(xq, xs, wp, sp, N, K)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("T", [2, 3, 4])
@pytest.mark.parametrize("N,K", [(2560, 1536), (1536, 12288), (1536, 256)])
def test_gemv_small_batch_bitexact(g4, oracle, T, N, K):
    rng = np.random.default_rng(T * 100 + N)
    _, _, wp, sp = packed_case(rng, N, K)
    xq, xs = oracle.quantize(activations(rng, T, K))
    out, dots = g4.linear(wp, sp, N, K, xq, xs, path=1, want_dots=True)
    assert np.array_equal(dots, oracle.linear_dots(xq, wp, N, K))
    assert np.array_equal(out.view(np.uint32), oracle.linear(xq, xs, wp, sp, N, K).view(np.uint32))


@pytest.mark.parametrize("T", [5, 64, 130, 512])
@pytest.mark.parametrize("N,K", [(2560, 1536), (1536, 4096), (1536, 256), (12288, 1536)])
def test_gemm_simt_bitexact(g4, oracle, T, N, K):
    rng = np.random.default_rng(T + N + K)
    _, _, wp, sp = packed_case(rng, N, K)
    xq, xs = oracle.quantize(activations(rng, T, K))
    out, dots = g4.linear(wp, sp, N, K, xq, xs, path=2, want_dots=True)
    assert np.array_equal(dots, oracle.linear_dots(xq, wp, N, K))
    assert np.array_equal(out.view(np.uint32), oracle.linear(xq, xs, wp, sp, N, K).view(np.uint32))


@pytest.mark.parametrize("T", [1, 5, 33, 64, 130, 512])
@pytest.mark.parametrize("N,K", [(2560, 1536), (1536, 4096), (1536, 256), (12288, 1536), (1536, 12288),
                                 (256, 1536), (2048, 1536)])
def test_gemm_tcgen05_bitexact(g4, oracle, T, N, K):
    """tcgen05 kind::i8 GEMM: exact int32 group dots on the tensor core, the
    reference's ordered fp32 chain in the epilogue -> bit-identical output.
    Up to 64 token rows it runs with transposed roles (128 weight rows as the
    MMA's M, the tokens as its N = 32 or 64)."""
    rng = np.random.default_rng(7 * T + N + K)
    _, _, wp, sp = packed_case(rng, N, K)
    xq, xs = oracle.quantize(activations(rng, T, K))
    out, _ = g4.linear(wp, sp, N, K, xq, xs, path=3)
    assert np.array_equal(out.view(np.uint32), oracle.linear(xq, xs, wp, sp, N, K).view(np.uint32))


@pytest.mark.parametrize("T", [1, 5, 8, 31, 33, 64])
@pytest.mark.parametrize("N,K", [(2560, 1536), (1536, 4096), (1536, 256), (12288, 1536), (1536, 12288),
                                 (256, 1536), (32768, 256), (65536, 256)])
def test_gemm_skinny_bitexact(g4, oracle, T, N, K):
    """Small-batch GEMM (mma.sync m16n8k32 s8 group dots, T <= 64 token rows):
    the same ordered fp32 chain -> bit-identical output. The shapes cover every
    row-block width it picks (16, 32, 64 and 128 output rows) and token tiles
    of 8, 16 and 32 rows per warp, with 4 or 8 groups per stage."""
    rng = np.random.default_rng(11 * T + N + K)
    _, _, wp, sp = packed_case(rng, N, K)
    xq, xs = oracle.quantize(activations(rng, T, K))
    out, _ = g4.linear(wp, sp, N, K, xq, xs, path=4)
    assert np.array_equal(out.view(np.uint32), oracle.linear(xq, xs, wp, sp, N, K).view(np.uint32))


def test_gemm_skinny_rejects_large_batches(g4, oracle):
    rng = np.random.default_rng(2)
    _, _, wp, sp = packed_case(rng, 256, 256)
    xq, xs = oracle.quantize(activations(rng, 65, 256))
    with pytest.raises(g4.G4Error):
        g4.linear(wp, sp, 256, 256, xq, xs, path=4)


def test_rmsnorm_quant(g4, oracle):
    rng = np.random.default_rng(3)
    x = activations(rng, 33, 1536)
    w = rng.uniform(0.5, 1.5, 1536).astype(np.float32)
    y, q, s = g4.rmsnorm_quant(x, w)
    yo = oracle.rmsnorm(x, w)
    # fp32 sum of squares in a different order: a few ulp of the normaliser
    np.testing.assert_allclose(y, yo, rtol=2e-6, atol=1e-7)
    qo, so = oracle.quantize(yo)
    # quantised values may flip by one step only where y itself moved across a rounding boundary
    diff = np.abs(q.astype(np.int32) - qo.astype(np.int32))
    assert diff.max() <= 1
    assert (diff != 0).mean() < 1e-3
    # quantising the kernel's own y is exact
    q2, s2 = oracle.quantize(y)
    assert np.array_equal(q, q2) and np.array_equal(s.view(np.uint32), s2.view(np.uint32))


def test_mma_i8_peak_runs(g4):
    """The int8 tensor-pipe microbenchmark (the measured denominator of the
    prefill GEMM roofline) completes without a device error, and its rate is
    within a plausible range for a B200 (between 0.5 and 1.2 x the 4.5 POP/s
    datasheet dense figure)."""
    ms, ops = g4.bench_mma_i8(4000)
    tops = ops / (ms * 1e-3) / 1e12
    assert 0.5 * 4500 < tops < 1.2 * 4500, tops
